// mla_combine.cuh -- log-sum-exp merge of split-KV partials, and the varlen
// planning kernel that expands cu_seqlens into the work list.
//
// The reference merges its fp16 split partials in mla_decode_combine
// (csrc/mla_decode_splitk_fwd.cuh:894-939): one 128-thread block per head,
// each thread looping serially over the splits and recomputing expf for every
// element.  Here one WARP owns one (sequence, head) row: the split weights
// w_i = exp(lse_i - max_i lse_i) are computed once per split, every lane
// accumulates 16 of the 512 columns with float4 loads, and the same kernel
// serves the intra-GPU split merge and the cross-GPU merge after an
// all-gather (any number of parts, fp16 or fp32 output, optional merged LSE).
#pragma once

#include "mla_common.cuh"

namespace mla {

constexpr int kCombineWarps = 8;

// rows = batch * num_heads; row r = (b, h).  Partial i of row (b, h) lives at
// part_o[(i * num_heads + h) * 512] and part_lse[i * num_heads + h], for i in
// item_range(b).  Normalized partials: O_i = sum_j p_j C_j / l_i and
// lse_i = ln(l_i) + max logit.  Merged: O = sum_i e^{lse_i - M} O_i / sum_i e^{lse_i - M}.
template <typename OutT>
__global__ void __launch_bounds__(kCombineWarps * 32) combine_kernel(
    const float *__restrict__ part_o, const float *__restrict__ part_lse, WorkList wl,
    int num_heads, long long rows, OutT *__restrict__ out, float *__restrict__ out_lse) {
    const int lane = threadIdx.x & 31;
    const long long row = (long long)blockIdx.x * kCombineWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int b = (int)(row / num_heads);
    const int h = (int)(row - (long long)b * num_heads);
    int i0, i1;
    item_range(wl, b, i0, i1);

    float mx = -INFINITY;
    for (int i = i0 + lane; i < i1; i += 32) mx = fmaxf(mx, part_lse[(size_t)i * num_heads + h]);
    mx = warp_max(mx);

    float4 acc[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    float wsum = 0.f;
    if (mx != -INFINITY) {
        for (int i = i0; i < i1; ++i) {
            const size_t pr = (size_t)i * num_heads + h;
            const float lse = part_lse[pr];
            if (lse == -INFINITY) continue;
            const float w = __expf(lse - mx);
            wsum += w;
            const float4 *src = reinterpret_cast<const float4 *>(part_o + pr * kDV);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 v = src[lane + 32 * k];
                acc[k].x = fmaf(w, v.x, acc[k].x);
                acc[k].y = fmaf(w, v.y, acc[k].y);
                acc[k].z = fmaf(w, v.z, acc[k].z);
                acc[k].w = fmaf(w, v.w, acc[k].w);
            }
        }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    OutT *dst = out + (size_t)row * kDV;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int col = 4 * (lane + 32 * k);
        const float4 v = make_float4(acc[k].x * inv, acc[k].y * inv, acc[k].z * inv, acc[k].w * inv);
        if constexpr (sizeof(OutT) == 4) {
            *reinterpret_cast<float4 *>(dst + col) = v;
        } else {
            __half2 a = __floats2half2_rn(v.x, v.y), c = __floats2half2_rn(v.z, v.w);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t *>(&a);
            u.y = *reinterpret_cast<uint32_t *>(&c);
            *reinterpret_cast<uint2 *>(dst + col) = u;
        }
    }
    if (out_lse != nullptr && lane == 0) out_lse[row] = wsum > 0.f ? mx + __logf(wsum) : -INFINITY;
}

// Expands cu_seqlens[B+1] into item_off[B+1] (exclusive prefix of per-sequence
// item counts) and items[] = {b, row_begin, row_end, 0}.  One block.
__global__ void __launch_bounds__(1024) plan_varlen_kernel(const int32_t *__restrict__ cu_seqlens,
                                                           int batch, int chunk,
                                                           int *__restrict__ item_off,
                                                           int4 *__restrict__ items,
                                                           int max_items) {
    __shared__ int warp_tot[32];
    __shared__ int carry_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) carry_s = 0;
    __syncthreads();
    for (int base = 0; base < batch; base += 1024) {
        const int b = base + tid;
        int cnt = 0;
        if (b < batch) {
            const int len = cu_seqlens[b + 1] - cu_seqlens[b];
            cnt = len > 0 ? (len + chunk - 1) / chunk : 0;
        }
        // block-wide inclusive scan of cnt
        int v = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += n;
        }
        if (lane == 31) warp_tot[warp] = v;
        __syncthreads();
        if (warp == 0) {
            int w = warp_tot[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += n;
            }
            warp_tot[lane] = w;
        }
        __syncthreads();
        const int carry = carry_s;
        const int excl = carry + (warp > 0 ? warp_tot[warp - 1] : 0) + v - cnt;
        if (b < batch) {
            item_off[b] = min(excl, max_items);
            const int r0 = cu_seqlens[b];
            const int r1 = cu_seqlens[b + 1];
            for (int c = 0; c < cnt && excl + c < max_items; ++c) {
                const int s = r0 + c * chunk;
                items[excl + c] = make_int4(b, s, min(s + chunk, r1), 0);
            }
        }
        __syncthreads();
        if (tid == 1023) carry_s = excl + cnt;
        __syncthreads();
    }
    if (tid == 0) item_off[batch] = min(carry_s, max_items);
}

}  // namespace mla
