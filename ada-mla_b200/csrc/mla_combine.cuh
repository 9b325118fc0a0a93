// mla_combine.cuh -- log-sum-exp merge of split-KV partials, and the varlen
// planning kernel that expands cu_seqlens into the work list.
//
// The reference merges its fp16 split partials in mla_decode_combine
// (csrc/mla_decode_splitk_fwd.cuh:894-939): one 128-thread block per head,
// each thread looping serially over the splits and recomputing expf for every
// element.  Here a block still owns one (sequence, head) row, but the split
// weights w_i = exp(lse_i - max_i lse_i) are computed once per split into
// shared memory and groups of threads stream disjoint splits of the row with
// several 16-byte loads in flight.  Partials are fp16 (as in the reference)
// when the output is fp16, fp32 otherwise.  The same kernel serves the intra-GPU split merge
// and the cross-GPU merge after an all-gather (any number of parts, fp16 or
// fp32 output, optional merged LSE).
#pragma once

#include <type_traits>

#include "mla_common.cuh"

namespace mla {

constexpr int kCombineThreads = 512;

// Two output elements (fp16 or bf16) packed into 32 bits.
template <typename OutT>
__device__ __forceinline__ uint32_t pack_out2(float a, float b) {
    if constexpr (std::is_same<OutT, __nv_bfloat16>::value) {
        __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&t);
    } else {
        __half2 t = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&t);
    }
}
constexpr int kCombineChunk = 1024;      // split weights staged per pass

// Unpacks one 16-byte vector of partial elements to fp32.
__device__ __forceinline__ void unpack16(const uint4 u, float (&v)[4]) {
    v[0] = __uint_as_float(u.x); v[1] = __uint_as_float(u.y);
    v[2] = __uint_as_float(u.z); v[3] = __uint_as_float(u.w);
}
__device__ __forceinline__ void unpack16(const uint4 u, float (&v)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[j]));
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
    }
}

// The same for bf16 partials, and the choice by partial type.
__device__ __forceinline__ void unpack16_bf16(const uint4 u, float (&v)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[j]));
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
    }
}

template <typename PartT, int N>
__device__ __forceinline__ void unpack_part(const uint4 u, float (&v)[N]) {
    if constexpr (std::is_same<PartT, __nv_bfloat16>::value) unpack16_bf16(u, v);
    else unpack16(u, v);
}

// rows = batch * num_heads; one block per row r = (b, h).  Partial i of row
// (b, h) lives at part_o[(i * num_heads + h) * 512] and part_lse[i * num_heads
// + h], for i in item_range(b).  Normalized partials: O_i = sum_j p_j C_j / l_i
// and lse_i = ln(l_i) + max logit.  Merged:
//   O = sum_i e^{lse_i - M} O_i / sum_i e^{lse_i - M},  M = max_i lse_i.
// The weights are computed once per split into shared memory.  A thread owns
// one 16-byte vector of the row (4 fp32 or 8 fp16 partial elements); the
// block's 512 threads form 4 (fp32) or 8 (fp16) groups that stream disjoint
// splits with 8 loads in flight each, and their sums meet in shared memory.
// skip_single: rows of sequences with exactly one item were already written
// by the decode kernel itself and are left alone.
// part_stride: elements from one partial's [num_heads, 512] block to the next
// (num_heads * 512 in the workspace; larger in a packed exchange buffer, where
// each part's LSE follows its O), lse_stride likewise for part_lse.
template <typename OutT, typename PartT>
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(
    const PartT *__restrict__ part_o, const float *__restrict__ part_lse, WorkList wl,
    int num_heads, long long rows, OutT *__restrict__ out, float *__restrict__ out_lse,
    int skip_single, size_t part_stride, size_t lse_stride) {
    constexpr int kVec = 16 / (int)sizeof(PartT);       // partial elements per thread
    constexpr int kTpr = kDV / kVec;                    // threads covering one row
    constexpr int kGroups = kCombineThreads / kTpr;     // split groups per block
    __shared__ float w_s[kCombineChunk];
    __shared__ float red[kCombineThreads / 32];
    __shared__ __align__(16) float acc_s[kGroups - 1][kDV];
    griddep_launch();  // the next decode may place its CTAs and set up
    griddep_wait();    // the partials are complete and visible
    const long long row = blockIdx.x;
    if (row >= rows) return;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int col = tid % kTpr, g = tid / kTpr;
    const int b = (int)(row / num_heads);
    const int h = (int)(row - (long long)b * num_heads);
    int i0, i1;
    item_range(wl, b, i0, i1);
    if (skip_single && i1 - i0 == 1) return;

    // this thread's first split's LSE stays in a register for the weights below
    // (one L2 round trip fewer for up to kCombineThreads splits)
    const float my_lse = i0 + tid < i1 ? part_lse[(size_t)(i0 + tid) * lse_stride + h] : -INFINITY;
    float mx = my_lse;
    for (int i = i0 + tid + kCombineThreads; i < i1; i += kCombineThreads)
        mx = fmaxf(mx, part_lse[(size_t)i * lse_stride + h]);
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kCombineThreads / 32; ++w) mx = fmaxf(mx, red[w]);

    float acc[kVec];
#pragma unroll
    for (int j = 0; j < kVec; ++j) acc[j] = 0.f;
    float wsum = 0.f;  // identical in every thread (same weights, same order)
    if (mx != -INFINITY) {
        const size_t step = part_stride / kVec;  // one split, in 16-byte vectors
        for (int c0 = i0; c0 < i1; c0 += kCombineChunk) {
            const int n = min(kCombineChunk, i1 - c0);
            __syncthreads();
            for (int k = tid; k < n; k += kCombineThreads) {
                const float lse = (c0 == i0 && k == tid) ? my_lse : part_lse[(size_t)(c0 + k) * lse_stride + h];
                w_s[k] = lse == -INFINITY ? 0.f : __expf(lse - mx);
            }
            __syncthreads();
            for (int k = 0; k < n; ++k) wsum += w_s[k];
            const uint4 *src = reinterpret_cast<const uint4 *>(part_o + (size_t)c0 * part_stride + (size_t)h * kDV) + col;
            // up to kInflight splits' loads in flight per thread (predicated at the end;
            // 12 measured no different on cfg3's 72 splits and 0.25 us slower on cfg1)
            constexpr int kInflight = 8;
            for (int k = g; k < n; k += kInflight * kGroups) {
                uint4 u[kInflight];
#pragma unroll
                for (int j = 0; j < kInflight; ++j)
                    if (k + j * kGroups < n) u[j] = __ldg(src + (size_t)(k + j * kGroups) * step);
#pragma unroll
                for (int j = 0; j < kInflight; ++j) {
                    if (k + j * kGroups < n) {
                        float v[kVec];
                        unpack_part<PartT>(u[j], v);
                        const float w = w_s[k + j * kGroups];
#pragma unroll
                        for (int e = 0; e < kVec; ++e) acc[e] = fmaf(w, v[e], acc[e]);
                    }
                }
            }
        }
    }
    if (g > 0) {
#pragma unroll
        for (int e = 0; e < kVec; ++e) acc_s[g - 1][col * kVec + e] = acc[e];
    }
    __syncthreads();
    if (g != 0) return;
#pragma unroll
    for (int o = 0; o < kGroups - 1; ++o) {
#pragma unroll
        for (int e = 0; e < kVec; ++e) acc[e] += acc_s[o][col * kVec + e];
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    OutT *dst = out + (size_t)row * kDV + col * kVec;
#pragma unroll
    for (int e0 = 0; e0 < kVec; e0 += 4) {
        const float4 v = make_float4(acc[e0] * inv, acc[e0 + 1] * inv, acc[e0 + 2] * inv, acc[e0 + 3] * inv);
        if constexpr (sizeof(OutT) == 4) {
            *reinterpret_cast<float4 *>(dst + e0) = v;
        } else {
            uint2 u;
            u.x = pack_out2<OutT>(v.x, v.y);
            u.y = pack_out2<OutT>(v.z, v.w);
            *reinterpret_cast<uint2 *>(dst + e0) = u;
        }
    }
    if (out_lse != nullptr && tid == 0) out_lse[row] = wsum > 0.f ? mx + __logf(wsum) : -INFINITY;
}

// Row-parallel merge for batches: one warp per (sequence, head) row and one
// block per 8 heads of one sequence, so a sequence's item range is read once
// per block and a block of a sequence decoded as a single item (already final)
// exits at once.  Lane l owns columns [16 l, 16 l + 16); the split weights
// e^{lse_i - M} live in the lanes (lane j holds split s0 + j) and are
// broadcast with shuffles while four splits' loads are in flight.
constexpr int kRowsPerCombineBlock = 8;

template <typename PartT>
__device__ __forceinline__ void load16(const PartT *row, int lane, uint4 (&u)[16 / (16 / (int)sizeof(PartT))]) {
    const uint4 *src = reinterpret_cast<const uint4 *>(row) + lane * (16 * (int)sizeof(PartT) / 16);
#pragma unroll
    for (int j = 0; j < 16 * (int)sizeof(PartT) / 16; ++j) u[j] = __ldg(src + j);
}

template <typename OutT, typename PartT>
__global__ void __launch_bounds__(32 * kRowsPerCombineBlock) combine_rows_kernel(
    const PartT *__restrict__ part_o, const float *__restrict__ part_lse, WorkList wl, int num_heads,
    OutT *__restrict__ out, float *__restrict__ out_lse, int skip_single) {
    constexpr int kU = 16 * (int)sizeof(PartT) / 16;  // 16-byte vectors per lane per split
    griddep_launch();
    griddep_wait();
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.y;
    const int h = blockIdx.x * kRowsPerCombineBlock + (threadIdx.x >> 5);
    int i0, i1;
    item_range(wl, b, i0, i1);
    if ((skip_single && i1 - i0 == 1) || h >= num_heads) return;
    const int n = i1 - i0;
    float mx = -INFINITY;
    for (int s = lane; s < n; s += 32) mx = fmaxf(mx, part_lse[(size_t)(i0 + s) * num_heads + h]);
    mx = warp_max(mx);
    float acc[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[e] = 0.f;
    float wsum = 0.f;
    if (mx != -INFINITY) {
        for (int s0 = 0; s0 < n; s0 += 32) {
            const int m = min(32, n - s0);
            float w = 0.f;
            if (lane < m) {
                const float lse = part_lse[(size_t)(i0 + s0 + lane) * num_heads + h];
                w = lse == -INFINITY ? 0.f : __expf(lse - mx);
            }
            wsum += warp_sum(w);
            const PartT *base = part_o + ((size_t)(i0 + s0) * num_heads + h) * kDV;
            const size_t step = (size_t)num_heads * kDV;
            for (int j = 0; j < m; j += 4) {
                uint4 u[4][kU];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (j + k < m) load16<PartT>(base + (size_t)(j + k) * step, lane, u[k]);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float wk = __shfl_sync(0xffffffffu, w, (j + k) & 31);
                    if (j + k < m) {
#pragma unroll
                        for (int q = 0; q < kU; ++q) {
                            float v[16 / kU];
                            unpack_part<PartT>(u[k][q], v);
#pragma unroll
                            for (int e = 0; e < 16 / kU; ++e) acc[q * (16 / kU) + e] = fmaf(wk, v[e], acc[q * (16 / kU) + e]);
                        }
                    }
                }
            }
        }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    OutT *dst = out + ((size_t)b * num_heads + h) * kDV + lane * 16;
    if constexpr (sizeof(OutT) == 4) {
#pragma unroll
        for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4 *>(dst + e) = make_float4(acc[e] * inv, acc[e + 1] * inv, acc[e + 2] * inv, acc[e + 3] * inv);
    } else {
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) pk[e] = pack_out2<OutT>(acc[2 * e] * inv, acc[2 * e + 1] * inv);
        reinterpret_cast<uint4 *>(dst)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        reinterpret_cast<uint4 *>(dst)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    }
    if (out_lse != nullptr && lane == 0)
        out_lse[(size_t)b * num_heads + h] = wsum > 0.f ? mx + __logf(wsum) : -INFINITY;
}

// Paged cache: per-sequence lengths (clamped to max_len) into offsets cu[B+1] on
// a virtual packed axis, which the schedules then walk like a packed batch.
// Called by all 1024 threads of one block; cu is complete and visible to the
// block on return.
__device__ void lens_to_offsets(const int32_t *lens, int batch, int max_len, int32_t *cu) {
    __shared__ int warp_tot[32];
    __shared__ int carry_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) carry_s = 0;
    __syncthreads();
    for (int base = 0; base < batch; base += 1024) {
        const int b = base + tid;
        const int len = b < batch ? min(max(lens[b], 0), max_len) : 0;
        int v = len;
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
        const int excl = carry_s + (warp > 0 ? warp_tot[warp - 1] : 0) + v - len;
        if (b < batch) cu[b] = excl;
        __syncthreads();
        if (tid == 1023) carry_s = excl + len;
        __syncthreads();
    }
    if (tid == 0) cu[batch] = carry_s;
    __syncthreads();
}

// Expands cu_seqlens[B+1] into item_off[B+1] (exclusive prefix of per-sequence
// item counts) and items[] = {b, row_begin, row_end, token offset in the
// sequence}.  One block.  With
// seq_lens (paged cache) the offsets are first built into cu_out from the
// lengths and used as cu_seqlens.
__global__ void __launch_bounds__(1024) plan_varlen_kernel(const int32_t *cu_seqlens,
                                                           int batch, int chunk,
                                                           int *__restrict__ item_off,
                                                           int4 *__restrict__ items,
                                                           int max_items,
                                                           const int32_t *seq_lens = nullptr,
                                                           int max_len = 0,
                                                           int32_t *cu_out = nullptr,
                                                           int group = 1, int dense_len = 0) {
    __shared__ int warp_tot[32];
    __shared__ int carry_s;
    griddep_launch();  // the decode kernel may start its set-up now
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (seq_lens != nullptr) {
        lens_to_offsets(seq_lens, batch, max_len, cu_out);
        cu_seqlens = cu_out;
    }
    if (tid == 0) carry_s = 0;
    __syncthreads();
    for (int base = 0; base < batch; base += 1024) {
        const int b = base + tid;
        int cnt = 0;
        if (b < batch) {
            const int len = seq_len_of(cu_seqlens, dense_len, group, b);
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
            const int r0 = (int)seq_row0_of(cu_seqlens, dense_len, group, b);
            const int r1 = r0 + seq_len_of(cu_seqlens, dense_len, group, b);
            for (int c = 0; c < cnt && excl + c < max_items; ++c) {
                const int s = r0 + c * chunk;
                items[excl + c] = make_int4(b, s, min(s + chunk, r1), c * chunk);
            }
        }
        __syncthreads();
        if (tid == 1023) carry_s = excl + cnt;
        __syncthreads();
    }
    if (tid == 0) item_off[batch] = min(carry_s, max_items);
}

// Balanced schedule, varlen: cost_off[b] = sum over b' < b of the cost of
// sequence b' (item_cost + its 96-row tiles, 0 for an empty sequence), and
// cost_off[B] the total.  One block; a block-wide scan per 1024 sequences.
__global__ void __launch_bounds__(1024) plan_balanced_kernel(const int32_t *cu_seqlens,
                                                             int batch, int item_cost,
                                                             int *__restrict__ cost_off,
                                                             const int32_t *seq_lens = nullptr,
                                                             int max_len = 0,
                                                             int32_t *cu_out = nullptr,
                                                             int group = 1, int dense_len = 0) {
    __shared__ int warp_tot[32];
    __shared__ int carry_s;
    griddep_launch();  // the decode kernel may start its set-up now
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (seq_lens != nullptr) {
        lens_to_offsets(seq_lens, batch, max_len, cu_out);
        cu_seqlens = cu_out;
    }
    if (tid == 0) carry_s = 0;
    __syncthreads();
    for (int base = 0; base < batch; base += 1024) {
        const int b = base + tid;
        int cost = 0;
        if (b < batch) {
            const int len = seq_len_of(cu_seqlens, dense_len, group, b);
            cost = len > 0 ? (len + kTile - 1) / kTile + item_cost : 0;
        }
        int v = cost;
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
        const int excl = carry_s + (warp > 0 ? warp_tot[warp - 1] : 0) + v - cost;
        if (b < batch) cost_off[b] = excl;
        __syncthreads();
        if (tid == 1023) carry_s = excl + cost;
        __syncthreads();
    }
    if (tid == 0) cost_off[batch] = carry_s;
}

}  // namespace mla
