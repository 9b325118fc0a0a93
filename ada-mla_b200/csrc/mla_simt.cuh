// mla_simt.cuh -- CUDA-core (SIMT) MLA decode kernels.
//
//  * naive_*        : the `naive` kernel name -- three launches with the
//                     attention matrix materialized in caller scratch,
//                     reference semantics of run_mla_decode_naive
//                     (csrc/mla_decode_naive_fwd.cu:4-31): scale 1/sqrt(D),
//                     all D output columns.
//  * simt_partial   : split-KV partial decode in fp32 arithmetic for fp32
//                     (and fp16) inputs; the fp32 `fused` kernel name
//                     (reference csrc/mla_decode_fused_fwd.cuh:50-352) runs on
//                     it.  Writes normalized partial O and its log-sum-exp per
//                     (work item, head); mla_combine.cuh merges them.
//
// fp32 has no tensor-core path here that keeps fp32 accuracy, so these are
// the fp32 kernels; fp16 decode runs on the tcgen05 kernel in mla_tc.cuh.
#pragma once

#include "mla_common.cuh"

namespace mla {

// ---------------------------------------------------------------------------
// naive: C[M x N] = alpha * A[M x K] . op(B),  op(B) = B^T ([N x K]) when
// TRANS_B, else B ([K x N]).  16x16 output tile per block, 16-wide K tiles.
// ---------------------------------------------------------------------------
template <bool TRANS_B>
__global__ void __launch_bounds__(256) naive_gemm_kernel(const float *__restrict__ A,
                                                         const float *__restrict__ B,
                                                         float *__restrict__ C, int M, int N,
                                                         int K, int ldc, float alpha) {
    __shared__ float As[16][17];
    __shared__ float Bs[16][17];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int row = blockIdx.y * 16 + ty;  // M index
    const int col = blockIdx.x * 16 + tx;  // N index
    float acc = 0.f;
    for (int k0 = 0; k0 < K; k0 += 16) {
        {
            const int k = k0 + tx;
            As[ty][tx] = (row < M && k < K) ? A[(size_t)row * K + k] : 0.f;
        }
        {
            // Bs[kk][n] = op(B)[k0+kk][blockIdx.x*16 + n]
            const int kk = ty, n = blockIdx.x * 16 + tx;
            const int k = k0 + kk;
            float v = 0.f;
            if (k < K && n < N) v = TRANS_B ? B[(size_t)n * K + k] : B[(size_t)k * ldc + n];
            Bs[kk][tx] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) acc += As[ty][kk] * Bs[kk][tx];
        __syncthreads();
    }
    if (row < M && col < N) C[(size_t)row * N + col] = alpha * acc;
}

// In-place row softmax of attn [rows x n] (one block per row).
__global__ void __launch_bounds__(256) naive_softmax_kernel(float *__restrict__ attn, int n) {
    __shared__ float red[8];
    float *r = attn + (size_t)blockIdx.x * n;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < n; j += blockDim.x) mx = fmaxf(mx, r[j]);
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, red[i]);
    __syncthreads();
    float s = 0.f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) s += expf(r[j] - mx);
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += red[i];
    const float inv = 1.f / s;
    for (int j = threadIdx.x; j < n; j += blockDim.x) r[j] = expf(r[j] - mx) * inv;
}

// ---------------------------------------------------------------------------
// simt_partial: one block per (work item, block of 16 heads).
//   S = scale * Q_blk . C_tile^T         (16 heads x 32 tokens, fp32 FMA)
//   online softmax in base 2 (running max m, running sum l, fp32)
//   O_blk += P . C_tile[:, :512]         (16 heads x 512, registers)
// and at the end writes O / l and lse = (m + log2 l) * ln2.
// ---------------------------------------------------------------------------
constexpr int kSimtHeads = 16;
constexpr int kSimtTok = 32;
constexpr int kSimtLd = kDK + 1;  // padded smem row: conflict-free column walks
constexpr size_t kSimtSmem =
    sizeof(float) * ((size_t)kSimtHeads * kSimtLd + (size_t)kSimtTok * kSimtLd +
                     kSimtHeads * kSimtTok + 3 * kSimtHeads);

template <typename T>
__global__ void __launch_bounds__(256) simt_partial_kernel(const T *__restrict__ q,
                                                           const T *__restrict__ cache,
                                                           WorkList wl, int num_heads,
                                                           float scale_log2,
                                                           float *__restrict__ part_o,
                                                           float *__restrict__ part_lse) {
    extern __shared__ float smem[];
    float *Qs = smem;                               // [16][577]
    float *Cs = Qs + kSimtHeads * kSimtLd;          // [32][577]
    float *Ps = Cs + kSimtTok * kSimtLd;            // [16][32]
    float *alpha_s = Ps + kSimtHeads * kSimtTok;    // [16]
    float *m_s = alpha_s + kSimtHeads;              // [16]
    float *l_s = m_s + kSimtHeads;                  // [16]

    const int item_idx = blockIdx.x;
    const Item it = get_item(wl, item_idx);
    const int h0 = blockIdx.y * kSimtHeads;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (it.len <= 0) {
        // Empty item (only possible past the end of a varlen list): no partial.
        return;
    }

    // Q block -> smem (fp32).
    const T *qb = q + ((size_t)it.b * num_heads + h0) * kDK;
    for (int e = tid; e < kSimtHeads * kDK; e += 256) {
        const int h = e / kDK, k = e - h * kDK;
        Qs[h * kSimtLd + k] = (h0 + h < num_heads) ? to_f32(qb[(size_t)h * kDK + k]) : 0.f;
    }

    // softmax state: warp w owns heads 2w, 2w+1 (lane-uniform registers)
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_run[2] = {0.f, 0.f};
    float oacc[kSimtHeads][2];
#pragma unroll
    for (int h = 0; h < kSimtHeads; ++h) oacc[h][0] = oacc[h][1] = 0.f;
    const int d0 = tid * 2;  // this thread's two output columns

    const T *cb = cache + (size_t)it.row0 * kDK;
    for (int t0 = 0; t0 < it.len; t0 += kSimtTok) {
        const int nt = min(kSimtTok, it.len - t0);
        __syncthreads();  // previous tile fully consumed (and Q visible on 1st pass)
        for (int e = tid; e < kSimtTok * kDK; e += 256) {
            const int t = e / kDK, k = e - t * kDK;
            Cs[t * kSimtLd + k] = (t < nt) ? to_f32(cb[(size_t)(t0 + t) * kDK + k]) : 0.f;
        }
        __syncthreads();
        // S: thread -> (head tid/16, tokens tid%16 and tid%16 + 16)
        {
            const int h = tid >> 4, t = tid & 15;
            const float *qr = Qs + h * kSimtLd;
            const float *c0 = Cs + t * kSimtLd;
            const float *c1 = Cs + (t + 16) * kSimtLd;
            float a0 = 0.f, a1 = 0.f;
#pragma unroll 8
            for (int k = 0; k < kDK; ++k) {
                const float qv = qr[k];
                a0 = fmaf(qv, c0[k], a0);
                a1 = fmaf(qv, c1[k], a1);
            }
            Ps[h * kSimtTok + t] = (t < nt) ? a0 * scale_log2 : -INFINITY;
            Ps[h * kSimtTok + t + 16] = (t + 16 < nt) ? a1 * scale_log2 : -INFINITY;
        }
        __syncthreads();
        // online softmax, base 2
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int h = warp * 2 + j;
            const float s = Ps[h * kSimtTok + lane];
            const float m_new = fmaxf(m_run[j], warp_max(s));
            const float p = (s == -INFINITY) ? 0.f : exp2f(s - m_new);
            const float alpha = (m_run[j] == -INFINITY) ? 0.f : exp2f(m_run[j] - m_new);
            l_run[j] = l_run[j] * alpha + warp_sum(p);
            m_run[j] = m_new;
            Ps[h * kSimtTok + lane] = p;
            if (lane == 0) alpha_s[h] = alpha;
        }
        __syncthreads();
        // O update
#pragma unroll
        for (int h = 0; h < kSimtHeads; ++h) {
            const float a = alpha_s[h];
            oacc[h][0] *= a;
            oacc[h][1] *= a;
        }
        for (int t = 0; t < nt; ++t) {
            const float c0 = Cs[t * kSimtLd + d0];
            const float c1 = Cs[t * kSimtLd + d0 + 1];
#pragma unroll
            for (int h = 0; h < kSimtHeads; ++h) {
                const float p = Ps[h * kSimtTok + t];
                oacc[h][0] = fmaf(p, c0, oacc[h][0]);
                oacc[h][1] = fmaf(p, c1, oacc[h][1]);
            }
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            m_s[warp * 2 + j] = m_run[j];
            l_s[warp * 2 + j] = l_run[j];
        }
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < kSimtHeads; ++h) {
        if (h0 + h >= num_heads) break;
        const float l = l_s[h];
        const float inv = l > 0.f ? 1.f / l : 0.f;
        float2 v = make_float2(oacc[h][0] * inv, oacc[h][1] * inv);
        const size_t row = (size_t)item_idx * num_heads + h0 + h;
        *reinterpret_cast<float2 *>(part_o + row * kDV + d0) = v;
        if (tid == 0) part_lse[row] = l > 0.f ? (m_s[h] + log2f(l)) * kLn2 : -INFINITY;
    }
}

}  // namespace mla
