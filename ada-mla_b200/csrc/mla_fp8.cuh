// mla_fp8.cuh -- Q* preparation for the e4m3 latent cache.
//
// With an fp8 cache, GEMM1 (S = Q* C^T) runs as tcgen05.mma kind::f8f6f4, which
// takes both operands in 8-bit formats.  One e4m3 copy of Q* would carry only
// 3 mantissa bits (a 2^-4 relative rounding per element), too coarse for the
// attention logits; Q* therefore goes in as two e4m3 planes, hi = e4m3(x) and
// lo = e4m3(x - hi), whose sum carries Q* to about 2^-8 relative, and GEMM1 is
// S = hi C^T + lo C^T (two MMAs per K-step, same count as the fp16 path's K=16
// steps).  Each (sequence, head) row is first scaled by a power of two that
// puts its largest magnitude in [128, 448) (e4m3's top binades), so small rows
// do not fall into e4m3's subnormal range; the kernel folds the inverse scale
// into that row's softmax scale.  (No reference counterpart: the reference's
// cache is fp16/fp32 only and lists fp8 as future work, README.md:407-408.)
#pragma once

#include <cuda_fp8.h>

#include "mla_common.cuh"

namespace mla {

// q [rows, 576] fp16 -> q8 [2, rows, 576] e4m3 (hi plane, then lo plane) and
// q_scale [rows] (Q* = (hi + lo) * q_scale).  One warp per row.
__global__ void __launch_bounds__(256) q8_prep_kernel(const __half *__restrict__ q, int rows,
                                                     uint8_t *__restrict__ q8,
                                                     float *__restrict__ q_scale) {
    griddep_launch();  // the decode kernel may start its set-up
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;
    const __half2 *src = reinterpret_cast<const __half2 *>(q + (size_t)row * kDK);
    // 576 values = 288 half2: 9 per lane
    float2 v[9];
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < 9; ++k) {
        v[k] = __half22float2(src[lane + 32 * k]);
        amax = fmaxf(amax, fmaxf(fabsf(v[k].x), fabsf(v[k].y)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    // 2^e with amax * 2^e in [128, 448), from the exponent field (exact)
    int e = 0;
    if (amax > 0.f) {
        int ex;
        frexpf(amax, &ex);  // amax = f * 2^ex, f in [0.5, 1)
        e = 9 - ex;         // amax * 2^e in [256, 512)
        if (ldexpf(amax, e) >= 448.f) --e;
    }
    const float s = ldexpf(1.f, e);
    uint16_t *hi = reinterpret_cast<uint16_t *>(q8 + (size_t)row * kDK);
    uint16_t *lo = reinterpret_cast<uint16_t *>(q8 + ((size_t)rows + row) * kDK);
#pragma unroll
    for (int k = 0; k < 9; ++k) {
        const float2 x = make_float2(v[k].x * s, v[k].y * s);
        const __nv_fp8x2_storage_t h = __nv_cvt_float2_to_fp8x2(x, __NV_SATFINITE, __NV_E4M3);
        const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(h, __NV_E4M3);
        const float2 hf = __half22float2(*reinterpret_cast<const __half2 *>(&hr));
        const float2 r = make_float2(x.x - hf.x, x.y - hf.y);
        const __nv_fp8x2_storage_t l = __nv_cvt_float2_to_fp8x2(r, __NV_SATFINITE, __NV_E4M3);
        hi[lane + 32 * k] = h;
        lo[lane + 32 * k] = l;
    }
    if (lane == 0) q_scale[row] = ldexpf(1.f, -e);
}

}  // namespace mla
