// mla_proj.cuh -- per-head projections on either side of the decode, tcgen05:
//
//   Q absorption   Q*[b, h, 0:512] = q_nope[b, h, :] . W_UK[h]   (W_UK[h]: [d, 512])
//   O projection   o[b, h, 0:d_v]  = O*[b, h, :]     . W_UV[h]   (W_UV[h]: [512, d_v])
//
// (lechebs/ada-mla README.md:74-110 describes both absorptions; the reference
// stops at O* and has no kernel for either.)  Both are Y[b, h, :] = X[b, h, :] .
// W[h] with a different weight per head, so they cannot join the decode's
// 128-row head tile.  At decode batch sizes they read far more weight than
// activation bytes (16 MB of W per projection at 128 heads in fp16), so the
// kernel is laid out to stream each weight byte from HBM exactly once:
//
//   * swap-AB: the weight is the MMA's A operand, M = output columns (128 per
//     tile), read MN-major (the output index is contiguous in W[h][k][:]);
//     the batch is N (16..256, zero-filled past B) with X K-major;
//   * a unit of work = (head, 128-column output tile, 256-row batch tile);
//     a persistent grid walks the units, K streamed in 64-deep stages through
//     a TMA ring (A: two 64-column SW128 boxes, B: one box of the batch rows);
//   * the fp32 accumulator [128 x N] lives in TMEM, double-buffered, so the
//     epilogue of one unit overlaps the MMAs of the next.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer and TMEM
// owner, warps 2-5 the epilogue (warp w reads TMEM lanes 32 (w % 4) ..: all
// 128 rows).  Every wait is bounded (a device error code, then wind-down).
#pragma once

#include "mla_tc_ptx.cuh"

namespace mla {
namespace proj {

constexpr int kThreads = 192;
constexpr int kTileM = 128;         // output columns per unit (MMA M)
constexpr int kStageK = 64;         // K per ring stage (one 128-byte swizzle row of X)
constexpr int kBoxA = 64 * kStageK * 2;  // 8 KB: one W box (64 output columns x 64 K rows)
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 200 * 1024;  // ring bytes
constexpr uint32_t kTmemCols = 512;      // two accumulators of up to 256 columns

struct ProjParams {
    int batch, heads, k_total, m_total;
    int n_box;        // batch rows per unit (multiple of 16, <= 256)
    int units_m, units_n, units;
    int stages;       // ring stages
    int stage_bytes;  // 2 * kBoxA + n_box * 128
    void *out;        // Y element (b, h, m) at out[b * out_b + h * out_h + m]
    long long out_b, out_h;
    int bf16;         // W, X and Y are bf16 (else fp16)
    // Q absorption: the rope columns q_rope[b, h, 0:64] go to out[.. + m_total + j]
    const void *rope;
};

enum : int { kBarFull = 0, kBarEmpty = kMaxStages, kBarAccFull = 2 * kMaxStages, kBarAccEmpty = kBarAccFull + 2,
             kBarDrain = kBarAccEmpty + 2, kNumBars = kBarDrain + 1 };

// wmap: W as (m_total, k_total, heads), box (64, 64, 1), SW128.
// xmap: X as (k_total, heads, batch), box (64, 1, n_box), SW128.
__global__ void __launch_bounds__(kThreads, 1)
    proj_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                const ProjParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = ptx::smem_u32(smem);
    const uint32_t bar0 = sbase + (uint32_t)(p.stages * p.stage_bytes);
    auto bar = [&](int id) -> uint32_t { return bar0 + 8u * id; };
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + p.stages * p.stage_bytes + kNumBars * 8);
    const uint32_t slot_addr = sbase + (uint32_t)(p.stages * p.stage_bytes + kNumBars * 8 + 8);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < p.stages; ++i) {
            ptx::mbar_init(bar(kBarFull + i), 1);
            ptx::mbar_init(bar(kBarEmpty + i), 1);
        }
        for (int i = 0; i < 2; ++i) {
            ptx::mbar_init(bar(kBarAccFull + i), 1);
            ptx::mbar_init(bar(kBarAccEmpty + i), 128);
        }
        ptx::mbar_init(bar(kBarDrain), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0 && lane == 0) {
        ptx::tma_prefetch_desc(&wmap);
        ptx::tma_prefetch_desc(&xmap);
    }
    if (warp == 1) {
        ptx::tmem_alloc(slot_addr, kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + p.stages * p.stage_bytes + kNumBars * 8 + 8);
    griddep_launch();  // a kernel launched after this one may start its set-up
    griddep_wait();    // X may come from the kernel before this one

    const int ksteps = p.k_total / kStageK;
    if (warp == 0) {
        // ---------------------------------------------------------- TMA producer
        if (lane == 0) {
            int slot = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
                const int h = u / (p.units_m * p.units_n);
                const int r = u - h * p.units_m * p.units_n;
                const int m0 = (r / p.units_n) * kTileM, n0 = (r % p.units_n) * p.n_box;
                for (int ks = 0; ks < ksteps; ++ks) {
                    if (*abort_flag || !ptx::mbar_wait(bar(kBarEmpty + slot), phase ^ 1, kErrWaitEmpty)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dst = sbase + (uint32_t)(slot * p.stage_bytes);
                    ptx::mbar_arrive_expect_tx(bar(kBarFull + slot), (uint32_t)p.stage_bytes);
                    ptx::tma_load_3d(dst, &wmap, m0, ks * kStageK, h, bar(kBarFull + slot));
                    ptx::tma_load_3d(dst + kBoxA, &wmap, m0 + 64, ks * kStageK, h, bar(kBarFull + slot));
                    ptx::tma_load_3d(dst + 2 * kBoxA, &xmap, ks * kStageK, h, n0, bar(kBarFull + slot));
                    if (++slot == p.stages) { slot = 0; phase ^= 1; }
                }
            }
            if (!ok) *abort_flag = 1;
            for (int k = 0; k < p.stages; ++k) {  // every issued load consumed (or the wait expires)
                ptx::mbar_wait(bar(kBarEmpty + slot), phase ^ 1, kErrWaitEmpty);
                if (++slot == p.stages) { slot = 0; phase ^= 1; }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0) {
            int slot = 0;
            uint32_t phase = 0;
            bool ok = true;
            // A: W^T tile, MN-major SW128: 64-column groups 8 KB apart (LBO), 8-row K
            // groups 1 KB apart (SBO); B: X rows K-major SW128.
            const uint32_t idesc = ptx::idesc_f16_f32(kTileM, p.n_box, 1, 0, p.bf16);
            int j = 0;
            for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++j) {
                const uint32_t ab = (uint32_t)(j & 1), use = (uint32_t)(j >> 1);
                if (*abort_flag || !ptx::mbar_spin(bar(kBarAccEmpty + ab), (use & 1) ^ 1, kErrWaitMma)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t d = tmem + ab * 256;
                for (int ks = 0; ks < ksteps; ++ks) {
                    if (!ptx::mbar_spin(bar(kBarFull + slot), phase, kErrWaitFull)) { ok = false; break; }
                    const uint32_t st = sbase + (uint32_t)(slot * p.stage_bytes);
                    const uint64_t a0 = ptx::sdesc_sw128(st, kBoxA, 1024);
                    const uint64_t b0 = ptx::sdesc_sw128(st + 2 * kBoxA, 16, 1024);
#pragma unroll
                    for (int kk = 0; kk < kStageK / 16; ++kk)
                        ptx::mma_ss(d, a0 + (uint64_t)((kk * 16 * 128) >> 4), b0 + (uint64_t)((kk * 32) >> 4), idesc,
                                    (ks > 0 || kk > 0) ? 1u : 0u);
                    ptx::mma_commit(bar(kBarEmpty + slot));
                    if (++slot == p.stages) { slot = 0; phase ^= 1; }
                }
                if (!ok) break;
                ptx::mma_commit(bar(kBarAccFull + ab));
            }
            if (!ok) *abort_flag = 1;
            // every MMA this thread issued has retired before TMEM is freed
            ptx::mma_commit(bar(kBarDrain));
            ptx::mbar_wait(bar(kBarDrain), 0, kErrWaitMma);
        }
    } else {
        // ---------------------------------------------------------- epilogue (warps 2-5)
        const int q = warp & 3;                   // TMEM lane quarter
        const int row = q * 32 + lane;            // output column within the tile
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        int j = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++j) {
            const uint32_t ab = (uint32_t)(j & 1), use = (uint32_t)(j >> 1);
            bool w = !*abort_flag && ptx::mbar_wait(bar(kBarAccFull + ab), use & 1, kErrWaitMma);
            w = __all_sync(0xffffffffu, w);
            if (!ptx::named_barrier_and(1, 128, w)) { ok = false; break; }
            ptx::tc_fence_after();
            const int h = u / (p.units_m * p.units_n);
            const int r = u - h * p.units_m * p.units_n;
            const int m = (r / p.units_n) * kTileM + row, n0 = (r % p.units_n) * p.n_box;
            const int nval = min(p.n_box, p.batch - n0);
            uint8_t *dst = static_cast<uint8_t *>(p.out) + 2 * ((long long)n0 * p.out_b + (long long)h * p.out_h + m);
            for (int c = 0; c < p.n_box; c += 32) {
                uint32_t v[32];
                ptx::tmem_ld_x32(tmem + lane_addr + ab * 256 + c, v);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    if (c + e < nval) {
                        const float f = __uint_as_float(v[e]);
                        unsigned short bits;
                        if (p.bf16) bits = __bfloat16_as_ushort(__float2bfloat16_rn(f));
                        else bits = __half_as_ushort(__float2half_rn(f));
                        *reinterpret_cast<unsigned short *>(dst + 2 * (long long)(c + e) * p.out_b) = bits;
                    }
                }
            }
            ptx::tc_fence_before();
            ptx::mbar_arrive(bar(kBarAccEmpty + ab));
        }
        if (!ok) *abort_flag = 1;
        // Q absorption: the rope columns, 16 bytes per thread, spread over the grid
        if (p.rope != nullptr) {
            const long long rows = (long long)p.batch * p.heads;  // rows of 64 elements = 8 vectors
            const uint4 *src = static_cast<const uint4 *>(p.rope);
            for (long long i = (long long)blockIdx.x * 128 + (tid - 64); i < rows * 8; i += (long long)gridDim.x * 128) {
                const long long rw = i >> 3;
                const long long b = rw / p.heads, hh = rw - b * p.heads;
                uint4 *o = reinterpret_cast<uint4 *>(static_cast<uint8_t *>(p.out) +
                                                     2 * (b * p.out_b + hh * p.out_h + p.m_total)) + (i & 7);
                *o = src[i];
            }
        }
    }

    // ---------------------------------------------------------------- teardown
    ptx::tc_fence_before();
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace proj
}  // namespace mla
