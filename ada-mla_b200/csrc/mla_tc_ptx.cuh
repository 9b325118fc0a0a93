// mla_tc_ptx.cuh -- thin inline-PTX wrappers for the sm_100a primitives the
// tensor-core decode kernel uses: mbarriers (local and cluster-remote), TMA
// tile loads, DSMEM bulk copies, tcgen05 (TMEM alloc / MMA / commit / ld / st
// / fences) and the UMMA shared-memory and instruction descriptors.
//
// Every wait here is bounded (mla::kWaitLimitNs): an expired wait records a
// device error code and returns false, the caller winds its loop down.
#pragma once

#include <cuda.h>  // CUtensorMap

#include "mla_common.cuh"

namespace mla {
namespace ptx {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Explicit shared-space vector accesses: generic loads of shared memory issued
// between global stores serialise behind them, these do not.
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ uint2 ld_shared_v2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t nclusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}

// Address of the same shared::cta offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// bar.sync / bar.red are .aligned: every lane of a warp must reach the same
// barrier instruction together, or the warp's arrival is miscounted.  Their
// callers come out of per-thread spin loops (mbarrier waits) and lane-divergent
// branches, so each helper first reconverges the warp.
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t count) {
    __syncwarp();
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// bar.red.or: returns true in every participating thread if any passed true.
__device__ __forceinline__ bool named_barrier_or(uint32_t id, uint32_t count, bool v) {
    __syncwarp();
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %3, 0;\n\t"
        "bar.red.or.pred q, %1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(id), "r"(count), "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

// bar.red.and: true in every participating thread iff all passed true.
__device__ __forceinline__ bool named_barrier_and(uint32_t id, uint32_t count, bool v) {
    __syncwarp();
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %3, 0;\n\t"
        "bar.red.and.pred q, %1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(id), "r"(count), "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init_cluster() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}

// Arrive (with expected transaction bytes) on a barrier of another CTA of the
// cluster; `remote_bar` is a shared::cluster address from mapa().  Relaxed:
// the arrive only posts the byte count of a bulk copy that follows, whose own
// complete_tx makes its data visible; a release here would make the thread
// wait for its outstanding memory operations (~1 us per message measured).
__device__ __forceinline__ void mbar_remote_arrive_expect_tx(uint32_t remote_bar, uint32_t bytes) {
    asm volatile(
        "mbarrier.arrive.expect_tx.relaxed.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(
            remote_bar),
        "r"(bytes)
        : "memory");
}

// try_wait with acquire semantics at CTA scope (barriers completed by this
// CTA's own TMA loads, tcgen05 commits and threads) or at cluster scope
// (barriers the partner CTA arrives on).  The cluster-scope acquire costs
// about 200 cycles even on a completed barrier, so it is used only where a
// remote arrival has to be ordered.
template <bool kCluster = false>
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    if constexpr (kCluster) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
    }
    return ok != 0;
}

// Waits for the phase of `bar` with the given parity to complete.  Bounded:
// after kWaitLimitNs records `err` and returns false.  The spin itself is just
// try_wait; the global timer is read only every 256 misses.
template <bool kCluster = false>
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int err,
                                          uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait<kCluster>(bar, parity)) return true;
    uint64_t t0 = 0;
    for (uint32_t n = 1;; ++n) {
        // back off: a hot try_wait loop competes with the tensor core's
        // shared-memory operand reads on the same SM
        __nanosleep(32);
        if (mbar_try_wait<kCluster>(bar, parity)) return true;
        if ((n & 255) == 0) {
            const uint64_t t = globaltimer_ns();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > limit_ns) {
                set_device_error(err);
                return false;
            }
        }
    }
}

// Non-blocking probe of a phase (CTA-scope acquire).  Cheaper than try_wait
// (~80 vs ~180 cycles on an already completed phase), which matters in the
// MMA-issuing thread: tcgen05.mma issue blocks on a shallow queue, so every
// cycle that thread spends waiting is a cycle the tensor pipe runs dry.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Spin on test_wait; same bound and error reporting as mbar_wait.
__device__ __forceinline__ bool mbar_spin(uint32_t bar, uint32_t parity, int err) {
    if (mbar_test_wait(bar, parity)) return true;
    uint64_t t0 = 0;
    for (uint32_t n = 1;; ++n) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((n & 1023) == 0) {
            const uint64_t t = globaltimer_ns();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > kWaitLimitNs) {
                set_device_error(err);
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// TMA and bulk copies
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled TMA load of box (x = innermost coordinate, y) into this CTA's smem.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// 3-D and 4-D tiled TMA loads (coordinates innermost first) into this CTA's smem.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *map, int x, int y, int z,
                                            int w, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar)
        : "memory");
}

// Bulk copy of `bytes` from this CTA's smem to another CTA's smem of the
// cluster (dst and bar are shared::cluster addresses); completion is signalled
// on the destination CTA's barrier.  Point to point: exactly one destination CTA.
__device__ __forceinline__ void bulk_copy_s2cluster(uint32_t dst, uint32_t src, uint32_t bytes,
                                                    uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(dst),
        "r"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16, fp32 accumulate.
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16, fp32 accumulate.
// Shared memory -> TMEM copy of a 128-row x 32-byte matrix (row r to lane r,
// the 32 bytes to 8 consecutive columns), read through a matrix descriptor
// like an MMA operand.  A later tcgen05.mma of this thread is ordered after it.
__device__ __forceinline__ void tmem_cp_128x256b(uint32_t d_tmem, uint64_t s_desc) {
    asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(d_tmem), "l"(s_desc) : "memory");
}

__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f8f6f4 (A, B e4m3 per the
// instruction descriptor), K = 32, fp32 accumulate.
__device__ __forceinline__ void mma_ts_f8(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f8f6f4, K = 32, fp32 accumulate.
__device__ __forceinline__ void mma_ss_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on a local mbarrier once all prior tcgen05 async ops of this thread finish.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

// Same, arriving on the barrier at this smem offset in every CTA of `mask`.
__device__ __forceinline__ void mma_commit_mc(uint32_t bar, uint16_t mask) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
        "[%0], %1;" ::"r"(bar),
        "h"(mask)
        : "memory");
}

#define MLA_TMEM_LD_X32(taddr, r)                                                               \
    asm volatile(                                                                               \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13," \
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"      \
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),   \
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),            \
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),         \
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),         \
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),         \
          "=r"(r[31])                                                                           \
        : "r"(taddr))

#define MLA_TMEM_ST_X32(taddr, r)                                                               \
    asm volatile(                                                                               \
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12," \
        "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"     \
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),         \
        "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]),         \
        "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]),     \
        "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),     \
        "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]))

__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
    MLA_TMEM_LD_X32(taddr, r);
}

__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    MLA_TMEM_ST_X32(taddr, r);
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---------------------------------------------------------------------------
// UMMA descriptors (bit layouts: PTX ISA "Shared memory descriptor" and
// "Instruction descriptor" for tcgen05.mma kind::f16)
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor, 128-byte swizzle.  addr/lbo/sbo in bytes.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);         // [0,14)  start address >> 4
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;    // [16,30) leading byte offset >> 4
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;    // [32,46) stride byte offset >> 4
    d |= (uint64_t)1 << 46;                        // [46,48) descriptor version 1 (sm_100)
    d |= (uint64_t)2 << 61;                        // [61,64) layout: SWIZZLE_128B
    return d;
}

// Same with 64-byte swizzle (rows of 64 B, 8-row atoms of 512 B).
__device__ __forceinline__ uint64_t sdesc_sw64(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)4 << 61;                        // layout: SWIZZLE_64B
    return d;
}

// Same with 32-byte swizzle (rows of 32 B, 8-row atoms of 256 B).
__device__ __forceinline__ uint64_t sdesc_sw32(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)6 << 61;                        // layout: SWIZZLE_32B
    return d;
}

// Instruction descriptor: f16 x f16 (or bf16 x bf16) -> f32, dense, no negate.
//   a_mn / b_mn: operand is MN-major (1) instead of K-major (0).
//   bf16: both operands bf16 (kind::f16 takes A and B of the same type).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n, int a_mn, int b_mn, int bf16 = 0) {
    return (1u << 4)                         // [4,6)   D format: f32
           | ((uint32_t)bf16 << 7)           // [7,10)  A format: 0 f16, 1 bf16
           | ((uint32_t)bf16 << 10)          // [10,13) B format
           | ((uint32_t)a_mn << 15)          // [15]    A major
           | ((uint32_t)b_mn << 16)          // [16]    B major
           | ((uint32_t)(n >> 3) << 17)      // [17,23) N >> 3
           | ((uint32_t)(m >> 4) << 24);     // [24,29) M >> 4
}

}  // namespace ptx
}  // namespace mla
