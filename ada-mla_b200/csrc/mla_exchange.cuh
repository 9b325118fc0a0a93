// mla_exchange.cuh -- the KV-split decode's cross-GPU exchange over NVLink peer
// memory, replacing an NCCL all-gather of the ranks' (O, LSE) partials.
//
// One process per GPU.  Every rank owns one exchange buffer (cudaMalloc, zeroed),
// mapped into every other rank's address space through CUDA IPC:
//
//   header [256 B]: flags[kMaxPeers] (u64: the last epoch rank g published into
//                   this buffer), epoch (u64: this rank's last published epoch),
//                   done (u32: blocks of the running put kernel that finished)
//   data:           [2 parities][world][stride] fp32, stride = rows * 513
//                   rounded up to 4 floats (O [rows, 512] normalized, then LSE)
//
// exchange_put_kernel (rank r, epoch e = its previous epoch + 1): every block
// copies its share of r's packed (O, LSE) into part r of parity e & 1 of every
// rank's buffer (own included) with plain stores over NVLink, fences at system
// scope and counts itself done; the last block publishes e in r's own header
// and stores e (release, system scope) into flags[r] of every rank's buffer.
//
// exchange_merge_kernel (rank r, epoch e read from its own header, written by
// its put kernel just before in stream order): thread 0 of every block waits,
// bounded by limit_ns, until flags[g] >= e for every g (acquire, system scope),
// then the block LSE-merges its row over the G parts of parity e & 1.
//
// exchange_fused_kernel does both in one launch (block = row: put the row,
// count done, wait for every flag, merge the row) when all its blocks fit on
// the device at once.  exchange_combine_kernel also merges the rank's own
// split-KV partials first, so the decode's merge kernel drops out of the step.
//
// Two parities make the reuse safe: rank A writes epoch e + 2 into B's parity
// (e & 1) only after its own merge of e + 1, which waited for B's flag e + 1,
// which B stored after its merge of e finished (stream order on B).
// No TMA, no multicast: plain loads and stores to peer memory.
#pragma once

#include "mla_combine.cuh"
#include "mla_common.cuh"

namespace mla {
namespace xchg {

constexpr int kMaxPeers = 16;
constexpr int kHeaderBytes = 256;
constexpr int kOffEpoch = kMaxPeers * 8;   // 128
constexpr int kOffDone = kOffEpoch + 8;    // 136
static_assert(kOffDone + 4 <= kHeaderBytes, "exchange header");

__host__ __device__ constexpr long long stride_floats(long long rows) { return (rows * (kDV + 1) + 3) / 4 * 4; }

__host__ __device__ constexpr size_t buffer_bytes(int world, long long rows) {
    return (size_t)kHeaderBytes + 2ull * (size_t)world * (size_t)stride_floats(rows) * sizeof(float);
}

struct Peers {
    uint8_t *buf[kMaxPeers];  // every rank's exchange buffer as mapped in this process (own included)
};

__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// part: this rank's packed (O, LSE), stride floats (16-byte aligned).
__global__ void __launch_bounds__(256) exchange_put_kernel(const float4 *__restrict__ part, long long n4,
                                                           Peers peers, int rank, int world, long long stride) {
    uint8_t *own = peers.buf[rank];
    // every block reads the previous epoch before any block can count itself done
    const unsigned long long e = *reinterpret_cast<volatile unsigned long long *>(own + kOffEpoch) + 1;
    const size_t off = ((size_t)(e & 1) * (size_t)world + (size_t)rank) * (size_t)stride;  // floats
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const float4 v = part[i];
        for (int g = 0; g < world; ++g)
            reinterpret_cast<float4 *>(reinterpret_cast<float *>(peers.buf[g] + kHeaderBytes) + off)[i] = v;
    }
    // The block's stores happen before thread 0's system-scope fence (bar.sync,
    // then the fence's cumulativity): one fence per block, not per thread (a
    // system fence waits for the thread's stores to be acknowledged over NVLink).
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        unsigned int *done = reinterpret_cast<unsigned int *>(own + kOffDone);
        if (atomicAdd(done, 1u) == gridDim.x - 1) {  // the last block: every block's data is out
            *done = 0u;
            *reinterpret_cast<volatile unsigned long long *>(own + kOffEpoch) = e;
            __threadfence_system();
            for (int g = 0; g < world; ++g)
                st_release_sys(reinterpret_cast<unsigned long long *>(peers.buf[g]) + rank, e);
        }
    }
}

// Block-wide LSE merge of row `row` over the `world` parts at `data` (parity
// base of a buffer's data region); 128 threads, thread t owns columns [4 t, 4 t + 4).
template <typename OutT>
__device__ __forceinline__ void merge_row(const float *data, int world, long long rows, long long stride,
                                          long long row, OutT *__restrict__ out, float *__restrict__ out_lse) {
    float mx = -INFINITY;
    for (int g = 0; g < world; ++g) mx = fmaxf(mx, __ldcg(data + (size_t)g * stride + (size_t)rows * kDV + row));
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float wsum = 0.f;
    if (mx != -INFINITY) {
        for (int g = 0; g < world; ++g) {
            const float *p = data + (size_t)g * stride;
            const float lse = __ldcg(p + (size_t)rows * kDV + row);
            const float w = lse == -INFINITY ? 0.f : __expf(lse - mx);
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(p + (size_t)row * kDV) + threadIdx.x);
            wsum += w;
            acc.x = fmaf(w, v.x, acc.x);
            acc.y = fmaf(w, v.y, acc.y);
            acc.z = fmaf(w, v.z, acc.z);
            acc.w = fmaf(w, v.w, acc.w);
        }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    OutT *dst = out + (size_t)row * kDV + threadIdx.x * 4;
    if constexpr (sizeof(OutT) == 4) {
        *reinterpret_cast<float4 *>(dst) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    } else {
        const __half2 a = __floats2half2_rn(acc.x * inv, acc.y * inv), b = __floats2half2_rn(acc.z * inv, acc.w * inv);
        uint2 u;
        u.x = *reinterpret_cast<const uint32_t *>(&a);
        u.y = *reinterpret_cast<const uint32_t *>(&b);
        *reinterpret_cast<uint2 *>(dst) = u;
    }
    if (out_lse != nullptr && threadIdx.x == 0) out_lse[row] = wsum > 0.f ? mx + __logf(wsum) : -INFINITY;
}

// One block of 128 threads per row; thread t owns columns [4 t, 4 t + 4).
template <typename OutT>
__global__ void __launch_bounds__(128) exchange_merge_kernel(const uint8_t *own, int world, long long rows,
                                                             long long stride, unsigned long long limit_ns,
                                                             OutT *__restrict__ out, float *__restrict__ out_lse) {
    __shared__ int ok_s;
    const long long row = blockIdx.x;
    const unsigned long long e = *reinterpret_cast<const volatile unsigned long long *>(own + kOffEpoch);
    if (threadIdx.x == 0) {
        const unsigned long long *flags = reinterpret_cast<const unsigned long long *>(own);
        int ok = 1;
        uint64_t t0 = 0;
        for (int g = 0; g < world && ok; ++g) {
            for (uint32_t n = 0; ld_acquire_sys(flags + g) < e; ++n) {
                if ((n & 255u) == 255u) {
                    const uint64_t t = globaltimer_ns();
                    if (t0 == 0) t0 = t;
                    else if (t - t0 > limit_ns) { set_device_error(kErrWaitPeer); ok = 0; break; }
                }
            }
        }
        ok_s = ok;
    }
    __syncthreads();
    if (!ok_s) return;
    merge_row(reinterpret_cast<const float *>(own + kHeaderBytes) + (size_t)(e & 1) * (size_t)world * (size_t)stride,
              world, rows, stride, row, out, out_lse);
}

// The whole exchange in one kernel: block `row` stores its row of this rank's
// packed (O, LSE) into every rank's buffer, the blocks count themselves done
// and the last one publishes the epoch (as exchange_put_kernel), then every
// block waits for every rank's flag and merges its row (as
// exchange_merge_kernel).  The blocks wait on each other through the done
// count, so all of them must be resident at once: the host launches it only
// when the grid fits the device's occupancy (else put + merge); a block that
// waits in vain (another kernel holding SMs) gives up after limit_ns with the
// peer-wait code, like the merge.
template <typename OutT>
__global__ void __launch_bounds__(128) exchange_fused_kernel(const float *__restrict__ part, long long rows,
                                                             Peers peers, int rank, int world, long long stride,
                                                             unsigned long long limit_ns, OutT *__restrict__ out,
                                                             float *__restrict__ out_lse) {
    __shared__ int ok_s;
    const long long row = blockIdx.x;
    uint8_t *own = peers.buf[rank];
    const unsigned long long e = *reinterpret_cast<volatile unsigned long long *>(own + kOffEpoch) + 1;
    const size_t base = (size_t)(e & 1) * (size_t)world * (size_t)stride;  // floats: this epoch's parity
    const size_t mine = base + (size_t)rank * (size_t)stride;
    {
        const float4 v = reinterpret_cast<const float4 *>(part + (size_t)row * kDV)[threadIdx.x];
        const float lse = part[(size_t)rows * kDV + row];
        for (int g = 0; g < world; ++g) {
            float *d = reinterpret_cast<float *>(peers.buf[g] + kHeaderBytes) + mine;
            reinterpret_cast<float4 *>(d + (size_t)row * kDV)[threadIdx.x] = v;
            if (threadIdx.x == 0) d[(size_t)rows * kDV + row] = lse;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        unsigned int *done = reinterpret_cast<unsigned int *>(own + kOffDone);
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0u;
            *reinterpret_cast<volatile unsigned long long *>(own + kOffEpoch) = e;
            __threadfence_system();
            for (int g = 0; g < world; ++g)
                st_release_sys(reinterpret_cast<unsigned long long *>(peers.buf[g]) + rank, e);
        }
        const unsigned long long *flags = reinterpret_cast<const unsigned long long *>(own);
        int ok = 1;
        uint64_t t0 = 0;
        for (int g = 0; g < world && ok; ++g) {
            for (uint32_t n = 0; ld_acquire_sys(flags + g) < e; ++n) {
                if ((n & 255u) == 255u) {
                    const uint64_t t = globaltimer_ns();
                    if (t0 == 0) t0 = t;
                    else if (t - t0 > limit_ns) { set_device_error(kErrWaitPeer); ok = 0; break; }
                }
            }
        }
        ok_s = ok;
    }
    __syncthreads();
    if (!ok_s) return;
    merge_row(reinterpret_cast<const float *>(own + kHeaderBytes) + base, world, rows, stride, row, out, out_lse);
}

// Where exchange_combine_kernel stores and waits: every rank's buffer, this
// rank's index, the part stride and the wait's limit.
struct XchgRows {
    Peers peers;
    int rank, world;
    long long stride;  // floats per part (stride_floats(rows))
    unsigned long long limit_ns;
};

// The local LSE merge of a decode's split partials fused with the exchange:
// block = row (b, h) of this rank's KV slice.  It merges the row's partials
// as combine_kernel does (or, for a sequence decoded as a single item, takes
// the (O, LSE) the decode kernel wrote straight into `direct`), stores the
// merged row and its LSE into every rank's buffer, counts itself done (the
// last block publishes the epoch), waits for every rank's flag and merges the
// G parts of its row into `out`.  One launch for the local merge, the
// exchange and the cross-GPU merge.  Like exchange_fused_kernel its blocks wait
// on each other: the host launches it only when the grid fits the device.
template <typename PartT, typename OutT>
__global__ void __launch_bounds__(kCombineThreads) exchange_combine_kernel(
    const PartT *__restrict__ part_o, const float *__restrict__ part_lse, WorkList wl, int num_heads,
    long long rows, const float *__restrict__ direct, XchgRows xr, OutT *__restrict__ out,
    float *__restrict__ out_lse) {
    const Peers &peers = xr.peers;
    const int rank = xr.rank, world = xr.world;
    const long long stride = xr.stride;
    constexpr int kVec = 16 / (int)sizeof(PartT);    // partial elements per thread
    constexpr int kTpr = kDV / kVec;                 // threads covering one row
    constexpr int kGroups = kCombineThreads / kTpr;  // split groups
    __shared__ float w_s[kCombineChunk];
    __shared__ float red[kCombineThreads / 32];
    __shared__ __align__(16) float acc_s[kGroups][kDV];
    __shared__ float lse_s;
    __shared__ int ok_s;
    const long long row = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = (int)(row / num_heads);
    const int h = (int)(row - (long long)b * num_heads);
    uint8_t *own = peers.buf[rank];
    const unsigned long long e = *reinterpret_cast<volatile unsigned long long *>(own + kOffEpoch) + 1;
    const size_t base = (size_t)(e & 1) * (size_t)world * (size_t)stride;
    const size_t mine = base + (size_t)rank * (size_t)stride;
    int i0, i1;
    item_range(wl, b, i0, i1);

    if (i1 - i0 == 1) {
        // the decode kernel finished this row itself: (O, LSE) are in `direct`
        if (tid < kDV / 4)
            reinterpret_cast<float4 *>(acc_s[0])[tid] = reinterpret_cast<const float4 *>(direct + (size_t)row * kDV)[tid];
        if (tid == 0) lse_s = direct[(size_t)rows * kDV + row];
    } else {
        const int col = tid % kTpr, g = tid / kTpr;
        float mx = -INFINITY;
        for (int i = i0 + tid; i < i1; i += kCombineThreads) mx = fmaxf(mx, part_lse[(size_t)i * num_heads + h]);
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
            const size_t step = (size_t)num_heads * kDV / kVec;  // one split, in 16-byte vectors
            for (int c0 = i0; c0 < i1; c0 += kCombineChunk) {
                const int n = min(kCombineChunk, i1 - c0);
                __syncthreads();
                for (int k = tid; k < n; k += kCombineThreads) {
                    const float lse = part_lse[(size_t)(c0 + k) * num_heads + h];
                    w_s[k] = lse == -INFINITY ? 0.f : __expf(lse - mx);
                }
                __syncthreads();
                for (int k = 0; k < n; ++k) wsum += w_s[k];
                const uint4 *src =
                    reinterpret_cast<const uint4 *>(part_o + (size_t)c0 * num_heads * kDV + (size_t)h * kDV) + col;
                for (int k = g; k < n; k += 8 * kGroups) {
                    uint4 u[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (k + j * kGroups < n) u[j] = __ldg(src + (size_t)(k + j * kGroups) * step);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        if (k + j * kGroups < n) {
                            float v[kVec];
                            unpack_part<PartT>(u[j], v);
                            const float w = w_s[k + j * kGroups];
#pragma unroll
                            for (int q = 0; q < kVec; ++q) acc[q] = fmaf(w, v[q], acc[q]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int q = 0; q < kVec; ++q) acc_s[g][col * kVec + q] = acc[q];
        __syncthreads();
        if (g == 0) {
            const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
            for (int q = 0; q < kVec; ++q) {
                float t = acc_s[0][col * kVec + q];
#pragma unroll
                for (int o = 1; o < kGroups; ++o) t += acc_s[o][col * kVec + q];
                acc_s[0][col * kVec + q] = t * inv;
            }
            if (tid == 0) lse_s = wsum > 0.f ? mx + __logf(wsum) : -INFINITY;
        }
    }
    __syncthreads();
    // the merged row into part `rank` of every rank's buffer
    if (tid < kDV / 4) {
        const float4 v = reinterpret_cast<const float4 *>(acc_s[0])[tid];
        for (int q = 0; q < world; ++q) {
            float *d = reinterpret_cast<float *>(peers.buf[q] + kHeaderBytes) + mine;
            reinterpret_cast<float4 *>(d + (size_t)row * kDV)[tid] = v;
            if (tid == 0) d[(size_t)rows * kDV + row] = lse_s;
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        unsigned int *done = reinterpret_cast<unsigned int *>(own + kOffDone);
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0u;
            *reinterpret_cast<volatile unsigned long long *>(own + kOffEpoch) = e;
            __threadfence_system();
            for (int q = 0; q < world; ++q)
                st_release_sys(reinterpret_cast<unsigned long long *>(peers.buf[q]) + rank, e);
        }
        const unsigned long long *flags = reinterpret_cast<const unsigned long long *>(own);
        int ok = 1;
        uint64_t t0 = 0;
        for (int q = 0; q < world && ok; ++q) {
            for (uint32_t n = 0; ld_acquire_sys(flags + q) < e; ++n) {
                if ((n & 255u) == 255u) {
                    const uint64_t t = globaltimer_ns();
                    if (t0 == 0) t0 = t;
                    else if (t - t0 > xr.limit_ns) { set_device_error(kErrWaitPeer); ok = 0; break; }
                }
            }
        }
        ok_s = ok;
    }
    __syncthreads();
    if (!ok_s || tid >= kDV / 4) return;
    merge_row(reinterpret_cast<const float *>(own + kHeaderBytes) + base, world, rows, stride, row, out, out_lse);
}

}  // namespace xchg
}  // namespace mla
