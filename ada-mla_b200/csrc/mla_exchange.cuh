// mla_exchange.cuh -- the KV-split decode's cross-GPU exchange over NVLink peer
// memory, replacing an NCCL all-gather of the ranks' (O, LSE) partials.
//
// One process per GPU.  Every rank owns one exchange buffer (cudaMalloc, zeroed),
// mapped into every other rank's address space through CUDA IPC:
//
//   header: epoch[rows] (u32: how many steps this rank has published for each
//           row), padded to a multiple of 256 bytes
//   data:   [2 parities][world parts][stride words]; one part = O [rows, 512
//           words] then LSE [rows words], 8-byte words (epoch << 32 | payload)
//
// Flags live in the data: every 8-byte word carries the epoch of the step that
// wrote it, and an aligned 8-byte store is seen whole or not at all.  A rank
// stores row r of its packed (O, LSE) as such words into its part of every
// rank's buffer (parity e & 1 for epoch e); a reader polls the words of its own
// buffer (volatile loads, bounded by limit_ns) until each carries e, and then
// LSE-merges the G parts.  No fence, no counter, no block waits for another
// block of its own grid.  O words hold one fp32 value (4 KB per row per peer:
// twice the bytes of the values) or, in the one-launch kernels with fp16
// output, two fp16 values (2 KB; the merged output is fp16 anyway); the LSE word
// is always fp32.  put + merge always use fp32 words, and every rank of a step
// takes the same form (same rows, same device).  The top bit of a word's epoch
// half names its payload format (set: fp16 pairs), so ranks that disagree on
// it (different output types) wait in vain and report code 4 instead of
// reading each other's words in the wrong format.
//
// Kernels (block = row, 128 threads own 4 columns each, unless noted):
//   exchange_put_kernel     epoch[r] += 1, then the stores (fp32 words)
//   exchange_merge_kernel   waits for epoch[r] in every part, merges (fp32 words)
//   exchange_fused_kernel   both, one launch (fp16 words for fp16 output)
//   exchange_combine_kernel (512 threads) merges the rank's own split-KV
//                           partials of the row first, then as the fused one
//
// Two parities make the reuse safe: rank A writes row r of epoch e + 2 into B's
// parity e & 1 only after its merge of e + 1 saw B's row r of e + 1, which B
// stored after its kernel of step e (the one reading that parity) had ended.
// No TMA, no multicast: plain loads and stores to peer memory.
#pragma once

#include "mla_combine.cuh"
#include "mla_common.cuh"

namespace mla {
namespace xchg {

constexpr int kMaxPeers = 16;

// header bytes: a u32 step count per row, padded to 256 bytes
__host__ __device__ constexpr size_t header_bytes(long long rows) { return ((size_t)rows * 4 + 255) / 256 * 256; }

// 8-byte words per part: O [rows, 512] then LSE [rows], rounded up to an even
// count so that every part's O rows start on a 16-byte boundary
__host__ __device__ constexpr long long stride_words(long long rows) { return (rows * (kDV + 1) + 1) / 2 * 2; }

__host__ __device__ constexpr size_t buffer_bytes(int world, long long rows) {
    return header_bytes(rows) + 2ull * (size_t)world * (size_t)stride_words(rows) * 8;
}

struct Peers {
    uint8_t *buf[kMaxPeers];  // every rank's exchange buffer as mapped in this process (own included)
};

// Where the exchange kernels store and wait: every rank's buffer, this rank's
// index, rows per part, the part stride and the wait's limit.
struct XchgRows {
    Peers peers;
    int rank, world;
    long long rows;
    long long stride;  // stride_words(rows)
    unsigned long long limit_ns;
};

__device__ __forceinline__ unsigned long long *data_of(uint8_t *buf, long long rows) {
    return reinterpret_cast<unsigned long long *>(buf + header_bytes(rows));
}

__device__ __forceinline__ unsigned long long word_of(float v, uint32_t e) {
    return ((unsigned long long)e << 32) | __float_as_uint(v);
}

__device__ __forceinline__ void st_words2(unsigned long long *p, unsigned long long a, unsigned long long b) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ void st_word(unsigned long long *p, unsigned long long a) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(a) : "memory");
}

__device__ __forceinline__ void ld_words2(const unsigned long long *p, unsigned long long &a, unsigned long long &b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ unsigned long long ld_word(const unsigned long long *p) {
    unsigned long long a;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
    return a;
}

__device__ __forceinline__ bool has_epoch(unsigned long long w, uint32_t e) { return (uint32_t)(w >> 32) == e; }

// The epoch half of a word: 31 bits of epoch, the top bit set for fp16 payload.
template <bool kHalf>
__device__ __forceinline__ uint32_t word_tag(uint32_t e) {
    return kHalf ? (e | 0x80000000u) : (e & 0x7fffffffu);
}

// Bounded poll step: false once more than limit_ns passed since the first call
// that had to wait (t0 = 0 before it).
__device__ __forceinline__ bool still_waiting(uint32_t n, uint64_t &t0, unsigned long long limit_ns) {
    if ((n & 63u) != 63u) return true;
    const uint64_t t = globaltimer_ns();
    if (t0 == 0) t0 = t;
    return t - t0 <= limit_ns;
}

__device__ __forceinline__ unsigned long long word_of_half2(float a, float b, uint32_t e) {
    const __half2 h = __floats2half2_rn(a, b);
    return ((unsigned long long)e << 32) | *reinterpret_cast<const uint32_t *>(&h);
}

// Thread t (< 128) stores columns [4 t, 4 t + 4) of row `row` (v) and, thread 0,
// its LSE, as epoch-e words into part `rank` of every rank's buffer.  Row r's O
// words start at word r * 512 (fp32 words: 512 of them; fp16 words: 256).
template <bool kHalf>
__device__ __forceinline__ void put_row(const XchgRows &xr, long long row, uint32_t e, float4 v, float lse) {
    const size_t base = ((size_t)(e & 1) * (size_t)xr.world + (size_t)xr.rank) * (size_t)xr.stride;
    const int t = threadIdx.x;
    const uint32_t tag = word_tag<kHalf>(e);
    const unsigned long long wl = word_of(lse, tag);
    if constexpr (kHalf) {
        const unsigned long long w0 = word_of_half2(v.x, v.y, tag), w1 = word_of_half2(v.z, v.w, tag);
        for (int q = 0; q < xr.world; ++q) {
            unsigned long long *d = data_of(xr.peers.buf[q], xr.rows) + base;
            st_words2(d + (size_t)row * kDV + 2 * t, w0, w1);
            if (t == 0) st_word(d + (size_t)xr.rows * kDV + row, wl);
        }
    } else {
        const unsigned long long w0 = word_of(v.x, tag), w1 = word_of(v.y, tag), w2 = word_of(v.z, tag),
                                 w3 = word_of(v.w, tag);
        for (int q = 0; q < xr.world; ++q) {
            unsigned long long *d = data_of(xr.peers.buf[q], xr.rows) + base;
            unsigned long long *o = d + (size_t)row * kDV + 4 * t;
            st_words2(o, w0, w1);
            st_words2(o + 2, w2, w3);
            if (t == 0) st_word(d + (size_t)xr.rows * kDV + row, wl);
        }
    }
}

// Thread t's words of one part's row (fp32 words: 4, fp16 words: 2), the test
// that they all carry epoch e, and their values.
template <bool kHalf>
__device__ __forceinline__ void load_part(const unsigned long long *p, unsigned long long (&w)[4]) {
    ld_words2(p, w[0], w[1]);
    if constexpr (!kHalf) ld_words2(p + 2, w[2], w[3]);
}

template <bool kHalf>
__device__ __forceinline__ bool part_ready(const unsigned long long (&w)[4], uint32_t e) {
    if constexpr (kHalf) return has_epoch(w[0], e) && has_epoch(w[1], e);
    return has_epoch(w[0], e) && has_epoch(w[1], e) && has_epoch(w[2], e) && has_epoch(w[3], e);
}

template <bool kHalf>
__device__ __forceinline__ float4 part_values(const unsigned long long (&w)[4]) {
    if constexpr (kHalf) {
        const uint32_t a = (uint32_t)w[0], b = (uint32_t)w[1];
        const float2 x = __half22float2(*reinterpret_cast<const __half2 *>(&a));
        const float2 y = __half22float2(*reinterpret_cast<const __half2 *>(&b));
        return make_float4(x.x, x.y, y.x, y.y);
    }
    return make_float4(__uint_as_float((uint32_t)w[0]), __uint_as_float((uint32_t)w[1]),
                       __uint_as_float((uint32_t)w[2]), __uint_as_float((uint32_t)w[3]));
}

// Block-wide: waits (bounded) until every part of row `row` in this rank's own
// buffer carries epoch e, then LSE-merges the parts into out / out_lse.  Every
// thread of the block calls it (barriers inside); threads 0..127 own 4 columns
// each and load four parts' words before testing any (one round trip to L2 per
// four parts, not per part).  Returns false, with nothing written and the
// peer-wait code recorded, when a wait ran out.
template <bool kHalf, typename OutT>
__device__ bool merge_row(const XchgRows &xr, long long row, uint32_t e, OutT *__restrict__ out,
                          float *__restrict__ out_lse) {
    __shared__ float lse_s[kMaxPeers];
    const int t = threadIdx.x;
    const int world = xr.world;
    const unsigned long long *d =
        data_of(xr.peers.buf[xr.rank], xr.rows) + (size_t)(e & 1) * (size_t)world * (size_t)xr.stride;
    const uint32_t tag = word_tag<kHalf>(e);
    bool ok = true;
    uint64_t t0 = 0;
    if (t < world) {
        const unsigned long long *p = d + (size_t)t * xr.stride + (size_t)xr.rows * kDV + row;
        unsigned long long w = ld_word(p);
        for (uint32_t n = 0; ok && !has_epoch(w, tag); ++n) {
            ok = still_waiting(n, t0, xr.limit_ns);
            w = ld_word(p);
        }
        lse_s[t] = __uint_as_float((uint32_t)w);
    }
    if (__syncthreads_or(!ok)) {
        if (t == 0) set_device_error(kErrWaitPeer);
        return false;
    }
    float mx = -INFINITY;
    for (int g = 0; g < world; ++g) mx = fmaxf(mx, lse_s[g]);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float wsum = 0.f;
    if (t < kDV / 4) {
        const size_t col = (size_t)row * kDV + (kHalf ? 2 : 4) * t;
        for (int g0 = 0; g0 < world && ok; g0 += 4) {
            unsigned long long w[4][4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (g0 + j < world) load_part<kHalf>(d + (size_t)(g0 + j) * xr.stride + col, w[j]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (g0 + j < world && ok) {
                    const unsigned long long *p = d + (size_t)(g0 + j) * xr.stride + col;
                    for (uint32_t n = 0; ok && !part_ready<kHalf>(w[j], tag); ++n) {
                        ok = still_waiting(n, t0, xr.limit_ns);
                        load_part<kHalf>(p, w[j]);
                    }
                    const float lse = lse_s[g0 + j];
                    const float wt = (mx == -INFINITY || lse == -INFINITY) ? 0.f : __expf(lse - mx);
                    const float4 v = part_values<kHalf>(w[j]);
                    wsum += wt;
                    acc.x = fmaf(wt, v.x, acc.x);
                    acc.y = fmaf(wt, v.y, acc.y);
                    acc.z = fmaf(wt, v.z, acc.z);
                    acc.w = fmaf(wt, v.w, acc.w);
                }
            }
        }
    }
    if (__syncthreads_or(!ok)) {
        if (t == 0) set_device_error(kErrWaitPeer);
        return false;
    }
    if (t < kDV / 4) {
        const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
        OutT *dst = out + (size_t)row * kDV + t * 4;
        if constexpr (sizeof(OutT) == 4) {
            *reinterpret_cast<float4 *>(dst) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        } else {
            const __half2 a = __floats2half2_rn(acc.x * inv, acc.y * inv), b = __floats2half2_rn(acc.z * inv, acc.w * inv);
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t *>(&a);
            u.y = *reinterpret_cast<const uint32_t *>(&b);
            *reinterpret_cast<uint2 *>(dst) = u;
        }
        if (out_lse != nullptr && t == 0) out_lse[row] = wsum > 0.f ? mx + __logf(wsum) : -INFINITY;
    }
    return true;
}

// This rank's step count for `row` (own header), advanced by one when `advance`;
// returns the step's epoch.  Block-wide (one barrier).
__device__ __forceinline__ uint32_t row_epoch(const XchgRows &xr, long long row, bool advance) {
    __shared__ uint32_t e_s;
    uint32_t *ep = reinterpret_cast<uint32_t *>(xr.peers.buf[xr.rank]) + row;
    if (threadIdx.x == 0) {
        const uint32_t e = *ep + (advance ? 1u : 0u);
        if (advance) *ep = e;  // read again only by this row's block of the next kernel
        e_s = e;
    }
    __syncthreads();
    return e_s;
}

// part: this rank's packed (O [rows, 512], LSE [rows]) fp32, 16-byte aligned.
__global__ void __launch_bounds__(128) exchange_put_kernel(const float *__restrict__ part, XchgRows xr) {
    const long long row = blockIdx.x;
    const uint32_t e = row_epoch(xr, row, true);
    const float4 v = reinterpret_cast<const float4 *>(part + (size_t)row * kDV)[threadIdx.x];
    put_row<false>(xr, row, e, v, part[(size_t)xr.rows * kDV + row]);
}

// The merge after exchange_put_kernel (which advanced the epoch).
template <typename OutT>
__global__ void __launch_bounds__(128) exchange_merge_kernel(XchgRows xr, OutT *__restrict__ out,
                                                             float *__restrict__ out_lse) {
    const long long row = blockIdx.x;
    const uint32_t e = row_epoch(xr, row, false);
    merge_row<false>(xr, row, e, out, out_lse);
}

// put + merge in one launch.  Blocks wait only on the same row's blocks of the
// other ranks; the host still launches it only when the whole grid fits the
// device at once, so that no rank's block r waits behind its own waiting blocks.
template <typename OutT>
__global__ void __launch_bounds__(128) exchange_fused_kernel(const float *__restrict__ part, XchgRows xr,
                                                             OutT *__restrict__ out, float *__restrict__ out_lse) {
    const long long row = blockIdx.x;
    const uint32_t e = row_epoch(xr, row, true);
    constexpr bool kHalf = sizeof(OutT) == 2;
    const float4 v = reinterpret_cast<const float4 *>(part + (size_t)row * kDV)[threadIdx.x];
    put_row<kHalf>(xr, row, e, v, part[(size_t)xr.rows * kDV + row]);
    merge_row<kHalf>(xr, row, e, out, out_lse);
}

// The local LSE merge of a decode's split partials fused with the exchange:
// block = row (b, h) of this rank's KV slice.  It merges the row's partials
// as combine_kernel does (or, for a sequence decoded as a single item, takes
// the (O, LSE) the decode kernel wrote straight into `direct`), stores the
// merged row into every rank's buffer and merges the G parts of its row into
// `out`: one launch for the local merge, the exchange and the cross-GPU merge.
// Launched, like exchange_fused_kernel, only when the grid fits the device.
template <typename PartT, typename OutT>
__global__ void __launch_bounds__(kCombineThreads) exchange_combine_kernel(
    const PartT *__restrict__ part_o, const float *__restrict__ part_lse, WorkList wl, int num_heads,
    const float *__restrict__ direct, XchgRows xr, OutT *__restrict__ out, float *__restrict__ out_lse) {
    constexpr int kVec = 16 / (int)sizeof(PartT);    // partial elements per thread
    constexpr int kTpr = kDV / kVec;                 // threads covering one row
    constexpr int kGroups = kCombineThreads / kTpr;  // split groups
    __shared__ float w_s[kCombineChunk];
    __shared__ float red[kCombineThreads / 32];
    __shared__ __align__(16) float acc_s[kGroups][kDV];
    __shared__ float lse_s;
    const long long row = blockIdx.x;
    const long long rows = xr.rows;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = (int)(row / num_heads);
    const int h = (int)(row - (long long)b * num_heads);
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
    constexpr bool kHalf = sizeof(OutT) == 2;
    const uint32_t e = row_epoch(xr, row, true);  // (its barrier publishes acc_s and lse_s)
    if (tid < kDV / 4) put_row<kHalf>(xr, row, e, reinterpret_cast<const float4 *>(acc_s[0])[tid], lse_s);
    merge_row<kHalf>(xr, row, e, out, out_lse);
}

}  // namespace xchg
}  // namespace mla
