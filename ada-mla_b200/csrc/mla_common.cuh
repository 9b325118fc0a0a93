// mla_common.cuh -- shapes, the split work list, the device error word and
// small device helpers shared by every MLA decode kernel.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "mla_b200.h"

namespace mla {

constexpr int kDK = MLA_B200_HEAD_DIM_K;  // 576: latent + rope
constexpr int kDV = MLA_B200_HEAD_DIM_V;  // 512: latent (value) columns
constexpr int kTile = 96;                 // tokens per tensor-core S tile; planned chunks are multiples
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---------------------------------------------------------------------------
// Split work list.
//
// A work item is a contiguous run of at most `chunk` cache rows of ONE
// sequence.  Items of sequence b are numbered consecutively; item i writes
// partial i (normalized O and its log-sum-exp) and the combine kernel merges
// the partials of each sequence.
//
//  dense  (items == nullptr): every sequence has seq_len rows at stride
//         seq_len; sequence b owns items [b*cps, (b+1)*cps).
//  varlen (items != nullptr): a plan kernel expanded cu_seqlens into
//         items[] = {b, row_begin, row_end, 0} and item_off[B+1]; launches are
//         sized for max_items and items >= item_off[B] are empty.
// ---------------------------------------------------------------------------
struct WorkList {
    const int4 *items;
    const int *item_off;
    int batch;
    int seq_len;   // dense only
    int chunk;     // rows per item (a multiple of kTile when planned)
    int cps;       // dense: chunks per sequence
    int max_items; // launch bound
};

struct Item {
    int b;
    long long row0;  // first cache row (index into the packed / dense cache)
    int len;         // rows in this item, 0 = empty
};

__device__ __forceinline__ Item get_item(const WorkList &w, int i) {
    Item it;
    if (w.items == nullptr) {
        const int b = i / w.cps;
        const int c = i - b * w.cps;
        const int start = c * w.chunk;
        it.b = b;
        it.row0 = (long long)b * w.seq_len + start;
        const int rem = w.seq_len - start;
        it.len = b < w.batch ? max(0, min(w.chunk, rem)) : 0;
    } else {
        const int n = w.item_off[w.batch];
        if (i < n) {
            const int4 v = w.items[i];
            it.b = v.x;
            it.row0 = v.y;
            it.len = v.z - v.y;
        } else {
            it.b = 0;
            it.row0 = 0;
            it.len = 0;
        }
    }
    return it;
}

__device__ __forceinline__ void item_range(const WorkList &w, int b, int &i0, int &i1) {
    if (w.items == nullptr) {
        i0 = b * w.cps;
        i1 = i0 + (w.seq_len > 0 ? w.cps : 0);
    } else {
        i0 = w.item_off[b];
        i1 = w.item_off[b + 1];
    }
}

// ---------------------------------------------------------------------------
// Device error word.  Kernels never trap: a bounded wait that expires stores a
// code here (first writer wins) and the kernel winds down.  Read and cleared by
// mla_b200_get_device_error().
// ---------------------------------------------------------------------------
enum DeviceError : int {
    kErrNone = 0,
    kErrWaitFull = 1,      // consumer waited too long for a TMA tile
    kErrWaitEmpty = 2,     // producer waited too long for a free stage
    kErrWaitMma = 3,       // waited too long for an MMA commit
    kErrWaitPeer = 4,      // waited too long for the partner CTA of a cluster
    kErrBadShape = 5,      // a kernel saw a shape its host checks should have rejected
};

__device__ int g_mla_error = 0;  // one translation unit (mla_b200.cu) includes this

__device__ __forceinline__ void set_device_error(int code) {
    atomicCAS(&g_mla_error, 0, code);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Upper bound of any single wait inside a kernel.  Ordinary waits last
// microseconds; this only fires when a pipeline is broken.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

}  // namespace mla
