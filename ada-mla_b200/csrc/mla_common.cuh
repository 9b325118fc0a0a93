// mla_common.cuh -- shapes, the split work list, the device error word and
// small device helpers shared by every MLA decode kernel.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
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
// A work item is a contiguous run of cache rows of ONE sequence, decoded by
// one worker (a 2-CTA cluster of the tensor-core kernel, or one SIMT block);
// item i writes partial i (normalized O and its log-sum-exp) and the combine
// kernel merges the partials of each sequence.  Two schedules:
//
// Chunked (chunk > 0): items of at most `chunk` rows, numbered consecutively
//   per sequence, dealt to the workers round-robin (explicit split counts and
//   the SIMT kernels).
//    dense  (items == nullptr): every sequence has seq_len rows at stride
//           seq_len; sequence b owns items [b*cps, (b+1)*cps).
//    varlen (items != nullptr): a plan kernel expanded cu_seqlens into
//           items[] = {b, row_begin, row_end, 0} and item_off[B+1]; launches
//           are sized for max_items and items >= item_off[B] are empty.
//
// Balanced (chunk == 0, tensor-core kernel with an automatic split): the
//   batch is laid out on a cost line.  Sequence b occupies the interval
//   [cost0_b, cost0_b + item_cost + tiles_b): item_cost units stand for the
//   fixed cost of a work item (Q load, epilogue), then one unit per 96-row
//   tile.  Worker c owns the units [c*quota, (c+1)*quota) and decodes, as one
//   item, the tiles of each sequence that fall into its units.  So every
//   worker gets the same work, whatever the lengths, and a sequence is split
//   only where a worker's share ends.  The item of (sequence b, worker c) has
//   id b + c: the ids of one sequence are consecutive and all ids are below
//   batch + workers (some ids stay unused).
//    dense : cost0_b = b * (item_cost + tiles), quota given by the host.
//    varlen: cost0_b = cost_off[b] (prefix computed by plan_balanced_kernel),
//            quota = ceil(cost_off[B] / nworkers), derived on the device.
// ---------------------------------------------------------------------------
// Fixed cost of one work item, in 96-row tiles: its Q load (always a 128-row
// box, 144 KB, whatever the head count), pipeline fill and its partial write
// (n_h x 1024 B; one SM writes ~45 GB/s).  2 tiles (measured at 128 heads: 3 or
// 4 moved nothing; at 16 heads, cfg4, 1 tile was 1-3.5 % slower).
__host__ __device__ constexpr int item_cost_for(int /*num_heads*/) { return 2; }

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start while its predecessor in the stream
// still runs (once every CTA of the predecessor has called griddep_launch() or
// exited); griddep_wait() returns when the predecessor grid has completed and
// its memory is visible.  Without the attribute both are no-ops.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// The decode and merge kernels call griddep_launch() at their start, so that
// a successor launched with the attribute (the host chains decode -> merge ->
// next decode for a few long sequences) can place its CTAs and set up early.
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

struct WorkList {
    const int4 *items;
    const int *item_off;
    int batch;
    int seq_len;   // dense only
    int chunk;     // chunked: rows per item (a multiple of kTile when planned); 0 = balanced
    int cps;       // chunked dense: chunks per sequence
    int max_items; // chunked: launch bound; balanced: batch + nworkers
    // balanced schedule
    const int *cost_off;        // varlen: [batch + 1] cost prefix (device)
    const int32_t *cu_seqlens;  // varlen: row offsets [batch + 1]
    int quota;                  // dense: cost units per worker
    int nworkers;               // varlen: workers the cost line is divided among
    int item_cost;              // fixed cost of an item in tiles (item_cost_for(num_heads))
    int group;                  // >= 1; see seq_len_of
};

// Length of (virtual) sequence b.  group == 1: sequence b itself (cu_seqlens,
// or dense_len for a dense cache).  group > 1 (multi-token decode with more
// draft tokens than one 128-row tile holds): sequence b is draft token
// d = b % group of real sequence b / group, reading that sequence's cache
// rows up to its causal limit len - (group - 1 - d).
__host__ __device__ __forceinline__ int seq_len_of(const int32_t *cu, int dense_len, int group, int b) {
    const int r = group > 1 ? b / group : b;
    int len = cu != nullptr ? cu[r + 1] - cu[r] : dense_len;
    if (group > 1) {
        len -= group - 1 - (b - r * group);
        if (len < 0) len = 0;
    }
    return len;
}

// First cache row of (virtual) sequence b.
__host__ __device__ __forceinline__ long long seq_row0_of(const int32_t *cu, int dense_len, int group, int b) {
    const int r = group > 1 ? b / group : b;
    return cu != nullptr ? (long long)cu[r] : (long long)r * dense_len;
}

struct Item {
    int b;
    long long row0;  // first cache row (index into the packed / dense cache)
    int len;         // rows in this item, 0 = empty
    int tok0;        // first token's position in its sequence
};

__device__ __forceinline__ Item get_item(const WorkList &w, int i) {
    Item it;
    if (w.items == nullptr) {
        const int b = i / w.cps;
        const int c = i - b * w.cps;
        const int start = c * w.chunk;
        it.b = b;
        it.row0 = (long long)b * w.seq_len + start;
        it.tok0 = start;
        const int rem = w.seq_len - start;
        it.len = b < w.batch ? max(0, min(w.chunk, rem)) : 0;
    } else {
        const int n = w.item_off[w.batch];
        if (i < n) {
            const int4 v = w.items[i];
            it.b = v.x;
            it.row0 = v.y;
            it.len = v.z - v.y;
            it.tok0 = v.w;
        } else {
            it.b = 0;
            it.row0 = 0;
            it.len = 0;
            it.tok0 = 0;
        }
    }
    return it;
}

// Balanced schedule: one sequence's place on the cost line.
struct SeqSpan {
    int cost0;       // first cost unit
    int tiles;       // 96-row tiles (its units after the item_cost fixed ones)
    long long row0;  // first cache row
    int len;         // rows
};

__device__ __forceinline__ SeqSpan seq_span(const WorkList &w, int b) {
    SeqSpan s;
    if (w.cost_off == nullptr) {
        s.len = w.seq_len;
        s.tiles = (w.seq_len + kTile - 1) / kTile;
        s.cost0 = b * (s.tiles > 0 ? s.tiles + w.item_cost : 0);
        s.row0 = (long long)b * w.seq_len;
    } else {
        s.cost0 = w.cost_off[b];
        s.row0 = seq_row0_of(w.cu_seqlens, w.seq_len, w.group, b);
        s.len = seq_len_of(w.cu_seqlens, w.seq_len, w.group, b);
        s.tiles = (s.len + kTile - 1) / kTile;
    }
    return s;
}

__device__ __forceinline__ int bal_total(const WorkList &w) {
    if (w.cost_off == nullptr) {
        const int t = (w.seq_len + kTile - 1) / kTile;
        return w.batch * (t > 0 ? t + w.item_cost : 0);
    }
    return w.cost_off[w.batch];
}

__device__ __forceinline__ int bal_quota(const WorkList &w) {
    if (w.cost_off == nullptr) return w.quota;
    const int n = max(w.nworkers, 1);
    return max(1, (w.cost_off[w.batch] + n - 1) / n);
}

// The sequence whose cost interval contains unit x (x < total).
__device__ __forceinline__ int bal_seq_at(const WorkList &w, int x) {
    if (w.cost_off == nullptr) {
        const int t = (w.seq_len + kTile - 1) / kTile;
        return x / (t + w.item_cost);
    }
    int lo = 0, hi = w.batch - 1;  // largest b with cost_off[b] <= x
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (w.cost_off[mid] <= x) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// Which schedule a kernel is compiled for: a kernel instantiated for one of
// them carries no code (and no registers) for the other.
enum SchedKind : int { kSchedAny = 0, kSchedChunked = 1, kSchedBalanced = 2 };

// Walks the items of worker `wid` in order.
struct ItemCursor {
    int next;    // chunked: next item index; balanced: next sequence
    int step;    // chunked: worker count
    int wid;     // balanced: this worker
    int x0, x1;  // balanced: this worker's cost units
};

template <int kSched = kSchedAny>
__device__ __forceinline__ ItemCursor items_begin(const WorkList &w, int wid, int nworkers) {
    ItemCursor c;
    c.wid = wid;
    c.step = nworkers;
    if (kSched == kSchedChunked || (kSched == kSchedAny && w.chunk > 0)) {
        c.next = wid;
        c.x0 = c.x1 = 0;
    } else {
        const int q = bal_quota(w), total = bal_total(w);
        c.x0 = min(wid * q, total);
        c.x1 = min(c.x0 + q, total);
        c.next = c.x0 < c.x1 ? bal_seq_at(w, c.x0) : w.batch;
    }
    return c;
}

// Next non-empty item of the cursor's worker: its id and rows.  False when done.
template <int kSched = kSchedAny>
__device__ __forceinline__ bool items_next(const WorkList &w, ItemCursor &c, Item &it, int &id) {
    if constexpr (kSched != kSchedBalanced) {
        if (kSched == kSchedChunked || w.chunk > 0) {
            while (c.next < w.max_items) {
                id = c.next;
                it = get_item(w, id);
                c.next += c.step;
                if (it.len > 0) return true;
            }
            return false;
        }
    }
    if constexpr (kSched != kSchedChunked) {
        while (c.next < w.batch) {
            const int b = c.next++;
            const SeqSpan s = seq_span(w, b);
            if (s.cost0 >= c.x1) {
                c.next = w.batch;
                return false;
            }
            const int base = s.cost0 + w.item_cost;  // cost unit of tile 0
            const int lo = max(c.x0 - base, 0), hi = min(c.x1 - base, s.tiles);
            if (hi <= lo) continue;
            id = b + c.wid;
            it.b = b;
            it.row0 = s.row0 + (long long)lo * kTile;
            it.len = min(hi * kTile, s.len) - lo * kTile;
            it.tok0 = lo * kTile;
            return true;
        }
    }
    return false;
}

// Ids [i0, i1) of the items of sequence b (its partials, for the combine).
template <int kSched = kSchedAny>
__device__ __forceinline__ void item_range(const WorkList &w, int b, int &i0, int &i1) {
    if (kSched == kSchedBalanced || (kSched == kSchedAny && w.chunk == 0)) {
        const SeqSpan s = seq_span(w, b);
        if (s.tiles <= 0) {
            i0 = i1 = 0;
            return;
        }
        const int q = bal_quota(w);
        const int base = s.cost0 + w.item_cost;
        i0 = b + base / q;
        i1 = b + (base + s.tiles - 1) / q + 1;
    } else if (w.items == nullptr) {
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
    kErrSelfTest = 6,      // the bounded-wait self test's wait ran out (expected)
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
