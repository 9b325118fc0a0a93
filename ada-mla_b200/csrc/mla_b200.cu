// mla_b200.cu -- the C ABI (include/mla_b200.h): argument checks, planning,
// workspace layout and kernel launches.  Every kernel of the library is in
// this one translation unit (the .cuh files), so no relocatable device code
// is needed for the shared device error word.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <utility>

#include <cudaTypedefs.h>

#include "mla_b200.h"
#include "mla_combine.cuh"
#include "mla_fp8.cuh"
#include "mla_common.cuh"
#include "mla_exchange.cuh"
#include "mla_proj.cuh"
#include "mla_simt.cuh"
#include "mla_tc.cuh"

using namespace mla;

namespace {

constexpr int kMaxDevices = 64;
constexpr float kRefScale = 0.07216878364870322f;  // 1/sqrt(HEAD_DIM + HEAD_DIM_ROPE) = 1/sqrt(192)

struct DevInfo {
    int sms = 0;
    int major = 0;
    bool simt_attr_set = false;
    bool proj_attr_set = false;
    int tc_clusters = 0;  // co-resident 2-CTA clusters of the tcgen05 decode kernel
};

std::mutex g_dev_mu;
DevInfo g_dev[kMaxDevices];

thread_local int t_last_cuda_error = 0;  // behind the last MLA_B200_ERR_CUDA of this thread

int cuda_failure(cudaError_t e) {
    t_last_cuda_error = (int)e;
    return MLA_B200_ERR_CUDA;
}

// Opts a tensor-core kernel instantiation (both schedules) into its dynamic
// shared memory.
template <bool kBf16, bool kPaged, bool kFp8 = false, bool kMtp = false, bool kRows = false>
bool set_tc_smem() {
    return cudaFuncSetAttribute(tc::tc_decode_kernel<kSchedChunked, kBf16, kPaged, kFp8, kMtp, kRows>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmemBytes) == cudaSuccess &&
           cudaFuncSetAttribute(tc::tc_decode_kernel<kSchedBalanced, kBf16, kPaged, kFp8, kMtp, kRows>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmemBytes) == cudaSuccess;
}

// Current device's properties (cached).  Returns a status.
int current_device(int *dev_out, DevInfo *info_out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return MLA_B200_ERR_NO_DEVICE;
    }
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DevInfo &d = g_dev[dev];
    if (d.sms == 0) {
        int sms = 0, major = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
            cudaGetLastError();
            return MLA_B200_ERR_NO_DEVICE;
        }
        d.sms = sms;
        d.major = major;
    }
    if (d.major != 10) return MLA_B200_ERR_NO_DEVICE;  // kernels are built for sm_100a only
    if (!d.simt_attr_set) {
        if (cudaFuncSetAttribute(simt_partial_kernel<float>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSimtSmem) !=
                cudaSuccess ||
            cudaFuncSetAttribute(simt_partial_kernel<__half>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSimtSmem) !=
                cudaSuccess) {
            return cuda_failure(cudaGetLastError());
        }
        d.simt_attr_set = true;
    }
    if (!d.proj_attr_set) {
        if (cudaFuncSetAttribute(proj::proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 proj::kSmemBudget + 4096) != cudaSuccess)
            return cuda_failure(cudaGetLastError());
        d.proj_attr_set = true;
    }
    if (d.tc_clusters == 0) {
        if (!set_tc_smem<false, false>() || !set_tc_smem<true, false>() ||
            !set_tc_smem<false, true>() || !set_tc_smem<true, true>() ||
            !set_tc_smem<false, false, true>() || !set_tc_smem<false, false, true, false, true>() ||
            !set_tc_smem<false, false, false, true>() ||
            !set_tc_smem<true, false, false, true>()) {
            return cuda_failure(cudaGetLastError());
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (d.sms / 2), 1, 1);
        cfg.blockDim = dim3(tc::kThreads, 1, 1);
        cfg.dynamicSmemBytes = tc::kSmemBytes;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, tc::tc_decode_kernel<kSchedChunked, false, false, false>, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = d.sms / 2;
        }
        d.tc_clusters = n;
    }
    *dev_out = dev;
    *info_out = d;
    return MLA_B200_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        cudaGetLastError();
    });
    return fn;
}

int encode_tmap(CUtensorMap *map, const void *base, cuuint32_t rank, const cuuint64_t *dims,
                const cuuint64_t *strides, const cuuint32_t *box, bool bf16,
                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B, bool bytes = false) {
    auto enc = tmap_encoder();
    if (enc == nullptr) return cuda_failure(cudaErrorSymbolNotFound);
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUtensorMapDataType dt = bytes ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const CUresult r = enc(map, dt, rank, const_cast<void *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MLA_B200_OK : cuda_failure(cudaErrorInvalidValue);
}

// e4m3 cache [rows, 576] (one byte per element), GEMM1 side: (64 B, rows, 9
// K-blocks) with 64-byte swizzle, one box = 3 K-blocks x 96 rows (an fp8 S slot).
// (Boxes of 128-byte rows with 128-byte swizzle, one K-block per 12 KB slot,
// measured slower: cfg3 89.8 vs 77.1 us per step.)
int make_tmap_fp8_s(CUtensorMap *map, const void *base, long long rows) {
    const cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(kDK / 64)};
    const cuuint64_t strides[2] = {(cuuint64_t)kDK, 64};
    const cuuint32_t box[3] = {64, (cuuint32_t)tc::kTS, (cuuint32_t)tc::kKbPerSlot};
    return encode_tmap(map, base, 3, dims, strides, box, false, CU_TENSOR_MAP_SWIZZLE_64B, true);
}

// e4m3 cache, GEMM2 side: (128 B, rows, 4 column groups) over the first 512
// columns, 128-byte swizzle, one box = a [32 x 512 B] C_N tile, GEMM2's MN-major B.
int make_tmap_fp8_o(CUtensorMap *map, const void *base, long long rows) {
    const cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)(kDV / 128)};
    const cuuint64_t strides[2] = {(cuuint64_t)kDK, 128};
    const cuuint32_t box[3] = {128, (cuuint32_t)tc::kTO, (cuuint32_t)(kDV / 128)};
    return encode_tmap(map, base, 3, dims, strides, box, false, CU_TENSOR_MAP_SWIZZLE_128B, true);
}

// Q8 [2 x rows, 576] e4m3 (hi plane then lo plane), box 64 B x 128 rows, SW64.
int make_tmap_q8(CUtensorMap *map, const void *base, long long rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)kDK, (cuuint64_t)(2 * rows)};
    const cuuint64_t strides[1] = {(cuuint64_t)kDK};
    const cuuint32_t box[2] = {64, 128};
    return encode_tmap(map, base, 2, dims, strides, box, false, CU_TENSOR_MAP_SWIZZLE_64B, true);
}

// 2-D view [rows, 576] with (64 x box_rows) boxes and 128-byte swizzle (the
// UMMA K-major / MN-major SW128 operand layout).
int make_tmap_576(CUtensorMap *map, const void *base, long long rows, int box_rows, bool bf16 = false) {
    const cuuint64_t dims[2] = {(cuuint64_t)kDK, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)kDK * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    return encode_tmap(map, base, 2, dims, strides, box, bf16);
}

// 3-D view (64 columns, rows, 9 column blocks) of the same [rows, 576] cache:
// the block axis (stride 128 B) is outermost, so one box of (64, box_rows,
// box_blocks) lands in shared memory as box_blocks consecutive [box_rows x 64]
// SW128 K-blocks -- the layout of box_blocks separate 2-D loads, in one
// instruction.
int make_tmap_blocks(CUtensorMap *map, const void *base, long long rows, int box_rows, int box_blocks,
                     bool bf16) {
    const cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(kDK / 64)};
    const cuuint64_t strides[2] = {(cuuint64_t)kDK * 2, 128};
    const cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)box_blocks};
    return encode_tmap(map, base, 3, dims, strides, box, bf16);
}

// 4-D view (64 columns, 8 rows, 9 column blocks, rows / 8 row groups) of a page
// pool with rows % 8 == 0.  A box (64, 8, 3, 4) takes 32 rows x 3 K-blocks and
// lands as 4 row groups of 3 interleaved 1 KB SW128 atoms: K-block j's 8-row
// groups sit 3 KB apart (the GEMM1 B descriptor's stride for paged tiles).
int make_tmap_pool_groups(CUtensorMap *map, const void *base, long long rows, bool bf16) {
    const cuuint64_t dims[4] = {64, 8, (cuuint64_t)(kDK / 64), (cuuint64_t)(rows / 8)};
    const cuuint64_t strides[3] = {(cuuint64_t)kDK * 2, 128, (cuuint64_t)kDK * 2 * 8};
    const cuuint32_t box[4] = {64, 8, (cuuint32_t)tc::kKbPerSlot, (cuuint32_t)(tc::kTO / 8)};
    return encode_tmap(map, base, 4, dims, strides, box, bf16);
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
inline long long cdiv(long long a, long long b) { return (a + b - 1) / b; }

// Split plan: rows per work item.  `units` is the number of workers one wave
// of the decode kernel has; the chunk is an even share of the batch's tiles
// plus the fixed per-item cost, which grows with the head count (the balanced
// schedule's quota, mla_common.cuh), but never longer than a sequence.
int plan_chunk(int batch, long long total_tokens, int max_seq_len, int num_sms, int num_heads) {
    const long long units = num_sms > 1 ? num_sms / 2 : 1;  // 2-CTA clusters per wave
    const long long cost = cdiv(total_tokens > 0 ? total_tokens : 1, kTile) +
                           (long long)item_cost_for(num_heads) * (batch > 0 ? batch : 1);
    long long chunk = cdiv(cost, units) * kTile;
    if (chunk < kTile) chunk = kTile;
    if (max_seq_len > 0) {
        const long long cap = cdiv(max_seq_len, kTile) * kTile;
        if (chunk > cap) chunk = cap;
    }
    if (chunk > (1 << 30)) chunk = 1 << 30;
    return (int)chunk;
}

int chunk_for(int batch, long long total_tokens, int max_seq_len, int num_splits, int num_sms,
              int num_heads) {
    if (num_splits > 0) {
        const long long n = max_seq_len > 0 ? max_seq_len : 1;
        long long c = cdiv(n, num_splits);
        return (int)(c < 1 ? 1 : c);
    }
    return plan_chunk(batch, total_tokens, max_seq_len, num_sms, num_heads);
}

long long max_items_for(int batch, long long total_tokens, int chunk) {
    return cdiv(total_tokens, chunk) + batch;
}

struct WsLayout {
    float *part_o = nullptr;
    float *part_lse = nullptr;
    int *item_off = nullptr;
    int4 *items = nullptr;
    int32_t *cu_virtual = nullptr;  // paged cache: sequence offsets built from seq_lens
    uint8_t *q8 = nullptr;          // fp8 cache: Q* as e4m3 hi and lo planes [2, B * n_h, 576]
    float *q_scale = nullptr;       // fp8 cache: [B * n_h]
    size_t bytes = 0;
};

WsLayout ws_layout(void *base, long long max_items, int num_heads, int batch, bool fp8 = false) {
    WsLayout L;
    size_t off = 0;
    const size_t o_bytes = (size_t)max_items * num_heads * kDV * sizeof(float);
    const size_t l_bytes = (size_t)max_items * num_heads * sizeof(float);
    const size_t off_bytes = (size_t)(batch + 1) * sizeof(int);
    const size_t it_bytes = (size_t)max_items * sizeof(int4);
    char *p = static_cast<char *>(base);
    L.part_o = reinterpret_cast<float *>(p + off);
    off = align_up(off + o_bytes, 256);
    L.part_lse = reinterpret_cast<float *>(p + off);
    off = align_up(off + l_bytes, 256);
    L.item_off = reinterpret_cast<int *>(p + off);
    off = align_up(off + off_bytes, 256);
    L.items = reinterpret_cast<int4 *>(p + off);
    off = align_up(off + it_bytes, 256);
    L.cu_virtual = reinterpret_cast<int32_t *>(p + off);
    off = align_up(off + off_bytes, 256);
    if (fp8) {
        const size_t rows = (size_t)batch * num_heads;
        L.q8 = reinterpret_cast<uint8_t *>(p + off);
        off = align_up(off + 2 * rows * kDK, 256);
        L.q_scale = reinterpret_cast<float *>(p + off);
        off = align_up(off + rows * sizeof(float), 256);
    }
    L.bytes = off;
    return L;
}

thread_local cudaEvent_t t_ev_start = nullptr;  // mla_b200_set_kernel_timing
thread_local cudaEvent_t t_ev_stop = nullptr;
thread_local unsigned long long *t_span = nullptr;  // mla_b200_set_kernel_span
thread_local int t_span_slots = 0, t_span_next = 0;

unsigned long long *next_span() {
    if (t_span == nullptr || t_span_slots <= 0) return nullptr;
    unsigned long long *p = t_span + 2 * (t_span_next % t_span_slots);
    t_span_next = (t_span_next + 1) % t_span_slots;
    return p;
}

// Inside stream capture a plain record only orders the capture; the external
// flag makes it a real event-record node of the graph, timed at replay.
inline void timing_mark(cudaEvent_t ev, cudaStream_t stream) {
    if (ev == nullptr) return;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) cs = cudaStreamCaptureStatusNone;
    if (cs == cudaStreamCaptureStatusActive)
        cudaEventRecordWithFlags(ev, stream, cudaEventRecordExternal);
    else
        cudaEventRecord(ev, stream);
}

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int launch_status() {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MLA_B200_OK : cuda_failure(e);
}

// A page pool [pool_rows / page_size, page_size, 576] with its block table
// [batch, max_blocks] and per-sequence lengths (device int32 arrays).
// An e4m3 latent cache [total_tokens, 576] (dense or packed like the fp16 one)
// and its per-tensor scale: C = C8 * kv_scale.
struct Fp8Args {
    const void *cache8;
    float kv_scale;
    const float *kv_scales;  // or null: per cache row scales [rows]
};

// Multi-token decode: each sequence carries `tokens` draft-token queries of
// `heads` heads each (rows token * heads + head); see tc_decode_kernel.
struct MtpArgs {
    int tokens;
    int heads;
};

// The split-KV multi-GPU step's exchange, fused into the decode's merge
// (xchg::exchange_combine_kernel): the decode writes single-item rows as fp32
// (O, LSE) into `direct` (the packed layout, O [rows, 512] then LSE [rows]).
struct XchgArgs {
    xchg::Peers peers;
    int rank, world;
    unsigned long long limit_ns;
    float *direct;
};

struct PagedArgs {
    const int32_t *block_table;
    const int32_t *seq_lens;
    int max_blocks;
    int page_size;
    long long pool_rows;
};

// Launch, with programmatic stream serialization when `dependent`: the kernel
// may then start while its predecessor in the stream runs (the predecessor
// allows it with griddep_launch) and waits for it (griddep_wait) before
// touching the predecessor's results.  Used on the plan -> decode edge (the
// decode kernel's set-up overlaps the plan) and on decode -> merge -> next
// decode for a few long sequences.
template <typename... Params, typename... Args>
void launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t stream, bool dependent, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dependent ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);  // errors: launch_status()
}

struct TcMaps {
    CUtensorMap cmap_s, cmap_o, qmap;
};

template <int kSched, bool kBf16, bool kPaged, bool kFp8 = false, bool kMtp = false, bool kRows = false>
void launch_tc(int clusters, const TcMaps &m, const tc::TcParams &tp, cudaStream_t stream, bool after_plan) {
    launch_dependent(tc::tc_decode_kernel<kSched, kBf16, kPaged, kFp8, kMtp, kRows>, dim3(2 * clusters),
                     dim3(tc::kThreads), tc::kSmemBytes, stream, after_plan, m.cmap_s, m.cmap_o, m.qmap, tp);
}

// Shared driver of the split-KV paths: plan -> partial kernel -> combine.
// pg (tensor-core path only): the cache is a page pool; cu_seqlens is ignored
// and the sequences' offsets on a virtual packed axis are built from
// pg->seq_lens by the plan kernel; total_tokens is an upper bound.
template <typename T>
int run_split_decode(const T *q, const T *cache, const int32_t *cu_seqlens, int batch,
                     int num_heads, long long total_tokens, int max_seq_len, float scale,
                     int num_splits, void *out, int out_dtype, float *out_lse, void *workspace,
                     size_t workspace_bytes, cudaStream_t stream, const PagedArgs *pg = nullptr,
                     const Fp8Args *f8 = nullptr, const MtpArgs *mtp = nullptr, int group = 1,
                     const XchgArgs *xa = nullptr) {
    int dev;
    DevInfo info;
    int st = current_device(&dev, &info);
    if (st != MLA_B200_OK) return st;
    if (batch == 0) return MLA_B200_OK;

    // The tensor-core kernel with an automatic split runs the balanced schedule
    // (every cluster gets an equal share of the batch's tiles); explicit split
    // counts and the SIMT kernels use fixed-size chunks.
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    const bool tc_path = !std::is_same<T, float>::value && num_heads <= 128;
    if (kBf16 && !tc_path) return MLA_B200_ERR_UNSUPPORTED;  // bf16 has no SIMT kernel
    if (pg != nullptr && !tc_path) return MLA_B200_ERR_UNSUPPORTED;  // paged: tensor-core kernel only
    if (f8 != nullptr && (!tc_path || kBf16 || pg != nullptr)) return MLA_B200_ERR_UNSUPPORTED;
    if (mtp != nullptr && (!tc_path || pg != nullptr || f8 != nullptr)) return MLA_B200_ERR_UNSUPPORTED;
    // group > 1: `batch` virtual sequences, `group` per real sequence, read the
    // real sequences' rows (seq_len_of); they always take a planned schedule
    // (work table or cost line), and plan with group x the real tokens.
    const bool virt = group > 1;
    if (virt && (!tc_path || pg != nullptr || f8 != nullptr || mtp != nullptr || batch % group != 0))
        return MLA_B200_ERR_UNSUPPORTED;
    const long long plan_total = virt ? total_tokens * group : total_tokens;
    if (xa != nullptr) {
        // fp16 inputs on the tensor-core kernel only (fp16 partials, fp32 direct
        // rows), and every block of the exchange kernel resident at once (they
        // wait on each other); checked before anything is launched
        if (!tc_path || kBf16 || pg != nullptr || f8 != nullptr || mtp != nullptr || virt)
            return MLA_B200_ERR_UNSUPPORTED;
        int per_sm = 0;
        const cudaError_t oe = out_dtype == MLA_B200_OUT_F16
            ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                  &per_sm, xchg::exchange_combine_kernel<__half, __half>, kCombineThreads, 0)
            : cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                  &per_sm, xchg::exchange_combine_kernel<__half, float>, kCombineThreads, 0);
        if (oe != cudaSuccess) return cuda_failure(oe);
        if ((long long)batch * num_heads > (long long)per_sm * info.sms) return MLA_B200_ERR_UNSUPPORTED;
    }
    // (A single sequence splits evenly in the chunked schedule already.)
    const bool balanced = tc_path && num_splits <= 0 && batch > 1;
    int chunk = chunk_for(batch, plan_total, max_seq_len, num_splits, info.sms, num_heads);
    // paged: items start on 96-token boundaries so every 32-row box sits in one page
    if (pg != nullptr) chunk = (int)std::min<long long>(cdiv(chunk, kTile) * kTile, 1 << 30);
    const long long max_items = balanced ? (long long)batch + info.tc_clusters
                                         : max_items_for(batch, plan_total, chunk);
    if (max_items > (1LL << 30)) return MLA_B200_ERR_UNSUPPORTED;
    WsLayout L = ws_layout(workspace, max_items, num_heads, batch, f8 != nullptr);
    if (workspace == nullptr || workspace_bytes < L.bytes) return MLA_B200_ERR_WORKSPACE;
    if (!aligned(workspace, 16)) return MLA_B200_ERR_INVALID_ARG;
    const int32_t *seq_lens = nullptr;
    if (pg != nullptr) {
        seq_lens = pg->seq_lens;
        cu_seqlens = L.cu_virtual;  // written by the plan kernel below
    }

    WorkList wl = {};
    wl.batch = batch;
    wl.chunk = balanced ? 0 : chunk;
    wl.item_cost = item_cost_for(num_heads);
    wl.group = group;
    const bool planned = cu_seqlens != nullptr || virt;  // a plan kernel precedes the decode
    int bal_clusters = 0;      // balanced: clusters to launch
    bool bal_split = true;     // balanced: some sequence has more than one item
    if (balanced) {
        wl.max_items = (int)max_items;
        if (!planned) {
            wl.seq_len = max_seq_len;
            const long long tiles = cdiv(max_seq_len, kTile);
            const long long cost = tiles > 0 ? tiles + wl.item_cost : 0;
            const long long total = (long long)batch * cost;
            if (total >= (1LL << 31)) return MLA_B200_ERR_UNSUPPORTED;
            const long long q = std::max(1LL, cdiv(total, info.tc_clusters));
            wl.quota = (int)q;
            bal_clusters = total > 0 ? (int)cdiv(total, q) : 0;
            bal_split = total == 0;  // empty sequences get their zeros from the combine
            for (long long b = 0; b < batch && tiles > 0; ++b) {
                const long long base = b * cost + wl.item_cost;
                if (base / q != (base + tiles - 1) / q) {
                    bal_split = true;
                    break;
                }
            }
        } else {
            wl.cost_off = L.item_off;
            wl.cu_seqlens = cu_seqlens;
            wl.seq_len = max_seq_len;  // the dense length of virtual sequences without cu_seqlens
            wl.nworkers = info.tc_clusters;
            bal_clusters = info.tc_clusters;
            plan_balanced_kernel<<<1, 1024, 0, stream>>>(cu_seqlens, batch, wl.item_cost, L.item_off, seq_lens,
                                                         max_seq_len, L.cu_virtual, group, max_seq_len);
        }
    } else if (!planned) {
        wl.items = nullptr;
        wl.item_off = nullptr;
        wl.seq_len = max_seq_len;
        wl.cps = max_seq_len > 0 ? (int)cdiv(max_seq_len, chunk) : 0;
        wl.max_items = batch * wl.cps;
    } else {
        wl.items = L.items;
        wl.item_off = L.item_off;
        wl.seq_len = 0;
        wl.cps = 0;
        wl.max_items = (int)max_items;
        wl.cu_seqlens = cu_seqlens;  // read by the paged kernel
        plan_varlen_kernel<<<1, 1024, 0, stream>>>(cu_seqlens, batch, chunk, L.item_off, L.items,
                                                   (int)max_items, seq_lens, max_seq_len, L.cu_virtual,
                                                   group, max_seq_len);
    }
    bool tc_direct = false;  // the tcgen05 kernel wrote single-item sequences itself
    // A few long sequences chain decode -> merge -> next decode with programmatic
    // launches (each kernel waits before it touches its predecessor's data): the
    // merge is one short wave there, and its launch gap is a tenth of the step.
    // Batches do not: the next decode's early CTAs would hold SMs that their
    // larger merge still needs (same-box A/B: cfg1 -1.2 us, cfg3 -1.4 us, cfg2
    // B=128 +3 us).
    const bool chain = batch < 8;
    if (wl.max_items > 0 && (!balanced || bal_clusters > 0)) {
        if (tc_path) {
            TcMaps maps;
            CUtensorMap &cmap_s = maps.cmap_s, &cmap_o = maps.cmap_o, &qmap = maps.qmap;
            // S-CTA: one box per ring slot (3 K-blocks x 96 rows); paged, one per
            // 32-row piece and slot.  O-CTA: one box per 32-row C tile (8 K-blocks).
            const long long map_rows = pg != nullptr ? pg->pool_rows : total_tokens;
            const long long qrows = (long long)batch * num_heads;
            if (f8 != nullptr) {
                st = make_tmap_fp8_s(&cmap_s, f8->cache8, map_rows);
                if (st == MLA_B200_OK) st = make_tmap_fp8_o(&cmap_o, f8->cache8, map_rows);
                if (st == MLA_B200_OK) st = make_tmap_q8(&qmap, L.q8, qrows);
                if (st != MLA_B200_OK) return st;
                // Q* -> e4m3 hi / lo planes and row scales; the decode kernel's
                // set-up overlaps it (programmatic launch)
                q8_prep_kernel<<<(unsigned)cdiv(qrows, 8), 256, 0, stream>>>(
                    reinterpret_cast<const __half *>(q), (int)qrows, L.q8, L.q_scale);
            } else {
                if (pg != nullptr)
                    st = make_tmap_pool_groups(&cmap_s, cache, map_rows, kBf16);
                else
                    st = make_tmap_blocks(&cmap_s, cache, map_rows, tc::kTS, tc::kKbPerSlot, kBf16);
                if (st == MLA_B200_OK) st = make_tmap_blocks(&cmap_o, cache, map_rows, tc::kTO, tc::kVBlocks, kBf16);
                if (st == MLA_B200_OK) st = make_tmap_576(&qmap, q, qrows, 128, kBf16);
                if (st != MLA_B200_OK) return st;
            }
            tc::TcParams tp{};
            tp.wl = wl;
            tp.num_heads = num_heads;
            tp.scale_log2 = scale * kLog2e;
            tp.part_o = L.part_o;
            tp.part_lse = L.part_lse;
            // 16-bit partials: fp16 for fp16 inputs (whatever the output type: a
            // normalized partial fits fp16 and its 2^-11 rounding is far inside the
            // error bar, and the epilogue and merge move half the bytes), bf16 for bf16
            // output; bf16 inputs with fp32 output keep fp32 partials (bf16's 2^-8
            // rounding would show at fp32 output precision)
            tp.part_kind = out_dtype == MLA_B200_OUT_BF16 ? tc::kOutBF16
                           : (out_dtype == MLA_B200_OUT_F16 || !kBf16) ? tc::kOutF16 : tc::kOutF32;
            tp.out = out;
            tp.out_kind = out_dtype == MLA_B200_OUT_F16 ? tc::kOutF16
                          : out_dtype == MLA_B200_OUT_BF16 ? tc::kOutBF16 : tc::kOutF32;
            tp.out_lse = out_lse;
            if (xa != nullptr) {  // single-item rows go to the exchange's direct buffer
                tp.out = xa->direct;
                tp.out_kind = tc::kOutF32;
                tp.out_lse = xa->direct + (size_t)batch * num_heads * kDV;
            }
            tp.max_blocks = pg != nullptr ? pg->max_blocks : 0;
            if (mtp != nullptr) tp.mtp = (mtp->tokens << 16) | mtp->heads;
            if (f8 != nullptr) {
                // S = kv_scale * q_scale[row] * (Q8.C8); O = kv_scale * (P8.C8) / l, the
                // weights' factor kP8Scale in l too (per-row scales: applied per column in
                // the kernel, kv_scale = 1 here)
                tp.scale_log2 = scale * kLog2e * (f8->kv_scales != nullptr ? 1.f : f8->kv_scale);
                tp.q_scale = L.q_scale;
                tp.o_scale = f8->kv_scales != nullptr ? 1.f : f8->kv_scale;
            } else {
                tp.block_table = pg != nullptr ? pg->block_table : nullptr;
                tp.page_size = pg != nullptr ? pg->page_size : 0;
            }
            tp.span = next_span();
            tp.kv_scales = f8 != nullptr ? f8->kv_scales : nullptr;
            tp.chain = chain ? 1 : 0;
            tc_direct = true;
            const int clusters = balanced ? bal_clusters : std::min(info.tc_clusters, wl.max_items);
            timing_mark(t_ev_start, stream);
            if (mtp != nullptr) {
                if (balanced) launch_tc<kSchedBalanced, kBf16, false, false, true>(clusters, maps, tp, stream, planned || chain);
                else launch_tc<kSchedChunked, kBf16, false, false, true>(clusters, maps, tp, stream, planned || chain);
            } else if (f8 != nullptr) {
                if constexpr (!kBf16) {  // (fp8 runs with fp16 Q*; the prep kernel precedes)
                    // per-row scales: their own instantiation (the per-row code in the
                    // per-tensor kernel cost it ~10 %)
                    if (f8->kv_scales != nullptr) {
                        if (balanced) launch_tc<kSchedBalanced, false, false, true, false, true>(clusters, maps, tp, stream, true);
                        else launch_tc<kSchedChunked, false, false, true, false, true>(clusters, maps, tp, stream, true);
                    } else {
                        if (balanced) launch_tc<kSchedBalanced, false, false, true>(clusters, maps, tp, stream, true);
                        else launch_tc<kSchedChunked, false, false, true>(clusters, maps, tp, stream, true);
                    }
                }
            } else if (pg != nullptr) {
                if (balanced) launch_tc<kSchedBalanced, kBf16, true>(clusters, maps, tp, stream, planned || chain);
                else launch_tc<kSchedChunked, kBf16, true>(clusters, maps, tp, stream, planned || chain);
            } else {
                if (balanced) launch_tc<kSchedBalanced, kBf16, false>(clusters, maps, tp, stream, planned || chain);
                else launch_tc<kSchedChunked, kBf16, false>(clusters, maps, tp, stream, planned || chain);
            }
            timing_mark(t_ev_stop, stream);
        } else if constexpr (!kBf16) {
            dim3 grid(wl.max_items, (unsigned)cdiv(num_heads, kSimtHeads));
            timing_mark(t_ev_start, stream);
            simt_partial_kernel<T><<<grid, 256, kSimtSmem, stream>>>(
                q, cache, wl, num_heads, scale * kLog2e, L.part_o, L.part_lse);
            timing_mark(t_ev_stop, stream);
        }
    }
    const long long rows = (long long)batch * num_heads;
    if (xa != nullptr) {
        // local merge + exchange + cross-GPU merge in one plain launch (its blocks
        // spin on the other ranks' flags, so none may start before the decode ends)
        const xchg::XchgRows xr = {xa->peers, xa->rank, xa->world, rows, xchg::stride_words(rows), xa->limit_ns};
        const __half *ph = reinterpret_cast<const __half *>(L.part_o);
        if (out_dtype == MLA_B200_OUT_F16)
            xchg::exchange_combine_kernel<__half, __half><<<(unsigned)rows, kCombineThreads, 0, stream>>>(
                ph, L.part_lse, wl, num_heads, xa->direct, xr, static_cast<__half *>(out), out_lse);
        else
            xchg::exchange_combine_kernel<__half, float><<<(unsigned)rows, kCombineThreads, 0, stream>>>(
                ph, L.part_lse, wl, num_heads, xa->direct, xr, static_cast<float *>(out), out_lse);
        return launch_status();
    }
    // A dense batch decoded as one item per sequence is complete already.
    if (tc_direct && !planned && (balanced ? !bal_split : wl.cps == 1)) return launch_status();
    const unsigned cgrid = (unsigned)rows;
    const int skip = tc_direct ? 1 : 0;
    // The tcgen05 kernel keeps fp16 partials for fp16 inputs and bf16 partials for
    // bf16 output (fp32 for bf16 inputs with fp32 output); the SIMT kernel's are fp32.
    // Batches merge row-parallel (a warp per row, few splits each); a few long
    // sequences merge split-parallel (a block per row, many splits).
    if (batch >= 8) {
        const dim3 rgrid((unsigned)cdiv(num_heads, kRowsPerCombineBlock), (unsigned)batch);
        const dim3 rblock(32 * kRowsPerCombineBlock);
        const float *po = L.part_o;
        const __half *ph = reinterpret_cast<const __half *>(L.part_o);
        if (out_dtype == MLA_B200_OUT_BF16)
            launch_dependent(combine_rows_kernel<__nv_bfloat16, __nv_bfloat16>, rgrid, rblock, 0, stream, chain,
                             reinterpret_cast<const __nv_bfloat16 *>(L.part_o), L.part_lse, wl, num_heads,
                             static_cast<__nv_bfloat16 *>(out), out_lse, skip);
        else if (out_dtype == MLA_B200_OUT_F16 && tc_direct)
            launch_dependent(combine_rows_kernel<__half, __half>, rgrid, rblock, 0, stream, chain, ph, L.part_lse,
                             wl, num_heads, static_cast<__half *>(out), out_lse, skip);
        else if (out_dtype == MLA_B200_OUT_F16)
            launch_dependent(combine_rows_kernel<__half, float>, rgrid, rblock, 0, stream, chain, po, L.part_lse,
                             wl, num_heads, static_cast<__half *>(out), out_lse, skip);
        else if (tc_direct && !kBf16)
            launch_dependent(combine_rows_kernel<float, __half>, rgrid, rblock, 0, stream, chain, ph, L.part_lse,
                             wl, num_heads, static_cast<float *>(out), out_lse, skip);
        else
            launch_dependent(combine_rows_kernel<float, float>, rgrid, rblock, 0, stream, chain, po, L.part_lse,
                             wl, num_heads, static_cast<float *>(out), out_lse, skip);
        return launch_status();
    }
    const float *po = L.part_o;
    const __half *ph = reinterpret_cast<const __half *>(L.part_o);
    const dim3 cblock(kCombineThreads);
    const size_t ps = (size_t)num_heads * kDV, ls = (size_t)num_heads;
    if (out_dtype == MLA_B200_OUT_BF16)
        launch_dependent(combine_kernel<__nv_bfloat16, __nv_bfloat16>, dim3(cgrid), cblock, 0, stream, chain,
                         reinterpret_cast<const __nv_bfloat16 *>(L.part_o), L.part_lse, wl, num_heads, rows,
                         static_cast<__nv_bfloat16 *>(out), out_lse, skip, ps, ls);
    else if (out_dtype == MLA_B200_OUT_F16 && tc_direct)
        launch_dependent(combine_kernel<__half, __half>, dim3(cgrid), cblock, 0, stream, chain, ph, L.part_lse,
                         wl, num_heads, rows, static_cast<__half *>(out), out_lse, skip, ps, ls);
    else if (out_dtype == MLA_B200_OUT_F16)
        launch_dependent(combine_kernel<__half, float>, dim3(cgrid), cblock, 0, stream, chain, po, L.part_lse,
                         wl, num_heads, rows, static_cast<__half *>(out), out_lse, skip, ps, ls);
    else if (tc_direct && !kBf16)
        launch_dependent(combine_kernel<float, __half>, dim3(cgrid), cblock, 0, stream, chain, ph, L.part_lse,
                         wl, num_heads, rows, static_cast<float *>(out), out_lse, skip, ps, ls);
    else
        launch_dependent(combine_kernel<float, float>, dim3(cgrid), cblock, 0, stream, chain, po, L.part_lse,
                         wl, num_heads, rows, static_cast<float *>(out), out_lse, skip, ps, ls);
    return launch_status();
}

}  // namespace

namespace {
template <typename T>
int decode_paged(const void *query, const void *kv_pages, const int32_t *block_table,
                 const int32_t *seq_lens, int batch, int num_heads, int num_pages, int page_size,
                 int max_blocks, int max_seq_len, float softmax_scale, int num_splits, void *out,
                 int out_dtype, float *out_lse, void *workspace, size_t workspace_bytes,
                 void *stream) {
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    if (batch < 0 || num_heads <= 0 || num_pages < 0 || page_size <= 0 || max_blocks < 0 ||
        max_seq_len < 0)
        return MLA_B200_ERR_INVALID_ARG;
    if (batch > 0 && (query == nullptr || out == nullptr || block_table == nullptr || seq_lens == nullptr))
        return MLA_B200_ERR_INVALID_ARG;
    if (num_pages > 0 && kv_pages == nullptr) return MLA_B200_ERR_INVALID_ARG;
    if (kBf16 ? (out_dtype != MLA_B200_OUT_BF16 && out_dtype != MLA_B200_OUT_F32)
              : (out_dtype != MLA_B200_OUT_F16 && out_dtype != MLA_B200_OUT_F32))
        return MLA_B200_ERR_INVALID_ARG;
    if (!(softmax_scale > 0.f) || !isfinite(softmax_scale)) return MLA_B200_ERR_INVALID_ARG;
    if (!aligned(query, 16) || !aligned(kv_pages, 16) || !aligned(out, 16) || !aligned(out_lse, 4) ||
        !aligned(block_table, 4) || !aligned(seq_lens, 4))
        return MLA_B200_ERR_INVALID_ARG;
    if (page_size % tc::kTO != 0) return MLA_B200_ERR_UNSUPPORTED;
    if ((long long)max_seq_len > (long long)max_blocks * page_size) return MLA_B200_ERR_INVALID_ARG;
    const long long pool_rows = (long long)num_pages * page_size;
    const long long bound = (long long)batch * max_seq_len;
    if (pool_rows >= (1LL << 31) || bound >= (1LL << 31)) return MLA_B200_ERR_UNSUPPORTED;
    if (num_heads > 128) return MLA_B200_ERR_UNSUPPORTED;
    if (batch == 0) return MLA_B200_OK;
    if (num_pages == 0 || max_seq_len == 0) {
        // every sequence is empty: O* = 0 and LSE = -inf, through the merge of no partials
        return run_split_decode<T>(static_cast<const T *>(query), static_cast<const T *>(kv_pages),
                                   nullptr, batch, num_heads, 0, 0, softmax_scale, num_splits, out,
                                   out_dtype, out_lse, workspace, workspace_bytes,
                                   static_cast<cudaStream_t>(stream));
    }
    PagedArgs pg{block_table, seq_lens, max_blocks, page_size, pool_rows};
    return run_split_decode<T>(static_cast<const T *>(query), static_cast<const T *>(kv_pages),
                               nullptr, batch, num_heads, bound, max_seq_len, softmax_scale,
                               num_splits, out, out_dtype, out_lse, workspace, workspace_bytes,
                               static_cast<cudaStream_t>(stream), &pg);
}
}  // namespace

namespace {
template <typename T>
int decode_mtp(const void *query, const void *cache, const int32_t *cu_seqlens, int batch,
               int num_tokens, int num_heads, long long total_tokens, int max_seq_len,
               float softmax_scale, int num_splits, void *out, int out_dtype, float *out_lse,
               void *workspace, size_t workspace_bytes, void *stream) {
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    if (batch < 0 || num_tokens <= 0 || num_heads <= 0 || total_tokens < 0 || max_seq_len < 0)
        return MLA_B200_ERR_INVALID_ARG;
    if (batch > 0 && (query == nullptr || out == nullptr)) return MLA_B200_ERR_INVALID_ARG;
    if (total_tokens > 0 && cache == nullptr) return MLA_B200_ERR_INVALID_ARG;
    if (kBf16 ? (out_dtype != MLA_B200_OUT_BF16 && out_dtype != MLA_B200_OUT_F32)
              : (out_dtype != MLA_B200_OUT_F16 && out_dtype != MLA_B200_OUT_F32))
        return MLA_B200_ERR_INVALID_ARG;
    if (!(softmax_scale > 0.f) || !isfinite(softmax_scale)) return MLA_B200_ERR_INVALID_ARG;
    if (!aligned(query, 16) || !aligned(cache, 16) || !aligned(out, 16) || !aligned(out_lse, 4))
        return MLA_B200_ERR_INVALID_ARG;
    if (cu_seqlens == nullptr && (long long)batch * max_seq_len != total_tokens)
        return MLA_B200_ERR_INVALID_ARG;
    if (cu_seqlens != nullptr && max_seq_len == 0 && total_tokens > 0)
        return MLA_B200_ERR_INVALID_ARG;
    if (total_tokens >= (1LL << 31)) return MLA_B200_ERR_UNSUPPORTED;
    if (num_heads > 128) return MLA_B200_ERR_UNSUPPORTED;
    if ((long long)num_tokens * num_heads <= 128) {
        // every draft token's rows in one 128-row tile: one pass over the cache
        MtpArgs m{num_tokens, num_heads};
        return run_split_decode<T>(static_cast<const T *>(query), static_cast<const T *>(cache),
                                   cu_seqlens, batch, num_tokens * num_heads, total_tokens, max_seq_len,
                                   softmax_scale, num_splits, out, out_dtype, out_lse, workspace,
                                   workspace_bytes, static_cast<cudaStream_t>(stream), nullptr, nullptr, &m);
    }
    // More rows than one tile: each draft token runs as its own sequence of
    // num_heads rows (query [batch, k, n_h] = [batch * k, n_h] sequences) over the
    // real sequence's rows up to its causal limit.  The drafts of a sequence are
    // neighbours on the balanced cost line, so their clusters read the same cache
    // tiles at about the same time and the second read comes from L2.
    if ((long long)batch * num_tokens >= (1LL << 31)) return MLA_B200_ERR_UNSUPPORTED;
    return run_split_decode<T>(static_cast<const T *>(query), static_cast<const T *>(cache), cu_seqlens,
                               batch * num_tokens, num_heads, total_tokens, max_seq_len, softmax_scale,
                               num_splits, out, out_dtype, out_lse, workspace, workspace_bytes,
                               static_cast<cudaStream_t>(stream), nullptr, nullptr, nullptr, num_tokens);
}
}  // namespace

namespace {
// Bounded-wait self test: one thread waits on an mbarrier that nothing will
// complete, with the given limit, through the same wait loop the decode kernels
// use; the wait records kErrSelfTest in the device error word and returns,
// and the kernel writes whether it returned to *done.
__global__ void wait_selftest_kernel(uint64_t limit_ns, int *done) {
    __shared__ __align__(8) uint64_t bar;
    const uint32_t b = ptx::smem_u32(&bar);
    ptx::mbar_init(b, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const bool ok = ptx::mbar_wait(b, 0, kErrSelfTest, limit_ns);  // phase 0 never completes
    *done = ok ? 2 : 1;
}
}  // namespace

namespace {
// Y[b, h, m] = sum_k X[b, h, k] W[h, k, m] for every head (proj::proj_kernel):
// X [batch, heads, k_total], W [heads, k_total, m_total], Y element (b, h, m)
// at out[b * out_b + h * out_h + m]; rope (or null): [batch, heads, 64] copied
// to out[b * out_b + h * out_h + m_total + j].
template <bool kBf16>
int run_proj(const void *x, const void *w, const void *rope, void *out, int batch, int heads, int k_total,
             int m_total, long long out_b, long long out_h, cudaStream_t stream) {
    if (batch < 0 || heads <= 0 || k_total <= 0 || m_total <= 0) return MLA_B200_ERR_INVALID_ARG;
    if (batch > 0 && (x == nullptr || w == nullptr || out == nullptr)) return MLA_B200_ERR_INVALID_ARG;
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(out, 16) || !aligned(rope, 16))
        return MLA_B200_ERR_INVALID_ARG;
    if (k_total % proj::kStageK != 0 || m_total % proj::kTileM != 0) return MLA_B200_ERR_UNSUPPORTED;
    if ((long long)batch * heads * (long long)(k_total > m_total ? k_total : m_total) >= (1LL << 40))
        return MLA_B200_ERR_UNSUPPORTED;
    int dev;
    DevInfo info;
    int st = current_device(&dev, &info);
    if (st != MLA_B200_OK) return st;
    if (batch == 0) return MLA_B200_OK;
    auto enc = tmap_encoder();
    if (enc == nullptr) return cuda_failure(cudaErrorSymbolNotFound);
    proj::ProjParams p;
    p.batch = batch;
    p.heads = heads;
    p.k_total = k_total;
    p.m_total = m_total;
    p.n_box = std::min(256, (batch + 15) / 16 * 16);
    p.units_m = m_total / proj::kTileM;
    p.units_n = (int)cdiv(batch, p.n_box);
    const long long units = (long long)heads * p.units_m * p.units_n;
    if (units >= (1LL << 31)) return MLA_B200_ERR_UNSUPPORTED;
    p.units = (int)units;
    p.stage_bytes = 2 * proj::kBoxA + p.n_box * 128;
    p.stages = std::max(2, std::min(proj::kMaxStages, proj::kSmemBudget / p.stage_bytes));
    p.out = out;
    p.out_b = out_b;
    p.out_h = out_h;
    p.bf16 = kBf16 ? 1 : 0;
    p.rope = rope;
    const CUtensorMapDataType dt = kBf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const cuuint32_t estr[3] = {1, 1, 1};
    CUtensorMap wmap, xmap;
    {
        const cuuint64_t dims[3] = {(cuuint64_t)m_total, (cuuint64_t)k_total, (cuuint64_t)heads};
        const cuuint64_t strides[2] = {(cuuint64_t)m_total * 2, (cuuint64_t)k_total * m_total * 2};
        const cuuint32_t box[3] = {64, (cuuint32_t)proj::kStageK, 1};
        if (enc(&wmap, dt, 3, const_cast<void *>(w), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cuda_failure(cudaErrorInvalidValue);
    }
    {
        const cuuint64_t dims[3] = {(cuuint64_t)k_total, (cuuint64_t)heads, (cuuint64_t)batch};
        const cuuint64_t strides[2] = {(cuuint64_t)k_total * 2, (cuuint64_t)heads * k_total * 2};
        const cuuint32_t box[3] = {(cuuint32_t)proj::kStageK, 1, (cuuint32_t)p.n_box};
        if (enc(&xmap, dt, 3, const_cast<void *>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cuda_failure(cudaErrorInvalidValue);
    }
    const size_t smem = (size_t)p.stages * p.stage_bytes + proj::kNumBars * 8 + 16 + 1024;
    const int grid = std::min(p.units, info.sms);
    timing_mark(t_ev_start, stream);
    launch_dependent(proj::proj_kernel, dim3(grid), dim3(proj::kThreads), smem, stream, false, wmap, xmap, p);
    timing_mark(t_ev_stop, stream);
    return launch_status();
}
}  // namespace

extern "C" {

int mla_b200_absorb_q_f16(const void *q_nope, const void *q_rope, const void *w_uk, void *q_star, int batch,
                          int num_heads, int head_dim, void *stream) {
    if (batch > 0 && q_rope == nullptr) return MLA_B200_ERR_INVALID_ARG;
    return run_proj<false>(q_nope, w_uk, q_rope, q_star, batch, num_heads, head_dim, kDV,
                           (long long)num_heads * kDK, kDK, static_cast<cudaStream_t>(stream));
}

int mla_b200_absorb_q_bf16(const void *q_nope, const void *q_rope, const void *w_uk, void *q_star, int batch,
                           int num_heads, int head_dim, void *stream) {
    if (batch > 0 && q_rope == nullptr) return MLA_B200_ERR_INVALID_ARG;
    return run_proj<true>(q_nope, w_uk, q_rope, q_star, batch, num_heads, head_dim, kDV,
                          (long long)num_heads * kDK, kDK, static_cast<cudaStream_t>(stream));
}

int mla_b200_project_o_f16(const void *o_star, const void *w_uv, void *out, int batch, int num_heads,
                           int head_dim_v, void *stream) {
    return run_proj<false>(o_star, w_uv, nullptr, out, batch, num_heads, kDV, head_dim_v,
                           (long long)num_heads * head_dim_v, head_dim_v, static_cast<cudaStream_t>(stream));
}

int mla_b200_project_o_bf16(const void *o_star, const void *w_uv, void *out, int batch, int num_heads,
                            int head_dim_v, void *stream) {
    return run_proj<true>(o_star, w_uv, nullptr, out, batch, num_heads, kDV, head_dim_v,
                          (long long)num_heads * head_dim_v, head_dim_v, static_cast<cudaStream_t>(stream));
}

const char *mla_b200_status_string(int status) {
    switch (status) {
        case MLA_B200_OK: return "ok";
        case MLA_B200_ERR_INVALID_ARG: return "invalid argument";
        case MLA_B200_ERR_UNSUPPORTED: return "unsupported shape";
        case MLA_B200_ERR_WORKSPACE: return "workspace missing or too small";
        case MLA_B200_ERR_CUDA: return "CUDA runtime error";
        case MLA_B200_ERR_DEVICE_TIMEOUT: return "a kernel's bounded wait expired";
        case MLA_B200_ERR_NO_DEVICE: return "no sm_100 device is current";
        default: return "unknown status";
    }
}

const char *mla_b200_version(void) { return "0.1.0"; }

int mla_b200_constant(const char *name) {
    if (name == nullptr) return -1;
    if (!strcmp(name, "NUM_HEADS")) return MLA_B200_NUM_HEADS;
    if (!strcmp(name, "HEAD_DIM")) return MLA_B200_HEAD_DIM;
    if (!strcmp(name, "HEAD_DIM_C")) return MLA_B200_HEAD_DIM_C;
    if (!strcmp(name, "HEAD_DIM_ROPE")) return MLA_B200_HEAD_DIM_ROPE;
    if (!strcmp(name, "HEAD_DIM_K")) return MLA_B200_HEAD_DIM_K;
    if (!strcmp(name, "HEAD_DIM_V")) return MLA_B200_HEAD_DIM_V;
    return -1;
}

int mla_b200_set_kernel_timing(void *ev_start, void *ev_stop) {
    if ((ev_start == nullptr) != (ev_stop == nullptr)) return MLA_B200_ERR_INVALID_ARG;
    t_ev_start = static_cast<cudaEvent_t>(ev_start);
    t_ev_stop = static_cast<cudaEvent_t>(ev_stop);
    return MLA_B200_OK;
}

int mla_b200_set_kernel_span(unsigned long long *span, int slots) {
    t_span = slots > 0 ? span : nullptr;
    t_span_slots = span != nullptr && slots > 0 ? slots : 0;
    t_span_next = 0;
    return MLA_B200_OK;
}

int mla_b200_device_info(int *num_sms, int *decode_clusters) {
    int dev;
    DevInfo info;
    const int st = current_device(&dev, &info);
    if (st != MLA_B200_OK) return st;
    if (num_sms) *num_sms = info.sms;
    if (decode_clusters) *decode_clusters = info.tc_clusters;
    return MLA_B200_OK;
}

int mla_b200_plan(int batch, int num_heads, long long total_tokens, int max_seq_len, int num_sms,
                  int *chunk_tokens, int *num_splits) {
    if (batch < 0 || num_heads <= 0 || total_tokens < 0 || max_seq_len < 0)
        return MLA_B200_ERR_INVALID_ARG;
    if (num_sms <= 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            num_sms = 148;
        }
    }
    const int chunk = plan_chunk(batch, total_tokens, max_seq_len, num_sms, num_heads);
    if (chunk_tokens) *chunk_tokens = chunk;
    if (num_splits) *num_splits = max_seq_len > 0 ? (int)cdiv(max_seq_len, chunk) : 0;
    return MLA_B200_OK;
}

namespace {
size_t workspace_bytes_for(int batch, int num_heads, long long total_tokens, int max_seq_len,
                           int num_splits, bool fp8) {
    if (batch < 0 || num_heads <= 0 || total_tokens < 0) return 0;
    int num_sms = 0, dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        num_sms = 148;
    }
    if (max_seq_len <= 0 && batch > 0) max_seq_len = (int)cdiv(total_tokens, batch);
    const int chunk = chunk_for(batch, total_tokens, max_seq_len, num_splits, num_sms, num_heads);
    long long max_items = max_items_for(batch, total_tokens, chunk);
    // an automatic split may run the balanced schedule: batch + one item per cluster
    if (num_splits <= 0) max_items = std::max(max_items, (long long)batch + std::max(1, num_sms / 2));
    return ws_layout(nullptr, max_items, num_heads, batch, fp8).bytes;
}
}  // namespace

size_t mla_b200_workspace_size(int batch, int num_heads, long long total_tokens, int max_seq_len,
                               int num_splits) {
    return workspace_bytes_for(batch, num_heads, total_tokens, max_seq_len, num_splits, false);
}

size_t mla_b200_workspace_size_fp8(int batch, int num_heads, long long total_tokens, int max_seq_len,
                                   int num_splits) {
    return workspace_bytes_for(batch, num_heads, total_tokens, max_seq_len, num_splits, true);
}

size_t mla_b200_workspace_size_mtp(int batch, int num_tokens, int num_heads, long long total_tokens,
                                   int max_seq_len, int num_splits) {
    if (batch < 0 || num_tokens <= 0 || num_heads <= 0 || total_tokens < 0) return 0;
    if ((long long)num_tokens * num_heads <= 128)
        return workspace_bytes_for(batch, num_tokens * num_heads, total_tokens, max_seq_len, num_splits, false);
    if (max_seq_len <= 0 && batch > 0) max_seq_len = (int)cdiv(total_tokens, batch);
    return workspace_bytes_for(batch * num_tokens, num_heads, total_tokens * num_tokens, max_seq_len,
                               num_splits, false);
}

int mla_b200_decode_split_f16(const void *query, const void *cache, void *out, int num_heads,
                              int seq_length, int num_splits, void *workspace,
                              size_t workspace_bytes, void *stream) {
    if (query == nullptr || out == nullptr || num_heads <= 0 || seq_length < 0 ||
        (seq_length > 0 && cache == nullptr))
        return MLA_B200_ERR_INVALID_ARG;
    if (!aligned(query, 16) || !aligned(cache, 16) || !aligned(out, 16))
        return MLA_B200_ERR_INVALID_ARG;
    return run_split_decode<__half>(static_cast<const __half *>(query),
                                    static_cast<const __half *>(cache), nullptr, 1, num_heads,
                                    seq_length, seq_length, kRefScale, num_splits, out,
                                    MLA_B200_OUT_F16, nullptr, workspace, workspace_bytes,
                                    static_cast<cudaStream_t>(stream));
}

int mla_b200_decode_batched_f16(const void *query, const void *cache, const int32_t *cu_seqlens,
                                int batch, int num_heads, long long total_tokens, int max_seq_len,
                                float softmax_scale, int num_splits, void *out, int out_dtype,
                                float *out_lse, void *workspace, size_t workspace_bytes,
                                void *stream) {
    if (batch < 0 || num_heads <= 0 || total_tokens < 0 || max_seq_len < 0)
        return MLA_B200_ERR_INVALID_ARG;
    if (batch > 0 && (query == nullptr || out == nullptr)) return MLA_B200_ERR_INVALID_ARG;
    if (total_tokens > 0 && cache == nullptr) return MLA_B200_ERR_INVALID_ARG;
    if (out_dtype != MLA_B200_OUT_F16 && out_dtype != MLA_B200_OUT_F32)
        return MLA_B200_ERR_INVALID_ARG;
    if (!(softmax_scale > 0.f) || !isfinite(softmax_scale)) return MLA_B200_ERR_INVALID_ARG;
    if (!aligned(query, 16) || !aligned(cache, 16) || !aligned(out, 16) || !aligned(out_lse, 4))
        return MLA_B200_ERR_INVALID_ARG;
    if (cu_seqlens == nullptr && (long long)batch * max_seq_len != total_tokens)
        return MLA_B200_ERR_INVALID_ARG;
    if (cu_seqlens != nullptr && max_seq_len == 0 && total_tokens > 0)
        return MLA_B200_ERR_INVALID_ARG;
    if (total_tokens >= (1LL << 31)) return MLA_B200_ERR_UNSUPPORTED;
    return run_split_decode<__half>(static_cast<const __half *>(query),
                                    static_cast<const __half *>(cache), cu_seqlens, batch,
                                    num_heads, total_tokens, max_seq_len, softmax_scale,
                                    num_splits, out, out_dtype, out_lse, workspace,
                                    workspace_bytes, static_cast<cudaStream_t>(stream));
}

int mla_b200_decode_batched_bf16(const void *query, const void *cache, const int32_t *cu_seqlens,
                                 int batch, int num_heads, long long total_tokens, int max_seq_len,
                                 float softmax_scale, int num_splits, void *out, int out_dtype,
                                 float *out_lse, void *workspace, size_t workspace_bytes, void *stream) {
    if (batch < 0 || num_heads <= 0 || total_tokens < 0 || max_seq_len < 0)
        return MLA_B200_ERR_INVALID_ARG;
    if (batch > 0 && (query == nullptr || out == nullptr)) return MLA_B200_ERR_INVALID_ARG;
    if (total_tokens > 0 && cache == nullptr) return MLA_B200_ERR_INVALID_ARG;
    if (out_dtype != MLA_B200_OUT_BF16 && out_dtype != MLA_B200_OUT_F32) return MLA_B200_ERR_INVALID_ARG;
    if (!(softmax_scale > 0.f) || !isfinite(softmax_scale)) return MLA_B200_ERR_INVALID_ARG;
    if (!aligned(query, 16) || !aligned(cache, 16) || !aligned(out, 16) || !aligned(out_lse, 4))
        return MLA_B200_ERR_INVALID_ARG;
    if (cu_seqlens == nullptr && (long long)batch * max_seq_len != total_tokens)
        return MLA_B200_ERR_INVALID_ARG;
    if (cu_seqlens != nullptr && max_seq_len == 0 && total_tokens > 0)
        return MLA_B200_ERR_INVALID_ARG;
    if (total_tokens >= (1LL << 31)) return MLA_B200_ERR_UNSUPPORTED;
    if (num_heads > 128) return MLA_B200_ERR_UNSUPPORTED;
    return run_split_decode<__nv_bfloat16>(static_cast<const __nv_bfloat16 *>(query),
                                           static_cast<const __nv_bfloat16 *>(cache), cu_seqlens, batch,
                                           num_heads, total_tokens, max_seq_len, softmax_scale,
                                           num_splits, out, out_dtype, out_lse, workspace,
                                           workspace_bytes, static_cast<cudaStream_t>(stream));
}

int mla_b200_decode_paged_f16(const void *query, const void *kv_pages, const int32_t *block_table,
                              const int32_t *seq_lens, int batch, int num_heads, int num_pages,
                              int page_size, int max_blocks_per_seq, int max_seq_len,
                              float softmax_scale, int num_splits, void *out, int out_dtype,
                              float *out_lse, void *workspace, size_t workspace_bytes, void *stream) {
    return decode_paged<__half>(query, kv_pages, block_table, seq_lens, batch, num_heads, num_pages,
                                page_size, max_blocks_per_seq, max_seq_len, softmax_scale, num_splits,
                                out, out_dtype, out_lse, workspace, workspace_bytes, stream);
}

int mla_b200_decode_paged_bf16(const void *query, const void *kv_pages, const int32_t *block_table,
                               const int32_t *seq_lens, int batch, int num_heads, int num_pages,
                               int page_size, int max_blocks_per_seq, int max_seq_len,
                               float softmax_scale, int num_splits, void *out, int out_dtype,
                               float *out_lse, void *workspace, size_t workspace_bytes, void *stream) {
    return decode_paged<__nv_bfloat16>(query, kv_pages, block_table, seq_lens, batch, num_heads,
                                       num_pages, page_size, max_blocks_per_seq, max_seq_len,
                                       softmax_scale, num_splits, out, out_dtype, out_lse, workspace,
                                       workspace_bytes, stream);
}

int mla_b200_decode_mtp_f16(const void *query, const void *cache, const int32_t *cu_seqlens,
                            int batch, int num_tokens, int num_heads, long long total_tokens,
                            int max_seq_len, float softmax_scale, int num_splits, void *out,
                            int out_dtype, float *out_lse, void *workspace, size_t workspace_bytes,
                            void *stream) {
    return decode_mtp<__half>(query, cache, cu_seqlens, batch, num_tokens, num_heads, total_tokens,
                              max_seq_len, softmax_scale, num_splits, out, out_dtype, out_lse,
                              workspace, workspace_bytes, stream);
}

int mla_b200_decode_mtp_bf16(const void *query, const void *cache, const int32_t *cu_seqlens,
                             int batch, int num_tokens, int num_heads, long long total_tokens,
                             int max_seq_len, float softmax_scale, int num_splits, void *out,
                             int out_dtype, float *out_lse, void *workspace, size_t workspace_bytes,
                             void *stream) {
    return decode_mtp<__nv_bfloat16>(query, cache, cu_seqlens, batch, num_tokens, num_heads,
                                     total_tokens, max_seq_len, softmax_scale, num_splits, out,
                                     out_dtype, out_lse, workspace, workspace_bytes, stream);
}

namespace {
int decode_fp8(const void *query, const void *cache, float kv_scale, const float *kv_scales,
               const int32_t *cu_seqlens, int batch, int num_heads, long long total_tokens, int max_seq_len,
               float softmax_scale, int num_splits, void *out, int out_dtype, float *out_lse, void *workspace,
               size_t workspace_bytes, void *stream);
}  // namespace

int mla_b200_decode_batched_fp8(const void *query, const void *cache, float kv_scale,
                                const int32_t *cu_seqlens, int batch, int num_heads,
                                long long total_tokens, int max_seq_len, float softmax_scale,
                                int num_splits, void *out, int out_dtype, float *out_lse,
                                void *workspace, size_t workspace_bytes, void *stream) {
    return decode_fp8(query, cache, kv_scale, nullptr, cu_seqlens, batch, num_heads, total_tokens, max_seq_len,
                      softmax_scale, num_splits, out, out_dtype, out_lse, workspace, workspace_bytes, stream);
}

int mla_b200_decode_batched_fp8_scaled(const void *query, const void *cache, const float *kv_scales,
                                       const int32_t *cu_seqlens, int batch, int num_heads,
                                       long long total_tokens, int max_seq_len, float softmax_scale,
                                       int num_splits, void *out, int out_dtype, float *out_lse,
                                       void *workspace, size_t workspace_bytes, void *stream) {
    if (total_tokens > 0 && (kv_scales == nullptr || !aligned(kv_scales, 4))) return MLA_B200_ERR_INVALID_ARG;
    return decode_fp8(query, cache, 1.f, kv_scales, cu_seqlens, batch, num_heads, total_tokens, max_seq_len,
                      softmax_scale, num_splits, out, out_dtype, out_lse, workspace, workspace_bytes, stream);
}

}  // extern "C"

namespace {
int decode_fp8(const void *query, const void *cache, float kv_scale, const float *kv_scales,
               const int32_t *cu_seqlens, int batch, int num_heads, long long total_tokens, int max_seq_len,
               float softmax_scale, int num_splits, void *out, int out_dtype, float *out_lse, void *workspace,
               size_t workspace_bytes, void *stream) {
    if (batch < 0 || num_heads <= 0 || total_tokens < 0 || max_seq_len < 0)
        return MLA_B200_ERR_INVALID_ARG;
    if (batch > 0 && (query == nullptr || out == nullptr)) return MLA_B200_ERR_INVALID_ARG;
    if (total_tokens > 0 && cache == nullptr) return MLA_B200_ERR_INVALID_ARG;
    if (out_dtype != MLA_B200_OUT_F16 && out_dtype != MLA_B200_OUT_F32) return MLA_B200_ERR_INVALID_ARG;
    if (!(softmax_scale > 0.f) || !isfinite(softmax_scale)) return MLA_B200_ERR_INVALID_ARG;
    if (!(kv_scale > 0.f) || !isfinite(kv_scale)) return MLA_B200_ERR_INVALID_ARG;
    if (!aligned(query, 16) || !aligned(cache, 16) || !aligned(out, 16) || !aligned(out_lse, 4))
        return MLA_B200_ERR_INVALID_ARG;
    if (cu_seqlens == nullptr && (long long)batch * max_seq_len != total_tokens)
        return MLA_B200_ERR_INVALID_ARG;
    if (cu_seqlens != nullptr && max_seq_len == 0 && total_tokens > 0)
        return MLA_B200_ERR_INVALID_ARG;
    if (total_tokens >= (1LL << 31)) return MLA_B200_ERR_UNSUPPORTED;
    if (num_heads > 128) return MLA_B200_ERR_UNSUPPORTED;
    Fp8Args f8{cache, kv_scale, kv_scales};
    // (the fp16 cache pointer is unused on this path; query is fp16)
    return run_split_decode<__half>(static_cast<const __half *>(query), nullptr, cu_seqlens, batch,
                                    num_heads, total_tokens, max_seq_len, softmax_scale, num_splits,
                                    out, out_dtype, out_lse, workspace, workspace_bytes,
                                    static_cast<cudaStream_t>(stream), nullptr, &f8);
}
}  // namespace

extern "C" {

int mla_b200_decode_fused_f32(const float *query, const float *cache, float *out, int num_heads,
                              int head_dim_c, int seq_length, void *workspace,
                              size_t workspace_bytes, void *stream) {
    if (query == nullptr || out == nullptr || num_heads <= 0 || seq_length < 0 ||
        (seq_length > 0 && cache == nullptr))
        return MLA_B200_ERR_INVALID_ARG;
    if (head_dim_c != kDK) return MLA_B200_ERR_UNSUPPORTED;
    if (!aligned(query, 16) || !aligned(cache, 16) || !aligned(out, 16))
        return MLA_B200_ERR_INVALID_ARG;
    return run_split_decode<float>(query, cache, nullptr, 1, num_heads, seq_length, seq_length,
                                   kRefScale, 0, out, MLA_B200_OUT_F32, nullptr, workspace,
                                   workspace_bytes, static_cast<cudaStream_t>(stream));
}

int mla_b200_decode_naive_f32(const float *query, const float *cache, float *attn, float *out,
                              int num_heads, int head_dim_c, int seq_length, void *stream) {
    if (query == nullptr || cache == nullptr || attn == nullptr || out == nullptr ||
        num_heads <= 0 || head_dim_c <= 0 || seq_length <= 0)
        return MLA_B200_ERR_INVALID_ARG;
    if ((long long)num_heads * seq_length >= (1LL << 31) ||
        (long long)seq_length * head_dim_c >= (1LL << 31))
        return MLA_B200_ERR_UNSUPPORTED;
    int dev;
    DevInfo info;
    int st = current_device(&dev, &info);
    if (st != MLA_B200_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float scale = (float)(1.0 / sqrt((double)head_dim_c));
    // attn = scale * Q . C^T   [num_heads x seq_length]
    naive_gemm_kernel<true><<<dim3((unsigned)cdiv(seq_length, 16), (unsigned)cdiv(num_heads, 16)),
                              256, 0, s>>>(query, cache, attn, num_heads, seq_length, head_dim_c,
                                           seq_length, scale);
    naive_softmax_kernel<<<num_heads, 256, 0, s>>>(attn, seq_length);
    // out = attn . C           [num_heads x head_dim_c]
    naive_gemm_kernel<false><<<dim3((unsigned)cdiv(head_dim_c, 16), (unsigned)cdiv(num_heads, 16)),
                               256, 0, s>>>(attn, cache, out, num_heads, head_dim_c, seq_length,
                                            head_dim_c, 1.0f);
    return launch_status();
}

int mla_b200_combine_f32(const float *part_o, const float *part_lse, int num_parts,
                         long long rows, void *out, int out_dtype, float *out_lse, void *stream) {
    if (num_parts < 0 || rows < 0 || rows >= (1LL << 31)) return MLA_B200_ERR_INVALID_ARG;
    if (rows == 0) return MLA_B200_OK;
    if (out == nullptr || (num_parts > 0 && (part_o == nullptr || part_lse == nullptr)))
        return MLA_B200_ERR_INVALID_ARG;
    if (out_dtype != MLA_B200_OUT_F16 && out_dtype != MLA_B200_OUT_F32)
        return MLA_B200_ERR_INVALID_ARG;
    if (!aligned(part_o, 16) || !aligned(out, 16)) return MLA_B200_ERR_INVALID_ARG;
    int dev;
    DevInfo info;
    int st = current_device(&dev, &info);
    if (st != MLA_B200_OK) return st;
    WorkList wl = {};
    wl.items = nullptr;
    wl.item_off = nullptr;
    wl.batch = 1;
    wl.seq_len = num_parts;  // one "row" per part: item_range(0) = [0, num_parts)
    wl.chunk = 1;
    wl.cps = num_parts;
    wl.max_items = num_parts;
    const unsigned cgrid = (unsigned)rows;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t ps = (size_t)rows * kDV, ls = (size_t)rows;
    if (out_dtype == MLA_B200_OUT_F16)
        combine_kernel<__half, float><<<cgrid, kCombineThreads, 0, s>>>(
            part_o, part_lse, wl, (int)rows, rows, static_cast<__half *>(out), out_lse, 0, ps, ls);
    else
        combine_kernel<float, float><<<cgrid, kCombineThreads, 0, s>>>(
            part_o, part_lse, wl, (int)rows, rows, static_cast<float *>(out), out_lse, 0, ps, ls);
    return launch_status();
}

int mla_b200_combine_packed_f32(const float *parts, int num_parts, long long rows,
                                long long part_stride, void *out, int out_dtype, float *out_lse,
                                void *stream) {
    if (num_parts < 0 || rows < 0 || rows >= (1LL << 31)) return MLA_B200_ERR_INVALID_ARG;
    if (rows == 0) return MLA_B200_OK;
    if (out == nullptr || (num_parts > 0 && parts == nullptr)) return MLA_B200_ERR_INVALID_ARG;
    if (part_stride < rows * (kDV + 1) || part_stride % 4 != 0) return MLA_B200_ERR_INVALID_ARG;
    if (out_dtype != MLA_B200_OUT_F16 && out_dtype != MLA_B200_OUT_F32)
        return MLA_B200_ERR_INVALID_ARG;
    if (!aligned(parts, 16) || !aligned(out, 16)) return MLA_B200_ERR_INVALID_ARG;
    int dev;
    DevInfo info;
    int st = current_device(&dev, &info);
    if (st != MLA_B200_OK) return st;
    WorkList wl = {};
    wl.batch = 1;
    wl.seq_len = num_parts;  // one "row" per part: item_range(0) = [0, num_parts)
    wl.chunk = 1;
    wl.cps = num_parts;
    wl.max_items = num_parts;
    const unsigned cgrid = (unsigned)rows;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float *lse0 = parts + (size_t)rows * kDV;
    if (out_dtype == MLA_B200_OUT_F16)
        combine_kernel<__half, float><<<cgrid, kCombineThreads, 0, s>>>(
            parts, lse0, wl, (int)rows, rows, static_cast<__half *>(out), out_lse, 0,
            (size_t)part_stride, (size_t)part_stride);
    else
        combine_kernel<float, float><<<cgrid, kCombineThreads, 0, s>>>(
            parts, lse0, wl, (int)rows, rows, static_cast<float *>(out), out_lse, 0,
            (size_t)part_stride, (size_t)part_stride);
    return launch_status();
}

// ---------------------------------------------------------------------------
// Cross-GPU exchange over peer memory (mla_exchange.cuh).
// ---------------------------------------------------------------------------
size_t mla_b200_exchange_bytes(int world, long long rows) {
    if (world <= 0 || world > xchg::kMaxPeers || rows < 0) return 0;
    return xchg::buffer_bytes(world, rows);
}

int mla_b200_exchange_alloc(int world, long long rows, void **buf) {
    if (buf == nullptr || world <= 0 || world > xchg::kMaxPeers || rows <= 0 || rows >= (1LL << 31))
        return MLA_B200_ERR_INVALID_ARG;
    *buf = nullptr;
    int dev;
    DevInfo info;
    int st = current_device(&dev, &info);
    if (st != MLA_B200_OK) return st;
    void *p = nullptr;
    const size_t bytes = xchg::buffer_bytes(world, rows);
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_failure(e);
    e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_failure(e);
    }
    *buf = p;
    return MLA_B200_OK;
}

int mla_b200_exchange_free(void *buf) {
    if (buf == nullptr) return MLA_B200_OK;
    const cudaError_t e = cudaFree(buf);
    return e == cudaSuccess ? MLA_B200_OK : cuda_failure(e);
}

int mla_b200_ipc_handle(const void *buf, void *handle_64_bytes) {
    if (buf == nullptr || handle_64_bytes == nullptr) return MLA_B200_ERR_INVALID_ARG;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(buf));
    if (e != cudaSuccess) return cuda_failure(e);
    std::memcpy(handle_64_bytes, &h, sizeof(h));
    return MLA_B200_OK;
}

int mla_b200_ipc_open(const void *handle_64_bytes, void **peer_buf) {
    if (handle_64_bytes == nullptr || peer_buf == nullptr) return MLA_B200_ERR_INVALID_ARG;
    *peer_buf = nullptr;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle_64_bytes, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? MLA_B200_OK : cuda_failure(e);
}

int mla_b200_ipc_close(void *peer_buf) {
    if (peer_buf == nullptr) return MLA_B200_OK;
    const cudaError_t e = cudaIpcCloseMemHandle(peer_buf);
    return e == cudaSuccess ? MLA_B200_OK : cuda_failure(e);
}

int mla_b200_exchange_put_f32(const float *part, long long rows, void *const *peer_bufs, int rank, int world,
                              void *stream) {
    if (world <= 0 || world > xchg::kMaxPeers || rank < 0 || rank >= world || rows <= 0 || rows >= (1LL << 31))
        return MLA_B200_ERR_INVALID_ARG;
    if (part == nullptr || peer_bufs == nullptr || !aligned(part, 16)) return MLA_B200_ERR_INVALID_ARG;
    xchg::Peers peers = {};
    for (int g = 0; g < world; ++g) {
        if (peer_bufs[g] == nullptr || !aligned(peer_bufs[g], 256)) return MLA_B200_ERR_INVALID_ARG;
        peers.buf[g] = static_cast<uint8_t *>(peer_bufs[g]);
    }
    int dev;
    DevInfo info;
    int st = current_device(&dev, &info);
    if (st != MLA_B200_OK) return st;
    const xchg::XchgRows xr = {peers, rank, world, rows, xchg::stride_words(rows), 0};
    // (plain launches: chaining put and merge as programmatic dependents measured
    // slower on the whole 2-GPU step, 83 vs 61 us)
    xchg::exchange_put_kernel<<<(unsigned)rows, 128, 0, static_cast<cudaStream_t>(stream)>>>(part, xr);
    return launch_status();
}

int mla_b200_exchange_f32(const float *part, long long rows, void *const *peer_bufs, int rank, int world, void *out,
                          int out_dtype, float *out_lse, unsigned long long wait_limit_ns, void *stream) {
    if (world <= 0 || world > xchg::kMaxPeers || rank < 0 || rank >= world || rows <= 0 || rows >= (1LL << 31))
        return MLA_B200_ERR_INVALID_ARG;
    if (part == nullptr || peer_bufs == nullptr || out == nullptr || !aligned(part, 16) || !aligned(out, 16))
        return MLA_B200_ERR_INVALID_ARG;
    if (out_dtype != MLA_B200_OUT_F16 && out_dtype != MLA_B200_OUT_F32) return MLA_B200_ERR_INVALID_ARG;
    if (wait_limit_ns == 0 || wait_limit_ns > 60000000000ull) return MLA_B200_ERR_INVALID_ARG;
    xchg::Peers peers = {};
    for (int g = 0; g < world; ++g) {
        if (peer_bufs[g] == nullptr || !aligned(peer_bufs[g], 256)) return MLA_B200_ERR_INVALID_ARG;
        peers.buf[g] = static_cast<uint8_t *>(peer_bufs[g]);
    }
    int dev;
    DevInfo info;
    int st = current_device(&dev, &info);
    if (st != MLA_B200_OK) return st;
    // every block must be resident at once (they wait on each other)
    int per_sm = 0;
    const cudaError_t oe = out_dtype == MLA_B200_OUT_F16
        ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, xchg::exchange_fused_kernel<__half>, 128, 0)
        : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, xchg::exchange_fused_kernel<float>, 128, 0);
    if (oe != cudaSuccess) return cuda_failure(oe);
    if (rows > (long long)per_sm * info.sms) return MLA_B200_ERR_UNSUPPORTED;
    const xchg::XchgRows xr = {peers, rank, world, rows, xchg::stride_words(rows), wait_limit_ns};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (out_dtype == MLA_B200_OUT_F16)
        xchg::exchange_fused_kernel<__half><<<(unsigned)rows, 128, 0, s>>>(part, xr, static_cast<__half *>(out), out_lse);
    else
        xchg::exchange_fused_kernel<float><<<(unsigned)rows, 128, 0, s>>>(part, xr, static_cast<float *>(out), out_lse);
    return launch_status();
}

int mla_b200_decode_exchange_f16(const void *query, const void *cache, const int32_t *cu_seqlens, int batch,
                                 int num_heads, long long total_tokens, int max_seq_len, float softmax_scale,
                                 int num_splits, void *const *peer_bufs, int rank, int world, float *direct,
                                 void *out, int out_dtype, float *out_lse, unsigned long long wait_limit_ns,
                                 void *workspace, size_t workspace_bytes, void *stream) {
    if (batch <= 0 || num_heads <= 0 || total_tokens < 0 || max_seq_len < 0) return MLA_B200_ERR_INVALID_ARG;
    if (query == nullptr || out == nullptr || direct == nullptr || peer_bufs == nullptr)
        return MLA_B200_ERR_INVALID_ARG;
    if (total_tokens > 0 && cache == nullptr) return MLA_B200_ERR_INVALID_ARG;
    if (out_dtype != MLA_B200_OUT_F16 && out_dtype != MLA_B200_OUT_F32) return MLA_B200_ERR_INVALID_ARG;
    if (!(softmax_scale > 0.f) || !isfinite(softmax_scale)) return MLA_B200_ERR_INVALID_ARG;
    if (!aligned(query, 16) || !aligned(cache, 16) || !aligned(out, 16) || !aligned(direct, 16) ||
        !aligned(out_lse, 4))
        return MLA_B200_ERR_INVALID_ARG;
    if (cu_seqlens == nullptr && (long long)batch * max_seq_len != total_tokens) return MLA_B200_ERR_INVALID_ARG;
    if (cu_seqlens != nullptr && max_seq_len == 0 && total_tokens > 0) return MLA_B200_ERR_INVALID_ARG;
    if (world <= 0 || world > xchg::kMaxPeers || rank < 0 || rank >= world) return MLA_B200_ERR_INVALID_ARG;
    if (wait_limit_ns == 0 || wait_limit_ns > 60000000000ull) return MLA_B200_ERR_INVALID_ARG;
    if (total_tokens >= (1LL << 31) || (long long)batch * num_heads >= (1LL << 31)) return MLA_B200_ERR_UNSUPPORTED;
    XchgArgs xa = {};
    for (int g = 0; g < world; ++g) {
        if (peer_bufs[g] == nullptr || !aligned(peer_bufs[g], 256)) return MLA_B200_ERR_INVALID_ARG;
        xa.peers.buf[g] = static_cast<uint8_t *>(peer_bufs[g]);
    }
    xa.rank = rank;
    xa.world = world;
    xa.limit_ns = wait_limit_ns;
    xa.direct = direct;
    return run_split_decode<__half>(static_cast<const __half *>(query), static_cast<const __half *>(cache),
                                    cu_seqlens, batch, num_heads, total_tokens, max_seq_len, softmax_scale,
                                    num_splits, out, out_dtype, out_lse, workspace, workspace_bytes,
                                    static_cast<cudaStream_t>(stream), nullptr, nullptr, nullptr, 1, &xa);
}

int mla_b200_exchange_merge_f32(const void *own_buf, int world, long long rows, void *out, int out_dtype,
                                float *out_lse, unsigned long long wait_limit_ns, void *stream) {
    if (world <= 0 || world > xchg::kMaxPeers || rows <= 0 || rows >= (1LL << 31)) return MLA_B200_ERR_INVALID_ARG;
    if (own_buf == nullptr || out == nullptr || !aligned(own_buf, 256) || !aligned(out, 16))
        return MLA_B200_ERR_INVALID_ARG;
    if (out_dtype != MLA_B200_OUT_F16 && out_dtype != MLA_B200_OUT_F32) return MLA_B200_ERR_INVALID_ARG;
    if (wait_limit_ns == 0 || wait_limit_ns > 60000000000ull) return MLA_B200_ERR_INVALID_ARG;
    int dev;
    DevInfo info;
    int st = current_device(&dev, &info);
    if (st != MLA_B200_OK) return st;
    // the merge reads only this rank's own buffer: it stands at index 0
    xchg::XchgRows xr = {};
    xr.peers.buf[0] = static_cast<uint8_t *>(const_cast<void *>(own_buf));
    xr.rank = 0;
    xr.world = world;
    xr.rows = rows;
    xr.stride = xchg::stride_words(rows);
    xr.limit_ns = wait_limit_ns;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (out_dtype == MLA_B200_OUT_F16)
        xchg::exchange_merge_kernel<__half><<<(unsigned)rows, 128, 0, s>>>(xr, static_cast<__half *>(out), out_lse);
    else
        xchg::exchange_merge_kernel<float><<<(unsigned)rows, 128, 0, s>>>(xr, static_cast<float *>(out), out_lse);
    return launch_status();
}

// ---------------------------------------------------------------------------
// Allocation-free split decode.  Its scratch is this file-scope device array;
// host code may not use the array's name as a device address, so each device
// resolves the address once with cudaGetSymbolAddress (with that device current).
// ---------------------------------------------------------------------------
}  // extern "C"

static __device__ __align__(256) unsigned char g_noalloc_scratch[MLA_B200_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kMaxDevices] = {};

int noalloc_scratch(int dev, void **ptr) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
            return cuda_failure(cudaGetLastError());
        }
        g_noalloc_ptr[dev] = p;
    }
    *ptr = g_noalloc_ptr[dev];
    return MLA_B200_OK;
}
}  // namespace

extern "C" {

int mla_b200_decode_split_f16_noalloc(const void *query, const void *cache, void *out,
                                      int num_heads, int seq_length, int num_splits,
                                      void *stream) {
    if (query == nullptr || out == nullptr || num_heads <= 0 || seq_length < 0 ||
        (seq_length > 0 && cache == nullptr))
        return MLA_B200_ERR_INVALID_ARG;
    if (!aligned(query, 16) || !aligned(cache, 16) || !aligned(out, 16))
        return MLA_B200_ERR_INVALID_ARG;
    const size_t cap = MLA_B200_NOALLOC_SCRATCH_BYTES;
    // Scratch bytes of an explicit split count (pure workspace arithmetic).
    auto bytes_for = [&](int splits) -> size_t {
        const int chunk = chunk_for(1, seq_length, seq_length, splits, 0, num_heads);
        return ws_layout(nullptr, max_items_for(1, seq_length, chunk), num_heads, 1).bytes;
    };
    int dev;
    DevInfo info;
    int st = current_device(&dev, &info);
    if (st != MLA_B200_OK) return st;
    int splits = num_splits;
    if (splits > 0) {
        if (bytes_for(splits) > cap) return MLA_B200_ERR_WORKSPACE;
    } else {
        // the planned split, clamped to the most items whose partials fit:
        // per item num_heads x 512 fp32 (+ its LSE and work-list entry)
        const int chunk = plan_chunk(1, seq_length, seq_length, info.sms, num_heads);
        splits = seq_length > 0 ? (int)cdiv(seq_length, chunk) : 1;
        const long long per_item = (long long)num_heads * (kDV + 1) * 4 + 16;
        const long long fit = std::max(1LL, ((long long)cap - 5 * 256) / per_item - 1);
        splits = (int)std::max(1LL, std::min((long long)splits, fit));
        while (splits > 1 && bytes_for(splits) > cap) --splits;  // alignment slack: at most a step or two
        if (bytes_for(splits) > cap) return MLA_B200_ERR_WORKSPACE;
    }
    void *scratch = nullptr;
    st = noalloc_scratch(dev, &scratch);
    if (st != MLA_B200_OK) return st;
    return run_split_decode<__half>(static_cast<const __half *>(query),
                                    static_cast<const __half *>(cache), nullptr, 1, num_heads,
                                    seq_length, seq_length, kRefScale, splits, out,
                                    MLA_B200_OUT_F16, nullptr, scratch, cap,
                                    static_cast<cudaStream_t>(stream));
}

int mla_b200_get_device_error(int *code, void *stream) {
    int v = 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyFromSymbolAsync(&v, g_mla_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s) !=
            cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        return cuda_failure(cudaGetLastError());
    }
    if (code) *code = v;
    if (v != 0) {
        const int zero = 0;
        if (cudaMemcpyToSymbolAsync(g_mla_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) !=
                cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess) {
            return cuda_failure(cudaGetLastError());
        }
        return MLA_B200_ERR_DEVICE_TIMEOUT;
    }
    return MLA_B200_OK;
}

int mla_b200_last_cuda_error(void) { return t_last_cuda_error; }

int mla_b200_selftest_wait_timeout(unsigned long long limit_ns, int *done, void *stream) {
    if (done == nullptr || limit_ns == 0 || limit_ns > 100000000ull) return MLA_B200_ERR_INVALID_ARG;
    int dev;
    DevInfo info;
    const int st = current_device(&dev, &info);
    if (st != MLA_B200_OK) return st;
    wait_selftest_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, done);
    return launch_status();
}

}  // extern "C"
