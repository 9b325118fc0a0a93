// mla_tc.cuh -- tcgen05 split-KV MLA decode for sm_100a (fp16 in, fp32 accumulate).
//
// Replaces the reference's mma.sync split kernel mla_decode_splitk_mma_fp16
// (csrc/mla_decode_splitk_fwd.cuh:559-892).  One work item = up to `chunk`
// cache rows of one sequence (mla_common.cuh WorkList); the item's partial
// (O normalized by its own sum, natural-log LSE) goes to the workspace and
// combine_kernel merges the items of each sequence.
//
// Why two CTAs per item.  For 128 heads the O accumulator is 128 x 512 fp32 =
// all 512 TMEM columns of an SM, leaving no room for S = Q.C^T.  So each item
// runs on a 2-CTA cluster (two SMs):
//
//   S-CTA (cluster rank 0)                 O-CTA (cluster rank 1)
//   Q* [128 x 576] fp16 in TMEM (288 col)    O [128 x 512] fp32 in TMEM (512 col)
//   TMA: C in K-blocks [96 tok x 64 col],    TMA: C tile [32 tok x 512] -> 4-slot ring
//     three per slot -> 4-slot ring          GEMM2 O += P.C_N (SS MMA, N=256,
//   GEMM1 S = Q.C^T (TS MMA, N=96)             C_N read MN-major from the tile)
//     into one of two S buffers (2 x 96 col)  rescale O rows when the S-CTA
//   online softmax (fp32 m, l; lazy             raised the running max; final
//     rescale, threshold 2^8)                   O / l and LSE to the workspace
//   P fp16 + per-row alpha ---DSMEM bulk copy (26 KB / 96 tokens)---> 3-slot ring
//
// Tile sizes come from tcgen05 costs measured on B200.  One thread issues an
// M=128 kind::f16 MMA at most every ~46 cycles and the tensor pipe queues ~8,
// so N=96 (48 cycles of work) is the smallest tile that keeps the pipe busy;
// Q (288 TMEM columns) leaves room for two N=96 S buffers, and TS MMAs (A in
// TMEM) issue faster than SS ones.  GEMM1's 576-deep K is streamed through the
// ring three 64-column blocks at a time, so every ring wait is followed by 12
// MMAs.  GEMM2 uses N=256.  GEMM1 (576 MACs/token/head) and GEMM2 (512) are
// balanced across the pair and no tensor work is duplicated.  The pair reads
// the same rows; the second read of each byte hits L2.
//
// Q reaches TMEM through the same ring as the cache: at the first item of a
// sequence the S-CTA's producer TMA-loads the nine 128 x 64 Q boxes into five
// ring slots, and the MMA thread copies each landed slot into TMEM with
// tcgen05.cp before the GEMM1 MMAs that read it (the copy and the MMAs are
// ordered in the tensor pipe), releasing the slot with a commit.
//
// Warp roles (256 threads): warp 0 TMA producer, warp 1 MMA issuer (one
// thread), warp 2 TMEM allocator, warps 4-7 the math warpgroup (softmax in
// the S-CTA, correction + epilogue in the O-CTA); thread h of the warpgroup
// owns TMEM lane h = head h.
//
// Heads: num_heads <= 128; rows >= num_heads carry the next rows of Q (or the
// TMA's zero fill) and their results are dropped, so fewer heads cost the same
// tensor work as 128.
#pragma once

#include "mla_tc_ptx.cuh"

namespace mla {
namespace tc {

constexpr int kTS = 96;                          // tokens per S tile (GEMM1 N)
constexpr int kTO = 32;                          // tokens per O tile (C_N ring granularity)
constexpr int kOPerS = kTS / kTO;                // 3
constexpr int kKBlocks = kDK / 64;               // 9 column blocks of 64
constexpr int kVBlocks = kDV / 64;               // 8
constexpr int kBoxS = kTS * 128;                 // 12288: one K-block box [96 tok x 64 col]
constexpr int kKbPerSlot = 3;                    // K-blocks per S ring slot (12 MMAs per wait)
constexpr int kSlotS = kKbPerSlot * kBoxS;       // 36864
constexpr int kSlotsPerTile = kKBlocks / kKbPerSlot;  // 3
constexpr int kPieceS = kKbPerSlot * kTO * 128;  // 12288: paged, one 32-row piece of a slot
constexpr int kSlotsS = 5;
constexpr int kBoxO = kTO * 128;                 // 4096: [32 tok x 64 col]
constexpr int kSlotO = kVBlocks * kBoxO;         // 32768: C tile [32 x 512]
constexpr int kSlotsO = 4;
constexpr int kQBoxBytes = 128 * 128;            // Q box: 128 rows x 64 fp16
constexpr int kQSlots = (kKBlocks + 1) / 2;      // 5 ring slots carry Q (two boxes each)
static_assert(2 * kQBoxBytes <= kSlotS, "two Q boxes per ring slot");

// FP8 (e4m3) cache.  S-CTA: C tiles as 64-byte K-blocks (SW64) in 18 KB slots
// (3 K-blocks x 96 rows), ten of them in the fp16 ring's space; Q* as fp8 hi
// and lo planes, one K-block of each per slot.  O-CTA: C8_N tiles [32 x 512 B]
// (4 column groups of 128 B, SW128: GEMM2's MN-major B) in eight 16 KB slots;
// the math warpgroup turns each fp16 P message into e4m3 hi and lo planes in
// place (3 K-steps x [128 rows x 32 B], SW32), GEMM2's K-major A.  (Splitting
// P in the S-CTA's softmax instead, from fp32 registers, measured slower: cfg3
// 85.7 vs 67 us.  The softmax warpgroup bounds the tile period and the
// conversions share the exp2 pipe; the O-CTA's warpgroup is otherwise idle.)
constexpr int kBoxS8 = kTS * 64;                 // 6144: one fp8 K-block [96 tok x 64 B]
constexpr int kSlotS8 = kKbPerSlot * kBoxS8;     // 18432
constexpr int kSlotsS8 = 10;
static_assert(kSlotsS8 * kSlotS8 <= kSlotsS * kSlotS, "fp8 S ring inside the fp16 one");
constexpr int kQBox8 = 128 * 64;                 // 8192: Q8 box [128 rows x 64 B]
static_assert(2 * kQBox8 <= kSlotS8, "Q8 hi + lo box per ring slot");
constexpr int kSlotO8 = kTO * kDV;               // 16384: C8_N tile [32 x 512 B]
constexpr int kSlotsO8 = 8;
constexpr int kPlaneP8 = kOPerS * 128 * kTO;     // 12288: one e4m3 P plane of a message
constexpr int kTmemQLo = 144;                    // fp8: Q lo plane's TMEM columns

// Message S-CTA -> O-CTA, one per S tile: P as three SW64 K-major sub-tiles of
// [128 rows x 32 tokens] (8 KB each), then per-row alpha, l, m.
constexpr int kSubP = 128 * kTO * 2;             // 8192
constexpr int kMsgP = kOPerS * kSubP;            // 24576
constexpr int kMsgAlpha = kMsgP;
constexpr int kMsgL = kMsgP + 512;
constexpr int kMsgM = kMsgP + 1024;
constexpr int kMsgBytes = kMsgP + 1536;          // 26112
constexpr int kMsgStride = 26 * 1024;
constexpr int kMsgSlots = 3;                     // O-CTA receive ring

constexpr int kRingSlots = kSlotsS8;             // the deepest ring (fp8 S-CTA)
static_assert(kRingSlots >= kSlotsS && kRingSlots >= kSlotsO, "ring barriers");
enum BarId {
    kBarFull = 0,                      // [4] ring slot landed            (count 1 + tx)
    kBarEmpty = kRingSlots,            // [4] ring slot consumed          (count 1, commit)
    kBarSFull = 2 * kRingSlots,        // [2] S-CTA: S tile in TMEM        (count 1, commit)
    kBarSEmpty = kBarSFull + 2,        // [2] S-CTA: S tile read           (count 128)
    kBarQFree = kBarSEmpty + 2,        // [2] S-CTA: an issuer's GEMM1s reading Q done (count 1, commit)
    kBarQReady = kBarQFree + 2,        //     S-CTA: a sequence's Q copied into TMEM (count 1, commit)
    kBarPFree = kBarQReady + 1,        // [3] GEMM2 done with message slot (count 1, commit arriving in both CTAs)
    kBarPFull = kBarPFree + kMsgSlots, // [3] O-CTA: message landed        (count 1 + tx, from the S-CTA)
    kBarCorr = kBarPFull + kMsgSlots,  // [3] O-CTA: O ready for GEMM2     (count 128)
    kBarMmaDone = kBarCorr + kMsgSlots,// [3] O-CTA: GEMM2 of a message done (count 1, commit)
    kBarDrain = kBarMmaDone + kMsgSlots,// [2] an MMA issuer's ops retired (teardown)
    kNumBars = kBarDrain + 2
};

// Shared-memory layout (offsets from a 1024-aligned base).  Each role has its
// own ring and message buffers; the barriers sit at the same offset in both
// CTAs (remote arrivals and the two-CTA commit address them by offset).
constexpr int kOffRing = 0;
constexpr int kOffStgS = kSlotsS * kSlotS;                       // 184320: S staging
constexpr int kOffMsgO = kSlotsO * kSlotO;                       // 131072: O receive ring [3]
static_assert(kSlotsO8 * kSlotO8 <= kOffMsgO, "C8_N ring inside the O ring");
static_assert(2 * kPlaneP8 <= kMsgAlpha, "e4m3 P planes inside the message's P");
constexpr int kEndS = kOffStgS + kMsgStride;                     // 210944
constexpr int kEndO = kOffMsgO + kMsgSlots * kMsgStride;         // 210944
constexpr int kOffBar = kEndS > kEndO ? kEndS : kEndO;
constexpr int kOffSlot = kOffBar + kNumBars * 8;
constexpr int kOffAbort = kOffSlot + 4;
constexpr int kOffZArg = kOffAbort + 4;                          // paged zero request: {tile, tail rows, stop}
constexpr int kOffEpi = (kOffZArg + 12 + 1023) / 1024 * 1024;    // O-CTA epilogue staging
constexpr int kEpiWarpBytes = 32 * 128;                          // one warp's 32 rows x 128 bytes
constexpr int kSmemBytes = kOffEpi + 4 * kEpiWarpBytes + 1024;   // + 1024 alignment slack
static_assert(kSmemBytes <= 232448, "dynamic shared memory limit");

constexpr int kThreads = 256;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemQ = 0;     // S-CTA: Q, 288 columns (2 fp16 per column)
constexpr uint32_t kTmemS = 288;   // S-CTA: two S buffers of kTS columns
static_assert(kTmemS + 2 * kTS <= kTmemCols, "TMEM budget");
constexpr float kRescaleLog2 = 8.0f;
// fp8 cache: P is scaled by 2^2 before its e4m3 hi/lo split (small weights
// reach e4m3's subnormals 4x later: their absolute error drops to 2^-12), and
// the lazy rescale keeps p <= 2^6: 2^2 * 64 = 256 stays under e4m3's 448.  (2^6
// with p <= 4 measured slower: O corrections become frequent.)
constexpr float kRescaleLog2Fp8 = 6.0f;
constexpr float kP8Scale = 4.0f;
// Per-row scales: the scale's exponent joins the softmax exponent, so within a
// tile the weights of small-scale rows sit lower by the tiles' scale spread.  A
// lower lazy-rescale threshold (2^3) leaves room for a larger factor: q = 16 *
// w * mantissa <= 16 * 8 * 2 = 256.  (2^4 with a factor of 8 left a 2^4.6
// scale spread at max-abs 0.0107, just over the bar.)
constexpr float kRescaleLog2Fp8Rows = 3.0f;
constexpr float kP8ScaleRows = 16.0f;  // times the scale's mantissa in [1, 2)
constexpr float kP8Log2Scale = 2.0f;      // log2 kP8Scale
constexpr float kP8Log2ScaleRows = 4.0f;  // log2 kP8ScaleRows

// s = 2^e * f with f in [1, 2), for a positive normal float (bit fields; e is
// clamped to +-125 so that 2^-e stays a normal float).
__device__ __forceinline__ int scale_exp(float s) {
    return min(125, max(-125, ((__float_as_int(s) >> 23) & 0xFF) - 127));
}
__device__ __forceinline__ float scale_mant(float s) {
    return __int_as_float((__float_as_int(s) & 0x007FFFFF) | 0x3F800000);
}
__device__ __forceinline__ float scale_pow2_inv(float s) { return __int_as_float((127 - scale_exp(s)) << 23); }

// GEMM1: M=128 heads, N=96 tokens; GEMM2: M=128 heads, N=256 dims, B MN-major.
template <bool kBf16> __host__ __device__ constexpr uint32_t idesc_s() { return ptx::idesc_f16_f32(128, kTS, 0, 0, kBf16 ? 1 : 0); }
template <bool kBf16> __host__ __device__ constexpr uint32_t idesc_o() { return ptx::idesc_f16_f32(128, 256, 0, 1, kBf16 ? 1 : 0); }
// kind::f8f6f4 with A and B e4m3 (format code 0), f32 accumulate: the same bits
// as the f16 descriptor.
__host__ __device__ constexpr uint32_t idesc_s8() { return ptx::idesc_f16_f32(128, kTS, 0, 0, 0); }

struct TcParams {
    WorkList wl;
    int num_heads;
    float scale_log2;  // softmax scale * log2(e)
    void *part_o;      // [max_items, num_heads, 512], element type part_kind
    float *part_lse;   // [max_items, num_heads]
    int part_kind;     // partial element type: kOutF32 / kOutF16 / kOutBF16
    union {
        int page_size;     // paged: a multiple of kTO
        float o_scale;     // fp8 cache: factor of the finished O (kv scale; 1 with per-row scales)
    };
    void *out;         // [batch, num_heads, 512]: written directly for single-item sequences
    int out_kind;      // out element type: kOutF32 / kOutF16 / kOutBF16
    union {
        int max_blocks;    // paged
        int mtp;           // multi-token: (draft tokens << 16) | heads per token
    };
    float *out_lse;    // [batch, num_heads] or null
    unsigned long long *span;  // or null: {first CTA start, last CTA end} %globaltimer of this launch
    int chain;                 // the merge after this launch is a programmatic dependent
    const float *kv_scales;    // fp8 cache: per cache row dequantisation scale (or null: per tensor)
    // Paged cache (kPaged): the maps address the page pool as rows
    // [num_pages * page_size, 576]; token t of sequence b lives in pool row
    // block_table[b * max_blocks + t / page_size] * page_size + t % page_size,
    // and wl.cu_seqlens holds the sequences' offsets on a virtual packed axis.
    // (page_size and max_blocks sit in alignment padding: the kernel's code
    // generation for the contiguous cache is sensitive to this struct's size.)
    union {
        const int32_t *block_table;
        const float *q_scale;  // fp8 cache: per (sequence, head) row, Q* = Q8 x q_scale
    };
};

// Zeroes rows [tail, 32) of a landed [32 x 512] C tile (8 SW128 K-blocks of
// 32 rows; whole 128-byte rows, so the swizzle does not matter), this lane's
// share of a warp's work, and orders the stores before the tensor core's
// operand reads.
__device__ __forceinline__ void zero_tail(uint32_t tile, int tail, int lane) {
    const int pieces = (kTO - tail) * kVBlocks * 8;  // 16-byte pieces
    for (int q = lane; q < pieces; q += 32) {
        const int rb = q >> 3;
        ptx::st_shared_v4(tile + (rb % kVBlocks) * kBoxO + (tail + rb / kVBlocks) * 128 + (q & 7) * 16, 0u, 0u, 0u, 0u);
    }
    ptx::fence_proxy_async_smem();
}

// fp8 cache: turns row h of a landed fp16 P message (3 SW64 K-major sub-tiles
// [128 x 32 tokens]) into e4m3 hi and lo planes of q (the weights as the
// softmax sent them, already times kP8Scale / kP8ScaleRows): hi and lo = e4m3(q
// - hi) carry q to ~2^-8 relative (one e4m3 plane would be 2^-4), written over
// the same bytes as GEMM2's A: plane x, K-step st at x * kPlaneP8 + st * 4096,
// row h's 32 bytes with 32-byte swizzle.  All of the warpgroup's reads must
// finish (a named barrier between the two halves) before any write.
struct P8Row {
    uint4 v[kOPerS * 4];  // the row's 96 fp16 values
};

__device__ __forceinline__ void p8_read(const uint8_t *msg, int h, P8Row &r) {
#pragma unroll
    for (int st = 0; st < kOPerS; ++st)
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4)
            r.v[st * 4 + c4] = *reinterpret_cast<const uint4 *>(msg + st * kSubP + h * 64 + ((c4 ^ ((h >> 1) & 3)) << 4));
}

__device__ __forceinline__ uint32_t e4m3x2_of(uint32_t h2) {  // two halves -> two e4m3 bytes
    const __half2_raw hr = *reinterpret_cast<const __half2_raw *>(&h2);
    return (uint32_t)__nv_cvt_halfraw2_to_fp8x2(hr, __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ uint32_t half2_of_e4m3x2(uint32_t b2) {
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)b2, __NV_E4M3);
    return (uint32_t)hr.x | ((uint32_t)hr.y << 16);
}

// hi: kExact, e4m3(q) decoded back (one conversion more per pair); else q
// rounded to 3 mantissa bits on the integer pipe (half an ulp added at bit 6 of
// each fp16, bits 0-6 cleared; q >= 0 so the low half cannot carry into the
// high one), which is exact in e4m3's normal range [2^-6, 448].  Below 2^-6
// (weights under 2^-8 of the running maximum) e4m3 is subnormal and the
// rounded hi may not be representable: an error of at most 2^-10 on such a q,
// as for the exact split.  Per-row cache scales push small-scale rows' weights
// lower, so they take the exact split.
template <bool kExact>
__device__ __forceinline__ void p8_write(uint8_t *msg, int h, const P8Row &r) {
#pragma unroll
    for (int st = 0; st < kOPerS; ++st) {
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
            const uint32_t in[4] = {r.v[st * 4 + c4].x, r.v[st * 4 + c4].y, r.v[st * 4 + c4].z, r.v[st * 4 + c4].w};
            uint32_t hb[4], lb[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                uint32_t hh;  // hi as two fp16
                if constexpr (kExact) {
                    hb[k] = e4m3x2_of(in[k]);
                    hh = half2_of_e4m3x2(hb[k]);
                } else {
                    hh = (in[k] + 0x00400040u) & 0xFF80FF80u;
                    hb[k] = e4m3x2_of(hh);
                }
                const __half2 d = __hsub2(*reinterpret_cast<const __half2 *>(&in[k]), *reinterpret_cast<const __half2 *>(&hh));
                lb[k] = e4m3x2_of(*reinterpret_cast<const uint32_t *>(&d));
            }
            hi[2 * c4] = hb[0] | (hb[1] << 16);
            hi[2 * c4 + 1] = hb[2] | (hb[3] << 16);
            lo[2 * c4] = lb[0] | (lb[1] << 16);
            lo[2 * c4 + 1] = lb[2] | (lb[3] << 16);
        }
        const int sw = (h >> 2) & 1;  // 32-byte swizzle: chunk ^= address bit 7
#pragma unroll
        for (int x = 0; x < 2; ++x) {
            const uint32_t *src = x == 0 ? hi : lo;
            uint8_t *row = msg + x * kPlaneP8 + st * 4096 + h * 32;
            *reinterpret_cast<uint4 *>(row + ((0 ^ sw) << 4)) = make_uint4(src[0], src[1], src[2], src[3]);
            *reinterpret_cast<uint4 *>(row + ((1 ^ sw) << 4)) = make_uint4(src[4], src[5], src[6], src[7]);
        }
    }
}

// Pool row of the 32-row box starting at token t (a multiple of kTO) of
// sequence b.  Boxes past the item's last token `last` re-read its last box:
// the softmax masks those columns, so the bytes only have to be addressable
// (and no block-table entry past the sequence's pages is read).
__device__ __forceinline__ int paged_row(const TcParams &p, int b, int t, int last) {
    const int tc = min(t, last & ~(kTO - 1));
    const int blk = tc / p.page_size;
    const int pg = p.block_table[(long long)b * p.max_blocks + blk];
    return pg * p.page_size + (tc - blk * p.page_size);
}

__device__ __forceinline__ uint32_t u32_of(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float f32_of(uint32_t u) { return __uint_as_float(u); }

enum OutKind : int { kOutF32 = 0, kOutF16 = 1, kOutBF16 = 2 };

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ uint32_t pack_bf162(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

template <bool kBf16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (kBf16) return pack_bf162(a, b);
    else return pack_half2(a, b);
}

// Ring position: slot index and phase bit of a producer/consumer cursor.
struct Ring {
    uint32_t slot = 0, phase = 0;
    __device__ __forceinline__ void next(int n) {
        if (++slot == (uint32_t)n) { slot = 0; phase ^= 1; }
    }
};

// cmap_s: the cache as (64 columns, rows, 9 K-blocks), one box = 3 K-blocks x
// 96 rows = one S ring slot; paged: the pool as (64, 8 rows, 9 K-blocks, row
// groups), one box = 3 K-blocks x 32 rows of one page, three per slot (the
// slot's K-blocks interleaved per 8-row group).  cmap_o: the cache as (64,
// rows, 9), one box = 8 K-blocks x 32 rows = one O ring slot.  qmap: query
// [B * n_h, 576], box 64 x 128.  All 128-byte swizzled.
// kSched: the work-list schedule this instantiation serves (kSchedChunked or
// kSchedBalanced); the other schedule's iteration code would cost registers in
// every role.  kBf16: Q* and the cache are bf16 (P goes to GEMM2 as bf16 too:
// the MMA takes A and B of one type); otherwise fp16.  kPaged: the cache is a
// page pool addressed through p.block_table.  kMtp: each sequence's rows are
// (draft token i, head) pairs, row = i * heads + head, and draft token i of k
// sees the sequence's first len - (k - 1 - i) tokens (its own KV being the
// cache's last k rows).  kFp8: the cache is e4m3 (cmap_s:
// 64-byte K-blocks, box 3 x 96 rows, SW64; cmap_o: (128 B, rows, 4) box of one
// [32 x 512 B] tile, SW128) and qmap addresses Q8 [2 x B * n_h, 576] e4m3
// (hi plane, then lo plane), box 64 x 128, SW64.  kRows (with kFp8): one
// dequantisation scale per cache row, p.kv_scales; a separate instantiation
// because the per-row code slowed the per-tensor kernel by ~10 %.
template <int kSched, bool kBf16, bool kPaged, bool kFp8, bool kMtp = false, bool kRows = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    tc_decode_kernel(const __grid_constant__ CUtensorMap cmap_s,
                     const __grid_constant__ CUtensorMap cmap_o,
                     const __grid_constant__ CUtensorMap qmap, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = ptx::smem_u32(smem);
    const uint32_t bar0 = sbase + kOffBar;
    auto bar = [&](int id) -> uint32_t { return bar0 + 8u * id; };
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + kOffAbort);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const uint32_t role = ptx::cluster_ctarank();  // 0 = S-CTA, 1 = O-CTA
    const int cid = (int)ptx::cluster_id_x();
    const int ncl = (int)ptx::nclusters_x();

    if (tid == 0) {
        for (int i = 0; i < kRingSlots; ++i) {
            ptx::mbar_init(bar(kBarFull + i), 1);
            ptx::mbar_init(bar(kBarEmpty + i), 1);
        }
        for (int i = 0; i < 2; ++i) {
            ptx::mbar_init(bar(kBarSFull + i), 1);
            ptx::mbar_init(bar(kBarSEmpty + i), 128);
        }
        for (int i = 0; i < kMsgSlots; ++i) {
            ptx::mbar_init(bar(kBarPFree + i), 1);
            ptx::mbar_init(bar(kBarPFull + i), 1);
            ptx::mbar_init(bar(kBarCorr + i), 128);
            ptx::mbar_init(bar(kBarMmaDone + i), 1);
        }
        for (int i = 0; i < 2; ++i) {
            ptx::mbar_init(bar(kBarQFree + i), 1);
            ptx::mbar_init(bar(kBarDrain + i), 1);
        }
        ptx::mbar_init(bar(kBarQReady), 1);
        if constexpr (kPaged) reinterpret_cast<volatile int *>(smem + kOffZArg)[2] = 0;
        *abort_flag = 0;
        ptx::fence_mbarrier_init_cluster();
    }
    if (warp == 0 && lane == 0) {
        ptx::tma_prefetch_desc(role == 0 ? &cmap_s : &cmap_o);
        if (role == 0) ptx::tma_prefetch_desc(&qmap);
    }
    if (warp == 2) {
        ptx::tmem_alloc(sbase + kOffSlot, kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    ptx::cluster_sync();
    ptx::tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + kOffSlot);
    // Set-up above overlaps the plan kernel (programmatic launch); the work list
    // is read below.
    if (p.chain) griddep_launch();  // the chained merge may place its CTAs
    griddep_wait();
    // the span starts when work can start (a chained launch may have started
    // early and waited above); it is published at teardown
    const unsigned long long t_start = globaltimer_ns();

    const WorkList &wl = p.wl;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            const int nslots = role == 0 ? (kFp8 ? kSlotsS8 : kSlotsS) : (kFp8 ? kSlotsO8 : kSlotsO);
            Ring rg;
            int prev_b = -1;
            bool ok = true;
            auto acquire = [&]() -> bool {
                return !*abort_flag && ptx::mbar_wait(bar(kBarEmpty + rg.slot), rg.phase ^ 1, kErrWaitEmpty);
            };
            ItemCursor cur = items_begin<kSched>(wl, cid, ncl);
            Item it;
            int i;
            while (ok && items_next<kSched>(wl, cur, it, i)) {
                // paged: pool rows of the current tile's three 32-row pieces, and
                // of the next tile's, read a tile ahead so the block-table
                // latency stays off the refill path (the first tile's overlaps
                // the Q loads)
                int last = 0, pr[kOPerS], pn[kOPerS];
                if constexpr (kPaged) {
                    last = it.tok0 + it.len - 1;
#pragma unroll
                    for (int c = 0; c < kOPerS; ++c) pr[c] = paged_row(p, it.b, it.tok0 + c * kTO, last);
                }
                if (kFp8 && role == 0 && it.b != prev_b) {
                    // Q8 of the new sequence: hi and lo boxes of one K-block per slot
                    const int qrow = it.b * p.num_heads, lo_row = wl.batch * p.num_heads + qrow;
                    for (int kb = 0; kb < kKBlocks; ++kb) {
                        if (!acquire()) { ok = false; break; }
                        const uint32_t dst = sbase + kOffRing + rg.slot * kSlotS8;
                        ptx::mbar_arrive_expect_tx(bar(kBarFull + rg.slot), 2 * kQBox8);
                        ptx::tma_load_2d(dst, &qmap, kb * 64, qrow, bar(kBarFull + rg.slot));
                        ptx::tma_load_2d(dst + kQBox8, &qmap, kb * 64, lo_row, bar(kBarFull + rg.slot));
                        rg.next(nslots);
                    }
                    prev_b = it.b;
                } else if (role == 0 && it.b != prev_b) {
                    // Q of the new sequence: two 128 x 64 boxes per ring slot
                    const int qrow = it.b * p.num_heads;
                    for (int kb = 0; kb < kKBlocks; kb += 2) {
                        if (!acquire()) { ok = false; break; }
                        const int nb = min(2, kKBlocks - kb);
                        const uint32_t dst = sbase + kOffRing + rg.slot * kSlotS;
                        ptx::mbar_arrive_expect_tx(bar(kBarFull + rg.slot), nb * kQBoxBytes);
                        for (int j = 0; j < nb; ++j)
                            ptx::tma_load_2d(dst + j * kQBoxBytes, &qmap, (kb + j) * 64, qrow, bar(kBarFull + rg.slot));
                        rg.next(nslots);
                    }
                    prev_b = it.b;
                }
                for (int t0 = 0; ok && t0 < it.len; t0 += kTS) {
                    const int row = (int)(it.row0 + t0);
                    if constexpr (kPaged) {
#pragma unroll
                        for (int c = 0; c < kOPerS; ++c) pn[c] = paged_row(p, it.b, it.tok0 + t0 + kTS + c * kTO, last);
                    }
                    if (role == 0) {
                        if constexpr (kPaged) {
                            for (int sl = 0; sl < kSlotsPerTile; ++sl) {
                                if (!acquire()) { ok = false; break; }
                                const uint32_t dst = sbase + kOffRing + rg.slot * kSlotS;
                                ptx::mbar_arrive_expect_tx(bar(kBarFull + rg.slot), kSlotS);
#pragma unroll
                                for (int c = 0; c < kOPerS; ++c)
                                    ptx::tma_load_4d(dst + c * kPieceS, &cmap_s, 0, 0, sl * kKbPerSlot, pr[c] >> 3, bar(kBarFull + rg.slot));
                                rg.next(nslots);
                            }
                        } else {
                            constexpr int kSlotBytes = kFp8 ? kSlotS8 : kSlotS;
                            for (int sl = 0; sl < kSlotsPerTile; ++sl) {
                                if (!acquire()) { ok = false; break; }
                                const uint32_t dst = sbase + kOffRing + rg.slot * kSlotBytes;
                                ptx::mbar_arrive_expect_tx(bar(kBarFull + rg.slot), kSlotBytes);
                                ptx::tma_load_3d(dst, &cmap_s, 0, row, sl * kKbPerSlot, bar(kBarFull + rg.slot));
                                rg.next(nslots);
                            }
                        }
                    } else {
                        const int nct = (min(kTS, it.len - t0) + kTO - 1) / kTO;
                        for (int ct = 0; ct < nct; ++ct) {
                            int r = row + ct * kTO;
                            if constexpr (kPaged) r = ct == 0 ? pr[0] : (ct == 1 ? pr[1] : pr[2]);
                            if (!acquire()) { ok = false; break; }
                            const uint32_t dst = sbase + kOffRing + rg.slot * (kFp8 ? kSlotO8 : kSlotO);
                            ptx::mbar_arrive_expect_tx(bar(kBarFull + rg.slot), kFp8 ? kSlotO8 : kSlotO);
                            ptx::tma_load_3d(dst, &cmap_o, 0, r, 0, bar(kBarFull + rg.slot));
                            rg.next(nslots);
                        }
                    }
                    if constexpr (kPaged) {
#pragma unroll
                        for (int c = 0; c < kOPerS; ++c) pr[c] = pn[c];
                    }
                }
            }
            if (!ok) *abort_flag = 1;
            // drain: every issued load has been consumed (or the wait expires)
            for (int k = 0; k < nslots; ++k, rg.next(nslots))
                ptx::mbar_wait(bar(kBarEmpty + rg.slot), rg.phase ^ 1, kErrWaitEmpty);
        }
    } else if (warp == 1 || (warp == 3 && role == 0)) {
        // ------------------------------------------------------------ MMA issuers
        // S-CTA: GEMM1 is issued by two threads, lane 0 of warps 1 and 3, taking
        // alternate S tiles (and so alternate S buffers).  One thread issues an
        // N=96 MMA every ~90 cycles in this kernel, twice the MMA's tensor time;
        // two issuers keep the tensor pipe busy.  At the first tile of a sequence
        // the tile's issuer copies Q into TMEM once every GEMM1 of the previous
        // sequence (its own and the other issuer's last tile) is done, and the
        // other issuer waits for the copy before its next tile.  Both walk the
        // same items and ring positions, skipping the other's slots.
        // O-CTA: lane 0 of warp 1 issues GEMM2.
        if (lane == 0) {
            const int nslots = role == 0 ? (kFp8 ? kSlotsS8 : kSlotsS) : (kFp8 ? kSlotsO8 : kSlotsO);
            const uint32_t me = warp == 1 ? 0u : 1u;
            Ring rg;
            uint32_t jt = 0, qphase = 0, nseq = 0, qready_seq = 0;
            int prev_b = -1;
            bool ok = true;
            ItemCursor cur = items_begin<kSched>(wl, cid, ncl);
            Item it;
            int i;
            while (ok && items_next<kSched>(wl, cur, it, i)) {
                const bool new_seq = role == 0 && it.b != prev_b;
                prev_b = it.b;
                for (int t0 = 0; ok && t0 < it.len; t0 += kTS, ++jt) {
                    if (role == 0) {
                        const bool mine = (jt & 1u) == me;
                        if (new_seq && t0 == 0) {
                            ++nseq;
                            if (mine) {
                                if (jt > 0) {
                                    // An MMA is not ordered before a later tcgen05.cp: every
                                    // GEMM1 reading the old Q completes first.
                                    ptx::mma_commit(bar(kBarQFree + me));
                                    if (!ptx::mbar_spin(bar(kBarQFree + me), qphase, kErrWaitMma)) { ok = false; break; }
                                    qphase ^= 1;
                                    const uint32_t pj = jt - 1;  // the other issuer's last tile
                                    if (!ptx::mbar_spin(bar(kBarSFull + (pj & 1)), (pj >> 1) & 1, kErrWaitMma)) { ok = false; break; }
                                    ptx::tc_fence_after();
                                }
                                // Ring slots filled by TMA need no tcgen05 fence: the full
                                // barrier's complete_tx orders the loaded bytes before the
                                // copy / MMA reads them.  (A fence stalls this thread until
                                // the tensor pipe drains, ~230 cycles.)
                                for (int kb = 0; ok && kb < kKBlocks; kb += kFp8 ? 1 : 2) {
                                    if (*abort_flag || !ptx::mbar_spin(bar(kBarFull + rg.slot), rg.phase, kErrWaitFull)) { ok = false; break; }
                                    if constexpr (kFp8) {
                                        // K-block kb of the hi and lo planes: 64 B per row, 16 columns each
                                        const uint32_t slot = sbase + kOffRing + rg.slot * kSlotS8;
#pragma unroll
                                        for (int c = 0; c < 2; ++c) {
                                            ptx::tmem_cp_128x256b(tmem + kTmemQ + kb * 16 + c * 8,
                                                                  ptx::sdesc_sw64(slot + c * 32, 16, 512));
                                            ptx::tmem_cp_128x256b(tmem + kTmemQ + kTmemQLo + kb * 16 + c * 8,
                                                                  ptx::sdesc_sw64(slot + kQBox8 + c * 32, 16, 512));
                                        }
                                    } else {
                                        const uint32_t slot = sbase + kOffRing + rg.slot * kSlotS;
                                        const int nb = min(2, kKBlocks - kb);
                                        for (int j = 0; j < nb; ++j) {
#pragma unroll
                                            for (int c = 0; c < 4; ++c)
                                                ptx::tmem_cp_128x256b(tmem + kTmemQ + ((kb + j) * 4 + c) * 8,
                                                                      ptx::sdesc_sw128(slot + j * kQBoxBytes + c * 32, 16, 1024));
                                        }
                                    }
                                    ptx::mma_commit(bar(kBarEmpty + rg.slot));
                                    rg.next(nslots);
                                }
                                if (!ok) break;
                                ptx::mma_commit(bar(kBarQReady));
                                qready_seq = nseq;
                            } else {
                                for (int q = 0; q < (kFp8 ? kKBlocks : kQSlots); ++q) rg.next(nslots);
                            }
                        }
                        if (!mine) {
                            for (int sl = 0; sl < kSlotsPerTile; ++sl) rg.next(nslots);
                            continue;
                        }
                        if (qready_seq != nseq) {  // the other issuer copied this sequence's Q
                            if (!ptx::mbar_spin(bar(kBarQReady), (nseq - 1) & 1, kErrWaitMma)) { ok = false; break; }
                            qready_seq = nseq;
                        }
                        const uint32_t sb = jt & 1, use = jt >> 1;
                        if (*abort_flag || !ptx::mbar_spin(bar(kBarSEmpty + sb), (use & 1) ^ 1, kErrWaitMma)) { ok = false; break; }
                        ptx::tc_fence_after();  // the softmax's loads of this S buffer (and Q's copy) come first
                        const uint32_t d = tmem + kTmemS + sb * kTS;
                        for (int sl = 0; sl < kSlotsPerTile; ++sl) {
                            if (!ptx::mbar_spin(bar(kBarFull + rg.slot), rg.phase, kErrWaitFull)) { ok = false; break; }
                            // descriptor of the slot, plus compile-time offsets per K-step: a
                            // short issue sequence between MMAs
                            const uint32_t acc0 = sl > 0 ? 1u : 0u;
                            if constexpr (kFp8) {
                                // K-block j, K-step ks (32 e4m3): S += Q8hi.C8 + Q8lo.C8
                                const uint64_t b0 = ptx::sdesc_sw64(sbase + kOffRing + rg.slot * kSlotS8, 16, 512);
                                const uint32_t a0 = tmem + kTmemQ + sl * (kKbPerSlot * 16);
#pragma unroll
                                for (int k = 0; k < kKbPerSlot * 2; ++k) {
                                    const uint64_t bk = b0 + (uint64_t)(((k >> 1) * kBoxS8 + (k & 1) * 32) >> 4);
                                    const uint32_t ak = a0 + (k >> 1) * 16 + (k & 1) * 8;
                                    ptx::mma_ts_f8(d, ak, bk, idesc_s8(), k > 0 ? 1u : acc0);
                                    ptx::mma_ts_f8(d, ak + kTmemQLo, bk, idesc_s8(), 1u);
                                }
                            } else {
                                // (paged slots interleave the K-blocks per 8-row group: stride 3 KB)
                                const uint64_t b0 = ptx::sdesc_sw128(sbase + kOffRing + rg.slot * kSlotS, 16, kPaged ? kKbPerSlot * 1024 : 1024);
                                const uint32_t a0 = tmem + kTmemQ + sl * (kKbPerSlot * 32);
                                constexpr int kKbStride = kPaged ? 1024 : kBoxS;
#pragma unroll
                                for (int k = 0; k < kKbPerSlot * 4; ++k)
                                    ptx::mma_ts(d, a0 + k * 8, b0 + (uint64_t)(((k >> 2) * kKbStride + (k & 3) * 32) >> 4),
                                                idesc_s<kBf16>(), k > 0 ? 1u : acc0);
                            }
                            ptx::mma_commit(bar(kBarEmpty + rg.slot));
                            rg.next(nslots);
                        }
                        if (!ok) break;
                        ptx::mma_commit(bar(kBarSFull + sb));
                    } else {
                        const uint32_t ms = jt % kMsgSlots, mu = jt / kMsgSlots;
                        if (*abort_flag || !ptx::mbar_wait<true>(bar(kBarPFull + ms), mu & 1, kErrWaitPeer) ||
                            !ptx::mbar_spin(bar(kBarCorr + ms), mu & 1, kErrWaitMma)) { ok = false; break; }
                        const int nct = (min(kTS, it.len - t0) + kTO - 1) / kTO;
                        // the correction's TMEM stores to O (and fp8: the e4m3 P planes the
                        // warpgroup wrote) come first
                        ptx::tc_fence_after();
                        const uint64_t p0 = ptx::sdesc_sw64(sbase + kOffMsgO + ms * kMsgStride, 16, 512);
                        for (int ct = 0; ct < nct; ++ct) {
                            if (!ptx::mbar_spin(bar(kBarFull + rg.slot), rg.phase, kErrWaitFull)) { ok = false; break; }
                            if constexpr (kPaged) {
                                // an item's last tile ending inside a 32-row piece: the rows past
                                // its end are zeroed by the whole warp (the other lanes wait at
                                // __syncwarp meanwhile).  Items split sequences on 96-token tile
                                // boundaries, so this is a sequence's end; elsewhere it would
                                // only zero rows whose P is 0.
                                const int tail = (it.len - t0) % kTO;
                                if (ct == nct - 1 && t0 + kTS >= it.len && tail != 0) {
                                    volatile int *za = reinterpret_cast<volatile int *>(smem + kOffZArg);
                                    const uint32_t tile = sbase + kOffRing + rg.slot * kSlotO;
                                    za[0] = (int)tile;
                                    za[1] = tail;
                                    __syncwarp();
                                    zero_tail(tile, tail, 0);
                                    __syncwarp();
                                    ptx::tc_fence_after();
                                }
                            }
                            const uint32_t acc0 = (t0 > 0 || ct > 0) ? 1u : 0u;
                            if constexpr (kFp8) {
                                // O += P8hi.C8 + P8lo.C8 (K = 32 tokens); C8_N MN-major: 128-column
                                // groups 4 KB apart (LBO), 8-row groups 1 KB apart (SBO)
                                const uint64_t c0 = ptx::sdesc_sw128(sbase + kOffRing + rg.slot * kSlotO8, 4096, 1024);
                                const uint32_t pm = sbase + kOffMsgO + ms * kMsgStride + ct * 4096;
#pragma unroll
                                for (int x = 0; x < 2; ++x)
#pragma unroll
                                    for (int nh = 0; nh < 2; ++nh)
                                        ptx::mma_ss_f8(tmem + nh * 256, ptx::sdesc_sw32(pm + x * kPlaneP8, 16, 256),
                                                       c0 + (uint64_t)((nh * 2 * 4096) >> 4), idesc_o<false>(),
                                                       x > 0 ? 1u : acc0);
                            } else {
                                const uint64_t c0 = ptx::sdesc_sw128(sbase + kOffRing + rg.slot * kSlotO, kBoxO, 1024);
                                const uint64_t pa = p0 + (uint64_t)(ct * (kSubP >> 4));
#pragma unroll
                                for (int kk = 0; kk < kTO / 16; ++kk) {
#pragma unroll
                                    for (int nh = 0; nh < 2; ++nh)
                                        ptx::mma_ss(tmem + nh * 256, pa + (uint64_t)((kk * 32) >> 4),
                                                    c0 + (uint64_t)((nh * 4 * kBoxO + kk * 16 * 128) >> 4), idesc_o<kBf16>(),
                                                    kk > 0 ? 1u : acc0);
                                }
                            }
                            ptx::mma_commit(bar(kBarEmpty + rg.slot));
                            rg.next(nslots);
                        }
                        if (!ok) break;
                        ptx::mma_commit_mc(bar(kBarPFree + ms), 0x3);
                        ptx::mma_commit(bar(kBarMmaDone + ms));
                    }
                }
            }
            if (!ok) *abort_flag = 1;
            if constexpr (kPaged) {
                if (role == 1) {  // release the helper lanes (every path out of the loop gets here)
                    reinterpret_cast<volatile int *>(smem + kOffZArg)[2] = 1;
                    __syncwarp();
                }
            }
            // every MMA this thread issued has retired before TMEM is freed
            ptx::mma_commit(bar(kBarDrain + me));
            ptx::mbar_wait(bar(kBarDrain + me), 0, kErrWaitMma);
        } else if (kPaged && role == 1) {
            // O-CTA, paged: lanes 1-31 of the GEMM2 warp.  Rows of a sequence's
            // last C tile past its end hold whatever the page held, not
            // necessarily finite numbers; P is 0 there, but 0 x NaN is NaN in
            // GEMM2.  The issuing lane posts such a tile (landed) and these lanes
            // zero its tail with it.  Between requests they wait inside
            // __syncwarp, issuing nothing.
            volatile int *za = reinterpret_cast<volatile int *>(smem + kOffZArg);
            for (;;) {
                __syncwarp();
                if (za[2] != 0) break;
                zero_tail((uint32_t)za[0], za[1], lane);
                __syncwarp();
            }
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ math warpgroup
        const int h = tid - 128;                              // head row = TMEM lane
        const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t trow = tmem + lane_addr;
        uint32_t jt = 0;
        bool ok = true;
        if (role == 0) {
            // ------------------------------------------------ S-CTA: softmax
            const uint32_t peer_pfull0 = ptx::mapa(bar(kBarPFull), 1);
            const uint32_t peer_msg0 = ptx::mapa(sbase + kOffMsgO, 1);
            // fp8: P leaves as fp16 q = K * w, the O-CTA splits it into e4m3 planes.
            // Per-tensor scale: w = p, K = kP8Scale.  Per-row scales s_t = 2^(e_t) *
            // f_t (f_t in [1, 2)): the exponent joins the logit in the online softmax
            // (y_t = z_t + e_t, so w_t = 2^(y_t - m) <= 2^3 whatever s_t) and the
            // weight is w_t * f_t with K = kP8ScaleRows; the row sum adds w_t *
            // 2^-e_t = p_t.  Either way q <= 256 < 448.  K enters through the
            // exponent (2^(y - m + log2 K)), so the row sum is K times the true one:
            // K cancels in O = sum(q c) / sum, and the LSE subtracts log2 K.
            constexpr bool rows_scaled = kFp8 && kRows;
            const float p8log2k = rows_scaled ? kP8Log2ScaleRows : kP8Log2Scale;
            ItemCursor cur = items_begin<kSched>(wl, cid, ncl);
            Item it;
            int i;
            while (ok && items_next<kSched>(wl, cur, it, i)) {
                float m_used = -INFINITY, l_run = 0.f;
                // fp8: this row's Q* scale joins the softmax scale
                float sl2 = p.scale_log2;
                if constexpr (kFp8) {
                    if (h < p.num_heads) sl2 *= p.q_scale[(size_t)it.b * p.num_heads + h];
                }
                // multi-token: this row's causal limit, as a token offset within the item
                int lim = 0;
                if constexpr (kMtp) {
                    const int mk = p.mtp >> 16, mnh = p.mtp & 0xFFFF;
                    const int tok = min(h / mnh, mk - 1);
                    const int slen = wl.cu_seqlens != nullptr ? wl.cu_seqlens[it.b + 1] - wl.cu_seqlens[it.b]
                                                              : wl.seq_len;
                    lim = slen - (mk - 1 - tok) - it.tok0;
                }
                for (int t0 = 0; t0 < it.len; t0 += kTS, ++jt) {
                    const uint32_t sb = jt & 1, use = jt >> 1;
                    const uint32_t ms = jt % kMsgSlots, mu = jt / kMsgSlots;
                    // Every decision below is made uniform across the warpgroup by the
                    // bar.red at the end of the tile, so an expired wait can never split
                    // a warp at a .sync.aligned tcgen05 op or strand a named barrier.
                    bool w = !*abort_flag && ptx::mbar_wait(bar(kBarSFull + sb), use & 1, kErrWaitMma);
                    w = __all_sync(0xffffffffu, w);
                    float alpha = 1.f;
                    const bool last = t0 + kTS >= it.len;
                    uint32_t pk[kTS / 2];
                    if (w) {
                        ptx::tc_fence_after();
                        uint32_t r[kTS];
                        {
                            uint32_t a[32], b[32], c[32];
                            ptx::tmem_ld_x32(trow + kTmemS + sb * kTS, a);
                            ptx::tmem_ld_x32(trow + kTmemS + sb * kTS + 32, b);
                            ptx::tmem_ld_x32(trow + kTmemS + sb * kTS + 64, c);
                            ptx::tmem_wait_ld();
#pragma unroll
                            for (int k = 0; k < 32; ++k) { r[k] = a[k]; r[32 + k] = b[k]; r[64 + k] = c[k]; }
                        }
                        ptx::tc_fence_before();
                        ptx::mbar_arrive(bar(kBarSEmpty + sb));
                        // fp8, per-row scales: r becomes y = sl2 * s * (Q8 . C8) + e (the log2
                        // domain, sl2 applied here), the tail masked below
                        const float *kvs = nullptr;
                        if constexpr (kFp8) {
                            if constexpr (rows_scaled) {
                                kvs = p.kv_scales + it.row0 + t0;
                                const int nv = min(kTS, it.len - t0);
#pragma unroll
                                for (int k = 0; k < kTS; ++k) {
                                    if (k < nv) {
                                        const float sc = __ldg(kvs + k);
                                        r[k] = u32_of(fmaf(f32_of(r[k]) * sc, sl2, (float)scale_exp(sc)));
                                    }
                                }
                            }
                        }

                        // Row max of the raw logits (scale > 0 commutes with max), with
                        // masked tail columns at -inf; 8 independent chains.
                        // (multi-token: per row; a row may see none of a tile)
                        const int valid = kMtp ? max(0, min(min(kTS, it.len - t0), lim - t0)) : min(kTS, it.len - t0);
                        if (valid < kTS) {
#pragma unroll
                            for (int k = 0; k < kTS; ++k)
                                if (k >= valid) r[k] = u32_of(-INFINITY);
                        }
                        float m8[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) m8[j] = f32_of(r[j]);
#pragma unroll
                        for (int k = 8; k < kTS; ++k) m8[k & 7] = fmaxf(m8[k & 7], f32_of(r[k]));
                        const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                                               fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * (rows_scaled ? 1.f : sl2);
                        if (mx > m_used + (kFp8 ? (rows_scaled ? kRescaleLog2Fp8Rows : kRescaleLog2Fp8) : kRescaleLog2)) {
                            alpha = (m_used == -INFINITY) ? 0.f : ptx::ex2(m_used - mx);
                            m_used = mx;
                        }
                        // p = 2^(s * scale_log2 - m_used): one FFMA + one EX2 per logit.
                        // (a row that has seen nothing yet keeps m_used = -inf: its p are 0)
                        const float neg_m = (kMtp && m_used == -INFINITY) ? 0.f : -m_used;
                        float s4[4] = {0.f, 0.f, 0.f, 0.f};
                        if constexpr (kFp8) {
                            // the per-row branch outside the unrolled loops (two copies)
                            const float nmk = neg_m + p8log2k;
                            if constexpr (rows_scaled) {
#pragma unroll
                                for (int k = 0; k < kTS; k += 2) {
                                    const float p0 = ptx::ex2(f32_of(r[k]) + nmk);
                                    const float p1 = ptx::ex2(f32_of(r[k + 1]) + nmk);
                                    // row sum of w * 2^-e; GEMM2 weight w * mantissa
                                    const float sc0 = k < valid ? __ldg(kvs + k) : 1.f;
                                    const float sc1 = k + 1 < valid ? __ldg(kvs + k + 1) : 1.f;
                                    s4[(k >> 1) & 3] += p0 * scale_pow2_inv(sc0) + p1 * scale_pow2_inv(sc1);
                                    pk[k >> 1] = pack2<false>(p0 * scale_mant(sc0), p1 * scale_mant(sc1));
                                }
                            } else {
#pragma unroll
                                for (int k = 0; k < kTS; k += 2) {
                                    const float p0 = ptx::ex2(fmaf(f32_of(r[k]), sl2, nmk));
                                    const float p1 = ptx::ex2(fmaf(f32_of(r[k + 1]), sl2, nmk));
                                    s4[(k >> 1) & 3] += p0 + p1;
                                    pk[k >> 1] = pack2<false>(p0, p1);
                                }
                            }
                        } else {
#pragma unroll
                            for (int k = 0; k < kTS; k += 2) {
                                const float p0 = ptx::ex2(fmaf(f32_of(r[k]), sl2, neg_m));
                                const float p1 = ptx::ex2(fmaf(f32_of(r[k + 1]), sl2, neg_m));
                                s4[(k >> 1) & 3] += p0 + p1;
                                pk[k >> 1] = pack2<kBf16>(p0, p1);
                            }
                        }
                        l_run = l_run * alpha + ((s4[0] + s4[1]) + (s4[2] + s4[3]));
                        // the peer's message slot is free once GEMM2 of S tile jt-3 finished
                        w = ptx::mbar_wait<true>(bar(kBarPFree + ms), (mu & 1) ^ 1, kErrWaitPeer);
                    }
                    // the previous tile's outgoing copy has finished reading the staging buffer
                    if (h == 0) ptx::bulk_wait_group_read<0>();
                    ptx::named_barrier(1, 128);
                    if (w) {
                        uint8_t *msg = smem + kOffStgS;
#pragma unroll
                        for (int st = 0; st < kOPerS; ++st) {
                            uint4 *prow = reinterpret_cast<uint4 *>(msg + st * kSubP + h * 64);  // SW64
#pragma unroll
                            for (int c4 = 0; c4 < 4; ++c4) {
                                const int q = st * 16 + c4 * 4;
                                prow[c4 ^ ((h >> 1) & 3)] = make_uint4(pk[q], pk[q + 1], pk[q + 2], pk[q + 3]);
                            }
                        }
                        reinterpret_cast<float *>(msg + kMsgAlpha)[h] = alpha;
                        if (last) {
                            reinterpret_cast<float *>(msg + kMsgL)[h] = l_run;
                            reinterpret_cast<float *>(msg + kMsgM)[h] = m_used;
                        }
                        ptx::fence_proxy_async_smem();
                    }
                    if (!ptx::named_barrier_and(1, 128, w)) { ok = false; break; }
                    if (h == 0) {
                        const uint32_t rbar = peer_pfull0 + 8u * ms;
                        ptx::mbar_remote_arrive_expect_tx(rbar, kMsgBytes);
                        ptx::bulk_copy_s2cluster(peer_msg0 + ms * kMsgStride, sbase + kOffStgS,
                                                 kMsgBytes, rbar);
                        ptx::bulk_commit_group();
                    }
                }
            }
            if (!ok) *abort_flag = 1;
            // The last messages were consumed by the peer's GEMM2 (so no remote
            // arrival is still in flight towards this CTA).
            for (uint32_t k = (jt >= (uint32_t)kMsgSlots ? jt - kMsgSlots : 0); k < jt; ++k)
                ptx::mbar_wait<true>(bar(kBarPFree + (k % kMsgSlots)), (k / kMsgSlots) & 1, kErrWaitPeer);
            if (h == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        } else {
            // ------------------------------------------------ O-CTA: correction + epilogue
            // GEMM2 of message x completes phase x / 3 of kBarMmaDone[x % 3].  The
            // warpgroup waits on it only to rescale or finish O; a parity wait is
            // unambiguous because the barrier is within one phase of the waited one:
            // message x+1 arrived only after GEMM2 x-2 finished (its slot was free),
            // and GEMM2 x+3 cannot start before this warpgroup releases it.
            auto gemm2_done = [&](uint32_t x) -> bool {
                return ptx::mbar_wait(bar(kBarMmaDone + x % kMsgSlots), (x / kMsgSlots) & 1, kErrWaitMma);
            };
            // fp8: O = (P8 . C8) * o_scale / l, o_scale = kv_scale per tensor, 1 with
            // per-row scales (host); the weights' factor K is in l as well, and the
            // LSE subtracts log2 K
            constexpr bool rows_scaled = kFp8 && kRows;
            constexpr float lse_k = rows_scaled ? kP8Log2ScaleRows : kP8Log2Scale;
            ItemCursor cur = items_begin<kSched>(wl, cid, ncl);
            Item it;
            int i;
            while (ok && items_next<kSched>(wl, cur, it, i)) {
                for (int t0 = 0; t0 < it.len; t0 += kTS, ++jt) {
                    const uint32_t ms = jt % kMsgSlots, mu = jt / kMsgSlots;
                    // As in the S-CTA, every branch is warpgroup-uniform (bar.red).
                    bool w = !*abort_flag && ptx::mbar_wait<true>(bar(kBarPFull + ms), mu & 1, kErrWaitPeer);
                    if (!ptx::named_barrier_and(2, 128, w)) { ok = false; break; }
                    const uint8_t *msg = smem + kOffMsgO + ms * kMsgStride;
                    if constexpr (kFp8) {
                        // P (fp16) -> e4m3 hi / lo planes in place, before Corr releases GEMM2.
                        // (A message slot is rewritten only after its GEMM2 finished: the
                        // S-CTA sends message x+3 after GEMM2 x freed the slot.)
                        P8Row pr;
                        p8_read(msg, h, pr);
                        ptx::named_barrier(2, 128);
                        if constexpr (rows_scaled) p8_write<true>(const_cast<uint8_t *>(msg), h, pr);
                        else p8_write<false>(const_cast<uint8_t *>(msg), h, pr);
                        ptx::fence_proxy_async_smem();
                    }
                    const float alpha = reinterpret_cast<const float *>(msg + kMsgAlpha)[h];
                    const bool last = t0 + kTS >= it.len;
                    float l_fin = 0.f, m_fin = 0.f;
                    if (last) {
                        l_fin = reinterpret_cast<const float *>(msg + kMsgL)[h];
                        m_fin = reinterpret_cast<const float *>(msg + kMsgM)[h];
                    }
                    if (t0 > 0 && ptx::named_barrier_or(2, 128, alpha != 1.f)) {
                        w = gemm2_done(jt - 1);
                        if (!ptx::named_barrier_and(2, 128, w)) { ok = false; break; }
                        ptx::tc_fence_after();
#pragma unroll 1
                        for (int c = 0; c < kDV / 32; ++c) {
                            uint32_t r[32];
                            ptx::tmem_ld_x32(trow + c * 32, r);
                            ptx::tmem_wait_ld();
#pragma unroll
                            for (int k = 0; k < 32; ++k) r[k] = u32_of(f32_of(r[k]) * alpha);
                            ptx::tmem_st_x32(trow + c * 32, r);
                        }
                        ptx::tmem_wait_st();
                    }
                    ptx::tc_fence_before();
                    ptx::mbar_arrive(bar(kBarCorr + ms));
                    if (last) {
                        w = gemm2_done(jt);
                        if (!ptx::named_barrier_and(2, 128, w)) { ok = false; break; }
                        ptx::tc_fence_after();
                        // A sequence covered by this one item gets its final output here;
                        // otherwise the item's partial goes to the workspace for the combine.
                        int ni0, ni1;
                        item_range<kSched>(wl, it.b, ni0, ni1);
                        const bool single = ni1 - ni0 == 1;
                        float inv_l = l_fin > 0.f ? 1.f / l_fin : 0.f;
                        if constexpr (kFp8) inv_l *= p.o_scale;
                        float lse = l_fin > 0.f ? (m_fin + __log2f(l_fin)) * kLn2 : -INFINITY;
                        if constexpr (kFp8) lse -= lse_k * kLn2;
                        // 16-bit output: fp16 from fp16 inputs, bf16 from bf16 inputs
                        const bool f16 = (single ? p.out_kind : p.part_kind) != kOutF32;
                        const size_t row_bytes = (size_t)kDV * (f16 ? 2 : 4);
                        uint8_t *dst = single ? static_cast<uint8_t *>(p.out) + (size_t)it.b * p.num_heads * row_bytes
                                              : static_cast<uint8_t *>(p.part_o) + (size_t)i * p.num_heads * row_bytes;
                        // Each pass moves a 128-byte segment of every row (64 fp16 or 32 fp32
                        // columns) through a per-warp swizzled 32-row staging tile, so that
                        // each store instruction covers 4 rows x 128 contiguous bytes.  (One
                        // SM writes global memory at ~45 GB/s whatever the pattern or the
                        // store path -- TMA stores measured slower -- so a 128 KB partial
                        // needs ~3 us; the stores are issued at once and drain meanwhile.)
                        const uint32_t stg = sbase + kOffEpi + (warp & 3) * kEpiWarpBytes;
                        const uint32_t srow = stg + lane * 128;
                        const int row0 = (warp & 3) * 32;  // first head of this warp
                        const int rr = lane >> 3, qq = lane & 7;
                        const int passes = f16 ? kDV / 64 : kDV / 32;
#pragma unroll 1
                        for (int c = 0; c < passes; ++c) {
                            uint32_t wv[32];
                            if (f16) {
                                uint32_t a[32], b[32];
                                ptx::tmem_ld_x32(trow + c * 64, a);
                                ptx::tmem_ld_x32(trow + c * 64 + 32, b);
                                ptx::tmem_wait_ld();
#pragma unroll
                                for (int j = 0; j < 16; ++j) {
                                    wv[j] = pack2<kBf16>(f32_of(a[2 * j]) * inv_l, f32_of(a[2 * j + 1]) * inv_l);
                                    wv[16 + j] = pack2<kBf16>(f32_of(b[2 * j]) * inv_l, f32_of(b[2 * j + 1]) * inv_l);
                                }
                            } else {
                                ptx::tmem_ld_x32(trow + c * 32, wv);
                                ptx::tmem_wait_ld();
#pragma unroll
                                for (int j = 0; j < 32; ++j) wv[j] = u32_of(f32_of(wv[j]) * inv_l);
                            }
                            __syncwarp();  // the previous pass has read the staging tile
#pragma unroll
                            for (int q = 0; q < 8; ++q)
                                ptx::st_shared_v4(srow + ((q ^ (lane & 7)) << 4), wv[4 * q], wv[4 * q + 1],
                                                  wv[4 * q + 2], wv[4 * q + 3]);
                            __syncwarp();
                            uint4 v[8];
#pragma unroll
                            for (int k = 0; k < 8; ++k) {
                                const int lr = 4 * k + rr;  // row within the warp
                                v[k] = ptx::ld_shared_v4(stg + lr * 128 + ((qq ^ (lr & 7)) << 4));
                            }
#pragma unroll
                            for (int k = 0; k < 8; ++k) {
                                const int head = row0 + 4 * k + rr;
                                if (head < p.num_heads)
                                    *reinterpret_cast<uint4 *>(dst + head * row_bytes + c * 128 + qq * 16) = v[k];
                            }
                        }
                        if (h < p.num_heads) {
                            if (single) {
                                if (p.out_lse != nullptr) p.out_lse[(size_t)it.b * p.num_heads + h] = lse;
                            } else {
                                p.part_lse[(size_t)i * p.num_heads + h] = lse;
                            }
                        }
                        ptx::tc_fence_before();
                    }
                }
            }
            if (!ok) *abort_flag = 1;
        }
    }

    // ---------------------------------------------------------------- teardown
    // (lane 0 of the producer and MMA warps arrives after its role loop: the
    // warp reconverges before the CTA and cluster barriers, which are .aligned)
    ptx::tc_fence_before();
    __syncwarp();
    __syncthreads();
    ptx::cluster_sync();  // neither CTA leaves while its partner may still target it
    if (warp == 2) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, kTmemCols);
    }
    if (tid == 0 && p.span != nullptr) {
        atomicMin(p.span, t_start);
        atomicMax(p.span + 1, (unsigned long long)globaltimer_ns());
    }
}

}  // namespace tc
}  // namespace mla
