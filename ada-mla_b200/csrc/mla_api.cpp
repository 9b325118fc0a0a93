// mla_api.cpp -- PyTorch extension boundary, mirroring the reference's
// csrc/mla_api.cpp (PYBIND11_MODULE(ada_mla), :115-120): the same three names
// with the same (query, cache) -> Tensor signatures, output shapes and dtypes,
// plus the batched/varlen entry point and the LSE merge used by the
// multi-GPU layer.  Every function validates device / dtype / contiguity /
// shape, allocates outputs and workspace from the caching allocator, and calls
// the C ABI (include/mla_b200.h) on the current torch stream; a non-zero status
// raises.  No torch types cross the C ABI.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "mla_b200.h"

namespace {

void check_status(int st, const char *what) {
    if (st == MLA_B200_ERR_CUDA) {
        const auto e = static_cast<cudaError_t>(mla_b200_last_cuda_error());
        TORCH_CHECK(false, what, " failed: ", mla_b200_status_string(st), " (status ", st, ", ",
                    cudaGetErrorName(e), ")");
    }
    TORCH_CHECK(st == MLA_B200_OK, what, " failed: ", mla_b200_status_string(st), " (status ", st,
                ")");
}

void check_cuda(const at::Tensor &t, const char *name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

void *stream_ptr() { return static_cast<void *>(at::cuda::getCurrentCUDAStream().stream()); }

at::Tensor workspace(const at::Tensor &like, size_t bytes) {
    return at::empty({(int64_t)std::max<size_t>(bytes, 256)},
                     at::TensorOptions().device(like.device()).dtype(at::kByte));
}

}  // namespace

// Reference: mla_decode_naive (csrc/mla_api.cpp:5-32).  fp32, scale
// 1/sqrt(head_dim_c), returns all head_dim_c columns: [n_h, head_dim_c].
at::Tensor mla_decode_naive(const at::Tensor &query, const at::Tensor &cache) {
    check_cuda(query, "query");
    check_cuda(cache, "cache");
    TORCH_CHECK(query.scalar_type() == at::kFloat && cache.scalar_type() == at::kFloat,
                "mla_decode_naive: query and cache must be float32");
    TORCH_CHECK(query.dim() == 2 && cache.dim() == 2 && query.size(1) == cache.size(1),
                "mla_decode_naive: expected query [n_h, D] and cache [N, D]");
    TORCH_CHECK(cache.size(0) > 0, "mla_decode_naive: empty cache");
    TORCH_CHECK(query.device() == cache.device(), "query and cache on different devices");
    c10::cuda::CUDAGuard g(query.device());
    const int64_t nh = query.size(0), d = query.size(1), n = cache.size(0);
    at::Tensor out = at::empty({nh, d}, query.options());
    at::Tensor attn = at::empty({nh, n}, query.options());
    check_status(mla_b200_decode_naive_f32(query.data_ptr<float>(), cache.data_ptr<float>(),
                                           attn.data_ptr<float>(), out.data_ptr<float>(), (int)nh,
                                           (int)d, (int)n, stream_ptr()),
                 "mla_decode_naive");
    return out;
}

static at::Tensor fused_f32(const at::Tensor &query, const at::Tensor &cache) {
    const int64_t nh = query.size(0), n = cache.size(0);
    at::Tensor out = at::empty({nh, MLA_B200_HEAD_DIM_V}, query.options());
    const size_t ws = mla_b200_workspace_size(1, (int)nh, n, (int)n, 0);
    at::Tensor w = workspace(query, ws);
    check_status(mla_b200_decode_fused_f32(query.data_ptr<float>(), cache.data_ptr<float>(),
                                           out.data_ptr<float>(), (int)nh,
                                           (int)query.size(1), (int)n, w.data_ptr(), w.numel(),
                                           stream_ptr()),
                 "mla_decode_fused");
    return out;
}

static void check_decode_inputs(const at::Tensor &query, const at::Tensor &cache, const char *fn) {
    check_cuda(query, "query");
    check_cuda(cache, "cache");
    TORCH_CHECK(query.device() == cache.device(), fn, ": query and cache on different devices");
    TORCH_CHECK(query.dim() == 2 && query.size(1) == MLA_B200_HEAD_DIM_K, fn,
                ": query must be [n_h, 576]");
    TORCH_CHECK(cache.dim() == 2 && cache.size(1) == MLA_B200_HEAD_DIM_K, fn,
                ": cache must be [N, 576]");
    TORCH_CHECK(query.scalar_type() == cache.scalar_type(), fn,
                ": query and cache must have the same dtype");
}

// Reference: mla_decode_fused (csrc/mla_api.cpp:34-54).  fp32 in, fp32
// [n_h, 512] out, scale 1/sqrt(192).
at::Tensor mla_decode_fused(const at::Tensor &query, const at::Tensor &cache) {
    check_decode_inputs(query, cache, "mla_decode_fused");
    TORCH_CHECK(query.scalar_type() == at::kFloat, "mla_decode_fused: float32 inputs expected");
    c10::cuda::CUDAGuard g(query.device());
    return fused_f32(query, cache);
}

// Reference: mla_decode_split (csrc/mla_api.cpp:86-113).  fp16 -> the split-KV
// decode, [n_h, 512] fp16; fp32 -> the fp32 kernel (the reference's fp32
// specialization is an empty stub, csrc/mla_decode_splitk_fwd_sm89.cu:9-24).
// num_splits <= 0 selects the heuristic (the reference hard-codes 4).
at::Tensor mla_decode_split(const at::Tensor &query, const at::Tensor &cache, int64_t num_splits) {
    check_decode_inputs(query, cache, "mla_decode_split");
    c10::cuda::CUDAGuard g(query.device());
    if (query.scalar_type() == at::kFloat) return fused_f32(query, cache);
    TORCH_CHECK(query.scalar_type() == at::kHalf,
                "mla_decode_split: float16 or float32 inputs expected");
    const int64_t nh = query.size(0), n = cache.size(0);
    at::Tensor out = at::empty({nh, MLA_B200_HEAD_DIM_V}, query.options());
    const size_t ws = mla_b200_workspace_size(1, (int)nh, n, (int)n, (int)num_splits);
    at::Tensor w = workspace(query, ws);
    check_status(mla_b200_decode_split_f16(query.data_ptr(), cache.data_ptr(), out.data_ptr(),
                                           (int)nh, (int)n, (int)num_splits, w.data_ptr(),
                                           w.numel(), stream_ptr()),
                 "mla_decode_split");
    return out;
}

// Batched / varlen decode (no reference counterpart).
//   query [B, n_h, 576] fp16 or bf16 (cache the same dtype); cache [B, N, 576]
//   (dense) or [T, 576] with cu_seqlens int32 [B+1] on the same device (packed).
// Returns (out [B, n_h, 512] in the input dtype, or fp32 when out_fp32,
// lse [B, n_h] fp32 or empty).
std::vector<at::Tensor> mla_decode_batched(const at::Tensor &query, const at::Tensor &cache,
                                           const c10::optional<at::Tensor> &cu_seqlens,
                                           int64_t max_seq_len, double softmax_scale,
                                           int64_t num_splits, bool return_lse,
                                           bool out_fp32, double kv_scale) {
    check_cuda(query, "query");
    check_cuda(cache, "cache");
    TORCH_CHECK(query.device() == cache.device(), "query and cache on different devices");
    const bool bf16 = query.scalar_type() == at::kBFloat16;
    const bool fp8 = cache.scalar_type() == at::kFloat8_e4m3fn;
    TORCH_CHECK((query.scalar_type() == at::kHalf || bf16) &&
                    (cache.scalar_type() == query.scalar_type() || (fp8 && !bf16)),
                "mla_decode_batched: float16 or bfloat16 inputs (query and cache alike), or a "
                "float16 query with a float8_e4m3fn cache, expected");
    TORCH_CHECK(query.dim() == 3 && query.size(2) == MLA_B200_HEAD_DIM_K,
                "mla_decode_batched: query must be [B, n_h, 576]");
    const int64_t b = query.size(0), nh = query.size(1);
    c10::cuda::CUDAGuard g(query.device());
    const int32_t *cu_ptr = nullptr;
    int64_t total = 0;
    if (cu_seqlens.has_value() && cu_seqlens->defined()) {
        const at::Tensor &cu = *cu_seqlens;
        check_cuda(cu, "cu_seqlens");
        TORCH_CHECK(cu.device() == query.device(), "cu_seqlens on a different device");
        TORCH_CHECK(cu.scalar_type() == at::kInt && cu.dim() == 1 && cu.size(0) == b + 1,
                    "cu_seqlens must be int32 [B+1]");
        TORCH_CHECK(cache.dim() == 2 && cache.size(1) == MLA_B200_HEAD_DIM_K,
                    "packed cache must be [T, 576]");
        total = cache.size(0);
        if (max_seq_len < 0) {
            max_seq_len = b > 0 ? (cu.slice(0, 1) - cu.slice(0, 0, b)).max().item<int64_t>() : 0;
        }
        cu_ptr = cu.data_ptr<int32_t>();
    } else {
        TORCH_CHECK(cache.dim() == 3 && cache.size(0) == b && cache.size(2) == MLA_B200_HEAD_DIM_K,
                    "dense cache must be [B, N, 576]");
        max_seq_len = cache.size(1);
        total = b * max_seq_len;
    }
    at::Tensor out = at::empty({b, nh, MLA_B200_HEAD_DIM_V},
                               query.options().dtype(out_fp32 ? at::kFloat
                                                              : query.scalar_type()));
    at::Tensor lse = return_lse ? at::empty({b, nh}, query.options().dtype(at::kFloat))
                                : at::Tensor();
    const size_t ws = (fp8 ? mla_b200_workspace_size_fp8 : mla_b200_workspace_size)(
        (int)b, (int)nh, total, (int)max_seq_len, (int)num_splits);
    at::Tensor w = workspace(query, ws);
    const int odt = out_fp32 ? MLA_B200_OUT_F32 : (bf16 ? MLA_B200_OUT_BF16 : MLA_B200_OUT_F16);
    float *lse_ptr = return_lse ? lse.data_ptr<float>() : nullptr;
    if (fp8) {
        check_status(mla_b200_decode_batched_fp8(
                         query.data_ptr(), cache.data_ptr(), (float)kv_scale, cu_ptr, (int)b, (int)nh,
                         total, (int)max_seq_len, (float)softmax_scale, (int)num_splits,
                         out.data_ptr(), odt, lse_ptr, w.data_ptr(), w.numel(), stream_ptr()),
                     "mla_decode_batched");
    } else {
        auto *fn = bf16 ? mla_b200_decode_batched_bf16 : mla_b200_decode_batched_f16;
        check_status(fn(query.data_ptr(), cache.data_ptr(), cu_ptr, (int)b, (int)nh, total,
                        (int)max_seq_len, (float)softmax_scale, (int)num_splits, out.data_ptr(), odt,
                        lse_ptr, w.data_ptr(), w.numel(), stream_ptr()),
                     "mla_decode_batched");
    }
    if (!return_lse) lse = at::empty({0}, query.options().dtype(at::kFloat));
    return {out, lse};
}

// Multi-token decode (no reference counterpart).
//   query [B, k, n_h, 576] fp16 or bf16 (n_h <= 128), cache as in
//   mla_decode_batched (same dtype); draft token i of sequence b sees its first
//   len_b - (k - 1 - i) tokens.  Returns (out [B, k, n_h, 512], lse [B, k, n_h] or empty).
std::vector<at::Tensor> mla_decode_mtp(const at::Tensor &query, const at::Tensor &cache,
                                       const c10::optional<at::Tensor> &cu_seqlens,
                                       int64_t max_seq_len, double softmax_scale,
                                       int64_t num_splits, bool return_lse, bool out_fp32) {
    check_cuda(query, "query");
    check_cuda(cache, "cache");
    TORCH_CHECK(query.device() == cache.device(), "query and cache on different devices");
    const bool bf16 = query.scalar_type() == at::kBFloat16;
    TORCH_CHECK((query.scalar_type() == at::kHalf || bf16) && cache.scalar_type() == query.scalar_type(),
                "mla_decode_mtp: float16 or bfloat16 inputs (query and cache alike) expected");
    TORCH_CHECK(query.dim() == 4 && query.size(3) == MLA_B200_HEAD_DIM_K,
                "mla_decode_mtp: query must be [B, k, n_h, 576]");
    const int64_t b = query.size(0), k = query.size(1), nh = query.size(2);
    c10::cuda::CUDAGuard g(query.device());
    const int32_t *cu_ptr = nullptr;
    int64_t total = 0;
    if (cu_seqlens.has_value() && cu_seqlens->defined()) {
        const at::Tensor &cu = *cu_seqlens;
        check_cuda(cu, "cu_seqlens");
        TORCH_CHECK(cu.device() == query.device(), "cu_seqlens on a different device");
        TORCH_CHECK(cu.scalar_type() == at::kInt && cu.dim() == 1 && cu.size(0) == b + 1,
                    "cu_seqlens must be int32 [B+1]");
        TORCH_CHECK(cache.dim() == 2 && cache.size(1) == MLA_B200_HEAD_DIM_K,
                    "packed cache must be [T, 576]");
        total = cache.size(0);
        if (max_seq_len < 0)
            max_seq_len = b > 0 ? (cu.slice(0, 1) - cu.slice(0, 0, b)).max().item<int64_t>() : 0;
        cu_ptr = cu.data_ptr<int32_t>();
    } else {
        TORCH_CHECK(cache.dim() == 3 && cache.size(0) == b && cache.size(2) == MLA_B200_HEAD_DIM_K,
                    "dense cache must be [B, N, 576]");
        max_seq_len = cache.size(1);
        total = b * max_seq_len;
    }
    at::Tensor out = at::empty({b, k, nh, MLA_B200_HEAD_DIM_V},
                               query.options().dtype(out_fp32 ? at::kFloat : query.scalar_type()));
    at::Tensor lse = return_lse ? at::empty({b, k, nh}, query.options().dtype(at::kFloat)) : at::Tensor();
    const size_t ws = mla_b200_workspace_size_mtp((int)b, (int)k, (int)nh, total, (int)max_seq_len,
                                                  (int)num_splits);
    at::Tensor w = workspace(query, ws);
    auto *fn = bf16 ? mla_b200_decode_mtp_bf16 : mla_b200_decode_mtp_f16;
    const int odt = out_fp32 ? MLA_B200_OUT_F32 : (bf16 ? MLA_B200_OUT_BF16 : MLA_B200_OUT_F16);
    check_status(fn(query.data_ptr(), cache.data_ptr(), cu_ptr, (int)b, (int)k, (int)nh, total,
                    (int)max_seq_len, (float)softmax_scale, (int)num_splits, out.data_ptr(), odt,
                    return_lse ? lse.data_ptr<float>() : nullptr, w.data_ptr(), w.numel(),
                    stream_ptr()),
                 "mla_decode_mtp");
    if (!return_lse) lse = at::empty({0}, query.options().dtype(at::kFloat));
    return {out, lse};
}

// Paged decode (no reference counterpart).
//   query [B, n_h, 576] fp16 or bf16; kv_pages [num_pages, page_size, 576] in the
//   same dtype; block_table int32 [B, max_blocks]; seq_lens int32 [B]; all on
//   one device.  max_seq_len < 0 reads max(seq_lens) from the device.
// Returns (out [B, n_h, 512] in the input dtype or fp32, lse [B, n_h] fp32 or empty).
std::vector<at::Tensor> mla_decode_paged(const at::Tensor &query, const at::Tensor &kv_pages,
                                         const at::Tensor &block_table, const at::Tensor &seq_lens,
                                         int64_t max_seq_len, double softmax_scale,
                                         int64_t num_splits, bool return_lse, bool out_fp32) {
    check_cuda(query, "query");
    check_cuda(kv_pages, "kv_pages");
    check_cuda(block_table, "block_table");
    check_cuda(seq_lens, "seq_lens");
    TORCH_CHECK(query.device() == kv_pages.device() && query.device() == block_table.device() &&
                    query.device() == seq_lens.device(),
                "mla_decode_paged: all tensors on one device");
    const bool bf16 = query.scalar_type() == at::kBFloat16;
    TORCH_CHECK((query.scalar_type() == at::kHalf || bf16) &&
                    kv_pages.scalar_type() == query.scalar_type(),
                "mla_decode_paged: float16 or bfloat16 inputs (query and kv_pages alike) expected");
    TORCH_CHECK(query.dim() == 3 && query.size(2) == MLA_B200_HEAD_DIM_K,
                "mla_decode_paged: query must be [B, n_h, 576]");
    TORCH_CHECK(kv_pages.dim() == 3 && kv_pages.size(2) == MLA_B200_HEAD_DIM_K,
                "mla_decode_paged: kv_pages must be [num_pages, page_size, 576]");
    const int64_t b = query.size(0), nh = query.size(1);
    TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.dim() == 2 &&
                    block_table.size(0) == b,
                "mla_decode_paged: block_table must be int32 [B, max_blocks]");
    TORCH_CHECK(seq_lens.scalar_type() == at::kInt && seq_lens.dim() == 1 && seq_lens.size(0) == b,
                "mla_decode_paged: seq_lens must be int32 [B]");
    c10::cuda::CUDAGuard g(query.device());
    const int64_t num_pages = kv_pages.size(0), page_size = kv_pages.size(1);
    const int64_t max_blocks = block_table.size(1);
    if (max_seq_len < 0) max_seq_len = b > 0 ? seq_lens.max().item<int64_t>() : 0;
    at::Tensor out = at::empty({b, nh, MLA_B200_HEAD_DIM_V},
                               query.options().dtype(out_fp32 ? at::kFloat
                                                              : query.scalar_type()));
    at::Tensor lse = return_lse ? at::empty({b, nh}, query.options().dtype(at::kFloat))
                                : at::Tensor();
    const size_t ws = mla_b200_workspace_size((int)b, (int)nh, b * max_seq_len, (int)max_seq_len,
                                              (int)num_splits);
    at::Tensor w = workspace(query, ws);
    auto *fn = bf16 ? mla_b200_decode_paged_bf16 : mla_b200_decode_paged_f16;
    const int odt = out_fp32 ? MLA_B200_OUT_F32 : (bf16 ? MLA_B200_OUT_BF16 : MLA_B200_OUT_F16);
    check_status(fn(query.data_ptr(), kv_pages.data_ptr(), block_table.data_ptr<int32_t>(),
                    seq_lens.data_ptr<int32_t>(), (int)b, (int)nh, (int)num_pages, (int)page_size,
                    (int)max_blocks, (int)max_seq_len, (float)softmax_scale, (int)num_splits,
                    out.data_ptr(), odt, return_lse ? lse.data_ptr<float>() : nullptr,
                    w.data_ptr(), w.numel(), stream_ptr()),
                 "mla_decode_paged");
    if (!return_lse) lse = at::empty({0}, query.options().dtype(at::kFloat));
    return {out, lse};
}

// LSE merge of partials: part_o [P, rows, 512] fp32, part_lse [P, rows] fp32.
std::vector<at::Tensor> mla_combine(const at::Tensor &part_o, const at::Tensor &part_lse,
                                    bool out_fp32) {
    check_cuda(part_o, "part_o");
    check_cuda(part_lse, "part_lse");
    TORCH_CHECK(part_o.scalar_type() == at::kFloat && part_lse.scalar_type() == at::kFloat,
                "mla_combine: float32 partials expected");
    TORCH_CHECK(part_o.dim() == 3 && part_o.size(2) == MLA_B200_HEAD_DIM_V && part_lse.dim() == 2 &&
                    part_lse.size(0) == part_o.size(0) && part_lse.size(1) == part_o.size(1),
                "mla_combine: expected part_o [P, rows, 512] and part_lse [P, rows]");
    c10::cuda::CUDAGuard g(part_o.device());
    const int64_t p = part_o.size(0), rows = part_o.size(1);
    at::Tensor out = at::empty({rows, MLA_B200_HEAD_DIM_V},
                               part_o.options().dtype(out_fp32 ? at::kFloat : at::kHalf));
    at::Tensor lse = at::empty({rows}, part_o.options());
    check_status(mla_b200_combine_f32(part_o.data_ptr<float>(), part_lse.data_ptr<float>(), (int)p,
                                      rows, out.data_ptr(),
                                      out_fp32 ? MLA_B200_OUT_F32 : MLA_B200_OUT_F16,
                                      lse.data_ptr<float>(), stream_ptr()),
                 "mla_combine");
    return {out, lse};
}

int64_t mla_get_device_error() {
    int code = 0;
    const int st = mla_b200_get_device_error(&code, stream_ptr());
    TORCH_CHECK(st == MLA_B200_OK || st == MLA_B200_ERR_DEVICE_TIMEOUT,
                "mla_get_device_error failed: ", mla_b200_status_string(st));
    return code;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.def("mla_decode_naive", &mla_decode_naive, "fp32 naive decode, reference semantics",
          py::arg("query"), py::arg("cache"));
    m.def("mla_decode_fused", &mla_decode_fused, "fp32 fused decode, reference semantics",
          py::arg("query"), py::arg("cache"));
    m.def("mla_decode_split", &mla_decode_split, "split-KV decode, reference semantics",
          py::arg("query"), py::arg("cache"), py::arg("num_splits") = -1);
    m.def("mla_decode_batched", &mla_decode_batched, "batched / varlen decode (fp16, bf16, fp8 cache)",
          py::arg("query"), py::arg("cache"), py::arg("cu_seqlens") = py::none(),
          py::arg("max_seq_len") = -1, py::arg("softmax_scale") = 0.07216878364870322,
          py::arg("num_splits") = -1, py::arg("return_lse") = false, py::arg("out_fp32") = false,
          py::arg("kv_scale") = 1.0);
    m.def("mla_decode_mtp", &mla_decode_mtp, "multi-token (draft) decode sharing each cache tile",
          py::arg("query"), py::arg("cache"), py::arg("cu_seqlens") = py::none(),
          py::arg("max_seq_len") = -1, py::arg("softmax_scale") = 0.07216878364870322,
          py::arg("num_splits") = -1, py::arg("return_lse") = false, py::arg("out_fp32") = false);
    m.def("mla_decode_paged", &mla_decode_paged, "decode over a paged latent cache",
          py::arg("query"), py::arg("kv_pages"), py::arg("block_table"), py::arg("seq_lens"),
          py::arg("max_seq_len") = -1, py::arg("softmax_scale") = 0.07216878364870322,
          py::arg("num_splits") = -1, py::arg("return_lse") = false, py::arg("out_fp32") = false);
    m.def("mla_combine", &mla_combine, "log-sum-exp merge of partial decodes", py::arg("part_o"),
          py::arg("part_lse"), py::arg("out_fp32") = false);
    m.def("mla_get_device_error", &mla_get_device_error,
          "read and clear the kernels' device error word");
    m.attr("NUM_HEADS") = MLA_B200_NUM_HEADS;
    m.attr("HEAD_DIM") = MLA_B200_HEAD_DIM;
    m.attr("HEAD_DIM_C") = MLA_B200_HEAD_DIM_C;
    m.attr("HEAD_DIM_ROPE") = MLA_B200_HEAD_DIM_ROPE;
    m.attr("HEAD_DIM_K") = MLA_B200_HEAD_DIM_K;
    m.attr("HEAD_DIM_V") = MLA_B200_HEAD_DIM_V;
}
