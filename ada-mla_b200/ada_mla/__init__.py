"""ada_mla -- B200 (sm_100a) MLA decode engine, drop-in for lechebs/ada-mla's
``ada_mla`` torch extension.

Same names, signatures, output shapes and dtypes as the reference's pybind
module (csrc/mla_api.cpp:115-120):

* ``mla_decode_naive(query, cache)``  fp32; softmax(Q C^T / sqrt(D)) C over all
  D columns, attention matrix materialized (reference csrc/mla_api.cpp:5-32).
* ``mla_decode_fused(query, cache)``  fp32 -> [n_h, 512] fp32, scale 1/sqrt(192)
  (reference csrc/mla_api.cpp:34-54).
* ``mla_decode_split(query, cache, num_splits=-1)``  fp16 -> [n_h, 512] fp16 on
  the split-KV kernels + LSE combine; fp32 -> the fp32 kernel (reference
  csrc/mla_api.cpp:86-113, whose fp32 branch is an empty stub).

plus ``mla_decode_batched`` (batch / varlen), ``mla_decode_paged`` (a paged
latent cache through a block table), ``mla_combine`` (the LSE merge the
multi-GPU layer uses), ``mla_get_device_error`` and the model constants the
reference left as a TODO in mla.py:29-34.

Importing never compiles: the native libraries are built in-tree by
``ada_mla._build.build()`` (or the repository's ``__graft_entry__.build()``).
If they are missing the import fails loudly -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import importlib.util
import os

import torch  # noqa: F401  (loads libtorch / libc10 before the extension)

from ._build import EXT_NAME, EXT_PATH, LIB_PATH

__all__ = [
    "mla_decode_naive", "mla_decode_fused", "mla_decode_split", "mla_decode_batched",
    "mla_decode_paged", "mla_decode_mtp",
    "mla_combine", "mla_get_device_error", "NUM_HEADS", "HEAD_DIM", "HEAD_DIM_C",
    "HEAD_DIM_ROPE", "HEAD_DIM_K", "HEAD_DIM_V", "SOFTMAX_SCALE", "lib_path", "ext_path",
]


def _load_extension():
    for path in (LIB_PATH, EXT_PATH):
        if not os.path.isfile(path):
            raise ImportError(
                f"ada_mla: native library {path} is missing; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` (repository root) "
                "or `python ada-mla_b200/ada_mla/_build.py`")
    # The extension links libmla_b200.so by soname; load it first, globally.
    ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
    spec = importlib.util.spec_from_file_location(EXT_NAME, EXT_PATH)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


_ext = _load_extension()

mla_decode_naive = _ext.mla_decode_naive
mla_decode_fused = _ext.mla_decode_fused
mla_decode_split = _ext.mla_decode_split
mla_combine = _ext.mla_combine
mla_get_device_error = _ext.mla_get_device_error

NUM_HEADS = _ext.NUM_HEADS
HEAD_DIM = _ext.HEAD_DIM
HEAD_DIM_C = _ext.HEAD_DIM_C
HEAD_DIM_ROPE = _ext.HEAD_DIM_ROPE
HEAD_DIM_K = _ext.HEAD_DIM_K
HEAD_DIM_V = _ext.HEAD_DIM_V
# The reference's fused/split softmax scale, 1/sqrt(HEAD_DIM + HEAD_DIM_ROPE)
# (csrc/mla_decode_splitk_fwd.cuh:446-450, mla.py:46).
SOFTMAX_SCALE = 1.0 / (HEAD_DIM + HEAD_DIM_ROPE) ** 0.5

lib_path = LIB_PATH
ext_path = EXT_PATH


def mla_decode_batched(query, cache, cu_seqlens=None, max_seq_len: int = -1,
                       softmax_scale: float = SOFTMAX_SCALE, num_splits: int = -1,
                       return_lse: bool = False, out_dtype=None, kv_scale=1.0):
    """Batched / variable-length decode: fp16 or bf16, or an fp8 (e4m3) cache.

    query  [B, n_h, 576] fp16 or bf16 (bf16 and fp8 cache: n_h <= 128).
    cache  dense [B, N, 576], or packed [T, 576] with ``cu_seqlens`` int32
           [B+1] (sequence b owns rows cu_seqlens[b]:cu_seqlens[b+1]), in the
           query's dtype -- or torch.float8_e4m3fn with an fp16 query, the
           cache then being ``cache * kv_scale``: a float (one scale for the
           tensor) or an fp32 CUDA tensor with one scale per cache row
           ([T] packed, [B, N] dense; a per-page or per-tile scale is its value
           repeated over the rows).  Pass ``max_seq_len`` to avoid a
           device->host read of the longest length.
    Returns O* [B, n_h, 512] (the query's dtype, or fp32 when
    ``out_dtype=torch.float32``) and, with ``return_lse``, the natural-log LSE
    [B, n_h] fp32 as a tuple.
    """
    if out_dtype not in (None, torch.float32, query.dtype):
        raise ValueError(f"mla_decode_batched: out_dtype must be None, float32 or {query.dtype}")
    out_fp32 = out_dtype == torch.float32
    if isinstance(kv_scale, torch.Tensor):
        from . import capi

        if cache.dtype != torch.float8_e4m3fn or query.dtype != torch.float16:
            raise ValueError("mla_decode_batched: per-row kv scales need an e4m3 cache and an fp16 query")
        rows = cache.shape[0] * (cache.shape[1] if cu_seqlens is None else 1)
        if (not kv_scale.is_cuda or kv_scale.dtype != torch.float32 or kv_scale.numel() != rows
                or not kv_scale.is_contiguous()):
            raise ValueError("mla_decode_batched: kv_scale tensor must be contiguous fp32 CUDA, one per cache row")
        if cu_seqlens is None:
            max_seq_len = cache.shape[1]
        elif max_seq_len < 0:
            max_seq_len = int((cu_seqlens[1:] - cu_seqlens[:-1]).max().item()) if cache.shape[0] else 0
        c2 = cache.reshape(-1, cache.shape[-1]) if cu_seqlens is None else cache
        res = capi.decode_batched_fp8_scaled(query, c2, kv_scale, cu_seqlens, int(max_seq_len), float(softmax_scale),
                                             int(num_splits), out_fp32=out_fp32, return_lse=return_lse)
        return res
    out, lse = _ext.mla_decode_batched(query, cache, cu_seqlens, int(max_seq_len),
                                       float(softmax_scale), int(num_splits),
                                       bool(return_lse), out_fp32, float(kv_scale))
    return (out, lse) if return_lse else out


def mla_decode_paged(query, kv_pages, block_table, seq_lens, max_seq_len: int = -1,
                     softmax_scale: float = SOFTMAX_SCALE, num_splits: int = -1,
                     return_lse: bool = False, out_dtype=None):
    """Decode over a paged latent cache.

    query        [B, n_h, 576] fp16 or bf16 (n_h <= 128).
    kv_pages     [num_pages, page_size, 576] page pool in the query's dtype;
                 page_size a multiple of 32.
    block_table  int32 [B, max_blocks]: token t of sequence b is row
                 t % page_size of page block_table[b, t // page_size].
    seq_lens     int32 [B].  Pass ``max_seq_len`` (>= every length) to avoid a
                 device->host read.
    Rows of a page past its sequence's end may hold anything.  Returns O*
    [B, n_h, 512] (input dtype, or fp32 with ``out_dtype=torch.float32``) and,
    with ``return_lse``, the natural-log LSE [B, n_h] fp32.
    """
    if out_dtype not in (None, torch.float32, query.dtype):
        raise ValueError(f"mla_decode_paged: out_dtype must be None, float32 or {query.dtype}")
    out, lse = _ext.mla_decode_paged(query, kv_pages, block_table, seq_lens, int(max_seq_len),
                                     float(softmax_scale), int(num_splits), bool(return_lse),
                                     out_dtype == torch.float32)
    return (out, lse) if return_lse else out


def mla_decode_mtp(query, cache, cu_seqlens=None, max_seq_len: int = -1,
                   softmax_scale: float = SOFTMAX_SCALE, num_splits: int = -1,
                   return_lse: bool = False, out_dtype=None):
    """Multi-token (speculative / MTP draft) decode.

    query  [B, k, n_h, 576] fp16 or bf16, n_h <= 128: k draft tokens per
           sequence whose own latent rows are the sequence's last k cache rows.
    cache  as for ``mla_decode_batched`` (dense [B, N, 576] or packed with
           ``cu_seqlens``), same dtype.  Draft token i of a sequence of length L
           sees its first L - (k - 1 - i) tokens.
    With k * n_h <= 128 the k drafts share every cache tile (rows token * n_h +
    head of one MMA tile): one pass over the cache for k tokens.  Above that
    (e.g. 128 heads) each draft is decoded as its own 128-row sequence next to
    the sequence's other drafts, whose repeated tile reads hit L2.  Returns O*
    [B, k, n_h, 512] (and the LSE [B, k, n_h] with ``return_lse``).
    """
    if out_dtype not in (None, torch.float32, query.dtype):
        raise ValueError(f"mla_decode_mtp: out_dtype must be None, float32 or {query.dtype}")
    out, lse = _ext.mla_decode_mtp(query, cache, cu_seqlens, int(max_seq_len), float(softmax_scale),
                                   int(num_splits), bool(return_lse), out_dtype == torch.float32)
    return (out, lse) if return_lse else out
