"""ctypes binding of the C ABI (``include/mla_b200.h``) in ``libmla_b200.so``.

This is the binding a maintainer of the reference would add to call the
engine without the torch extension: plain pointers, sizes and a
``cudaStream_t``, every call returning a status.  Buffers here are torch
CUDA tensors only for convenience (their ``data_ptr()`` crosses the ABI).
The GPU parity tests call through this module to exercise the ABI itself.
"""
from __future__ import annotations

import ctypes
import os

import torch

from ._build import LIB_PATH

OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED = 2
ERR_WORKSPACE = 3
ERR_CUDA = 4
ERR_DEVICE_TIMEOUT = 5
ERR_NO_DEVICE = 6
OUT_F16 = 0
OUT_F32 = 1
OUT_BF16 = 2

_c_int, _c_ll, _c_size, _c_float = ctypes.c_int, ctypes.c_longlong, ctypes.c_size_t, ctypes.c_float
_vp = ctypes.c_void_p

# (name, restype, argtypes) for every symbol declared in include/mla_b200.h
SIGNATURES = {
    "mla_b200_status_string": (ctypes.c_char_p, [_c_int]),
    "mla_b200_version": (ctypes.c_char_p, []),
    "mla_b200_constant": (_c_int, [ctypes.c_char_p]),
    "mla_b200_set_kernel_timing": (_c_int, [_vp, _vp]),
    "mla_b200_set_kernel_span": (_c_int, [_vp, _c_int]),
    "mla_b200_device_info": (_c_int, [ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    "mla_b200_plan": (_c_int, [_c_int, _c_int, _c_ll, _c_int, _c_int,
                               ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    "mla_b200_workspace_size": (_c_size, [_c_int, _c_int, _c_ll, _c_int, _c_int]),
    "mla_b200_workspace_size_fp8": (_c_size, [_c_int, _c_int, _c_ll, _c_int, _c_int]),
    "mla_b200_workspace_size_mtp": (_c_size, [_c_int, _c_int, _c_int, _c_ll, _c_int, _c_int]),
    "mla_b200_decode_split_f16": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _vp, _c_size, _vp]),
    "mla_b200_decode_split_f16_noalloc": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _vp]),
    "mla_b200_decode_batched_f16": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_ll, _c_int, _c_float,
                                             _c_int, _vp, _c_int, _vp, _vp, _c_size, _vp]),
    "mla_b200_decode_batched_bf16": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_ll, _c_int, _c_float,
                                              _c_int, _vp, _c_int, _vp, _vp, _c_size, _vp]),
    "mla_b200_decode_batched_fp8": (_c_int, [_vp, _vp, _c_float, _vp, _c_int, _c_int, _c_ll, _c_int,
                                             _c_float, _c_int, _vp, _c_int, _vp, _vp, _c_size, _vp]),
    "mla_b200_decode_batched_fp8_scaled": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_ll, _c_int,
                                                    _c_float, _c_int, _vp, _c_int, _vp, _vp, _c_size, _vp]),
    "mla_b200_decode_mtp_f16": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _c_ll, _c_int, _c_float,
                                         _c_int, _vp, _c_int, _vp, _vp, _c_size, _vp]),
    "mla_b200_decode_mtp_bf16": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _c_ll, _c_int, _c_float,
                                          _c_int, _vp, _c_int, _vp, _vp, _c_size, _vp]),
    "mla_b200_decode_paged_f16": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                           _c_int, _c_float, _c_int, _vp, _c_int, _vp, _vp, _c_size, _vp]),
    "mla_b200_decode_paged_bf16": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                            _c_int, _c_float, _c_int, _vp, _c_int, _vp, _vp, _c_size, _vp]),
    "mla_b200_decode_fused_f32": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _vp, _c_size, _vp]),
    "mla_b200_decode_naive_f32": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp]),
    "mla_b200_combine_f32": (_c_int, [_vp, _vp, _c_int, _c_ll, _vp, _c_int, _vp, _vp]),
    "mla_b200_combine_packed_f32": (_c_int, [_vp, _c_int, _c_ll, _c_ll, _vp, _c_int, _vp, _vp]),
    "mla_b200_absorb_q_f16": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp]),
    "mla_b200_absorb_q_bf16": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp]),
    "mla_b200_project_o_f16": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _vp]),
    "mla_b200_project_o_bf16": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _vp]),
    "mla_b200_get_device_error": (_c_int, [ctypes.POINTER(_c_int), _vp]),
    "mla_b200_last_cuda_error": (_c_int, []),
    "mla_b200_selftest_wait_timeout": (_c_int, [ctypes.c_ulonglong, _vp, _vp]),
    "mla_b200_exchange_bytes": (_c_size, [_c_int, _c_ll]),
    "mla_b200_exchange_alloc": (_c_int, [_c_int, _c_ll, ctypes.POINTER(_vp)]),
    "mla_b200_exchange_free": (_c_int, [_vp]),
    "mla_b200_ipc_handle": (_c_int, [_vp, _vp]),
    "mla_b200_ipc_open": (_c_int, [_vp, ctypes.POINTER(_vp)]),
    "mla_b200_ipc_close": (_c_int, [_vp]),
    "mla_b200_exchange_put_f32": (_c_int, [_vp, _c_ll, ctypes.POINTER(_vp), _c_int, _c_int, _vp]),
    "mla_b200_exchange_merge_f32": (_c_int, [_vp, _c_int, _c_ll, _vp, _c_int, _vp, ctypes.c_ulonglong, _vp]),
    "mla_b200_exchange_f32": (_c_int, [_vp, _c_ll, ctypes.POINTER(_vp), _c_int, _c_int, _vp, _c_int, _vp,
                                       ctypes.c_ulonglong, _vp]),
    "mla_b200_decode_exchange_f16": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_ll, _c_int, _c_float, _c_int,
                                              ctypes.POINTER(_vp), _c_int, _c_int, _vp, _vp, _c_int, _vp,
                                              ctypes.c_ulonglong, _vp, _c_size, _vp]),
}

_lib: ctypes.CDLL | None = None


class MlaError(RuntimeError):
    def __init__(self, fn: str, status: int):
        detail = ""
        if status == ERR_CUDA and _lib is not None:
            detail = f", cudaError {_lib.mla_b200_last_cuda_error()}"
        super().__init__(f"{fn}: {status_string(status)} (status {status}{detail})")
        self.status = status


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.isfile(LIB_PATH):
            raise ImportError(f"{LIB_PATH} missing; run ada_mla._build.build()")
        l = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def status_string(status: int) -> str:
    return lib().mla_b200_status_string(status).decode()


def _check(fn: str, status: int) -> None:
    if status != OK:
        raise MlaError(fn, status)


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def constant(name: str) -> int:
    return lib().mla_b200_constant(name.encode())


def set_kernel_timing(start: "torch.cuda.Event | None", stop: "torch.cuda.Event | None") -> None:
    """Record `start`/`stop` around every later main decode-kernel launch of this
    host thread (None, None turns it off)."""
    a = None if start is None else start.cuda_event
    b = None if stop is None else stop.cuda_event
    _check("mla_b200_set_kernel_timing", lib().mla_b200_set_kernel_timing(a, b))


def set_kernel_span(span: "torch.Tensor | None") -> None:
    """Record the device-side span of each later main decode-kernel launch of
    this host thread into `span` (int64 CUDA tensor [slots, 2], each pair set
    to (UINT64_MAX, 0) beforehand); None turns it off."""
    if span is None:
        _check("mla_b200_set_kernel_span", lib().mla_b200_set_kernel_span(None, 0))
    else:
        _check("mla_b200_set_kernel_span", lib().mla_b200_set_kernel_span(span.data_ptr(), span.shape[0]))


def device_info():
    """(num_sms, resident 2-CTA decode clusters) of the current device."""
    sms, cl = _c_int(0), _c_int(0)
    _check("mla_b200_device_info", lib().mla_b200_device_info(ctypes.byref(sms), ctypes.byref(cl)))
    return sms.value, cl.value


def plan(batch: int, num_heads: int, total_tokens: int, max_seq_len: int, num_sms: int = 0):
    chunk, splits = _c_int(0), _c_int(0)
    _check("mla_b200_plan", lib().mla_b200_plan(batch, num_heads, total_tokens, max_seq_len,
                                                num_sms, ctypes.byref(chunk), ctypes.byref(splits)))
    return chunk.value, splits.value


def workspace_size(batch: int, num_heads: int, total_tokens: int, max_seq_len: int,
                   num_splits: int = 0) -> int:
    return int(lib().mla_b200_workspace_size(batch, num_heads, total_tokens, max_seq_len, num_splits))


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def decode_split_f16(query: torch.Tensor, cache: torch.Tensor, num_splits: int = -1,
                     out: torch.Tensor | None = None, workspace: torch.Tensor | None = None):
    nh, n = query.shape[0], cache.shape[0]
    if out is None:
        out = torch.empty((nh, 512), dtype=torch.float16, device=query.device)
    if workspace is None:
        workspace = _workspace(workspace_size(1, nh, n, n, num_splits), query.device)
    _check("mla_b200_decode_split_f16", lib().mla_b200_decode_split_f16(
        _ptr(query), _ptr(cache), _ptr(out), nh, n, num_splits, _ptr(workspace),
        workspace.numel(), _stream()))
    return out


def decode_split_f16_noalloc(query: torch.Tensor, cache: torch.Tensor, num_splits: int = -1,
                             out: torch.Tensor | None = None):
    """The allocation-free split decode: scratch comes from the library's static
    device array, so only the output is passed (and allocated here if absent)."""
    nh, n = query.shape[0], cache.shape[0]
    if out is None:
        out = torch.empty((nh, 512), dtype=torch.float16, device=query.device)
    _check("mla_b200_decode_split_f16_noalloc", lib().mla_b200_decode_split_f16_noalloc(
        _ptr(query), _ptr(cache), _ptr(out), nh, n, num_splits, _stream()))
    return out


def decode_batched_f16(query: torch.Tensor, cache: torch.Tensor, cu_seqlens: torch.Tensor | None,
                       max_seq_len: int, softmax_scale: float, num_splits: int = -1,
                       out_fp32: bool = False, return_lse: bool = False,
                       workspace: torch.Tensor | None = None):
    """Batched / varlen decode; the entry point follows query.dtype (fp16 ->
    mla_b200_decode_batched_f16, bf16 -> mla_b200_decode_batched_bf16) and the
    16-bit output takes the input dtype."""
    b, nh = query.shape[0], query.shape[1]
    bf16 = query.dtype == torch.bfloat16
    total = cache.shape[0] if cu_seqlens is not None else b * max_seq_len
    out = torch.empty((b, nh, 512), dtype=torch.float32 if out_fp32 else query.dtype,
                      device=query.device)
    lse = torch.empty((b, nh), dtype=torch.float32, device=query.device) if return_lse else None
    if workspace is None:
        workspace = _workspace(workspace_size(b, nh, total, max_seq_len, num_splits), query.device)
    name = "mla_b200_decode_batched_bf16" if bf16 else "mla_b200_decode_batched_f16"
    odt = OUT_F32 if out_fp32 else (OUT_BF16 if bf16 else OUT_F16)
    _check(name, getattr(lib(), name)(
        _ptr(query), _ptr(cache), _ptr(cu_seqlens), b, nh, total, max_seq_len,
        float(softmax_scale), num_splits, _ptr(out), odt,
        _ptr(lse), _ptr(workspace), workspace.numel(), _stream()))
    return (out, lse) if return_lse else out


decode_batched = decode_batched_f16


def decode_batched_fp8(query: torch.Tensor, cache: torch.Tensor, kv_scale: float,
                       cu_seqlens: torch.Tensor | None, max_seq_len: int, softmax_scale: float,
                       num_splits: int = -1, out_fp32: bool = False, return_lse: bool = False):
    """Decode over an e4m3 cache (C = cache * kv_scale) with an fp16 query."""
    b, nh = query.shape[0], query.shape[1]
    total = cache.shape[0] if cu_seqlens is not None else b * max_seq_len
    out = torch.empty((b, nh, 512), dtype=torch.float32 if out_fp32 else torch.float16,
                      device=query.device)
    lse = torch.empty((b, nh), dtype=torch.float32, device=query.device) if return_lse else None
    ws_bytes = lib().mla_b200_workspace_size_fp8(b, nh, total, max_seq_len, num_splits)
    ws = _workspace(ws_bytes, query.device)
    _check("mla_b200_decode_batched_fp8", lib().mla_b200_decode_batched_fp8(
        _ptr(query), _ptr(cache), float(kv_scale), _ptr(cu_seqlens), b, nh, total, max_seq_len,
        float(softmax_scale), num_splits, _ptr(out), OUT_F32 if out_fp32 else OUT_F16, _ptr(lse),
        _ptr(ws), ws.numel(), _stream()))
    return (out, lse) if return_lse else out


def decode_batched_fp8_scaled(query: torch.Tensor, cache: torch.Tensor, kv_scales: torch.Tensor,
                              cu_seqlens: torch.Tensor | None, max_seq_len: int, softmax_scale: float,
                              num_splits: int = -1, out_fp32: bool = False, return_lse: bool = False):
    """Decode over an e4m3 cache with one scale per cache row (C[t] = cache[t] * kv_scales[t])."""
    b, nh = query.shape[0], query.shape[1]
    total = cache.shape[0] if cu_seqlens is not None else b * max_seq_len
    out = torch.empty((b, nh, 512), dtype=torch.float32 if out_fp32 else torch.float16, device=query.device)
    lse = torch.empty((b, nh), dtype=torch.float32, device=query.device) if return_lse else None
    ws = _workspace(lib().mla_b200_workspace_size_fp8(b, nh, total, max_seq_len, num_splits), query.device)
    _check("mla_b200_decode_batched_fp8_scaled", lib().mla_b200_decode_batched_fp8_scaled(
        _ptr(query), _ptr(cache), _ptr(kv_scales), _ptr(cu_seqlens), b, nh, total, max_seq_len,
        float(softmax_scale), num_splits, _ptr(out), OUT_F32 if out_fp32 else OUT_F16, _ptr(lse),
        _ptr(ws), ws.numel(), _stream()))
    return (out, lse) if return_lse else out


def decode_paged(query: torch.Tensor, kv_pages: torch.Tensor, block_table: torch.Tensor,
                 seq_lens: torch.Tensor, max_seq_len: int, softmax_scale: float,
                 num_splits: int = -1, out_fp32: bool = False, return_lse: bool = False,
                 workspace: torch.Tensor | None = None):
    """Paged decode through mla_b200_decode_paged_f16 / _bf16 (by query.dtype)."""
    b, nh = query.shape[0], query.shape[1]
    bf16 = query.dtype == torch.bfloat16
    out = torch.empty((b, nh, 512), dtype=torch.float32 if out_fp32 else query.dtype,
                      device=query.device)
    lse = torch.empty((b, nh), dtype=torch.float32, device=query.device) if return_lse else None
    if workspace is None:
        workspace = _workspace(workspace_size(b, nh, b * max_seq_len, max_seq_len, num_splits),
                               query.device)
    name = "mla_b200_decode_paged_bf16" if bf16 else "mla_b200_decode_paged_f16"
    odt = OUT_F32 if out_fp32 else (OUT_BF16 if bf16 else OUT_F16)
    _check(name, getattr(lib(), name)(
        _ptr(query), _ptr(kv_pages), _ptr(block_table), _ptr(seq_lens), b, nh,
        kv_pages.shape[0], kv_pages.shape[1], block_table.shape[1], max_seq_len,
        float(softmax_scale), num_splits, _ptr(out), odt, _ptr(lse), _ptr(workspace),
        workspace.numel(), _stream()))
    return (out, lse) if return_lse else out


def decode_fused_f32(query: torch.Tensor, cache: torch.Tensor):
    nh, d, n = query.shape[0], query.shape[1], cache.shape[0]
    out = torch.empty((nh, 512), dtype=torch.float32, device=query.device)
    ws = _workspace(workspace_size(1, nh, n, n, 0), query.device)
    _check("mla_b200_decode_fused_f32", lib().mla_b200_decode_fused_f32(
        _ptr(query), _ptr(cache), _ptr(out), nh, d, n, _ptr(ws), ws.numel(), _stream()))
    return out


def decode_naive_f32(query: torch.Tensor, cache: torch.Tensor):
    nh, d, n = query.shape[0], query.shape[1], cache.shape[0]
    out = torch.empty((nh, d), dtype=torch.float32, device=query.device)
    attn = torch.empty((nh, n), dtype=torch.float32, device=query.device)
    _check("mla_b200_decode_naive_f32", lib().mla_b200_decode_naive_f32(
        _ptr(query), _ptr(cache), _ptr(attn), _ptr(out), nh, d, n, _stream()))
    return out


def combine_f32(part_o: torch.Tensor, part_lse: torch.Tensor, out_fp32: bool = True):
    p, rows = part_o.shape[0], part_o.shape[1]
    out = torch.empty((rows, 512), dtype=torch.float32 if out_fp32 else torch.float16,
                      device=part_o.device)
    lse = torch.empty((rows,), dtype=torch.float32, device=part_o.device)
    _check("mla_b200_combine_f32", lib().mla_b200_combine_f32(
        _ptr(part_o), _ptr(part_lse), p, rows, _ptr(out), OUT_F32 if out_fp32 else OUT_F16,
        _ptr(lse), _stream()))
    return out, lse


def absorb_q(q_nope: torch.Tensor, q_rope: torch.Tensor, w_uk: torch.Tensor,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Q* [B, n_h, 576] = [q_nope . W_UK[h], q_rope] (mla_b200_absorb_q_f16 / _bf16)."""
    b, nh, d = q_nope.shape
    if out is None:
        out = torch.empty((b, nh, 576), dtype=q_nope.dtype, device=q_nope.device)
    name = "mla_b200_absorb_q_bf16" if q_nope.dtype == torch.bfloat16 else "mla_b200_absorb_q_f16"
    _check(name, getattr(lib(), name)(_ptr(q_nope), _ptr(q_rope), _ptr(w_uk), _ptr(out), b, nh, d, _stream()))
    return out


def project_o(o_star: torch.Tensor, w_uv: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out [B, n_h, d_v] = O*[b, h, :] . W_UV[h] (mla_b200_project_o_f16 / _bf16)."""
    b, nh, _ = o_star.shape
    dv = w_uv.shape[2]
    if out is None:
        out = torch.empty((b, nh, dv), dtype=o_star.dtype, device=o_star.device)
    name = "mla_b200_project_o_bf16" if o_star.dtype == torch.bfloat16 else "mla_b200_project_o_f16"
    _check(name, getattr(lib(), name)(_ptr(o_star), _ptr(w_uv), _ptr(out), b, nh, dv, _stream()))
    return out


def get_device_error() -> int:
    code = _c_int(0)
    st = lib().mla_b200_get_device_error(ctypes.byref(code), _stream())
    if st not in (OK, ERR_DEVICE_TIMEOUT):
        raise MlaError("mla_b200_get_device_error", st)
    return code.value
