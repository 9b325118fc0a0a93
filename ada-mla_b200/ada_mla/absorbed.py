"""The steps on either side of the decode kernel: weight absorption into Q* and
the per-head value projection of O* (README.md:76-110 of the reference, which
stops at O* and leaves both to the caller).

For head i, with decoupled RoPE (DeepSeek-V2),

    q*_i = [ q_nope_i W_UK_i , q_rope_i ]             (1 x 576)
    o*_i = softmax(scale * q*_i C^T) C_N              (1 x 512, the decode kernel)
    o_i  = o*_i W_UV_i                                 (1 x d_v)

W_UK_i [d x 512] maps head i's key space to the latent and W_UV_i [512 x d_v]
the latent to its value space; absorbing them makes every head attend over the
same latent rows.  Both projections are per-head GEMMs with the batch as the
small dimension (each head has its own weights, so they do not join the
decode's 128-row head tile).  They run on this library's tcgen05 projection
kernel (mla_b200_absorb_q_* / mla_b200_project_o_*), which streams each weight
byte once with the weights on the MMA's M side; the three launches share the
caller's stream, the absorption signalling early completion so the decode's
set-up overlaps its tail.
"""
from __future__ import annotations

import torch

from . import SOFTMAX_SCALE, capi, mla_decode_batched


def _check_inputs(*ts):
    for t in ts:
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError("absorbed: inputs must be contiguous CUDA tensors")
    if len({t.dtype for t in ts}) != 1 or ts[0].dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("absorbed: inputs must all be float16 or all bfloat16")


def absorb_query(q_nope: torch.Tensor, q_rope: torch.Tensor, w_uk: torch.Tensor) -> torch.Tensor:
    """q_nope [B, n_h, d], q_rope [B, n_h, 64], w_uk [n_h, d, 512] -> Q* [B, n_h, 576]."""
    b, nh, dn = q_nope.shape
    if w_uk.shape != (nh, dn, 512) or q_rope.shape != (b, nh, 64):
        raise ValueError("absorb_query: expected q_nope [B, n_h, d], q_rope [B, n_h, 64], w_uk [n_h, d, 512]")
    _check_inputs(q_nope, q_rope, w_uk)
    return capi.absorb_q(q_nope, q_rope, w_uk)


def project_output(o_star: torch.Tensor, w_uv: torch.Tensor) -> torch.Tensor:
    """o_star [B, n_h, 512], w_uv [n_h, 512, d_v] -> per-head outputs [B, n_h, d_v]."""
    b, nh, _ = o_star.shape
    if w_uv.shape[:2] != (nh, 512):
        raise ValueError("project_output: expected w_uv [n_h, 512, d_v]")
    w_uv = w_uv.to(o_star.dtype)
    _check_inputs(o_star, w_uv)
    return capi.project_o(o_star, w_uv)


def mla_decode_absorbed(q_nope, q_rope, w_uk, cache, w_uv, cu_seqlens=None, max_seq_len: int = -1,
                        softmax_scale: float = SOFTMAX_SCALE, num_splits: int = -1):
    """One MLA decode step from the per-head compressed query to the per-head
    attention outputs: absorb W_UK into Q*, decode over the latent cache
    (``mla_decode_batched``: dense or packed, fp16 or bf16), project by W_UV.
    Returns [B, n_h, d_v] in the query's dtype (the W_O projection follows)."""
    q_star = absorb_query(q_nope, q_rope, w_uk)
    o_star = mla_decode_batched(q_star, cache, cu_seqlens, max_seq_len=max_seq_len,
                                softmax_scale=softmax_scale, num_splits=num_splits)
    return project_output(o_star, w_uv)
