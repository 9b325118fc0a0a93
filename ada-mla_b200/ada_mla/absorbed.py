"""The steps on either side of the decode kernel: weight absorption into Q* and
the per-head value projection of O* (README.md:76-110 of the reference, which
stops at O* and leaves both to the caller).

For head i, with decoupled RoPE (DeepSeek-V2),

    q*_i = [ q_nope_i W_UK_i^T , q_rope_i ]          (1 x 576)
    o*_i = softmax(scale * q*_i C^T) C_N              (1 x 512, the decode kernel)
    o_i  = o*_i W_UV_i                                 (1 x 128)

W_UK_i [128 x 512] maps the latent to head i's key space and W_UV_i [512 x 128]
to its value space; absorbing them makes every head attend over the same latent
rows.  Both projections are per-head GEMMs with the batch as M (each head has its
own weights, so they do not join the decode's 128-row head tile); they run as
plain batched library GEMMs on the same stream, around our decode kernel.
"""
from __future__ import annotations

import torch

from . import mla_decode_batched, SOFTMAX_SCALE


def absorb_query(q_nope: torch.Tensor, q_rope: torch.Tensor, w_uk: torch.Tensor) -> torch.Tensor:
    """q_nope [B, n_h, 128], q_rope [B, n_h, 64], w_uk [n_h, 128, 512] -> Q* [B, n_h, 576]."""
    b, nh, dn = q_nope.shape
    if w_uk.shape != (nh, dn, 512) or q_rope.shape != (b, nh, 64):
        raise ValueError("absorb_query: expected q_nope [B, n_h, d], q_rope [B, n_h, 64], w_uk [n_h, d, 512]")
    q_star = torch.empty((b, nh, 576), dtype=q_nope.dtype, device=q_nope.device)
    # [n_h, B, d] @ [n_h, d, 512] -> [n_h, B, 512]
    q_star[:, :, :512] = torch.bmm(q_nope.transpose(0, 1), w_uk).transpose(0, 1)
    q_star[:, :, 512:] = q_rope
    return q_star


def project_output(o_star: torch.Tensor, w_uv: torch.Tensor) -> torch.Tensor:
    """o_star [B, n_h, 512], w_uv [n_h, 512, d_v] -> per-head outputs [B, n_h, d_v]."""
    b, nh, _ = o_star.shape
    if w_uv.shape[:2] != (nh, 512):
        raise ValueError("project_output: expected w_uv [n_h, 512, d_v]")
    return torch.bmm(o_star.transpose(0, 1), w_uv.to(o_star.dtype)).transpose(0, 1)


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
