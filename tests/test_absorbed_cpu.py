"""CPU check of the weight-absorption algebra around the decode
(ada_mla.absorbed): absorbing W_UK into Q* and projecting O* by W_UV equals
per-head attention over up-projected keys and values.  The decode step itself
is a torch fp32 restatement here, and so are the two projections (the
definitions the tcgen05 projection kernels implement; their parity is covered
on the GPU)."""
import numpy as np
import torch



def absorb_ref(q_nope, q_rope, w_uk):
    """Q*[b, h] = [q_nope[b, h] . W_UK[h], q_rope[b, h]]"""
    return torch.cat([torch.einsum("bhd,hdc->bhc", q_nope, w_uk), q_rope], dim=-1)


def project_ref(o_star, w_uv):
    """o[b, h] = O*[b, h] . W_UV[h]"""
    return torch.einsum("bhc,hcv->bhv", o_star, w_uv)


def _decode_fp32(q_star, c, scale):
    s = torch.einsum("bhk,bnk->bhn", q_star, c) * scale
    return torch.einsum("bhn,bnc->bhc", torch.softmax(s, dim=-1), c[:, :, :512])


def test_absorption_algebra():
    torch.manual_seed(3)
    b, nh, n, dn, dv = 2, 8, 50, 128, 64
    scale = 1.0 / np.sqrt(192)
    c = torch.randn(b, n, 576, dtype=torch.float64)
    q_nope = torch.randn(b, nh, dn, dtype=torch.float64)
    q_rope = torch.randn(b, nh, 64, dtype=torch.float64)
    w_uk = torch.randn(nh, dn, 512, dtype=torch.float64) / 512 ** 0.5
    w_uv = torch.randn(nh, 512, dv, dtype=torch.float64) / 512 ** 0.5
    q_star = absorb_ref(q_nope, q_rope, w_uk)
    assert q_star.shape == (b, nh, 576)
    out = project_ref(_decode_fp32(q_star, c, scale), w_uv)
    k_nope = torch.einsum("bnc,hdc->bhnd", c[:, :, :512], w_uk)
    v = torch.einsum("bnc,hcv->bhnv", c[:, :, :512], w_uv)
    logits = (torch.einsum("bhd,bhnd->bhn", q_nope, k_nope)
              + torch.einsum("bhr,bnr->bhn", q_rope, c[:, :, 512:])) * scale
    ref = torch.einsum("bhn,bhnv->bhv", torch.softmax(logits, dim=-1), v)
    assert torch.allclose(out, ref, atol=1e-10, rtol=1e-10)


def test_shape_errors():
    import pytest

    from ada_mla import absorbed

    with pytest.raises(ValueError):
        absorbed.absorb_query(torch.zeros(1, 4, 128), torch.zeros(1, 4, 64), torch.zeros(4, 64, 512))
    with pytest.raises(ValueError):
        absorbed.project_output(torch.zeros(1, 4, 512), torch.zeros(3, 512, 128))
    with pytest.raises(ValueError):  # the kernels take CUDA tensors only: no CPU path
        absorbed.absorb_query(torch.zeros(1, 4, 128), torch.zeros(1, 4, 64), torch.zeros(4, 128, 512))
