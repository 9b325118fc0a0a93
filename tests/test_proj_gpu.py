"""The tcgen05 per-head projection kernels on either side of the decode
(mla_b200_absorb_q_* and mla_b200_project_o_*, through the C ABI) against an
fp32 einsum of the same fp16 / bf16 inputs.  The reference derives both
products (README.md:74-110) and has no kernel for them.

Tolerance: fp32 accumulation on both sides, so the difference is the output's
own rounding: |y| <= ~5 here, fp16 2^-11 relative (max-abs 1e-2, mean-abs
1e-3) and bf16 2^-8 relative (max-abs 4e-2, mean-abs 4e-3)."""
import numpy as np
import pytest
import torch

from conftest import assert_close_parity

pytestmark = pytest.mark.gpu

TOL = {torch.float16: (1e-2, 1e-3), torch.bfloat16: (4e-2, 4e-3)}


def _rand(shape, gen, scale, dtype):
    return (torch.randn(shape, generator=gen) * scale).to(dtype).cuda()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("b,nh,d", [(1, 128, 128), (7, 16, 128), (64, 128, 128), (300, 128, 128), (33, 8, 192)])
def test_absorb_q(b, nh, d, dtype):
    from ada_mla import capi

    g = torch.Generator().manual_seed(b * 1000 + nh + d)
    q_nope = _rand((b, nh, d), g, 1.0, dtype)
    q_rope = _rand((b, nh, 64), g, 1.0, dtype)
    w_uk = _rand((nh, d, 512), g, 1.0 / np.sqrt(d), dtype)
    out = torch.full((b, nh, 576), float("nan"), dtype=dtype, device="cuda")
    capi.absorb_q(q_nope, q_rope, w_uk, out)
    torch.cuda.synchronize()
    ref = torch.einsum("bhd,hdc->bhc", q_nope.float(), w_uk.float())
    mx, mean = TOL[dtype]
    assert_close_parity(out[:, :, :512].float().cpu().numpy(), ref.cpu().numpy(), mx, mean,
                        what=f"absorb b={b} nh={nh} d={d} {dtype}")
    assert torch.equal(out[:, :, 512:], q_rope), "rope columns are copied unchanged"
    assert capi.get_device_error() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("b,nh,dv", [(1, 128, 128), (9, 16, 128), (300, 128, 256), (256, 4, 128)])
def test_project_o(b, nh, dv, dtype):
    from ada_mla import capi

    g = torch.Generator().manual_seed(b * 7 + nh + dv)
    o_star = _rand((b, nh, 512), g, 1.0, dtype)
    w_uv = _rand((nh, 512, dv), g, 1.0 / np.sqrt(512), dtype)
    out = torch.full((b, nh, dv), float("nan"), dtype=dtype, device="cuda")
    capi.project_o(o_star, w_uv, out)
    torch.cuda.synchronize()
    ref = torch.einsum("bhc,hcv->bhv", o_star.float(), w_uv.float())
    mx, mean = TOL[dtype]
    assert_close_parity(out.float().cpu().numpy(), ref.cpu().numpy(), mx, mean,
                        what=f"project b={b} nh={nh} dv={dv} {dtype}")
    assert capi.get_device_error() == 0


def test_projection_rejects_bad_shapes():
    from ada_mla import capi

    lib = capi.lib()
    z = torch.zeros(64, dtype=torch.float16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    # head_dim not a multiple of 64, head_dim_v not a multiple of 128, null rope
    assert lib.mla_b200_absorb_q_f16(z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), 1, 1, 100, s) \
        == capi.ERR_UNSUPPORTED
    assert lib.mla_b200_project_o_f16(z.data_ptr(), z.data_ptr(), z.data_ptr(), 1, 1, 64, s) == capi.ERR_UNSUPPORTED
    assert lib.mla_b200_absorb_q_f16(z.data_ptr(), None, z.data_ptr(), z.data_ptr(), 1, 1, 128, s) \
        == capi.ERR_INVALID_ARG
