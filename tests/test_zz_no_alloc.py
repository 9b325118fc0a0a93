"""The allocation-free split decode (mla_b200_decode_split_f16_noalloc) against
the workspace entry point, through the C ABI.

It exists for callers that cannot allocate device memory while decoding (an FFI
host without a CUDA allocator, or a server whose pool already holds the GPU):
the scratch is a static device array inside the library.  This file is named to
be collected last, and it must pass alone in a fresh process as well as after
the other tests."""
import pytest
import torch

from conftest import MAX_ABS_TOL, MEAN_ABS_TOL, assert_close_parity

pytestmark = pytest.mark.gpu


def _inputs(nh, n, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(nh, 576, generator=g).half().cuda()
    c = torch.randn(n, 576, generator=g).half().cuda()
    return q, c


def test_noalloc_matches_workspace_entry_on_two_calls():
    from ada_mla import capi

    lib = capi.lib()
    stream = torch.cuda.current_stream().cuda_stream
    # two calls in a row: the shared scratch keeps the first call's contents,
    # which must not leak into the second result
    for seed, (nh, n) in enumerate([(128, 4096), (128, 1000)]):
        q, c = _inputs(nh, n, seed=100 + seed)
        ref = capi.decode_split_f16(q, c)
        out = torch.full((nh, 512), float("nan"), dtype=torch.float16, device="cuda")
        st = lib.mla_b200_decode_split_f16_noalloc(q.data_ptr(), c.data_ptr(), out.data_ptr(),
                                                   nh, n, -1, stream)
        assert st == capi.OK, capi.status_string(st)
        torch.cuda.synchronize()
        assert_close_parity(out.float().cpu().numpy(), ref.float().cpu().numpy(),
                            MAX_ABS_TOL, MEAN_ABS_TOL, what=f"noalloc call {seed}")
    assert capi.get_device_error() == 0


def test_noalloc_rejects_oversized_split_request():
    from ada_mla import capi

    q, c = _inputs(128, 4096, seed=7)
    out = torch.empty((128, 512), dtype=torch.float16, device="cuda")
    # 4096 splits of one token need ~1 GiB of partials: far above the scratch
    st = capi.lib().mla_b200_decode_split_f16_noalloc(q.data_ptr(), c.data_ptr(), out.data_ptr(),
                                                      128, 4096, 4096,
                                                      torch.cuda.current_stream().cuda_stream)
    assert st == capi.ERR_WORKSPACE
