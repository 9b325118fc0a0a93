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


@pytest.mark.parametrize("splits", [1, 4, 16])
def test_noalloc_explicit_splits_match_workspace_entry_and_oracle(splits):
    import numpy as np

    import oracle
    from ada_mla import capi

    lib = capi.lib()
    stream = torch.cuda.current_stream().cuda_stream
    q, c = _inputs(128, 4000, seed=200 + splits)
    ref = capi.decode_split_f16(q, c, splits)
    want = oracle.mla_decode_oracle(q.float().cpu().numpy(), c.float().cpu().numpy(),
                                    1.0 / np.sqrt(192.0), threads=8)
    out = torch.full((128, 512), float("nan"), dtype=torch.float16, device="cuda")
    for call in range(2):
        st = lib.mla_b200_decode_split_f16_noalloc(q.data_ptr(), c.data_ptr(), out.data_ptr(), 128, 4000,
                                                   splits, stream)
        assert st == capi.OK, capi.status_string(st)
        torch.cuda.synchronize()
        if call == 0:
            free0, _ = torch.cuda.mem_get_info()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0  # the second call took no device memory
    got = out.float().cpu().numpy()
    assert_close_parity(got, ref.float().cpu().numpy(), MAX_ABS_TOL, MEAN_ABS_TOL, what=f"splits={splits}")
    assert_close_parity(got, want, MAX_ABS_TOL, MEAN_ABS_TOL, what=f"splits={splits} vs oracle")


def test_noalloc_rejects_oversized_split_request():
    from ada_mla import capi

    q, c = _inputs(128, 4096, seed=7)
    out = torch.empty((128, 512), dtype=torch.float16, device="cuda")
    # 4096 splits of one token need ~1 GiB of partials: far above the scratch
    st = capi.lib().mla_b200_decode_split_f16_noalloc(q.data_ptr(), c.data_ptr(), out.data_ptr(),
                                                      128, 4096, 4096,
                                                      torch.cuda.current_stream().cuda_stream)
    assert st == capi.ERR_WORKSPACE
