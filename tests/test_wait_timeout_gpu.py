"""The bounded waits' wind-down path on the GPU, without a fault: a one-thread
kernel waits, through the same wait loop as the decode kernels, on an mbarrier
phase that nothing completes, with a 1 ms limit
(mla_b200_selftest_wait_timeout).  The wait must give up, record its code in
the device error word and return, and the context must stay usable."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from conftest import assert_close_parity

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports():
    from ada_mla import capi

    lib = capi.lib()
    stream = torch.cuda.current_stream().cuda_stream
    assert capi.get_device_error() == 0  # clean start
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = lib.mla_b200_selftest_wait_timeout(1_000_000, done.data_ptr(), stream)
    assert st == capi.OK, capi.status_string(st)
    torch.cuda.synchronize()
    assert done.item() == 1, "the wait returned after giving up"
    code = ctypes.c_int(0)
    st = lib.mla_b200_get_device_error(ctypes.byref(code), stream)
    assert st == capi.ERR_DEVICE_TIMEOUT and code.value == 6
    assert capi.get_device_error() == 0, "reading the word clears it"

    # the context is still usable: a decode right after is correct
    g = torch.Generator().manual_seed(5)
    q = torch.randn(128, 576, generator=g).half()
    c = torch.randn(500, 576, generator=g).half()
    out = capi.decode_split_f16(q.cuda(), c.cuda())
    torch.cuda.synchronize()
    ref = oracle.mla_decode_oracle(q.float().numpy(), c.float().numpy(), 1.0 / np.sqrt(192.0), threads=8)
    assert_close_parity(out.float().cpu().numpy(), ref, what="decode after the self test")
    assert capi.get_device_error() == 0


def test_selftest_rejects_bad_limits():
    from ada_mla import capi

    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert capi.lib().mla_b200_selftest_wait_timeout(0, done.data_ptr(), s) == capi.ERR_INVALID_ARG
    assert capi.lib().mla_b200_selftest_wait_timeout(10**9, done.data_ptr(), s) == capi.ERR_INVALID_ARG
    assert capi.lib().mla_b200_selftest_wait_timeout(1000, None, s) == capi.ERR_INVALID_ARG
