"""The peer-memory exchange kernels of the split-KV multi-GPU step
(mla_b200_exchange_put_f32 / _merge_f32) on one GPU: a single rank's buffer
goes through put + merge for several steps (both parities of the buffer), the
merged output against a numpy LSE merge of the same packed partials; and a
peer that never publishes makes the merge's bounded wait run out (a flag that
nothing sets: no fault), report the peer-wait code and leave the rows alone.
The two-rank path runs in tests/test_multigpu_gpu.py."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _packed(rows, world, gen):
    """world packed parts [rows*512 O, rows LSE], each padded to a multiple of 4 floats."""
    from ada_mla.multigpu import packed_stride

    stride = packed_stride(rows)
    parts = torch.zeros(world, stride)
    for g in range(world):
        parts[g, :rows * 512] = torch.randn(rows * 512, generator=gen)
        parts[g, rows * 512:rows * 513] = torch.randn(rows, generator=gen) * 3
    return parts, stride


def _np_merge(parts, rows):
    o = parts[:, :rows * 512].reshape(parts.shape[0], rows, 512).double().numpy()
    lse = parts[:, rows * 512:rows * 513].double().numpy()
    m = lse.max(axis=0)
    w = np.exp(lse - m)
    return (w[:, :, None] * o).sum(axis=0) / w.sum(axis=0)[:, None], m + np.log(w.sum(axis=0))


def test_single_rank_put_merge_steps():
    from ada_mla import capi
    from ada_mla.multigpu import PeerExchange

    rows = 40
    ex = PeerExchange(rows)
    try:
        g = torch.Generator().manual_seed(3)
        for step in range(4):  # epochs 1..4: parities 1, 0, 1, 0
            parts, _ = _packed(rows, 1, g)
            ex.put(parts[0].cuda())
            out, lse = ex.merge(torch.float32, device="cuda")
            torch.cuda.synchronize()
            ref_o, ref_lse = _np_merge(parts, rows)
            np.testing.assert_allclose(out.cpu().numpy(), ref_o, rtol=0, atol=1e-5, err_msg=f"step {step}")
            np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, rtol=0, atol=1e-5)
        assert capi.get_device_error() == 0
    finally:
        ex.close()


def test_single_rank_fused_exchange_matches_put_merge():
    """The one-kernel exchange (mla_b200_exchange_f32) against the numpy merge,
    steps alternating with put + merge on the same buffer (the epochs and
    parities stay in step between the two forms)."""
    from ada_mla import capi
    from ada_mla.multigpu import PeerExchange

    rows = 136
    ex = PeerExchange(rows)
    try:
        g = torch.Generator().manual_seed(5)
        for step in range(5):
            parts, _ = _packed(rows, 1, g)
            if step % 2 == 0:
                out, lse = ex.exchange(parts[0].cuda(), torch.float32, device="cuda")
            else:
                ex.put(parts[0].cuda())
                out, lse = ex.merge(torch.float32, device="cuda")
            torch.cuda.synchronize()
            ref_o, ref_lse = _np_merge(parts, rows)
            np.testing.assert_allclose(out.cpu().numpy(), ref_o, rtol=0, atol=1e-5, err_msg=f"step {step}")
            np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, rtol=0, atol=1e-5)
        assert capi.get_device_error() == 0
    finally:
        ex.close()


def test_fused_exchange_wait_runs_out_when_a_peer_never_publishes():
    from ada_mla import capi

    lib = capi.lib()
    rows, world = 8, 2
    buf = ctypes.c_void_p()
    assert lib.mla_b200_exchange_alloc(world, rows, ctypes.byref(buf)) == capi.OK
    try:
        parts, _ = _packed(rows, 1, torch.Generator().manual_seed(6))
        part = parts[0].cuda()
        s = torch.cuda.current_stream().cuda_stream
        peers = (ctypes.c_void_p * world)(buf.value, buf.value)
        out = torch.full((rows, 512), 7.0, device="cuda")
        assert lib.mla_b200_exchange_f32(part.data_ptr(), rows, peers, 0, world, out.data_ptr(), capi.OUT_F32,
                                         None, 2_000_000, s) == capi.OK
        torch.cuda.synchronize()
        code = ctypes.c_int(0)
        assert lib.mla_b200_get_device_error(ctypes.byref(code), s) == capi.ERR_DEVICE_TIMEOUT
        assert code.value == 4
        assert bool((out == 7.0).all())
    finally:
        torch.cuda.synchronize()
        lib.mla_b200_exchange_free(buf.value)


def test_merge_wait_runs_out_when_a_peer_never_publishes():
    """A two-rank buffer whose rank 1 never puts: rank 0's merge gives up after
    its 2 ms limit with the peer-wait code, and leaves out untouched."""
    from ada_mla import capi

    lib = capi.lib()
    rows, world = 8, 2
    buf = ctypes.c_void_p()
    assert lib.mla_b200_exchange_alloc(world, rows, ctypes.byref(buf)) == capi.OK
    try:
        parts, _ = _packed(rows, 1, torch.Generator().manual_seed(4))
        part = parts[0].cuda()
        s = torch.cuda.current_stream().cuda_stream
        peers = (ctypes.c_void_p * world)(buf.value, buf.value)  # both parts land in this buffer
        assert lib.mla_b200_exchange_put_f32(part.data_ptr(), rows, peers, 0, world, s) == capi.OK
        out = torch.full((rows, 512), 7.0, device="cuda")
        assert lib.mla_b200_exchange_merge_f32(buf.value, world, rows, out.data_ptr(), capi.OUT_F32, None,
                                               2_000_000, s) == capi.OK
        torch.cuda.synchronize()
        code = ctypes.c_int(0)
        assert lib.mla_b200_get_device_error(ctypes.byref(code), s) == capi.ERR_DEVICE_TIMEOUT
        assert code.value == 4, "the peer-wait code"
        assert bool((out == 7.0).all()), "rows are left alone when the wait runs out"
        assert capi.get_device_error() == 0, "reading the word cleared it"
    finally:
        torch.cuda.synchronize()
        lib.mla_b200_exchange_free(buf.value)


def test_exchange_rejects_bad_arguments():
    from ada_mla import capi

    lib = capi.lib()
    buf = ctypes.c_void_p()
    assert lib.mla_b200_exchange_alloc(0, 8, ctypes.byref(buf)) == capi.ERR_INVALID_ARG
    assert lib.mla_b200_exchange_alloc(17, 8, ctypes.byref(buf)) == capi.ERR_INVALID_ARG
    assert lib.mla_b200_exchange_bytes(2, 8) == 256 + 2 * 2 * (8 * 513) * 4
    s = torch.cuda.current_stream().cuda_stream
    z = torch.zeros(16, device="cuda")
    assert lib.mla_b200_exchange_merge_f32(z.data_ptr(), 1, 8, z.data_ptr(), capi.OUT_F32, None, 0, s) \
        == capi.ERR_INVALID_ARG
