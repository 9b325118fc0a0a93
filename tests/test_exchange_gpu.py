"""The peer-memory exchange kernels of the split-KV multi-GPU step
(mla_b200_exchange_put_f32 / _merge_f32 / _f32, mla_b200_decode_exchange_f16)
on one GPU: a single rank's buffer goes through put + merge for several steps
(both parities of the buffer), the merged output against a numpy LSE merge of
the same packed partials; the decode with its merge fused into the exchange
against the plain decode; and a peer that never publishes makes the bounded
wait run out (a flag that nothing sets: no fault), report the peer-wait code
and leave the rows alone.  The two-rank path runs in tests/test_multigpu_gpu.py."""
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
    assert lib.mla_b200_exchange_bytes(2, 8) == 256 + 2 * 2 * (8 * 513) * 8  # header, 2 parities x 2 parts
    assert lib.mla_b200_exchange_bytes(1, 65) == 512 + 2 * (65 * 513 + 1) * 8  # stride rounded up to even
    s = torch.cuda.current_stream().cuda_stream
    z = torch.zeros(16, device="cuda")
    assert lib.mla_b200_exchange_merge_f32(z.data_ptr(), 1, 8, z.data_ptr(), capi.OUT_F32, None, 0, s) \
        == capi.ERR_INVALID_ARG


def _plain_decode(q, c, scale, out_fp32):
    """mla_b200_decode_batched_f16 on a dense batch: (out, lse)."""
    from ada_mla import capi

    b, nh, n = q.shape[0], q.shape[1], c.shape[1]
    ws = torch.empty(max(256, capi.workspace_size(b, nh, b * n, n, -1)), dtype=torch.uint8, device="cuda")
    out = torch.empty(b * nh, 512, dtype=torch.float32 if out_fp32 else torch.float16, device="cuda")
    lse = torch.empty(b * nh, device="cuda")
    assert capi.lib().mla_b200_decode_batched_f16(
        q.data_ptr(), c.data_ptr(), None, b, nh, b * n, n, scale, -1, out.data_ptr(),
        capi.OUT_F32 if out_fp32 else capi.OUT_F16, lse.data_ptr(), ws.data_ptr(), ws.numel(),
        torch.cuda.current_stream().cuda_stream) == capi.OK
    return out, lse


@pytest.mark.parametrize("b,nh,n,out_fp32", [
    (1, 128, 5000, False),  # one long sequence: many splits per row
    (100, 2, 192, False),   # a batch on the balanced schedule: single-item rows and split rows
    (2, 64, 777, True),     # fp32 output
])
def test_decode_exchange_single_rank_matches_decode(b, nh, n, out_fp32):
    """mla_b200_decode_exchange_f16 with one rank (its own buffer the only peer)
    over several steps: the decode's split merge, the put and the merge of one
    part give the plain decode's output, and its LSE."""
    from ada_mla import capi
    from ada_mla.multigpu import PeerExchange, packed_stride

    g = torch.Generator().manual_seed(b * 1000 + n)
    q = (torch.randn(b, nh, 576, generator=g) / 192 ** 0.5).half().cuda()
    c = torch.randn(b, n, 576, generator=g).half().cuda()
    scale = 1.0 / 192 ** 0.5
    ref_o, ref_lse = _plain_decode(q, c, scale, out_fp32)
    rows = b * nh
    ex = PeerExchange(rows)
    try:
        ws = torch.empty(max(256, capi.workspace_size(b, nh, b * n, n, -1)), dtype=torch.uint8, device="cuda")
        direct = torch.empty(packed_stride(rows), device="cuda")
        for step in range(3):
            res = ex.decode_exchange(q, c, scale, ws, direct, torch.float32 if out_fp32 else torch.float16)
            assert res is not None
            out, lse = res
            torch.cuda.synchronize()
            d = (out.float() - ref_o.float()).abs()
            assert float(d.max()) <= (1e-6 if out_fp32 else 1e-3), (step, float(d.max()))
            assert float((lse - ref_lse).abs().max()) <= 1e-5, step
        assert capi.get_device_error() == 0
    finally:
        ex.close()


def test_decode_exchange_rejects_rows_that_do_not_fit():
    """More rows than the exchange kernel can hold resident at once: refused
    before anything is launched (the caller falls back to decode + exchange)."""
    from ada_mla import capi
    from ada_mla.multigpu import PeerExchange, packed_stride

    b, nh, n = 19, 128, 96  # 2432 rows: more than 148 SMs x 4 blocks of 512 threads
    q = torch.zeros(b, nh, 576, dtype=torch.float16, device="cuda")
    c = torch.zeros(b, n, 576, dtype=torch.float16, device="cuda")
    ex = PeerExchange(b * nh)
    try:
        ws = torch.empty(max(256, capi.workspace_size(b, nh, b * n, n, -1)), dtype=torch.uint8, device="cuda")
        direct = torch.full((packed_stride(b * nh),), 5.0, device="cuda")
        assert ex.decode_exchange(q, c, 0.1, ws, direct) is None
        torch.cuda.synchronize()
        assert bool((direct == 5.0).all()), "nothing ran"
    finally:
        ex.close()


def test_ranks_that_disagree_on_the_word_format_time_out():
    """Two ranks' buffers in one process: "rank 1" exchanges with fp32 output
    (fp32 payload words) and "rank 0" with fp16 output (fp16 payload words).
    Rank 0 must not read rank 1's words as fp16 pairs: the format bit in each
    word's epoch half keeps them from matching, its wait runs out (code 4) and
    its rows stay untouched.  (Rank 1's own wait runs out first: rank 0 has not
    put yet when it runs.)"""
    from ada_mla import capi

    lib = capi.lib()
    rows, world = 8, 2
    bufs = [ctypes.c_void_p(), ctypes.c_void_p()]
    for b in bufs:
        assert lib.mla_b200_exchange_alloc(world, rows, ctypes.byref(b)) == capi.OK
    try:
        parts, _ = _packed(rows, 1, torch.Generator().manual_seed(8))
        part = parts[0].cuda()
        s = torch.cuda.current_stream().cuda_stream
        peers = (ctypes.c_void_p * world)(bufs[0].value, bufs[1].value)
        code = ctypes.c_int(0)
        out1 = torch.full((rows, 512), 7.0, device="cuda")
        assert lib.mla_b200_exchange_f32(part.data_ptr(), rows, peers, 1, world, out1.data_ptr(), capi.OUT_F32,
                                         None, 2_000_000, s) == capi.OK
        torch.cuda.synchronize()
        assert lib.mla_b200_get_device_error(ctypes.byref(code), s) == capi.ERR_DEVICE_TIMEOUT
        out0 = torch.full((rows, 512), 7.0, dtype=torch.float16, device="cuda")
        assert lib.mla_b200_exchange_f32(part.data_ptr(), rows, peers, 0, world, out0.data_ptr(), capi.OUT_F16,
                                         None, 2_000_000, s) == capi.OK
        torch.cuda.synchronize()
        assert lib.mla_b200_get_device_error(ctypes.byref(code), s) == capi.ERR_DEVICE_TIMEOUT
        assert code.value == 4
        assert bool((out0 == 7.0).all()), "no row merged from words of the other format"
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            lib.mla_b200_exchange_free(b.value)
