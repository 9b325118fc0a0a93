"""GPU parity of the decode entry points against the CPU oracle.

Inputs are seeded; fp16 kernels are compared with the oracle run on the same
fp16-rounded inputs upcast to fp32, on the north-star bar
(max-abs <= 1e-2, mean-abs <= 1e-3 on O*)."""
import os

import numpy as np
import pytest
import torch

import oracle
from conftest import assert_close_parity

pytestmark = pytest.mark.gpu

REF_SCALE = 1.0 / np.sqrt(192.0)
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mla_ref_golden.npz")


@pytest.fixture(scope="module")
def mla():
    import ada_mla

    return ada_mla


@pytest.fixture(scope="module")
def capi():
    from ada_mla import capi

    return capi


def _inputs(nh, n, seed, dtype=torch.float16, qscale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(nh, 576, generator=g) * qscale).to(dtype)
    c = torch.randn(n, 576, generator=g).to(dtype)
    return q, c


def _np(t):
    return t.detach().float().cpu().numpy()


def _no_device_error(mla):
    assert mla.mla_get_device_error() == 0


@pytest.mark.parametrize("n", [1, 15, 16, 17, 63, 64, 65, 1000, 4096, 4097])
@pytest.mark.parametrize("nh", [16, 128])
def test_split_f16_parity(mla, nh, n):
    q, c = _inputs(nh, n, seed=nh * 7 + n)
    out = mla.mla_decode_split(q.cuda(), c.cuda())
    assert out.shape == (nh, 512) and out.dtype == torch.float16
    ref = oracle.mla_decode_oracle(_np(q), _np(c), REF_SCALE, threads=8)
    assert_close_parity(_np(out), ref, what=f"split nh={nh} n={n}")
    _no_device_error(mla)


@pytest.mark.parametrize("splits", [1, 2, 3, 4, 7, 64, 148, 5000])
def test_split_f16_explicit_splits(mla, splits):
    q, c = _inputs(128, 4100, seed=splits)
    out = mla.mla_decode_split(q.cuda(), c.cuda(), splits)
    ref = oracle.mla_decode_oracle(_np(q), _np(c), REF_SCALE, threads=8)
    assert_close_parity(_np(out), ref, what=f"splits={splits}")


def test_split_f16_through_capi(capi):
    q, c = _inputs(128, 777, seed=3)
    out = capi.decode_split_f16(q.cuda(), c.cuda())
    torch.cuda.synchronize()
    ref = oracle.mla_decode_oracle(_np(q), _np(c), REF_SCALE, threads=8)
    assert_close_parity(_np(out), ref, what="capi split")
    assert capi.get_device_error() == 0


def test_split_empty_sequence_gives_zeros(capi):
    q, _ = _inputs(128, 1, seed=4)
    c = torch.empty(0, 576, dtype=torch.float16, device="cuda")
    out = capi.decode_split_f16(q.cuda(), c)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0


def test_golden_fixtures_on_gpu(mla):
    """The reference's own outputs (folded-scale fp16 cases) reproduced on the GPU."""
    z = np.load(GOLDEN)
    names = sorted({k.split("__")[0] for k in z.files if k.startswith("folded")})
    assert names
    for name in names:
        q = torch.from_numpy(z[f"{name}__q"]).cuda()
        c = torch.from_numpy(z[f"{name}__c"]).cuda()
        ref = z[f"{name}__out"][:, :512]
        out = mla.mla_decode_batched(q[None], c[None], softmax_scale=1.0, out_dtype=torch.float32)
        assert_close_parity(_np(out[0]), ref, what=name)


def test_fused_f32_parity(mla):
    q, c = _inputs(128, 1000, seed=5, dtype=torch.float32)
    out = mla.mla_decode_fused(q.cuda(), c.cuda())
    assert out.shape == (128, 512) and out.dtype == torch.float32
    ref = oracle.mla_decode_oracle(_np(q), _np(c), REF_SCALE, threads=8)
    assert_close_parity(_np(out), ref, max_tol=1e-4, mean_tol=1e-5, what="fused f32")
    # mla_decode_split with fp32 inputs works (the reference's fp32 branch is a stub)
    out2 = mla.mla_decode_split(q.cuda(), c.cuda())
    assert_close_parity(_np(out2), ref, max_tol=1e-4, mean_tol=1e-5, what="split f32")


@pytest.mark.parametrize("nh,n,d", [(128, 1000, 576), (5, 33, 576), (7, 19, 100)])
def test_naive_f32_reference_semantics(mla, capi, nh, n, d):
    g = torch.Generator().manual_seed(nh + n)
    q = torch.randn(nh, d, generator=g)
    c = torch.randn(n, d, generator=g)
    ref = oracle.run_mla_decode_cpu(_np(q), _np(c), threads=8)  # all d columns, 1/sqrt(d)
    out = mla.mla_decode_naive(q.cuda(), c.cuda())
    assert out.shape == (nh, d)
    assert_close_parity(_np(out), ref, max_tol=1e-4, mean_tol=1e-5, what="naive")
    out2 = capi.decode_naive_f32(q.cuda(), c.cuda())
    torch.cuda.synchronize()
    assert_close_parity(_np(out2), ref, max_tol=1e-4, mean_tol=1e-5, what="naive capi")


def test_batched_dense(mla):
    b, nh, n = 3, 16, 300
    g = torch.Generator().manual_seed(11)
    q = (torch.randn(b, nh, 576, generator=g) / np.sqrt(192)).half()
    c = torch.randn(b, n, 576, generator=g).half()
    out, lse = mla.mla_decode_batched(q.cuda(), c.cuda(), softmax_scale=1.0, return_lse=True)
    for i in range(b):
        ref = oracle.mla_decode_oracle(_np(q[i]), _np(c[i]), 1.0, threads=8)
        assert_close_parity(_np(out[i]), ref, what=f"dense b={i}")
        _, ref_lse = oracle.lse_partial_oracle(_np(q[i]), _np(c[i]), 1.0)
        np.testing.assert_allclose(_np(lse[i]), ref_lse, atol=2e-3, rtol=0)


def test_batched_varlen_with_empty(mla, capi):
    lens = [5, 0, 64, 129, 1, 700]
    nh = 128
    g = torch.Generator().manual_seed(12)
    q = (torch.randn(len(lens), nh, 576, generator=g) / np.sqrt(192)).half()
    c = torch.randn(sum(lens), 576, generator=g).half()
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    for num_splits in (-1, 1, 3):
        out = mla.mla_decode_batched(q.cuda(), c.cuda(), cu.cuda(), max_seq_len=max(lens),
                                     softmax_scale=1.0, num_splits=num_splits)
        out_c = capi.decode_batched_f16(q.cuda(), c.cuda(), cu.cuda(), max(lens), 1.0,
                                        num_splits=num_splits)
        torch.cuda.synchronize()
        lo = 0
        for i, n in enumerate(lens):
            if n == 0:
                assert torch.count_nonzero(out[i]).item() == 0
            else:
                ref = oracle.mla_decode_oracle(_np(q[i]), _np(c[lo:lo + n]), 1.0, threads=8)
                assert_close_parity(_np(out[i]), ref, what=f"varlen b={i} s={num_splits}")
                assert_close_parity(_np(out_c[i]), ref, what=f"varlen capi b={i}")
            lo += n


def test_combine_matches_numpy_merge(capi):
    rng = np.random.default_rng(4)
    p, rows = 5, 37
    po = rng.standard_normal((p, rows, 512)).astype(np.float32)
    pl = rng.standard_normal((p, rows)).astype(np.float32) * 3
    pl[1, :5] = -np.inf   # empty slices
    pl[:, 7] = -np.inf    # a row with no data at all
    out, lse = capi.combine_f32(torch.from_numpy(po).cuda(), torch.from_numpy(pl).cuda())
    torch.cuda.synchronize()
    m = pl.max(axis=0)
    mm = np.where(np.isfinite(m), m, 0)
    w = np.where(np.isfinite(pl), np.exp(pl - mm), 0)
    s = w.sum(axis=0)
    ref = np.einsum("pr,prd->rd", w, po) / np.where(s > 0, s, 1)[:, None]
    np.testing.assert_allclose(_np(out), ref, atol=1e-5, rtol=1e-5)
    assert np.all(_np(out)[7] == 0) and np.isneginf(_np(lse)[7])
    fin = np.isfinite(m)
    np.testing.assert_allclose(_np(lse)[fin], (m + np.log(np.where(s > 0, s, 1)))[fin], atol=1e-5)


def test_errors_raise(mla):
    q, c = _inputs(128, 64, seed=1)
    with pytest.raises(RuntimeError):
        mla.mla_decode_split(q.cuda(), c.cuda()[:, :512].contiguous())
    with pytest.raises(RuntimeError):
        mla.mla_decode_split(q.cuda(), c)  # cache on the host
    with pytest.raises(RuntimeError):
        mla.mla_decode_fused(q.cuda(), c.cuda())  # fp16 into the fp32 kernel name


@pytest.mark.parametrize("nh", [128, 16])
def test_balanced_schedule_varlen(mla, nh):
    """Automatic split of a mixed-length batch: the balanced schedule cuts sequences
    wherever a cluster's share ends (and skips empty ones); every sequence must
    still match the oracle."""
    rng = np.random.default_rng(21 + nh)
    lens = [int(x) for x in rng.integers(1, 1500, size=61)]
    lens[5] = 0
    lens[17] = 96
    lens[40] = 97
    g = torch.Generator().manual_seed(22)
    q = (torch.randn(len(lens), nh, 576, generator=g) / np.sqrt(192)).half()
    c = torch.randn(sum(lens), 576, generator=g).half()
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    out, lse = mla.mla_decode_batched(q.cuda(), c.cuda(), cu.cuda(), max_seq_len=max(lens),
                                      softmax_scale=1.0, return_lse=True)
    torch.cuda.synchronize()
    lo = 0
    for i, n in enumerate(lens):
        if n == 0:
            assert torch.count_nonzero(out[i]).item() == 0
        else:
            ref = oracle.mla_decode_oracle(_np(q[i]), _np(c[lo:lo + n]), 1.0, threads=8)
            assert_close_parity(_np(out[i]), ref, what=f"balanced varlen b={i} n={n}")
            if i % 10 == 0:
                _, ref_lse = oracle.lse_partial_oracle(_np(q[i]), _np(c[lo:lo + n]), 1.0)
                np.testing.assert_allclose(_np(lse[i]), ref_lse, atol=2e-3, rtol=0)
        lo += n
    _no_device_error(mla)


@pytest.mark.parametrize("b,n", [(37, 500), (3, 9000), (200, 96)])
def test_balanced_schedule_dense(mla, b, n):
    nh = 128
    g = torch.Generator().manual_seed(b + n)
    q = (torch.randn(b, nh, 576, generator=g) / np.sqrt(192)).half()
    c = torch.randn(b, n, 576, generator=g).half()
    out = mla.mla_decode_batched(q.cuda(), c.cuda(), softmax_scale=1.0)
    torch.cuda.synchronize()
    for i in range(0, b, max(1, b // 12)):
        ref = oracle.mla_decode_oracle(_np(q[i]), _np(c[i]), 1.0, threads=8)
        assert_close_parity(_np(out[i]), ref, what=f"balanced dense b={i}")
    _no_device_error(mla)


# bf16 inputs: O* is checked at the north-star bar with fp32 output (P enters the
# second GEMM as bf16, a 2^-9 relative rounding against fp16's 2^-11).  bf16
# output adds the rounding of the bf16 split partials and of the output, each up
# to half a bf16 ulp (2^-9 * |O*|), so that check is elementwise
# |got - ref| <= 1e-2 + 2^-8 * |ref| with mean-abs <= 2e-3.
def _assert_bf16_out(got, ref, what):
    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    d = np.abs(g - r)
    assert np.isfinite(g).all(), f"{what}: non-finite output"
    assert np.all(d <= 1e-2 + 2.0 ** -8 * np.abs(r)), f"{what}: max-abs {d.max():.3g}"
    assert d.mean() <= 2e-3, f"{what}: mean-abs {d.mean():.3g}"


@pytest.mark.parametrize("b,nh,n", [(3, 128, 300), (2, 16, 1), (40, 128, 257)])
def test_bf16_batched_dense(mla, b, nh, n):
    g = torch.Generator().manual_seed(31 + n)
    q = (torch.randn(b, nh, 576, generator=g) / np.sqrt(192)).bfloat16()
    c = torch.randn(b, n, 576, generator=g).bfloat16()
    out32, lse = mla.mla_decode_batched(q.cuda(), c.cuda(), softmax_scale=1.0, return_lse=True,
                                        out_dtype=torch.float32)
    out16 = mla.mla_decode_batched(q.cuda(), c.cuda(), softmax_scale=1.0)
    assert out16.dtype == torch.bfloat16 and out32.dtype == torch.float32
    torch.cuda.synchronize()
    for i in range(0, b, max(1, b // 8)):
        ref = oracle.mla_decode_oracle(_np(q[i]), _np(c[i]), 1.0, threads=8)
        assert_close_parity(_np(out32[i]), ref, what=f"bf16 dense fp32-out b={i}")
        _assert_bf16_out(_np(out16[i]), ref, what=f"bf16 dense bf16-out b={i}")
        _, ref_lse = oracle.lse_partial_oracle(_np(q[i]), _np(c[i]), 1.0)
        np.testing.assert_allclose(_np(lse[i]), ref_lse, atol=2e-3, rtol=0)
    _no_device_error(mla)


def test_bf16_batched_varlen(mla, capi):
    lens = [5, 0, 64, 96, 97, 129, 1, 700, 2500]
    nh = 128
    g = torch.Generator().manual_seed(32)
    q = (torch.randn(len(lens), nh, 576, generator=g) / np.sqrt(192)).bfloat16()
    c = torch.randn(sum(lens), 576, generator=g).bfloat16()
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    refs, lo = [], 0
    for n in lens:
        refs.append(oracle.mla_decode_oracle(_np(q[len(refs)]), _np(c[lo:lo + n]), 1.0, threads=8)
                    if n else None)
        lo += n
    for num_splits in (-1, 1, 3):
        out = mla.mla_decode_batched(q.cuda(), c.cuda(), cu.cuda(), max_seq_len=max(lens),
                                     softmax_scale=1.0, num_splits=num_splits)
        out_c = capi.decode_batched(q.cuda(), c.cuda(), cu.cuda(), max(lens), 1.0,
                                    num_splits=num_splits, out_fp32=True)
        torch.cuda.synchronize()
        for i, n in enumerate(lens):
            if n == 0:
                assert torch.count_nonzero(out[i]).item() == 0
                assert torch.count_nonzero(out_c[i]).item() == 0
            else:
                _assert_bf16_out(_np(out[i]), refs[i], what=f"bf16 varlen b={i} s={num_splits}")
                assert_close_parity(_np(out_c[i]), refs[i], what=f"bf16 varlen capi b={i}")
    _no_device_error(mla)


def test_bf16_beyond_fp16_range(mla):
    """bf16 carries magnitudes fp16 cannot (|x| > 65504): the cache is scaled by
    1e5 and the query by 1e-5 so the scores stay moderate while O* ~ 1e5; the
    partials stay fp32, so O* matches the oracle relative to that scale."""
    b, nh, n, s = 4, 128, 1000, 1e5
    g = torch.Generator().manual_seed(33)
    q = (torch.randn(b, nh, 576, generator=g) / np.sqrt(192) / s).bfloat16()
    c = (torch.randn(b, n, 576, generator=g) * s).bfloat16()
    out = mla.mla_decode_batched(q.cuda(), c.cuda(), softmax_scale=1.0, out_dtype=torch.float32)
    torch.cuda.synchronize()
    for i in range(b):
        ref = oracle.mla_decode_oracle(_np(q[i]), _np(c[i]), 1.0, threads=8)
        assert_close_parity(_np(out[i]) / s, ref / s, what=f"bf16 large b={i}")
    _no_device_error(mla)


def test_bf16_rejects_mixed_dtypes(mla):
    q = torch.randn(1, 16, 576).bfloat16().cuda()
    c = torch.randn(1, 64, 576).half().cuda()
    with pytest.raises(RuntimeError):
        mla.mla_decode_batched(q, c)
    with pytest.raises(ValueError):
        mla.mla_decode_batched(q, c.bfloat16(), out_dtype=torch.float16)


# ---------------------------------------------------------------------------
# Paged latent cache


def _paged(lens, page_size, nh, seed, dtype=torch.float16, spare_pages=3):
    """Packed per-sequence caches scattered over a shuffled page pool whose unused
    rows hold NaN; block-table slots past a sequence's pages hold -1."""
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(len(lens), nh, 576, generator=g) / np.sqrt(192)).to(dtype)
    packed = torch.randn(sum(lens), 576, generator=g).to(dtype)
    npg = [-(-n // page_size) for n in lens]
    num_pages = sum(npg) + spare_pages
    perm = torch.randperm(num_pages, generator=g)
    pool = torch.full((num_pages, page_size, 576), float("nan"), dtype=dtype)
    max_blocks = max(max(npg), 1) + 1
    bt = torch.full((len(lens), max_blocks), -1, dtype=torch.int32)
    lo, used = 0, 0
    for b, n in enumerate(lens):
        for k in range(npg[b]):
            pg = int(perm[used])
            used += 1
            bt[b, k] = pg
            rows = packed[lo + k * page_size: lo + min(n, (k + 1) * page_size)]
            pool[pg, :rows.shape[0]] = rows
        lo += n
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    return q, packed, cu, pool, bt, torch.tensor(lens, dtype=torch.int32)


@pytest.mark.parametrize("page_size", [32, 64, 128])
@pytest.mark.parametrize("nh", [128, 16])
def test_paged_matches_packed_and_oracle(mla, page_size, nh):
    """Automatic split: the paged decode runs the same schedule as the packed
    varlen decode of the same sequences, so the outputs agree bit for bit; both
    match the oracle.  NaN in unused page rows must not reach the result."""
    lens = [1, 31, 32, 33, 0, 64, 95, 96, 97, 128, 129, 700, 2500]
    q, packed, cu, pool, bt, sl = _paged(lens, page_size, nh, seed=40 + page_size + nh)
    out_p, lse_p = mla.mla_decode_paged(q.cuda(), pool.cuda(), bt.cuda(), sl.cuda(),
                                        max_seq_len=max(lens), softmax_scale=1.0, return_lse=True)
    out_v, lse_v = mla.mla_decode_batched(q.cuda(), packed.cuda(), cu.cuda(), max_seq_len=max(lens),
                                          softmax_scale=1.0, return_lse=True)
    torch.cuda.synchronize()
    assert torch.equal(out_p, out_v)
    assert torch.equal(lse_p[sl.cuda() > 0], lse_v[sl.cuda() > 0])
    lo = 0
    for i, n in enumerate(lens):
        if n == 0:
            assert torch.count_nonzero(out_p[i]).item() == 0
        else:
            ref = oracle.mla_decode_oracle(_np(q[i]), _np(packed[lo:lo + n]), 1.0, threads=8)
            assert_close_parity(_np(out_p[i]), ref, what=f"paged ps={page_size} b={i} n={n}")
        lo += n
    _no_device_error(mla)


@pytest.mark.parametrize("num_splits", [-1, 1, 3, 7])
def test_paged_single_long_sequence(mla, capi, num_splits):
    lens = [20000 + 17]
    q, packed, cu, pool, bt, sl = _paged(lens, 64, 128, seed=50)
    ref = oracle.mla_decode_oracle(_np(q[0]), _np(packed), REF_SCALE, threads=8)
    out = mla.mla_decode_paged(q.cuda(), pool.cuda(), bt.cuda(), sl.cuda(), max_seq_len=lens[0],
                               softmax_scale=REF_SCALE, num_splits=num_splits)
    out_c = capi.decode_paged(q.cuda(), pool.cuda(), bt.cuda(), sl.cuda(), lens[0], REF_SCALE,
                              num_splits=num_splits, out_fp32=True)
    torch.cuda.synchronize()
    assert_close_parity(_np(out[0]), ref, what=f"paged long s={num_splits}")
    assert_close_parity(_np(out_c[0]), ref, what=f"paged long capi s={num_splits}")
    _no_device_error(mla)


@pytest.mark.parametrize("num_splits", [1, 2, 5])
def test_paged_explicit_splits_batch(mla, num_splits):
    lens = [300, 0, 1, 4097, 96, 1000]
    q, packed, cu, pool, bt, sl = _paged(lens, 128, 128, seed=51 + num_splits)
    out = mla.mla_decode_paged(q.cuda(), pool.cuda(), bt.cuda(), sl.cuda(), max_seq_len=max(lens),
                               softmax_scale=1.0, num_splits=num_splits)
    torch.cuda.synchronize()
    lo = 0
    for i, n in enumerate(lens):
        if n == 0:
            assert torch.count_nonzero(out[i]).item() == 0
        else:
            ref = oracle.mla_decode_oracle(_np(q[i]), _np(packed[lo:lo + n]), 1.0, threads=8)
            assert_close_parity(_np(out[i]), ref, what=f"paged splits={num_splits} b={i}")
        lo += n
    _no_device_error(mla)


def test_paged_bf16(mla):
    lens = [5, 0, 64, 97, 1500, 33]
    q, packed, cu, pool, bt, sl = _paged(lens, 64, 128, seed=52, dtype=torch.bfloat16)
    out = mla.mla_decode_paged(q.cuda(), pool.cuda(), bt.cuda(), sl.cuda(), softmax_scale=1.0,
                               out_dtype=torch.float32)
    out_v = mla.mla_decode_batched(q.cuda(), packed.cuda(), cu.cuda(), max_seq_len=max(lens),
                                   softmax_scale=1.0, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(out, out_v)
    lo = 0
    for i, n in enumerate(lens):
        if n:
            ref = oracle.mla_decode_oracle(_np(q[i]), _np(packed[lo:lo + n]), 1.0, threads=8)
            assert_close_parity(_np(out[i]), ref, what=f"paged bf16 b={i}")
        lo += n
    _no_device_error(mla)


def test_paged_rejects_bad_shapes(mla):
    q = torch.randn(2, 16, 576).half().cuda()
    pool = torch.randn(4, 48, 576).half().cuda()   # page size not a multiple of 32
    bt = torch.zeros(2, 2, dtype=torch.int32).cuda()
    sl = torch.tensor([10, 20], dtype=torch.int32).cuda()
    with pytest.raises(RuntimeError):
        mla.mla_decode_paged(q, pool, bt, sl)
    with pytest.raises(RuntimeError):
        mla.mla_decode_paged(q, pool[:, :32].contiguous(), bt[:1], sl)  # block table rows != B


# ---------------------------------------------------------------------------
# FP8 (e4m3) latent cache: the oracle runs on the dequantized cache (the
# e4m3 values times kv_scale, exact in fp32) with the same fp16 Q*.  The
# kernel rounds Q* to two e4m3 planes (about 2^-8 relative, like bf16) and
# keeps P fp16: the north-star bar applies unchanged.


def _fp8_inputs(lens, nh, seed, kv_scale, dense_n=None):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(len(lens), nh, 576, generator=g) / np.sqrt(192)).half()
    total = sum(lens)
    c = (torch.randn(total, 576, generator=g) / kv_scale).to(torch.float8_e4m3fn)
    deq = c.float() * kv_scale
    return q, c, deq


@pytest.mark.parametrize("kv_scale", [1.0, 1.0 / 16])
def test_fp8_dense(mla, kv_scale):
    b, nh, n = 3, 128, 300
    q, c, deq = _fp8_inputs([n] * b, nh, seed=61, kv_scale=kv_scale)
    out32, lse = mla.mla_decode_batched(q.cuda(), c.view(b, n, 576).cuda(), softmax_scale=1.0,
                                        return_lse=True, out_dtype=torch.float32, kv_scale=kv_scale)
    out16 = mla.mla_decode_batched(q.cuda(), c.view(b, n, 576).cuda(), softmax_scale=1.0,
                                   kv_scale=kv_scale)
    torch.cuda.synchronize()
    assert out16.dtype == torch.float16
    for i in range(b):
        rows = deq[i * n:(i + 1) * n].numpy()
        ref = oracle.mla_decode_oracle(_np(q[i]), rows, 1.0, threads=8)
        assert_close_parity(_np(out32[i]), ref, what=f"fp8 dense fp32-out b={i}")
        assert_close_parity(_np(out16[i]), ref, what=f"fp8 dense fp16-out b={i}")
        _, ref_lse = oracle.lse_partial_oracle(_np(q[i]), rows, 1.0)
        np.testing.assert_allclose(_np(lse[i]), ref_lse, atol=2e-3, rtol=0)
    _no_device_error(mla)


@pytest.mark.parametrize("num_splits", [-1, 1, 3])
def test_fp8_varlen(mla, capi, num_splits):
    lens = [5, 0, 64, 95, 96, 97, 129, 1, 700, 2500]
    q, c, deq = _fp8_inputs(lens, 128, seed=62, kv_scale=0.25)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    out = mla.mla_decode_batched(q.cuda(), c.cuda(), cu.cuda(), max_seq_len=max(lens),
                                 softmax_scale=1.0, num_splits=num_splits, kv_scale=0.25)
    out_c = capi.decode_batched_fp8(q.cuda(), c.cuda(), 0.25, cu.cuda(), max(lens), 1.0,
                                    num_splits=num_splits, out_fp32=True)
    torch.cuda.synchronize()
    lo = 0
    for i, n in enumerate(lens):
        if n == 0:
            assert torch.count_nonzero(out[i]).item() == 0
        else:
            ref = oracle.mla_decode_oracle(_np(q[i]), deq[lo:lo + n].numpy(), 1.0, threads=8)
            assert_close_parity(_np(out[i]), ref, what=f"fp8 varlen b={i} n={n} s={num_splits}")
            assert_close_parity(_np(out_c[i]), ref, what=f"fp8 varlen capi b={i}")
        lo += n
    _no_device_error(mla)


@pytest.mark.parametrize("b,nh,n", [(40, 16, 257), (1, 128, 20017)])
def test_fp8_batches_and_long(mla, b, nh, n):
    q, c, deq = _fp8_inputs([n] * b, nh, seed=63 + b, kv_scale=0.5)
    out = mla.mla_decode_batched(q.cuda(), c.view(b, n, 576).cuda(), softmax_scale=1.0,
                                 out_dtype=torch.float32, kv_scale=0.5)
    torch.cuda.synchronize()
    for i in range(0, b, max(1, b // 8)):
        ref = oracle.mla_decode_oracle(_np(q[i]), deq[i * n:(i + 1) * n].numpy(), 1.0, threads=8)
        assert_close_parity(_np(out[i]), ref, what=f"fp8 b={i}")
    _no_device_error(mla)


def _fp8_row_scaled_inputs(lens, nh, seed, block):
    """e4m3 cache with one scale per row, constant over blocks of `block` rows
    (a per-tile / per-page scaling) and spread over 2^-2 .. 2^2.6 (a 2^4.6
    span, inside the documented ~2^5 per-tile envelope)."""
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(len(lens), nh, 576, generator=g) / np.sqrt(192)).half()
    total = sum(lens)
    nb = -(-total // block)
    sblk = torch.pow(2.0, torch.randint(-2, 3, (nb,), generator=g).float()) * \
        (1 + 0.5 * torch.rand(nb, generator=g))
    scales = sblk.repeat_interleave(block)[:total].contiguous()
    c = (torch.randn(total, 576, generator=g) / scales[:, None]).to(torch.float8_e4m3fn)
    deq = c.float() * scales[:, None]
    return q, c, scales, deq


@pytest.mark.parametrize("block", [32, 96, 1])
@pytest.mark.parametrize("num_splits", [-1, 2])
def test_fp8_row_scales_varlen(mla, block, num_splits):
    """Per-tile (32 or 96 rows) and per-row scales on a packed varlen batch."""
    lens = [7, 96, 130, 1000, 2500, 0, 64]
    q, c, scales, deq = _fp8_row_scaled_inputs(lens, 128, seed=64 + block, block=block)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    out = mla.mla_decode_batched(q.cuda(), c.cuda(), cu.cuda(), max_seq_len=max(lens), softmax_scale=1.0,
                                 num_splits=num_splits, out_dtype=torch.float32, kv_scale=scales.cuda())
    torch.cuda.synchronize()
    lo = 0
    for i, n in enumerate(lens):
        if n == 0:
            assert torch.count_nonzero(out[i]).item() == 0
        else:
            ref = oracle.mla_decode_oracle(_np(q[i]), deq[lo:lo + n].numpy(), 1.0, threads=8)
            assert_close_parity(_np(out[i]), ref, what=f"fp8 row scales block={block} b={i} n={n}")
        lo += n
    _no_device_error(mla)


def test_fp8_row_scales_dense_long(mla):
    b, nh, n = 2, 128, 9000
    q, c, scales, deq = _fp8_row_scaled_inputs([n] * b, nh, seed=69, block=64)
    out16, lse = mla.mla_decode_batched(q.cuda(), c.view(b, n, 576).cuda(), softmax_scale=1.0, return_lse=True,
                                        kv_scale=scales.view(b, n).cuda())
    torch.cuda.synchronize()
    for i in range(b):
        rows = deq[i * n:(i + 1) * n].numpy()
        ref = oracle.mla_decode_oracle(_np(q[i]), rows, 1.0, threads=8)
        assert_close_parity(_np(out16[i]), ref, what=f"fp8 row scales dense b={i}")
        _, ref_lse = oracle.lse_partial_oracle(_np(q[i]), rows, 1.0)
        np.testing.assert_allclose(_np(lse[i]), ref_lse, atol=2e-3, rtol=0)
    _no_device_error(mla)


# ---------------------------------------------------------------------------
# Multi-token (draft) decode: draft token i of k sees the first L - (k-1-i)
# tokens of its sequence; the oracle runs each (sequence, token) separately.


def _mtp_check(mla, q, c_rows, lens, out, what, lse=None):
    k = q.shape[1]
    lo = 0
    for b, n in enumerate(lens):
        for i in range(k):
            vis = n - (k - 1 - i)
            if vis <= 0:
                assert torch.count_nonzero(out[b, i]).item() == 0, f"{what} b={b} i={i}"
                continue
            rows = c_rows[lo:lo + vis]
            ref = oracle.mla_decode_oracle(_np(q[b, i]), _np(rows), 1.0, threads=8)
            assert_close_parity(_np(out[b, i]), ref, what=f"{what} b={b} i={i} n={n}")
            if lse is not None and i == k - 1 and b % 3 == 0:
                _, ref_lse = oracle.lse_partial_oracle(_np(q[b, i]), _np(rows), 1.0)
                np.testing.assert_allclose(_np(lse[b, i]), ref_lse, atol=2e-3, rtol=0)
        lo += n


@pytest.mark.parametrize("k,nh", [(8, 16), (2, 64), (1, 128)])
def test_mtp_dense(mla, k, nh):
    b, n = 12, 700
    g = torch.Generator().manual_seed(71 + k)
    q = (torch.randn(b, k, nh, 576, generator=g) / np.sqrt(192)).half()
    c = torch.randn(b, n, 576, generator=g).half()
    out, lse = mla.mla_decode_mtp(q.cuda(), c.cuda(), softmax_scale=1.0, return_lse=True)
    torch.cuda.synchronize()
    assert out.shape == (b, k, nh, 512)
    _mtp_check(mla, q, c.view(-1, 576), [n] * b, out, f"mtp dense k={k}", lse)
    if k == 1:  # one draft token is the plain batched decode, bit for bit
        ref = mla.mla_decode_batched(q[:, 0].contiguous().cuda(), c.cuda(), softmax_scale=1.0)
        torch.cuda.synchronize()
        assert torch.equal(out[:, 0], ref)
    _no_device_error(mla)


@pytest.mark.parametrize("num_splits", [-1, 1, 4])
def test_mtp_varlen_short_and_split(mla, num_splits):
    """Sequences shorter than, equal to and just past the draft count, a split
    landing inside the last k-1 tokens (97 = 96 + 1), and long ones."""
    k, nh = 8, 16
    lens = [3, 8, 9, 96, 97, 100, 1500, 40]
    g = torch.Generator().manual_seed(72)
    q = (torch.randn(len(lens), k, nh, 576, generator=g) / np.sqrt(192)).bfloat16()
    c = torch.randn(sum(lens), 576, generator=g).bfloat16()
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    out = mla.mla_decode_mtp(q.cuda(), c.cuda(), cu.cuda(), max_seq_len=max(lens), softmax_scale=1.0,
                             num_splits=num_splits, out_dtype=torch.float32)
    torch.cuda.synchronize()
    _mtp_check(mla, q, c, lens, out, f"mtp varlen s={num_splits}")
    _no_device_error(mla)


@pytest.mark.parametrize("k", [2, 4])
def test_mtp_128_heads_dense(mla, k):
    """k x 128 rows do not fit one MMA tile: each draft token runs as its own
    128-row sequence over the same cache rows, up to its causal limit."""
    b, nh, n = 3, 128, 2000
    g = torch.Generator().manual_seed(90 + k)
    q = (torch.randn(b, k, nh, 576, generator=g) / np.sqrt(192)).half()
    c = torch.randn(b, n, 576, generator=g).half()
    out, lse = mla.mla_decode_mtp(q.cuda(), c.cuda(), softmax_scale=1.0, return_lse=True)
    torch.cuda.synchronize()
    assert out.shape == (b, k, nh, 512) and lse.shape == (b, k, nh)
    _mtp_check(mla, q, c.view(-1, 576), [n] * b, out, f"mtp128 dense k={k}", lse)
    _no_device_error(mla)


@pytest.mark.parametrize("num_splits", [-1, 3])
def test_mtp_128_heads_varlen(mla, num_splits):
    """Packed varlen bf16 with 128 heads and 4 drafts: sequences shorter than
    the draft count (some drafts see nothing), a split boundary inside the
    last k-1 tokens, a single long sequence."""
    k, nh = 4, 128
    lens = [2, 4, 97, 1300, 5000]
    g = torch.Generator().manual_seed(95)
    q = (torch.randn(len(lens), k, nh, 576, generator=g) / np.sqrt(192)).bfloat16()
    c = torch.randn(sum(lens), 576, generator=g).bfloat16()
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    out = mla.mla_decode_mtp(q.cuda(), c.cuda(), cu.cuda(), max_seq_len=max(lens), softmax_scale=1.0,
                             num_splits=num_splits, out_dtype=torch.float32)
    torch.cuda.synchronize()
    _mtp_check(mla, q, c, lens, out, f"mtp128 varlen s={num_splits}")
    _no_device_error(mla)


def test_mtp_128_heads_draft_equals_batched_decode(mla):
    """The last draft token sees the whole sequence: it equals the batched
    decode of that token's queries, bit for bit (same kernel, same split of a
    sequence of the same length on the cost line is not guaranteed, so the
    check is the parity bar against the batched result)."""
    b, k, nh, n = 2, 2, 128, 4096
    g = torch.Generator().manual_seed(97)
    q = (torch.randn(b, k, nh, 576, generator=g) / np.sqrt(192)).half().cuda()
    c = torch.randn(b, n, 576, generator=g).half().cuda()
    out = mla.mla_decode_mtp(q, c, softmax_scale=1.0)
    ref = mla.mla_decode_batched(q[:, k - 1].contiguous(), c, softmax_scale=1.0)
    torch.cuda.synchronize()
    assert_close_parity(_np(out[:, k - 1]), _np(ref), what="mtp128 last draft vs batched")
    _no_device_error(mla)


# ---------------------------------------------------------------------------
# Weight absorption around the decode: the absorbed pipeline equals per-head
# attention over up-projected keys and values (fp32 torch reference).


def test_absorbed_pipeline_matches_unabsorbed_attention(mla):
    from ada_mla import absorbed

    torch.manual_seed(81)
    b, nh, n, dn, dv = 4, 16, 300, 128, 128
    scale = 1.0 / np.sqrt(dn + 64)
    c = torch.randn(b, n, 576) * 0.5
    q_nope = torch.randn(b, nh, dn) * 0.5
    q_rope = torch.randn(b, nh, 64) * 0.5
    w_uk = torch.randn(nh, dn, 512) / np.sqrt(512)
    w_uv = torch.randn(nh, 512, dv) / np.sqrt(512)
    # reference: keys k_j,i = c_j,N W_UK_i^T, values v_j,i = c_j,N W_UV_i, rope part shared
    k_nope = torch.einsum("bnc,hdc->bhnd", c[:, :, :512], w_uk)           # [b, h, n, d]
    v = torch.einsum("bnc,hcv->bhnv", c[:, :, :512], w_uv)                # [b, h, n, dv]
    logits = (torch.einsum("bhd,bhnd->bhn", q_nope, k_nope) +
              torch.einsum("bhr,bnr->bhn", q_rope, c[:, :, 512:])) * scale
    ref = torch.einsum("bhn,bhnv->bhv", torch.softmax(logits, dim=-1), v)
    out = absorbed.mla_decode_absorbed(q_nope.half().cuda(), q_rope.half().cuda(), w_uk.half().cuda(),
                                       c.half().cuda(), w_uv.half().cuda(), softmax_scale=scale)
    torch.cuda.synchronize()
    assert out.shape == (b, nh, dv)
    # fp16 operands and an fp16 O* between the steps: relative error ~1e-3 of |ref| ~ 0.1-1
    assert_close_parity(_np(out), ref.numpy(), max_tol=2e-2, mean_tol=2e-3, what="absorbed pipeline")
    _no_device_error(mla)
