"""The CPU oracle against the reference's own outputs (golden fixtures) and,
where it was built here, against the reference function itself."""
import os

import numpy as np
import pytest

import oracle
from conftest import assert_close_parity

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mla_ref_golden.npz")


def _cases():
    z = np.load(GOLDEN)
    names = sorted({k.split("__")[0] for k in z.files})
    return [(n, z[f"{n}__q"], z[f"{n}__c"], z[f"{n}__out"]) for n in names]


@pytest.mark.parametrize("name,q,c,out", _cases(), ids=lambda v: v if isinstance(v, str) else "")
def test_oracle_matches_reference_golden(name, q, c, out):
    q32 = q.astype(np.float32)
    if name.startswith("folded"):
        q32 = (q32 * np.float32(24.0)).astype(np.float32)
    got = oracle.run_mla_decode_cpu(q32, c.astype(np.float32))
    # The restatement follows the reference's arithmetic order: bit-exact.
    np.testing.assert_array_equal(got, out)


def test_golden_fixture_shapes():
    for name, q, c, out in _cases():
        assert q.shape[1] == 576 and c.shape[1] == 576
        assert out.shape == (q.shape[0], 576)
        if name.startswith("folded"):
            assert q.dtype == np.float16 and c.dtype == np.float16


def test_oracle_vs_double_precision():
    rng = np.random.default_rng(3)
    q = rng.standard_normal((16, 576), dtype=np.float32)
    c = rng.standard_normal((257, 576), dtype=np.float32)
    a = oracle.run_mla_decode_cpu(q, c)
    b = oracle.mla_decode_f64(q, c, 1.0 / 24.0, 576)
    assert np.abs(a - b).max() < 1e-5


@pytest.mark.skipif(not oracle.have_ref(), reason="reference CPU kernel not built here")
@pytest.mark.parametrize("nh,n", [(1, 1), (3, 5), (16, 64), (128, 96)])
def test_oracle_bitexact_with_reference_build(nh, n):
    rng = np.random.default_rng(nh * 1000 + n)
    q = rng.standard_normal((nh, 576), dtype=np.float32)
    c = rng.standard_normal((n, 576), dtype=np.float32)
    np.testing.assert_array_equal(oracle.run_mla_decode_cpu(q, c),
                                  oracle.run_mla_decode_cpu(q, c, impl="reference"))


def test_oracle_threads_identical():
    rng = np.random.default_rng(5)
    q = rng.standard_normal((37, 576), dtype=np.float32)
    c = rng.standard_normal((70, 576), dtype=np.float32)
    np.testing.assert_array_equal(oracle.run_mla_decode_cpu(q, c, threads=1),
                                  oracle.run_mla_decode_cpu(q, c, threads=4))


def test_folded_scale_adapter():
    """Q * scale * sqrt(576) through the reference kernel == softmax(scale Q C^T) C[:, :512]."""
    rng = np.random.default_rng(11)
    q = (rng.standard_normal((8, 576)) / np.sqrt(192)).astype(np.float16).astype(np.float32)
    c = rng.standard_normal((100, 576)).astype(np.float16).astype(np.float32)
    for scale in (1.0, 1.0 / np.sqrt(192.0)):
        a = oracle.mla_decode_oracle(q, c, scale)
        b = oracle.mla_decode_f64(q, c, scale, 512)
        assert a.shape == (8, 512)
        assert np.abs(a - b).max() < 2e-5


def test_lse_partials_merge_to_full():
    """Merging per-slice (O, lse) with weights e^{lse_i - max} reproduces the full decode."""
    rng = np.random.default_rng(2)
    q = rng.standard_normal((4, 576)) / np.sqrt(192)
    c = rng.standard_normal((300, 576))
    full, full_lse = oracle.lse_partial_oracle(q, c, 1.0)
    cuts = [0, 0, 17, 150, 300]  # includes an empty slice
    parts = [oracle.lse_partial_oracle(q, c[a:b], 1.0) for a, b in zip(cuts[:-1], cuts[1:])]
    lse = np.stack([p[1] for p in parts])
    m = lse.max(axis=0)
    w = np.exp(lse - m)
    merged = sum(w[i][:, None] * parts[i][0] for i in range(len(parts))) / w.sum(axis=0)[:, None]
    assert np.abs(merged - full).max() < 1e-12
    assert np.abs(m + np.log(w.sum(axis=0)) - full_lse).max() < 1e-12


def test_parity_helper_rejects_out_of_tolerance():
    """A mistake planted in the oracle output must fail the parity bar."""
    rng = np.random.default_rng(9)
    q = (rng.standard_normal((4, 576)) / np.sqrt(192)).astype(np.float32)
    c = rng.standard_normal((64, 576)).astype(np.float32)
    ref = oracle.mla_decode_oracle(q, c, 1.0)
    assert_close_parity(ref + 1e-4, ref)
    bad = ref.copy()
    bad[1, 3] += 0.05
    with pytest.raises(AssertionError):
        assert_close_parity(bad, ref)
