"""GPU parity at the benchmark configurations' full sizes, through the schedules
the benchmark runs (automatic split), against the CPU oracle (the reference's
run_mla_decode_cpu, csrc/mla_decode_naive_fp32_cpu.cpp:5-61, restated in
oracle/mla_oracle.c) on all host threads.

  cfg 1  B=1, n_h=128, N=4096: 43 single-tile items + the split merge
  cfg 2  B=128, n_h=128, N_b ~ U[1024, 8192], packed: the balanced schedule over
         all 74 clusters + the row-parallel merge; every sequence checked
  cfg 3  B=1, n_h=128, N=131072: 72 items of 1824 tokens + the split merge
  cfg 4  B=256, n_h=16, N=2048, dense: the balanced schedule, sequences split
         where a cluster's share ends; every sequence checked

Inputs are the benchmark's own seeded generators (ada_mla.workloads, seed 0).
Bar: the north star's max-abs <= 1e-2 and mean-abs <= 1e-3 on O*, per
sequence, with the fp16 output compared to the oracle on the same
fp16-rounded inputs."""
import os

import numpy as np
import pytest
import torch

import oracle
from conftest import assert_close_parity

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1


@pytest.fixture(scope="module")
def mla():
    import ada_mla

    return ada_mla


def _decode(mla, wl):
    out, lse = mla.mla_decode_batched(wl.query, wl.cache, wl.cu_seqlens, max_seq_len=wl.max_seq_len,
                                      softmax_scale=1.0, return_lse=True)
    torch.cuda.synchronize()
    assert mla.mla_get_device_error() == 0
    return out.float().cpu().numpy(), lse.cpu().numpy()


def _check_sequences(wl, out, lse, seqs, what):
    q = wl.query.float().cpu().numpy()
    worst = 0.0
    for b in seqs:
        c = wl.cache_rows(b).float().cpu().numpy()
        ref = oracle.mla_decode_oracle(q[b], c, 1.0, threads=THREADS)
        mx, _ = assert_close_parity(out[b], ref, what=f"{what} sequence {b} (N={c.shape[0]})")
        worst = max(worst, mx)
        # the LSE is the natural log of the softmax denominator: check it in fp64
        s = q[b].astype(np.float64) @ c.T.astype(np.float64)
        m = s.max(axis=1)
        ref_lse = m + np.log(np.exp(s - m[:, None]).sum(axis=1))
        assert np.abs(lse[b] - ref_lse).max() < 1e-3, f"{what} sequence {b}: LSE"
    return worst


@pytest.mark.parametrize("cfg", [1, 3])
def test_single_sequence_configs_full_size(mla, cfg):
    from ada_mla import capi
    from ada_mla.workloads import make_workload

    wl = make_workload(cfg, seed=0, device="cuda")
    chunk, splits = capi.plan(1, wl.num_heads, wl.total_tokens, wl.max_seq_len)
    assert splits > 1  # the split path and its merge run
    out, lse = _decode(mla, wl)
    _check_sequences(wl, out, lse, [0], f"cfg{cfg} ({splits} items of {chunk} tokens)")


def test_cfg2_varlen_batch_full_size(mla):
    from ada_mla.workloads import make_workload

    wl = make_workload(2, seed=0, device="cuda")
    assert wl.batch == 128 and wl.cu_seqlens is not None
    out, lse = _decode(mla, wl)
    _check_sequences(wl, out, lse, range(wl.batch), "cfg2")


def test_cfg4_few_heads_batch_full_size(mla):
    from ada_mla.workloads import make_workload

    wl = make_workload(4, seed=0, device="cuda")
    assert wl.batch == 256 and wl.num_heads == 16
    out, lse = _decode(mla, wl)
    _check_sequences(wl, out, lse, range(wl.batch), "cfg4")


def test_cfg3_paged_full_size_matches_contiguous(mla):
    """The 128K sequence through the paged entry (shuffled 64-token pages)
    against the oracle."""
    from ada_mla.workloads import make_workload, paged_layout

    wl = make_workload(3, seed=0, device="cuda")
    pl = paged_layout(wl, 64, seed=1)
    pool = pl.scatter(wl.cache)
    out = mla.mla_decode_paged(wl.query, pool, pl.block_table, pl.seq_lens, max_seq_len=wl.max_seq_len,
                               softmax_scale=1.0)
    torch.cuda.synchronize()
    assert mla.mla_get_device_error() == 0
    q = wl.query.float().cpu().numpy()
    ref = oracle.mla_decode_oracle(q[0], wl.cache[0].float().cpu().numpy(), 1.0, threads=THREADS)
    assert_close_parity(out[0].float().cpu().numpy(), ref, what="cfg3 paged")
