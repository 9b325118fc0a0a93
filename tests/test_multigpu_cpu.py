"""Host logic of the multi-GPU layer on CPU ``gloo`` ranks (world size 2 and 3):
partitioning, packing, the all-gather and the LSE merge.  The per-rank decode
is the CPU oracle (float64 partials), injected in place of the CUDA kernel."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from ada_mla import multigpu


def test_shard_sequences_lpt_balance_and_coverage():
    lens = [8000, 1100, 4096, 7000, 1024, 5000, 3000, 2000, 6500, 1500]
    for world in (1, 2, 3, 4, 8):
        plan = multigpu.shard_sequences(lens, world)
        assert sorted(i for p in plan for i in p) == list(range(len(lens)))
        loads = [sum(lens[i] for i in p) for p in plan]
        # LPT bound: max load <= mean + largest item
        assert max(loads) <= sum(lens) / world + max(lens)
        assert plan == multigpu.shard_sequences(lens, world)  # deterministic


def test_packed_stride_aligns_every_part():
    for rows in (1, 3, 16, 128, 129, 2048):
        st = multigpu.packed_stride(rows)
        assert st >= rows * 513 and st % 4 == 0 and st - rows * 513 < 4


def test_kv_split_bounds_cover_and_align():
    for n in (0, 1, 95, 96, 4096, 131072, 131071):
        for world in (1, 2, 4, 8):
            b = multigpu.kv_split_bounds(n, world)
            assert b[0][0] == 0 and b[-1][1] == n
            for (lo, hi), (lo2, _) in zip(b, b[1:]):
                assert hi == lo2 and lo <= hi
            for lo, _ in b:
                assert lo % multigpu.KV_ALIGN == 0 or lo == n


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_partial(query, cache, scale, o_out, lse_out, workspace):
    """In-place per-rank decode (float64 oracle partials) into the exchange buffer's views."""
    q = query.numpy()
    c = cache.numpy()
    for b in range(q.shape[0]):
        o, lse = oracle.lse_partial_oracle(q[b], c[b], scale)
        o_out[b] = torch.tensor(o, dtype=torch.float32)
        lse_out[b] = torch.tensor(lse, dtype=torch.float32)


def _cpu_merge(packed, parts, rows, stride, out_dtype):
    """LSE merge read straight from the gathered buffer: part g's O at
    g * stride, its LSE right after the O block."""
    views = packed.view(parts, stride)
    part_o = views[:, :rows * 512].reshape(parts, rows, 512)
    part_lse = views[:, rows * 512:rows * 513]
    lse = part_lse.double()
    m = lse.max(dim=0).values
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w = torch.where(torch.isfinite(lse), torch.exp(lse - m), torch.zeros_like(lse))
    s = w.sum(dim=0)
    out = (w[:, :, None] * part_o.double()).sum(dim=0) / torch.where(s > 0, s, torch.ones_like(s))[:, None]
    return out.to(out_dtype), (m + torch.log(s)).float()


def _kv_worker(rank, world, port, n, seed, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(seed)
        b, nh = 2, 8
        q = torch.randn(b, nh, 576, generator=g) / 192 ** 0.5
        c = torch.randn(b, n, 576, generator=g)
        dec = multigpu.KvSplitDecoder(local_decode=_cpu_partial, merge=_cpu_merge,
                                      make_workspace=lambda q, c: None)
        lo, hi = dec.bounds(n)
        out, lse = dec(q, c[:, lo:hi].contiguous(), 1.0, out_dtype=torch.float64, return_lse=True)
        full = [oracle.lse_partial_oracle(q[i].numpy(), c[i].numpy(), 1.0) for i in range(b)]
        ref = np.stack([f[0] for f in full])
        ref_lse = np.stack([f[1] for f in full])
        results[rank] = (float(np.abs(out.numpy() - ref).max()), float(np.abs(lse.numpy() - ref_lse).max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n", [(2, 300), (3, 100), (2, 50)])  # n=100/50: some slices empty
def test_kv_split_gloo_merge_matches_full_decode(world, n):
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_kv_worker, args=(r, world, port, n, 7, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert len(results) == world
    for r in range(world):
        err_o, err_lse = results[r]
        assert err_o < 1e-6 and err_lse < 1e-6, (r, err_o, err_lse)


def _shard_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(3)
        bl, nh, n = 2, 4, 40
        qs = torch.randn(world, bl, nh, 576, generator=g) / 192 ** 0.5
        cs = torch.randn(world, bl, n, 576, generator=g)

        def local(q, c, cu, scale):
            return torch.tensor(np.stack([oracle.lse_partial_oracle(q[i].numpy(), c[i].numpy(), scale)[0]
                                          for i in range(q.shape[0])]), dtype=torch.float32)

        full = multigpu.decode_sharded(qs[rank], cs[rank], softmax_scale=1.0, gather=True,
                                       local_decode=local)
        ref = np.concatenate([local(qs[r], cs[r], None, 1.0).numpy() for r in range(world)])
        results[rank] = float(np.abs(full.numpy() - ref).max())
    finally:
        dist.destroy_process_group()


def test_sequence_sharded_gather_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert all(results[r] == 0.0 for r in range(world))
