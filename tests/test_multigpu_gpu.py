"""Multi-GPU decode (needs >= 2 GPUs; skipped otherwise): the KV-length split
with its NCCL all-gather + LSE merge or its peer-memory exchange (the slice's
merge fused into the exchange kernel or not, and one rank fused while the other
is not), and sequence sharding, all against the CPU oracle."""
import os
import socket

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, results):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "ada-mla_b200")]
    import torch.distributed as dist

    from ada_mla import multigpu

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        g = torch.Generator().manual_seed(11)
        if mode.startswith("kv"):
            # kv_p2p: decode + one exchange kernel (the slice's merge fused in);
            # kv_p2p_unfused: decode, merge, exchange kernel; kv_p2p_empty: rank 1's
            # slice is empty, so it takes the unfused kernels while rank 0 fuses
            b, nh, n = 1, 128, 90 if mode == "kv_p2p_empty" else 5000
            q = (torch.randn(b, nh, 576, generator=g) / 192 ** 0.5).half()
            c = torch.randn(b, n, 576, generator=g).half()
            dec = multigpu.KvSplitDecoder(exchange="nccl" if mode == "kv" else "p2p",
                                          fuse=mode != "kv_p2p_unfused")
            lo, hi = dec.bounds(n)
            qd, cd = q.cuda(), c[:, lo:hi].contiguous().cuda()
            outs = [dec(qd, cd, 1.0) for _ in range(3)]  # three steps: both exchange parities
            torch.cuda.synchronize()
            fused = dec._fused_ok.get((b, nh), False)
            assert fused == (mode == "kv_p2p" or (mode == "kv_p2p_empty" and rank == 0)), (mode, rank, fused)
            ref = oracle.mla_decode_oracle(q[0].float().numpy(), c[0].float().numpy(), 1.0, threads=4)
            d = np.abs(outs[-1][0].float().cpu().numpy() - ref)
            assert all(torch.equal(o, outs[0]) for o in outs), "every step gives the same result"
            from ada_mla import capi
            assert capi.get_device_error() == 0
            dec.close()
        else:
            bl, nh, n = 2, 128, 700
            qs = (torch.randn(world, bl, nh, 576, generator=g) / 192 ** 0.5).half()
            cs = torch.randn(world, bl, n, 576, generator=g).half()
            full = multigpu.decode_sharded(qs[rank].cuda(), cs[rank].cuda(), softmax_scale=1.0, gather=True)
            ref = np.concatenate([np.stack([oracle.mla_decode_oracle(qs[r, i].float().numpy(),
                                                                     cs[r, i].float().numpy(), 1.0, threads=4)
                                            for i in range(bl)]) for r in range(world)])
            d = np.abs(full.float().cpu().numpy() - ref)
        results[rank] = (float(d.max()), float(d.mean()))
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


@needs_two
@pytest.mark.parametrize("mode", ["kv", "kv_p2p", "kv_p2p_unfused", "kv_p2p_empty", "shard"])
def test_two_gpu_decode(mode):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    for r in range(2):
        mx, mean = results[r]
        assert mx <= 1e-2 and mean <= 1e-3, (mode, r, mx, mean)
