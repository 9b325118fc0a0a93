"""The synthetic workloads and the paged layout helper used by bench.py (CPU)."""
import torch

from ada_mla.workloads import CONFIGS, make_workload, paged_layout, seqlens_for


def test_config_shapes():
    for cfg in (1, 2, 4):
        wl = make_workload(cfg, seed=0, device="cpu", batch=3)
        c = CONFIGS[cfg]
        assert wl.query.shape == (3, c["heads"], 576)
        assert wl.cache_bytes == wl.total_tokens * 576 * wl.cache.element_size()
        for b in range(3):
            assert wl.cache_rows(b).shape == (wl.seqlens[b], 576)
    lens = seqlens_for(2, seed=0)
    assert len(lens) == 128 and all(1024 <= n <= 8192 for n in lens)
    assert lens == seqlens_for(2, seed=0)  # seeded


def test_paged_layout_round_trip():
    for cfg, ps in ((2, 64), (4, 128), (2, 32)):
        wl = make_workload(cfg, seed=1, device="cpu", batch=5)
        pl = paged_layout(wl, ps, seed=3, spare_pages=2)
        pool = pl.scatter(wl.cache)
        assert pool.shape == (pl.num_pages, ps, 576)
        used = set()
        for b in range(wl.batch):
            n = wl.seqlens[b]
            npg = -(-n // ps)
            pages = pl.block_table[b, :npg].tolist()
            assert all(0 <= p < pl.num_pages for p in pages)
            assert not used & set(pages)  # no page shared between sequences
            used |= set(pages)
            assert (pl.block_table[b, npg:] == -1).all()
            t = torch.arange(n)
            rows = pl.block_table[b].long()[t // ps] * ps + t % ps
            assert torch.equal(pool.view(-1, 576)[rows], wl.cache_rows(b))
        assert torch.equal(pl.seq_lens, torch.tensor(wl.seqlens, dtype=torch.int32))
