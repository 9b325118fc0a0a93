"""Seeded synthetic decode inputs with the shapes and value distributions of the
five benchmark configurations (the reference measures on random inputs only:
mla.py:104-110, :122-126; there is no dataset).

Every config draws C ~ N(0, 1) and Q* ~ N(0, 1) / sqrt(192) in fp32 from a
seeded torch generator and casts to fp16 (config 0 stays fp32).  The softmax
scale is folded into Q*, so the kernels run with ``softmax_scale = 1``.

  cfg 0  CPU oracle case: B=1, n_h=128, N=4096, fp32
  cfg 1  B=1, n_h=128, N=4096, fp16
  cfg 2  B=128, n_h=128, N_b ~ U[1024, 8192] (seeded, separate generator), packed cache
  cfg 3  B=1, n_h=128, N=131072
  cfg 4  B=256, n_h=16, N=2048, dense [B, N, 576] cache
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

HEAD_DIM_K = 576
HEAD_DIM_V = 512
Q_SCALE = 1.0 / (192.0 ** 0.5)


@dataclass
class Workload:
    cfg: int
    query: torch.Tensor            # [B, n_h, 576]
    cache: torch.Tensor            # packed [T, 576] or dense [B, N, 576]
    cu_seqlens: torch.Tensor | None  # int32 [B+1] (packed) or None (dense)
    seqlens: list[int]
    max_seq_len: int
    softmax_scale: float = 1.0

    @property
    def batch(self) -> int:
        return self.query.shape[0]

    @property
    def num_heads(self) -> int:
        return self.query.shape[1]

    @property
    def total_tokens(self) -> int:
        return int(sum(self.seqlens))

    @property
    def cache_bytes(self) -> int:
        """Algorithmic latent-cache bytes one decode step reads."""
        return self.total_tokens * HEAD_DIM_K * self.cache.element_size()

    @property
    def flops(self) -> int:
        return 2 * self.num_heads * (HEAD_DIM_K + HEAD_DIM_V) * self.total_tokens

    def cache_rows(self, b: int) -> torch.Tensor:
        """Rows of sequence b as a [N_b, 576] view."""
        if self.cu_seqlens is None:
            return self.cache[b]
        lo = sum(self.seqlens[:b])
        return self.cache[lo:lo + self.seqlens[b]]


CONFIGS = {
    0: dict(batch=1, heads=128, seqlen=4096, dtype=torch.float32),
    1: dict(batch=1, heads=128, seqlen=4096, dtype=torch.float16),
    2: dict(batch=128, heads=128, seqlen=(1024, 8192), dtype=torch.float16),
    3: dict(batch=1, heads=128, seqlen=131072, dtype=torch.float16),
    4: dict(batch=256, heads=16, seqlen=2048, dtype=torch.float16),
}


def seqlens_for(cfg: int, seed: int = 0) -> list[int]:
    c = CONFIGS[cfg]
    if isinstance(c["seqlen"], tuple):
        g = torch.Generator().manual_seed(seed + 7919)
        lo, hi = c["seqlen"]
        return torch.randint(lo, hi + 1, (c["batch"],), generator=g).tolist()
    return [c["seqlen"]] * c["batch"]


def _randn(shape, gen, device, dtype, scale=1.0, chunk_elems=1 << 26):
    out = torch.empty(shape, dtype=dtype, device=device)
    flat = out.view(-1)
    for s in range(0, flat.numel(), chunk_elems):
        e = min(flat.numel(), s + chunk_elems)
        x = torch.randn(e - s, generator=gen, device=device, dtype=torch.float32)
        if scale != 1.0:
            x.mul_(scale)
        flat[s:e].copy_(x)
    return out


def make_workload(cfg: int, seed: int = 0, device: str | torch.device = "cpu",
                  batch: int | None = None, seqlens: list[int] | None = None,
                  heads: int | None = None) -> Workload:
    """Build config ``cfg`` (optionally overriding batch / seqlens / heads) on ``device``."""
    c = CONFIGS[cfg]
    dtype = c["dtype"]
    nh = heads or c["heads"]
    if seqlens is None:
        seqlens = seqlens_for(cfg, seed)
        if batch is not None:
            seqlens = (seqlens * (batch // len(seqlens) + 1))[:batch]
    b = len(seqlens)
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed)
    q = _randn((b, nh, HEAD_DIM_K), gen, dev, dtype, Q_SCALE)
    varlen = isinstance(c["seqlen"], tuple)
    if varlen:
        cache = _randn((int(sum(seqlens)), HEAD_DIM_K), gen, dev, dtype)
        cu = torch.zeros(b + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(torch.tensor(seqlens, dtype=torch.int64), 0).to(torch.int32)
        cu = cu.to(dev)
    else:
        n = seqlens[0]
        assert all(s == n for s in seqlens)
        cache = _randn((b, n, HEAD_DIM_K), gen, dev, dtype)
        cu = None
    return Workload(cfg=cfg, query=q, cache=cache, cu_seqlens=cu, seqlens=list(seqlens),
                    max_seq_len=max(seqlens) if seqlens else 0)


@dataclass
class PagedLayout:
    """A page pool layout of a workload's sequences: sequence b's token t lives
    in row t % page_size of page block_table[b, t // page_size]."""
    page_size: int
    num_pages: int
    block_table: torch.Tensor  # int32 [B, max_blocks]
    seq_lens: torch.Tensor     # int32 [B]
    pool_rows: torch.Tensor    # int64 [T]: pool row of each packed cache row

    def scatter(self, cache: torch.Tensor, pool: torch.Tensor | None = None) -> torch.Tensor:
        """Copies a workload cache (dense or packed) into a [num_pages,
        page_size, 576] pool (allocated when absent; rows past a sequence's end
        are left as they were)."""
        if pool is None:
            pool = torch.empty((self.num_pages, self.page_size, HEAD_DIM_K), dtype=cache.dtype,
                               device=cache.device)
        pool.view(-1, HEAD_DIM_K).index_copy_(0, self.pool_rows.to(cache.device),
                                              cache.reshape(-1, HEAD_DIM_K))
        return pool


def paged_layout(wl: Workload, page_size: int, seed: int = 0, spare_pages: int = 0) -> PagedLayout:
    """Shuffled page assignment (seeded) for ``wl``'s sequences, as a serving
    engine's page allocator would leave it after churn."""
    npg = [-(-n // page_size) for n in wl.seqlens]
    num_pages = sum(npg) + spare_pages
    g = torch.Generator().manual_seed(seed + 104729)
    perm = torch.randperm(num_pages, generator=g)
    max_blocks = max(max(npg, default=0), 1)
    bt = torch.full((wl.batch, max_blocks), -1, dtype=torch.int32)
    rows = []
    used = 0
    for b, n in enumerate(wl.seqlens):
        pages = perm[used:used + npg[b]]
        used += npg[b]
        bt[b, :npg[b]] = pages.to(torch.int32)
        t = torch.arange(n, dtype=torch.int64)
        rows.append(pages.to(torch.int64)[t // page_size] * page_size + t % page_size)
    dev = wl.query.device
    pool_rows = torch.cat(rows) if rows else torch.zeros(0, dtype=torch.int64)
    return PagedLayout(page_size=page_size, num_pages=num_pages, block_table=bt.to(dev),
                       seq_lens=torch.tensor(wl.seqlens, dtype=torch.int32).to(dev),
                       pool_rows=pool_rows.to(dev))
