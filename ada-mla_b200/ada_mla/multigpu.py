"""Multi-GPU MLA decode over ``torch.distributed`` (NCCL over NVLink / NVSwitch).

The reference has no distributed code (it runs one sequence on one GPU).  This
layer scales the same decode across the G GPUs of a node, one process per GPU:

* **Sequence sharding** (batch >= G): every rank owns whole sequences, chosen by
  longest-processing-time assignment on their lengths, and decodes them with no
  collective on the data path (``shard_sequences`` + ``decode_sharded``).  An
  optional all-gather returns the full batch of outputs to every rank.
* **KV-length split** (batch < G): rank r owns cache rows
  ``kv_split_bounds(N, G)[r]`` of every sequence, decodes them into a partial
  ``(O normalized, LSE)`` in fp32, and one ``all_gather_into_tensor`` of
  ``n_h x (512 + 1)`` floats per sequence gives every rank all G partials,
  which the LSE-merge kernel (``mla_combine``) reduces to the exact result
  (``KvSplitDecoder``).

The per-rank decode and the merge are injectable so that the host logic
(partitioning, packing, the collective, unpacking) can be exercised by CPU
``gloo`` ranks; the defaults are the CUDA kernels, and they require CUDA
tensors.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

HEAD_DIM_V = 512
KV_ALIGN = 96  # the tensor-core kernel's token tile; KV slices start on it


# ---------------------------------------------------------------------------
# partitioning (pure host logic)
# ---------------------------------------------------------------------------
def shard_sequences(seqlens: list[int], world: int) -> list[list[int]]:
    """Longest-processing-time assignment of sequences to ranks.

    Returns, per rank, the sorted indices of its sequences.  Ties are broken by
    sequence index and rank index so every rank computes the same plan.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    owned: list[list[int]] = [[] for _ in range(world)]
    order = sorted(range(len(seqlens)), key=lambda i: (-int(seqlens[i]), i))
    for i in order:
        load, r = heapq.heappop(heap)
        owned[r].append(i)
        heapq.heappush(heap, (load + int(seqlens[i]), r))
    return [sorted(o) for o in owned]


def kv_split_bounds(n: int, world: int, align: int = KV_ALIGN) -> list[tuple[int, int]]:
    """[start, end) of each rank's slice of an N-row cache (aligned starts;
    trailing ranks may get empty slices when N is small)."""
    if world <= 0:
        raise ValueError("world must be positive")
    per = -(-n // world)
    per = -(-per // align) * align if per > 0 else 0
    out = []
    for r in range(world):
        lo = min(n, r * per)
        hi = min(n, (r + 1) * per)
        out.append((lo, hi))
    return out


# ---------------------------------------------------------------------------
# defaults: the CUDA kernels
# ---------------------------------------------------------------------------
def _cuda_partial(query: torch.Tensor, cache: torch.Tensor, softmax_scale: float):
    """(O [B, n_h, 512] fp32 normalized, LSE [B, n_h] fp32) of one KV slice."""
    import ada_mla

    if not (query.is_cuda and cache.is_cuda):
        raise RuntimeError("the multi-GPU decode runs on CUDA tensors")
    return ada_mla.mla_decode_batched(query, cache, softmax_scale=softmax_scale, return_lse=True,
                                      out_dtype=torch.float32)


def _cuda_merge(part_o: torch.Tensor, part_lse: torch.Tensor, out_dtype: torch.dtype):
    import ada_mla

    if not part_o.is_cuda:
        raise RuntimeError("the LSE merge runs on CUDA tensors")
    out, lse = ada_mla.mla_combine(part_o, part_lse, out_fp32=out_dtype == torch.float32)
    return out, lse


@dataclass
class KvSplitDecoder:
    """KV-length-split decode across the ranks of ``group``.

    ``local_decode(query, cache_slice, scale) -> (O fp32 [B, n_h, 512], LSE
    fp32 [B, n_h])`` and ``merge(part_o [G, rows, 512], part_lse [G, rows],
    out_dtype) -> (out [rows, 512], lse [rows])`` default to the CUDA kernels.
    """

    group: dist.ProcessGroup | None = None
    local_decode: Callable | None = None
    merge: Callable | None = None

    def __post_init__(self):
        self.local_decode = self.local_decode or _cuda_partial
        self.merge = self.merge or _cuda_merge

    @property
    def world(self) -> int:
        return dist.get_world_size(self.group)

    @property
    def rank(self) -> int:
        return dist.get_rank(self.group)

    def bounds(self, n: int) -> tuple[int, int]:
        return kv_split_bounds(n, self.world)[self.rank]

    def __call__(self, query: torch.Tensor, cache_slice: torch.Tensor, softmax_scale: float,
                 out_dtype: torch.dtype = torch.float16, return_lse: bool = False):
        """query [B, n_h, 576] (identical on every rank); cache_slice
        [B, N_r, 576] = this rank's rows of a dense cache (N_r may be 0).
        Returns O* [B, n_h, 512] on every rank."""
        b, nh = query.shape[0], query.shape[1]
        rows = b * nh
        if cache_slice.shape[1] > 0:
            o, lse = self.local_decode(query, cache_slice, softmax_scale)
        else:  # an empty slice contributes nothing to the merge
            o = torch.zeros((b, nh, HEAD_DIM_V), dtype=torch.float32, device=query.device)
            lse = torch.full((b, nh), float("-inf"), dtype=torch.float32, device=query.device)
        packed = torch.cat([o.reshape(rows, HEAD_DIM_V).float(), lse.reshape(rows, 1).float()], dim=1)
        gathered = torch.empty((self.world * rows, HEAD_DIM_V + 1), dtype=packed.dtype,
                               device=packed.device)
        dist.all_gather_into_tensor(gathered, packed.contiguous(), group=self.group)
        gathered = gathered.view(self.world, rows, HEAD_DIM_V + 1)
        part_o = gathered[:, :, :HEAD_DIM_V].contiguous()
        part_lse = gathered[:, :, HEAD_DIM_V].contiguous()
        out, out_lse = self.merge(part_o, part_lse, out_dtype)
        out = out.reshape(b, nh, HEAD_DIM_V)
        return (out, out_lse.reshape(b, nh)) if return_lse else out


def decode_sharded(query_local: torch.Tensor, cache_local: torch.Tensor,
                   cu_seqlens_local: torch.Tensor | None = None, max_seq_len: int = -1,
                   softmax_scale: float = 1.0 / 192 ** 0.5, gather: bool = False,
                   group: dist.ProcessGroup | None = None, local_decode: Callable | None = None):
    """Sequence-sharded decode: every rank decodes the sequences it owns
    (already resident on its GPU) with no data-path collective.  With
    ``gather`` the per-rank outputs (same shape on every rank) are all-gathered
    into [G * B_local, n_h, 512] in rank order."""
    if local_decode is None:
        import ada_mla

        out = ada_mla.mla_decode_batched(query_local, cache_local, cu_seqlens_local,
                                         max_seq_len=max_seq_len, softmax_scale=softmax_scale)
    else:
        out = local_decode(query_local, cache_local, cu_seqlens_local, softmax_scale)
    if not gather:
        return out
    world = dist.get_world_size(group)
    full = torch.empty((world * out.shape[0],) + tuple(out.shape[1:]), dtype=out.dtype,
                       device=out.device)
    dist.all_gather_into_tensor(full, out.contiguous(), group=group)
    return full
