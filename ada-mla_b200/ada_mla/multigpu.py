"""Multi-GPU MLA decode over ``torch.distributed`` (NCCL over NVLink / NVSwitch).

The reference has no distributed code (it runs one sequence on one GPU).  This
layer scales the same decode across the G GPUs of a node, one process per GPU:

* **Sequence sharding** (batch >= G): every rank owns whole sequences, chosen by
  longest-processing-time assignment on their lengths, and decodes them with no
  collective on the data path (``shard_sequences`` + ``decode_sharded``).  An
  optional all-gather returns the full batch of outputs to every rank.
* **KV-length split** (batch < G): rank r owns cache rows
  ``kv_split_bounds(N, G)[r]`` of every sequence and decodes them straight
  into a packed exchange buffer (O normalized, then LSE, fp32); one
  ``all_gather_into_tensor`` of ``n_h x (512 + 1)`` floats per sequence gives
  every rank all G partials, which the LSE-merge kernel reads in place and
  reduces to the exact result (``KvSplitDecoder``).  With ``exchange="p2p"``
  the all-gather is replaced by this library's own kernels over NVLink peer
  memory (``PeerExchange``: CUDA IPC mappings, plain stores into every rank's
  buffer of 8-byte words that each carry the step's epoch, readers polling their
  own buffer with bounded waits).

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
def packed_stride(rows: int) -> int:
    """Floats per rank in the packed (O, LSE) exchange buffer: O [rows, 512]
    then LSE [rows], padded to a multiple of 4 floats so that every rank's O
    starts on a 16-byte boundary."""
    return -(-rows * (HEAD_DIM_V + 1) // 4) * 4


def _cuda_partial(query: torch.Tensor, cache: torch.Tensor, softmax_scale: float,
                  o_out: torch.Tensor, lse_out: torch.Tensor, workspace: torch.Tensor) -> None:
    """Decodes one dense KV slice into o_out [B, n_h, 512] fp32 (normalized) and
    lse_out [B, n_h] fp32, in place (views into the exchange buffer)."""
    from ada_mla import capi

    if not (query.is_cuda and cache.is_cuda):
        raise RuntimeError("the multi-GPU decode runs on CUDA tensors")
    b, nh, n = query.shape[0], query.shape[1], cache.shape[1]
    bf16 = query.dtype == torch.bfloat16
    name = "mla_b200_decode_batched_bf16" if bf16 else "mla_b200_decode_batched_f16"
    st = getattr(capi.lib(), name)(
        query.data_ptr(), cache.data_ptr(), None, b, nh, b * n, n, float(softmax_scale), -1,
        o_out.data_ptr(), capi.OUT_F32, lse_out.data_ptr(), workspace.data_ptr(),
        workspace.numel(), torch.cuda.current_stream().cuda_stream)
    if st != capi.OK:
        raise capi.MlaError(name, st)


def _cuda_workspace(query: torch.Tensor, cache: torch.Tensor) -> torch.Tensor:
    from ada_mla import capi

    b, nh, n = query.shape[0], query.shape[1], cache.shape[1]
    return torch.empty(max(256, capi.workspace_size(b, nh, b * n, n, -1)), dtype=torch.uint8,
                       device=query.device)


def _cuda_merge(packed: torch.Tensor, parts: int, rows: int, stride: int, out_dtype: torch.dtype):
    """LSE merge straight from the gathered exchange buffer (mla_b200_combine_packed_f32)."""
    from ada_mla import capi

    if not packed.is_cuda:
        raise RuntimeError("the LSE merge runs on CUDA tensors")
    out = torch.empty((rows, HEAD_DIM_V), dtype=torch.float32 if out_dtype == torch.float32
                      else torch.float16, device=packed.device)
    lse = torch.empty((rows,), dtype=torch.float32, device=packed.device)
    st = capi.lib().mla_b200_combine_packed_f32(
        packed.data_ptr(), parts, rows, stride, out.data_ptr(),
        capi.OUT_F32 if out_dtype == torch.float32 else capi.OUT_F16, lse.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    if st != capi.OK:
        raise capi.MlaError("mla_b200_combine_packed_f32", st)
    return out, lse


class PeerExchange:
    """The split-KV step's exchange over NVLink peer memory, instead of an NCCL
    all-gather: every rank owns one exchange buffer (mla_b200_exchange_alloc),
    maps every other rank's through CUDA IPC (handles swapped once with
    ``all_gather_object``), stores its packed (O, LSE) straight into every
    rank's buffer (``put``) and merges the G parts in its own buffer once their
    words carry this step's epoch (``merge``, a bounded wait).  Both are stream-ordered
    kernels, so the step captures in a CUDA graph.  Set up and ``close()`` on
    every rank together (both end with a barrier)."""

    WAIT_LIMIT_NS = 1_000_000_000  # a peer that has not published within 1 s is an error

    def __init__(self, rows: int, group: dist.ProcessGroup | None = None):
        import ctypes

        from ada_mla import capi

        self.rows = rows
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        lib = capi.lib()
        own = ctypes.c_void_p()
        capi._check("mla_b200_exchange_alloc", lib.mla_b200_exchange_alloc(self.world, rows, ctypes.byref(own)))
        self.own = own.value
        handle = ctypes.create_string_buffer(64)
        capi._check("mla_b200_ipc_handle", lib.mla_b200_ipc_handle(self.own, handle))
        handles = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, handle.raw, group=group)
        else:
            handles[0] = handle.raw
        ptrs, self._opened = [], []
        for g, h in enumerate(handles):
            if g == self.rank:
                ptrs.append(self.own)
                continue
            p = ctypes.c_void_p()
            capi._check("mla_b200_ipc_open", lib.mla_b200_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p)))
            ptrs.append(p.value)
            self._opened.append(p.value)
        self._peer_array = (ctypes.c_void_p * self.world)(*ptrs)  # host array of device pointers
        if self.world > 1:
            dist.barrier(group=group)  # every mapping exists before the first put

    def put(self, packed: torch.Tensor) -> None:
        """packed: this rank's [packed_stride(rows)] fp32 (O then LSE)."""
        from ada_mla import capi

        capi._check("mla_b200_exchange_put_f32", capi.lib().mla_b200_exchange_put_f32(
            packed.data_ptr(), self.rows, self._peer_array, self.rank, self.world,
            torch.cuda.current_stream().cuda_stream))

    def merge(self, out_dtype: torch.dtype = torch.float16, device=None):
        """The merged [rows, 512] output and its [rows] LSE, on this rank."""
        from ada_mla import capi

        out = torch.empty((self.rows, HEAD_DIM_V), dtype=torch.float32 if out_dtype == torch.float32
                          else torch.float16, device=device)
        lse = torch.empty((self.rows,), dtype=torch.float32, device=device)
        capi._check("mla_b200_exchange_merge_f32", capi.lib().mla_b200_exchange_merge_f32(
            self.own, self.world, self.rows, out.data_ptr(),
            capi.OUT_F32 if out_dtype == torch.float32 else capi.OUT_F16, lse.data_ptr(),
            self.WAIT_LIMIT_NS, torch.cuda.current_stream().cuda_stream))
        return out, lse

    def exchange(self, packed: torch.Tensor, out_dtype: torch.dtype = torch.float16, device=None):
        """put + merge as one kernel (mla_b200_exchange_f32) when its blocks fit
        the device at once, else the two kernels; returns (out, lse)."""
        from ada_mla import capi

        out = torch.empty((self.rows, HEAD_DIM_V), dtype=torch.float32 if out_dtype == torch.float32
                          else torch.float16, device=device)
        lse = torch.empty((self.rows,), dtype=torch.float32, device=device)
        st = capi.lib().mla_b200_exchange_f32(
            packed.data_ptr(), self.rows, self._peer_array, self.rank, self.world, out.data_ptr(),
            capi.OUT_F32 if out_dtype == torch.float32 else capi.OUT_F16, lse.data_ptr(),
            self.WAIT_LIMIT_NS, torch.cuda.current_stream().cuda_stream)
        if st == capi.ERR_UNSUPPORTED:
            self.put(packed)
            return self.merge(out_dtype, device=device)
        capi._check("mla_b200_exchange_f32", st)
        return out, lse

    def decode_exchange(self, query: torch.Tensor, cache_slice: torch.Tensor, softmax_scale: float,
                        workspace: torch.Tensor, direct: torch.Tensor, out_dtype: torch.dtype = torch.float16):
        """This rank's decode of its dense KV slice and the whole exchange, the
        slice's split merge included, in one decode launch and ONE exchange
        kernel (mla_b200_decode_exchange_f16); ``direct`` is [packed_stride(rows)]
        fp32 scratch.  Returns (out, lse), or None when the exchange kernel's rows
        do not fit the device at once (nothing was launched then)."""
        from ada_mla import capi

        b, nh, n = query.shape[0], query.shape[1], cache_slice.shape[1]
        out = torch.empty((self.rows, HEAD_DIM_V), dtype=torch.float32 if out_dtype == torch.float32
                          else torch.float16, device=query.device)
        lse = torch.empty((self.rows,), dtype=torch.float32, device=query.device)
        st = capi.lib().mla_b200_decode_exchange_f16(
            query.data_ptr(), cache_slice.data_ptr(), None, b, nh, b * n, n, float(softmax_scale), -1,
            self._peer_array, self.rank, self.world, direct.data_ptr(), out.data_ptr(),
            capi.OUT_F32 if out_dtype == torch.float32 else capi.OUT_F16, lse.data_ptr(),
            self.WAIT_LIMIT_NS, workspace.data_ptr(), workspace.numel(),
            torch.cuda.current_stream().cuda_stream)
        if st == capi.ERR_UNSUPPORTED:
            return None
        capi._check("mla_b200_decode_exchange_f16", st)
        return out, lse

    def close(self) -> None:
        from ada_mla import capi

        if self.own is None:
            return
        torch.cuda.synchronize()
        lib = capi.lib()
        for p in self._opened:
            lib.mla_b200_ipc_close(p)
        self._opened = []
        if self.world > 1:
            dist.barrier(group=self.group)  # no peer maps the buffer any more
        lib.mla_b200_exchange_free(self.own)
        self.own = None


@dataclass
class KvSplitDecoder:
    """KV-length-split decode across the ranks of ``group``.

    Each rank decodes its slice straight into its part of a packed exchange
    buffer (O [rows, 512] fp32 then LSE [rows] fp32, rows = B x n_h), one
    ``all_gather_into_tensor`` gives every rank all G parts, and the merge reads
    the gathered buffer in place: no concatenation or unpacking copies.

    ``local_decode(query, cache_slice, scale, o_out, lse_out, workspace)``
    writes in place; ``merge(packed [G * stride], G, rows, stride, out_dtype) ->
    (out [rows, 512], lse [rows])``.  Both default to the CUDA kernels and are
    injectable (the CPU tests run the host logic on gloo ranks).

    ``exchange="p2p"`` replaces the all-gather and the merge by ``PeerExchange``:
    the packed partial goes straight into every rank's buffer over NVLink and is
    merged there (CUDA only; ``close()`` releases the mappings on every rank).
    With the default CUDA decode, fp16 inputs and a non-empty slice, the slice's
    own split merge joins that kernel too (``PeerExchange.decode_exchange``;
    ``fuse=False`` keeps it a kernel of its own).
    """

    group: dist.ProcessGroup | None = None
    local_decode: Callable | None = None
    merge: Callable | None = None
    make_workspace: Callable | None = None
    exchange: str = "nccl"
    fuse: bool = True  # p2p: the slice's split merge joins the exchange kernel where it applies

    def __post_init__(self):
        self.local_decode = self.local_decode or _cuda_partial
        self.merge = self.merge or _cuda_merge
        self.make_workspace = self.make_workspace or _cuda_workspace
        self._bufs: dict = {}
        self._peers: dict = {}
        self._fused_ok: dict = {}  # (B, n_h) -> the one-kernel exchange fits the device
        if self.exchange not in ("nccl", "p2p"):
            raise ValueError(f"exchange must be 'nccl' or 'p2p', not {self.exchange!r}")

    def _peer_exchange(self, rows: int) -> PeerExchange:
        if rows not in self._peers:
            self._peers[rows] = PeerExchange(rows, self.group)
        return self._peers[rows]

    def close(self) -> None:
        for ex in self._peers.values():
            ex.close()
        self._peers = {}

    @property
    def world(self) -> int:
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    @property
    def rank(self) -> int:
        return dist.get_rank(self.group) if dist.is_initialized() else 0

    def bounds(self, n: int) -> tuple[int, int]:
        return kv_split_bounds(n, self.world)[self.rank]

    def _gather(self, recv: torch.Tensor, send: torch.Tensor) -> None:
        if self.world > 1:
            dist.all_gather_into_tensor(recv, send, group=self.group)
        else:  # a single rank: its own part is the whole exchange
            recv.copy_(send)

    def _barrier(self) -> None:
        if self.world > 1:
            dist.barrier(group=self.group)

    def _buffers(self, query: torch.Tensor, cache_slice: torch.Tensor):
        """Exchange buffers and the decode workspace, allocated once per shape
        (so the step can be captured in a CUDA graph)."""
        b, nh = query.shape[0], query.shape[1]
        key = (b, nh, cache_slice.shape[1], query.dtype, query.device)
        if key not in self._bufs:
            stride = packed_stride(b * nh)
            send = torch.empty(stride, dtype=torch.float32, device=query.device)
            recv = torch.empty(self.world * stride, dtype=torch.float32, device=query.device)
            ws = self.make_workspace(query, cache_slice) if cache_slice.shape[1] > 0 else None
            self._bufs[key] = (stride, send, recv, ws)
        return self._bufs[key]

    def _local(self, query, cache_slice, softmax_scale):
        b, nh = query.shape[0], query.shape[1]
        rows = b * nh
        stride, send, recv, ws = self._buffers(query, cache_slice)
        o = send[:rows * HEAD_DIM_V].view(b, nh, HEAD_DIM_V)
        lse = send[rows * HEAD_DIM_V:rows * (HEAD_DIM_V + 1)].view(b, nh)
        if cache_slice.shape[1] > 0:
            self.local_decode(query, cache_slice, softmax_scale, o, lse, ws)
        else:  # an empty slice contributes nothing to the merge
            o.zero_()
            lse.fill_(float("-inf"))
        return stride, send, recv

    def _fused(self, query: torch.Tensor, cache_slice: torch.Tensor, softmax_scale: float,
               out_dtype: torch.dtype):
        """The decode + one-kernel exchange of ``PeerExchange.decode_exchange``
        where it applies, else None."""
        if (self.exchange != "p2p" or not self.fuse or self.local_decode is not _cuda_partial
                or query.dtype != torch.float16 or cache_slice.shape[1] == 0
                or not self._fused_ok.get(tuple(query.shape[:2]), True)):
            return None
        b, nh = query.shape[0], query.shape[1]
        _, send, _, ws = self._buffers(query, cache_slice)
        res = self._peer_exchange(b * nh).decode_exchange(query, cache_slice, softmax_scale, ws, send, out_dtype)
        self._fused_ok[(b, nh)] = res is not None
        return res

    def __call__(self, query: torch.Tensor, cache_slice: torch.Tensor, softmax_scale: float,
                 out_dtype: torch.dtype = torch.float16, return_lse: bool = False):
        """query [B, n_h, 576] (identical on every rank); cache_slice
        [B, N_r, 576] = this rank's rows of a dense cache (N_r may be 0).
        Returns O* [B, n_h, 512] on every rank."""
        b, nh = query.shape[0], query.shape[1]
        fused = self._fused(query, cache_slice, softmax_scale, out_dtype)
        if fused is not None:
            out, out_lse = fused
            out = out.reshape(b, nh, HEAD_DIM_V)
            return (out, out_lse.reshape(b, nh)) if return_lse else out
        stride, send, recv = self._local(query, cache_slice, softmax_scale)
        if self.exchange == "p2p":
            out, out_lse = self._peer_exchange(b * nh).exchange(send, out_dtype, device=query.device)
        else:
            self._gather(recv, send)
            out, out_lse = self.merge(recv, self.world, b * nh, stride, out_dtype)
        out = out.reshape(b, nh, HEAD_DIM_V)
        return (out, out_lse.reshape(b, nh)) if return_lse else out

    def stage_times_us(self, query: torch.Tensor, cache_slice: torch.Tensor, softmax_scale: float,
                       reps: int = 20) -> dict:
        """Device time of each stage (local decode, all-gather, merge; p2p: local
        decode, exchange, and decode + exchange as one step where fused): each
        stage captured `reps` times in a CUDA graph, one replay between CUDA
        events on this rank's stream (launch overhead excluded, as in the timed
        step), after one untimed run of the stage that aligns the ranks on the
        device.  Every rank must call it (the exchange stages are collective)."""
        b, nh = query.shape[0], query.shape[1]
        stride, send, recv = self._local(query, cache_slice, softmax_scale)
        times = {}
        if self.exchange == "p2p":
            ex = self._peer_exchange(b * nh)
            stages = {
                "local_decode": lambda: self._local(query, cache_slice, softmax_scale),
                "p2p_exchange": lambda: ex.exchange(send, torch.float16, device=query.device),
            }
            if self._fused(query, cache_slice, softmax_scale, torch.float16) is not None:
                stages["decode_exchange"] = lambda: self._fused(query, cache_slice, softmax_scale, torch.float16)
        else:
            stages = {
                "local_decode": lambda: self._local(query, cache_slice, softmax_scale),
                "all_gather": lambda: self._gather(recv, send),
                "merge": lambda: self.merge(recv, self.world, b * nh, stride, torch.float16),
            }
        for name, fn in stages.items():
            fn()
            torch.cuda.synchronize()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                for _ in range(reps):
                    fn()
            torch.cuda.synchronize()
            self._barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            fn()  # a collective stage completes on every rank together: the events start aligned
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            times[name] = e0.elapsed_time(e1) * 1e3 / reps
            del graph
        return times


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
