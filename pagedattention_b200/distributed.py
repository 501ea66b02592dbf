"""Multi-GPU decode, one process per GPU (torch.distributed over NCCL).

The decode path spreads over devices in two ways:

* Sequence sharding — no collective.  Sequences are independent, so each rank
  decodes its own; ``shard_sequences`` balances ranks by tokens
  (longest-processing-time-first), since KV bytes, not sequence count, set
  the time.  With fewer sequences than ranks, ``shard_heads`` splits by
  (sequence, kv head) instead and ``lens_of_units`` gives a rank the
  lengths of its units only.
* Context split — one exchange.  A context too long for one device's share
  is cut into contiguous token ranges, one per rank (``context_ranges``).
  Each rank decodes its range of every sequence into a packed (o, lse) state
  (``paged_attention_states``), one NCCL all-gather moves the states
  (num_seqs * num_q_heads * (head_size + 1) floats per rank), and
  ``merge_packed_states`` combines them: the reference's log-sum-exp reduce
  (src/kernel_triton.py:120-174) applied across devices.  Any rank's
  output is the full-context result.  With a ``PeerExchange`` the gather and
  the merge are one kernel over peer memory instead (NVLink stores into
  every rank's exchange buffer, mapped with CUDA IPC; an epoch flag per rank;
  a bounded wait), launched by the decode call itself in place of its reduce
  kernel (``paged_attention_exchange``: the exchange kernel also folds the
  heads the decode split), which saves the NCCL launch, the reduce launch
  and the separate merge.

The reference has no multi-device code; this module is new.
"""
from __future__ import annotations

import ctypes
import heapq

import torch
import torch.distributed as dist

from . import _lib
from .kernel_b200 import (merge_packed_states, paged_attention_exchange, paged_attention_states,
                          state_numel)

_OUT_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16,
               torch.float32: _lib.DTYPE_F32}
IPC_HANDLE_BYTES = 64


def shard_sequences(lens, world_size: int) -> list[list[int]]:
    """Assign sequence indices to ranks, balancing total tokens (LPT greedy:
    longest first onto the least-loaded rank).  Every rank's list is sorted."""
    lens = [int(x) for x in lens]
    heap = [(0, r) for r in range(world_size)]
    shards = [[] for _ in range(world_size)]
    for i in sorted(range(len(lens)), key=lambda i: (-lens[i], i)):
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + lens[i], r))
    return [sorted(s) for s in shards]


def shard_heads(lens, world_size: int) -> list[list[tuple[int, int]]]:
    """Assign (sequence, kv head) units to ranks, balancing tokens (LPT, as
    ``shard_sequences``) — for batches with fewer sequences than ranks.
    ``lens``: (num_seqs, num_kv_heads) lengths.  Every rank's list is sorted."""
    lens = torch.as_tensor(lens)
    B, Hkv = lens.shape
    flat = [int(x) for x in lens.reshape(-1).tolist()]
    heap = [(0, r) for r in range(world_size)]
    shards = [[] for _ in range(world_size)]
    for i in sorted(range(len(flat)), key=lambda i: (-flat[i], i)):
        load, r = heapq.heappop(heap)
        shards[r].append(divmod(i, Hkv))
        heapq.heappush(heap, (load + flat[i], r))
    return [sorted(s) for s in shards]


def lens_of_units(lens, units):
    """Per-(sequence, kv head) lengths of a rank that owns ``units``: the
    others become 0 (an empty head: no pages read, a zero output row that the
    owning rank overwrites in its own result)."""
    lens = torch.as_tensor(lens)
    out = torch.zeros_like(lens)
    for s, h in units:
        out[s, h] = lens[s, h]
    return out


def context_ranges(lens, world_size: int, align: int):
    """Token range [start, end) of every sequence owned by each rank.

    Each sequence is cut into ceil(L / align) chunks of ``align`` tokens (a
    multiple of the block size, so ranges start on page boundaries) and rank
    r takes chunks [floor(r*n/W), floor((r+1)*n/W)).  Returns int64 tensors
    starts, ends of shape [world_size, num_seqs]; empty ranges have
    start == end.
    """
    lens = torch.as_tensor(lens, dtype=torch.int64)
    n = (lens + align - 1) // align
    r = torch.arange(world_size + 1, dtype=torch.int64)[:, None]
    bounds = torch.minimum((r * n[None, :]) // world_size * align, lens[None, :])
    return bounds[:-1].clone(), bounds[1:].clone()


def local_view(block_tables, lens, start, end, block_size: int):
    """Block table and lengths of a rank's token ranges.

    block_tables: [B, max_blocks] (block ids per sequence, shared by all kv
    heads); start/end: [B] token ranges with start a multiple of block_size.
    Returns (bt_local [B, max_local] int32, lens_local [B] int32); entries
    past a sequence's local page count are 0 and never read.
    """
    start = torch.as_tensor(start, dtype=torch.int64)
    end = torch.as_tensor(end, dtype=torch.int64)
    if bool((start % block_size != 0).any()):
        raise ValueError("range starts must be multiples of block_size")
    lens_local = (end - start).clamp_min(0)
    first = start // block_size
    npages = (lens_local + block_size - 1) // block_size
    max_local = max(int(npages.max()) if npages.numel() else 0, 1)
    cols = torch.arange(max_local, dtype=torch.int64)[None, :]
    idx = (first[:, None] + cols).clamp_max(block_tables.shape[1] - 1)
    bt = torch.gather(block_tables.to(torch.int64).cpu(), 1, idx)
    bt = torch.where(cols < npages[:, None], bt, torch.zeros_like(bt))
    return bt.to(torch.int32), lens_local.to(torch.int32)


def all_gather_states(state: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather one flat float32 state per rank into an (N, S) tensor."""
    world = dist.get_world_size(group)
    out = torch.empty((world, state.numel()), dtype=state.dtype, device=state.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, state, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), state, group=group)
    return out


class PeerExchange:
    """Exchange buffers of the ranks of one node for the fused exchange +
    merge (``pab200_exchange_merge``), mapped into every rank with CUDA IPC.

    Collective: every rank of ``group`` constructs it with the same shape,
    on its own current CUDA device (one process per GPU).  Each rank's
    buffer holds two parities of ``world`` packed states plus control words;
    the handles travel once through ``all_gather_object``.  ``wait_limit_s``
    bounds the wait for peers inside the kernel: when it runs out the kernel
    sets ``STATUS_WAIT_TIMEOUT`` in ``status`` and merges what arrived, and
    all ranks must then call ``reset()`` before the next exchange.  Every
    rank must make the same sequence of exchange calls.
    """

    def __init__(self, num_seqs: int, num_q_heads: int, head_size: int, group=None,
                 wait_limit_s: float = 1.0):
        self.lib = lib = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.shape = (num_seqs, num_q_heads, head_size)
        self.rows = num_seqs * num_q_heads
        self.nbytes = lib.pab200_exchange_buffer_bytes(self.world, self.rows, head_size)
        if not self.nbytes:
            raise ValueError(f"unsupported exchange shape {self.shape} for world {self.world}")
        self.wait_limit_ns = max(int(wait_limit_s * 1e9), 1)
        buf = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * IPC_HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            _lib.check(lib, lib.pab200_exchange_buffer_create(self.nbytes, ctypes.byref(buf),
                                                              handle),
                       "pab200_exchange_buffer_create")
        self._own = buf.value
        self._opened: list[int] = []
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        ptrs = []
        try:
            with torch.cuda.device(self.device):
                for r, h in enumerate(handles):
                    if r == self.rank:
                        ptrs.append(self._own)
                        continue
                    pb = ctypes.c_void_p()
                    hb = (ctypes.c_ubyte * IPC_HANDLE_BYTES).from_buffer_copy(h)
                    _lib.check(lib, lib.pab200_exchange_buffer_open(hb, ctypes.byref(pb)),
                               "pab200_exchange_buffer_open")
                    self._opened.append(pb.value)
                    ptrs.append(pb.value)
        except Exception:
            self._release()
            raise
        self.bufs = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.state = torch.empty(state_numel(*self.shape), dtype=torch.float32,
                                 device=self.device)
        dist.barrier(group)

    def exchange_merge(self, state: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Merge every rank's packed ``state`` into ``out`` (num_seqs,
        num_q_heads, head_size), on the current stream."""
        code = _OUT_DTYPES.get(out.dtype)
        if code is None:
            raise TypeError(f"unsupported out dtype {out.dtype}")
        if (tuple(out.shape) != self.shape or not out.is_contiguous()
                or out.device != self.device):
            raise ValueError(f"out must be a contiguous {self.shape} tensor on {self.device}")
        if (state.dtype != torch.float32 or not state.is_contiguous()
                or state.numel() < state_numel(*self.shape) or state.device != self.device):
            raise ValueError("state must be a contiguous float32 tensor of state_numel() elements")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = self.lib.pab200_exchange_merge(
            ctypes.c_void_p(state.data_ptr()), ctypes.c_void_p(self.bufs.data_ptr()), self.rank,
            self.world, self.rows, self.shape[2], ctypes.c_void_p(out.data_ptr()), self.shape[2],
            code, self.wait_limit_ns, ctypes.c_void_p(self.status.data_ptr()),
            ctypes.c_void_p(stream))
        _lib.check(self.lib, rc, "pab200_exchange_merge")
        return out

    def read_status(self) -> int:
        """Status bits of the exchanges so far (synchronises the device)."""
        return int(self.status.item()) & 0xFFFFFFFF

    def reset(self) -> None:
        """Zero this rank's buffer and status; collective (all ranks, with no
        exchange in flight), e.g. after a timed-out exchange."""
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(self.lib, self.lib.pab200_exchange_buffer_reset(
            ctypes.c_void_p(self._own), self.nbytes, ctypes.c_void_p(stream)),
            "pab200_exchange_buffer_reset")
        self.status.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)

    def _release(self) -> None:
        with torch.cuda.device(self.device):
            for p in self._opened:
                self.lib.pab200_exchange_buffer_close(ctypes.c_void_p(p))
            self._opened = []
            if self._own:
                self.lib.pab200_exchange_buffer_destroy(ctypes.c_void_p(self._own))
                self._own = None

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's; collective."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                self.lib.pab200_exchange_buffer_close(ctypes.c_void_p(p))
        self._opened = []
        dist.barrier(self.group)
        self._release()


def decode_context_parallel(query, key_cache, value_cache, block_tables, context_lens, scale,
                            block_size, group=None, kv_layout="HND", out=None, exchange=None):
    """Decode with every sequence's context split across the ranks of ``group``.

    Each rank passes ITS token range: block_tables / context_lens describe
    only the pages it holds (see ``local_view``), query is the full query on
    every rank.  Returns out (num_seqs, num_q_heads, head_size) in query's
    dtype, identical on all ranks.  ``exchange`` (a ``PeerExchange`` of this
    shape) replaces the NCCL all-gather + merge with the fused kernel over
    peer memory.
    """
    B, Hq, D = query.shape
    if exchange is not None:
        # decode, fold and exchange in one call (pab200_decode_exchange)
        return paged_attention_exchange(query, key_cache, value_cache, block_tables, context_lens,
                                        scale, block_size, exchange, out=out, kv_layout=kv_layout)
    state = torch.empty(state_numel(B, Hq, D), dtype=torch.float32, device=query.device)
    paged_attention_states(query, key_cache, value_cache, block_tables, context_lens, scale,
                           block_size, kv_layout=kv_layout, state=state)
    gathered = all_gather_states(state, group)
    return merge_packed_states(gathered, B, Hq, D, out=out, out_dtype=query.dtype)
