"""Multi-GPU decode, one process per GPU (torch.distributed over NCCL).

The decode path spreads over devices in two ways:

* Sequence sharding — no collective.  Sequences are independent, so each rank
  decodes its own; ``shard_sequences`` balances ranks by tokens
  (longest-processing-time-first), since KV bytes, not sequence count, set
  the time.
* Context split — one exchange.  A context too long for one device's share
  is cut into contiguous token ranges, one per rank (``context_ranges``).
  Each rank decodes its range of every sequence into a packed (o, lse) state
  (``paged_attention_states``), one NCCL all-gather moves the states
  (num_seqs * num_q_heads * (head_size + 1) floats per rank), and
  ``merge_packed_states`` combines them: the reference's log-sum-exp reduce
  (src/kernel_triton.py:120-174) applied across devices.  Any rank's
  output is the full-context result.

The reference has no multi-device code; this module is new.
"""
from __future__ import annotations

import heapq

import torch
import torch.distributed as dist

from .kernel_b200 import merge_packed_states, paged_attention_states, state_numel


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


def decode_context_parallel(query, key_cache, value_cache, block_tables, context_lens, scale,
                            block_size, group=None, kv_layout="HND", out=None):
    """Decode with every sequence's context split across the ranks of ``group``.

    Each rank passes ITS token range: block_tables / context_lens describe
    only the pages it holds (see ``local_view``), query is the full query on
    every rank.  Returns out (num_seqs, num_q_heads, head_size) in query's
    dtype, identical on all ranks.
    """
    B, Hq, D = query.shape
    S = state_numel(B, Hq, D)
    state = torch.empty(S, dtype=torch.float32, device=query.device)
    paged_attention_states(query, key_cache, value_cache, block_tables, context_lens, scale,
                           block_size, kv_layout=kv_layout, state=state)
    gathered = all_gather_states(state, group)
    return merge_packed_states(gathered, B, Hq, D, out=out, out_dtype=query.dtype)
