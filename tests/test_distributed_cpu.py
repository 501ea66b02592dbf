"""Host-side multi-device logic on CPU: sharding arithmetic, and the context
split's gather + log-sum-exp merge exercised by two gloo ranks with the oracle
standing in for the per-rank device decode."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import eager as oracle
from pagedattention_b200.distributed import (all_gather_states, context_ranges, local_view,
                                             shard_sequences)


def test_shard_sequences_balances_tokens():
    lens = [16, 16384, 2048, 300, 9000, 50, 4096, 4096, 1, 700]
    shards = shard_sequences(lens, 3)
    assert sorted(i for s in shards for i in s) == list(range(len(lens)))
    loads = [sum(lens[i] for i in s) for s in shards]
    assert max(loads) - min(loads) <= max(lens)
    assert shard_sequences(lens, 1) == [list(range(len(lens)))]


def test_shard_sequences_more_ranks_than_sequences():
    shards = shard_sequences([5, 7], 4)
    assert sorted(len(s) for s in shards) == [0, 0, 1, 1]


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_context_ranges_partition_each_sequence(world):
    lens = [0, 1, 511, 512, 513, 32768, 131072]
    starts, ends = context_ranges(lens, world, 512)
    for s, L in enumerate(lens):
        pos = 0
        for r in range(world):
            assert int(starts[r, s]) == pos
            assert int(starts[r, s]) % 512 == 0 or int(starts[r, s]) == L
            pos = int(ends[r, s])
        assert pos == L


def test_local_view_selects_the_range_pages():
    bs = 16
    bt = torch.arange(100, dtype=torch.int32).reshape(2, 50) + 1000
    lens = torch.tensor([700, 33])
    starts, ends = context_ranges(lens, 2, 64)
    bt0, l0 = local_view(bt, lens, starts[0], ends[0], bs)
    bt1, l1 = local_view(bt, lens, starts[1], ends[1], bs)
    assert int(l0[0] + l1[0]) == 700 and int(l0[1] + l1[1]) == 33
    first1 = int(starts[1, 0]) // bs
    assert int(bt1[0, 0]) == int(bt[0, first1])
    n1 = (int(l1[0]) + bs - 1) // bs
    assert torch.equal(bt1[0, :n1], bt[0, first1:first1 + n1])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(123)
        B, Hkv, G, D, bs = 2, 2, 4, 64, 16
        lens = [700, 33]
        q = rng.standard_normal((B, Hkv * G, D)).astype(np.float32)
        K = [[(rng.standard_normal((L, D)) * 2).astype(np.float32) for _ in range(Hkv)] for L in lens]
        V = [[rng.standard_normal((L, D)).astype(np.float32) for _ in range(Hkv)] for L in lens]
        starts, ends = context_ranges(lens, world, 64)
        rows = B * Hkv * G
        S = rows * D + ((rows + 3) // 4) * 4
        state = torch.zeros(S, dtype=torch.float32)
        o = state[:rows * D].view(B, Hkv * G, D)
        lse = state[rows * D:rows * D + rows].view(B, Hkv * G)
        for s in range(B):
            a, b = int(starts[rank, s]), int(ends[rank, s])
            for h in range(Hkv):
                so, sl = oracle.split_state(q[s, h * G:(h + 1) * G], K[s][h][a:b], V[s][h][a:b],
                                            D ** -0.5)
                o[s, h * G:(h + 1) * G] = torch.from_numpy(so)
                lse[s, h * G:(h + 1) * G] = torch.from_numpy(sl)
        gathered = all_gather_states(state)
        go = gathered[:, :rows * D].reshape(world, B, Hkv * G, D).numpy()
        gl = gathered[:, rows * D:rows * D + rows].reshape(world, B, Hkv * G).numpy()
        merged = oracle.merge_states(go, gl)
        full = np.stack([np.concatenate([oracle._one_head(q[s, h * G:(h + 1) * G], K[s][h],
                                                          V[s][h], D ** -0.5)
                                         for h in range(Hkv)]) for s in range(B)])
        result_q.put((rank, float(np.abs(merged - full).max())))
    finally:
        dist.destroy_process_group()


def test_context_split_gather_merge_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert max(res.values()) < 1e-4, res


def test_shard_heads_covers_every_unit_and_balances():
    from pagedattention_b200.distributed import lens_of_units, shard_heads
    lens = torch.tensor([[32768, 30000, 100, 5], [65536, 0, 7, 900]])
    shards = shard_heads(lens, 4)
    units = sorted(u for sh in shards for u in sh)
    assert units == [(s, h) for s in range(2) for h in range(4)]
    loads = [sum(int(lens[s, h]) for s, h in sh) for sh in shards]
    assert max(loads) - min(loads) <= int(lens.max())
    total = sum(lens_of_units(lens, sh) for sh in shards)
    assert torch.equal(total, lens)
    assert int(lens_of_units(lens, shards[0]).count_nonzero()) <= len(shards[0])
