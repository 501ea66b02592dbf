"""GPU, two or more devices: sequence sharding, the NCCL context split and
the fused exchange + merge over peer memory, one process per GPU.  Skipped
where fewer than two GPUs are visible.

NVLS is switched off (NCCL_NVLS_ENABLE=0) and every process group has a short
timeout, so a failing rank ends the test with an error instead of a hang."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs"),
]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from pagedattention_b200 import flash_attn_with_kvcache_wrapper_b200 as decode
    from pagedattention_b200.distributed import (PeerExchange, context_ranges,
                                                 decode_context_parallel, lens_of_units,
                                                 local_view, shard_heads, shard_sequences)
    from pagedattention_b200.workloads import WORKLOADS, make_inputs
    from tests.util import ATOL, RTOL, run_oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        # 1) context split: every rank holds the whole (small) pool but
        #    decodes only its token range; the merged output is the full one.
        w = WORKLOADS["long_context"]
        lens = torch.tensor([3000, 9000, 17, 0], dtype=torch.int32)
        inp = make_inputs(w, seed=3, lens=lens)          # CPU, identical on all ranks
        starts, ends = context_ranges(lens, world, w.partition_tokens)
        btl, ll = local_view(inp.block_tables, lens, starts[rank], ends[rank], w.block_size)
        out = decode_context_parallel(inp.q.to(dev), inp.k_pool.to(dev), inp.v_pool.to(dev),
                                      btl.to(dev), ll.to(dev), inp.scale, w.block_size)
        ref = run_oracle(*inp.reference_layout(), inp.scale)[:, 0]
        ok_split = bool(torch.isclose(out.float().cpu(), ref, atol=ATOL, rtol=RTOL).all())
        # 1b) the same split through the fused exchange + merge: five calls
        #     cover both buffer parities and epoch reuse; every call matches
        #     the NCCL path's output to one bf16 rounding step
        ex = PeerExchange(*inp.q.shape, wait_limit_s=5.0)
        outs = [decode_context_parallel(inp.q.to(dev), inp.k_pool.to(dev), inp.v_pool.to(dev),
                                        btl.to(dev), ll.to(dev), inp.scale, w.block_size,
                                        exchange=ex) for _ in range(5)]
        ok_split = ok_split and ex.read_status() == 0
        ok_split = ok_split and all(torch.allclose(o.float(), out.float(), atol=1e-3, rtol=8e-3)
                                    for o in outs)
        ok_split = ok_split and bool(torch.isclose(outs[-1].float().cpu(), ref, atol=ATOL,
                                                   rtol=RTOL).all())
        ex.close()
        # 2) sequence sharding: each rank decodes its LPT shard of one batch
        w = WORKLOADS["llama70b_mixed"]
        inp = make_inputs(w, seed=5, num_seqs=12)
        shard = shard_sequences(inp.context_lens.tolist(), world)[rank]
        q4, kp, vp, sl, bt = inp.reference_layout()
        idx = torch.tensor(shard, dtype=torch.long)
        mine = decode(q4[idx].to(dev), kp.to(dev), vp.to(dev), sl[idx].to(dev), bt[idx].to(dev),
                      inp.scale)
        ref = run_oracle(q4[idx], kp, vp, sl[idx], bt[idx], inp.scale)
        ok_shard = bool(torch.isclose(mine.float().cpu(), ref, atol=ATOL, rtol=RTOL).all())
        # 3) fewer sequences than ranks: (sequence, kv head) units; every rank
        #    decodes the batch with only its units' lengths and owns those rows
        w = WORKLOADS["llama8b_gqa"]
        inp = make_inputs(w, seed=9, lens=torch.tensor([3000], dtype=torch.int32))
        q4, kp, vp, sl, bt = inp.reference_layout()
        units = shard_heads(sl, world)[rank]
        outh = decode(q4.to(dev), kp.to(dev), vp.to(dev), lens_of_units(sl, units).to(dev),
                      bt.to(dev), inp.scale).float().cpu()
        ref = run_oracle(q4, kp, vp, sl, bt, inp.scale)
        G = q4.shape[2] // sl.shape[1]
        ok_heads = len(units) > 0 and all(
            bool(torch.isclose(outh[s, 0, h * G:(h + 1) * G], ref[s, 0, h * G:(h + 1) * G],
                               atol=ATOL, rtol=RTOL).all()) for s, h in units)
        q.put((rank, ok_split, ok_shard and ok_heads))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_multi_gpu_context_split_and_sharding(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [q.get(timeout=10) for _ in range(world)]
    assert all(r[1] for r in res), res
    assert all(r[2] for r in res), res


def _timeout_worker(rank, world, port, q):
    """Rank 0 exchanges once; the others never call, so rank 0's bounded wait
    for their epoch flags runs out and reports it in the status word."""
    import torch.distributed as dist

    from pagedattention_b200 import _lib
    from pagedattention_b200.distributed import PeerExchange

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        B, Hq, D = 2, 8, 128
        ex = PeerExchange(B, Hq, D, wait_limit_s=0.2)
        status = 0
        if rank == 0:
            state = torch.zeros_like(ex.state)
            out = torch.empty((B, Hq, D), dtype=torch.bfloat16, device=dev)
            ex.exchange_merge(state, out)
            torch.cuda.synchronize()
            status = ex.read_status()
        ex.reset()
        after = ex.read_status()
        ex.close()
        q.put((rank, status, after, _lib.STATUS_WAIT_TIMEOUT))
    finally:
        dist.destroy_process_group()


def test_exchange_wait_limit_reports_timeout():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_timeout_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = {r: (st, after, bit) for r, st, after, bit in (q.get(timeout=10) for _ in range(world))}
    assert res[0][0] & res[0][2], res
    assert res[1][0] == 0 and all(v[1] == 0 for v in res.values()), res
