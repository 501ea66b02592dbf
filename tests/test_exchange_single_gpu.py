"""GPU, one device: the fused decode + exchange of a context split
(pab200_decode_exchange) with a one-rank group.  With one rank the exchange
stores to no peer and merges only this rank's state, so its output must be
the whole decode: the exchange kernel's fold of the heads the decode split
over several warps (in place of the reduce kernel) is checked against the
oracle, and against the in-place decode, on one GPU.

Tolerance: atol = rtol = 2e-2 (scripts/benchmark.py:63-72)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist

from pagedattention_b200 import paged_attention
from pagedattention_b200.distributed import PeerExchange, decode_context_parallel
from tests.util import assert_close, run_oracle

pytestmark = pytest.mark.gpu


def _pool_case(B, Hkv, G, D, bs, lens, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    lens = torch.as_tensor(lens, dtype=torch.int32)
    nblk = (lens + bs - 1) // bs
    maxb = int(nblk.max()) + 1
    nb = int(nblk.sum()) + 3
    k = torch.randn((nb, Hkv, bs, D), generator=g).to(dtype)
    v = torch.randn((nb, Hkv, bs, D), generator=g).to(dtype)
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.zeros((B, maxb), dtype=torch.int32)
    off = 0
    for s in range(B):
        n = int(nblk[s])
        bt[s, :n] = perm[off:off + n]
        off += n
    q = torch.randn((B, Hkv * G, D), generator=g).to(dtype)
    return q, k, v, bt, lens, D ** -0.5


def _reference(q, k, v, bt, lens):
    nb, Hkv, bs, D = k.shape
    B = q.shape[0]
    heads = torch.arange(Hkv, dtype=torch.int32)
    bt3 = bt[:, None, :] * Hkv + heads[None, :, None]
    return (q[:, None], k.reshape(nb * Hkv, bs, D), v.reshape(nb * Hkv, bs, D),
            lens[:, None].expand(B, Hkv).contiguous(), bt3)


@pytest.fixture
def one_rank_group():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60))
    try:
        yield
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("G,D,bs,dtype", [(4, 128, 16, torch.bfloat16), (8, 64, 32, torch.float16),
                                          (2, 256, 16, torch.bfloat16)])
def test_fused_exchange_one_rank_matches_oracle(cuda_device, one_rank_group, G, D, bs, dtype):
    dev = cuda_device
    B, Hkv = 3, 2
    # long heads are split over many warps (folded by the exchange kernel),
    # short ones are whole, one is empty
    q, k, v, bt, lens, scale = _pool_case(B, Hkv, G, D, bs, [9000, 40, 0], dtype, seed=G + D)
    ref = run_oracle(*_reference(q, k, v, bt, lens), scale)[:, 0]
    qd, kd, vd, btd, ld = (t.to(dev) for t in (q, k, v, bt, lens))
    ex = PeerExchange(B, Hkv * G, D, wait_limit_s=5.0)
    try:
        outs = [decode_context_parallel(qd, kd, vd, btd, ld, scale, bs, exchange=ex)
                for _ in range(3)]  # both buffer parities
        plain = torch.empty_like(qd)
        paged_attention(plain, qd, kd, vd, btd, ld, scale, bs)
        torch.cuda.synchronize(dev)
        assert ex.read_status() == 0
        for i, out in enumerate(outs):
            assert_close(out, ref, what=f"fused exchange call {i + 1}")
            assert torch.allclose(out.float(), plain.float(), atol=1e-2, rtol=1e-2)
    finally:
        ex.close()
