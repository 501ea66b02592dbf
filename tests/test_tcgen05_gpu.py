"""GPU parity of the tcgen05 decode path (PAB200_TC=1): query groups of 9-32
heads at head size 64, scores and P.V on the 5th-generation tensor cores
with TMEM accumulators, against the fp32 oracle.

Tolerance everywhere: torch.isclose(atol=2e-2, rtol=2e-2), the reference's
parity bar (scripts/benchmark.py:63-72, 161).
"""
import pytest
import torch

from pagedattention_b200 import (_lib, flash_attn_with_kvcache_wrapper_b200, merge_packed_states,
                                 paged_attention, paged_attention_states, read_status, state_numel)
from pagedattention_b200.distributed import context_ranges, local_view
from pagedattention_b200.workloads import WORKLOADS, make_inputs
from tests.util import assert_close, random_case, run_oracle

pytestmark = pytest.mark.gpu

TC_KERNEL = "64, 2, 64, false, true, true>"  # decode_kernel<T, 64, 2, 64, CORE, PAIR, TC>


@pytest.fixture
def tc(monkeypatch):
    monkeypatch.setenv("PAB200_TC", "1")
    return monkeypatch


def _decode(*args, **kw):
    return flash_attn_with_kvcache_wrapper_b200(*args, **kw)


def _lens(B, Hkv, bs, seed):
    # 0, 1, page edges, the 64-token stage edges, and long heads
    pool = [0, 1, bs - 1, bs, bs + 1, 63, 64, 65, 127, 128, 129, 200, 513, 1000, 3001]
    return [[pool[(s * Hkv + h * 7 + seed) % len(pool)] for h in range(Hkv)] for s in range(B)]


@pytest.mark.parametrize("G,bs,dtype", [
    (32, 8, torch.float16), (32, 16, torch.bfloat16), (32, 32, torch.float16),
    (32, 64, torch.bfloat16), (24, 32, torch.float16), (16, 16, torch.bfloat16),
    (9, 8, torch.float16), (12, 64, torch.float16),
])
def test_random_vs_oracle(cuda_device, tc, G, bs, dtype):
    B, Hkv = 3, 2
    lens = _lens(B, Hkv, bs, G)
    q, k, v, sl, bt, scale = random_case(B, Hkv, G, 64, bs, lens, dtype, seed=G * 10 + bs,
                                         k_scale=4.0)
    dev = cuda_device
    out = _decode(q.to(dev), k.to(dev), v.to(dev), sl.to(dev), bt.to(dev), scale)
    assert_close(out, run_oracle(q, k, v, sl, bt, scale), what=f"tc G{G} bs{bs} {dtype}")


@pytest.mark.parametrize("early", ["0", "1"])
def test_with_and_without_early_start(cuda_device, tc, early):
    """The decode grid plans its own ranges from the lengths before the
    planner has finished (early start, the default at most 1024 heads), or
    reads the planner's plan first; both give the same result."""
    tc.setenv("PAB200_EARLY", early)
    lens = _lens(4, 3, 8, 5)
    q, k, v, sl, bt, scale = random_case(4, 3, 32, 64, 8, lens, torch.float16, seed=77,
                                         k_scale=4.0)
    dev = cuda_device
    args = [t.to(dev) for t in (q, k, v, sl, bt)]
    out = _decode(*args, scale)
    assert_close(out, run_oracle(q, k, v, sl, bt, scale), what=f"early={early}")
    assert torch.equal(out, _decode(*args, scale))


def test_runs_the_tcgen05_kernel(cuda_device, tc):
    """The switch selects the tcgen05 kernel (no silent fallback)."""
    q, k, v, sl, bt, scale = random_case(2, 1, 32, 64, 8, [[700], [90]], torch.float16, seed=1)
    dev = cuda_device
    args = [t.to(dev) for t in (q, k, v, sl, bt)]
    _decode(*args, scale)
    torch.cuda.synchronize()
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        _decode(*args, scale)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if "decode_kernel" in e.name]
    assert names, "the profiler saw no decode kernel"
    assert any(TC_KERNEL in n for n in names), names


@pytest.mark.parametrize("steal_m", ["0", "2", "8"])
def test_tail_chunks_and_stealing(cuda_device, tc, steal_m):
    """Static ranges, and ranges with run-time claimed / stolen tail chunks
    (one-stage chunks): every split head is merged from its segments."""
    tc.setenv("PAB200_STEAL_M", steal_m)
    tc.setenv("PAB200_STEAL_MIN_STAGES", "1")
    lens = [[5000, 37, 0, 1200], [1, 2600, 700, 16], [9000, 64, 65, 3]]
    q, k, v, sl, bt, scale = random_case(3, 4, 32, 64, 8, lens, torch.float16, seed=5,
                                         k_scale=4.0)
    dev = cuda_device
    args = [t.to(dev) for t in (q, k, v, sl, bt)]
    out = _decode(*args, scale)
    assert_close(out, run_oracle(q, k, v, sl, bt, scale), what=f"steal_m={steal_m}")
    assert torch.equal(out, _decode(*args, scale))


@pytest.mark.parametrize("num_splits", [0, 1, 2, 7])
def test_num_splits(cuda_device, tc, num_splits):
    q, k, v, sl, bt, scale = random_case(2, 3, 32, 64, 16, [[700, 5, 64], [0, 333, 1024]],
                                         torch.bfloat16, seed=7)
    dev = cuda_device
    out = _decode(q.to(dev), k.to(dev), v.to(dev), sl.to(dev), bt.to(dev), scale,
                  num_splits=num_splits)
    assert_close(out, run_oracle(q, k, v, sl, bt, scale), what=f"num_splits={num_splits}")


def test_one_long_head_over_every_unit(cuda_device, tc):
    """One 150k-token head cut over every unit of the grid (static prefixes
    and tail chunks), merged from hundreds of partial states."""
    tc.setenv("PAB200_STEAL_MIN_STAGES", "1")
    q, k, v, sl, bt, scale = random_case(1, 1, 32, 64, 16, [[150_000]], torch.float16, seed=23,
                                         poison=False)
    dev = cuda_device
    args = [t.to(dev) for t in (q, k, v, sl, bt)]
    out = _decode(*args, scale)
    assert_close(out, run_oracle(q, k, v, sl, bt, scale), what="one 150k-token head")
    assert torch.equal(out, _decode(*args, scale))


def test_matches_mma_sync_path(cuda_device, monkeypatch):
    """Both arithmetic paths agree with the oracle on the same inputs."""
    lens = [[4096, 77], [1, 3000]]
    q, k, v, sl, bt, scale = random_case(2, 2, 32, 64, 8, lens, torch.float16, seed=31,
                                         k_scale=4.0)
    dev = cuda_device
    args = [t.to(dev) for t in (q, k, v, sl, bt)]
    ref = run_oracle(q, k, v, sl, bt, scale)
    monkeypatch.setenv("PAB200_TC", "0")
    base = _decode(*args, scale)
    monkeypatch.setenv("PAB200_TC", "1")
    tcout = _decode(*args, scale)
    assert_close(base, ref, what="mma.sync")
    assert_close(tcout, ref, what="tcgen05")


def _pool_case(B, Hkv, G, D, bs, lens, dtype, seed, extra_blocks=5):
    g = torch.Generator().manual_seed(seed)
    lens = torch.as_tensor(lens, dtype=torch.int32)
    nblk = (lens + bs - 1) // bs
    maxb = int(nblk.max()) + 1
    nb = int(nblk.sum()) + extra_blocks
    pool_k = torch.randn((nb, Hkv, bs, D), generator=g).to(dtype)
    pool_v = torch.randn((nb, Hkv, bs, D), generator=g).to(dtype)
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.zeros((B, maxb), dtype=torch.int32)
    off = 0
    for s in range(B):
        n = int(nblk[s])
        bt[s, :n] = perm[off:off + n]
        off += n
    q = torch.randn((B, Hkv * G, D), generator=g).to(dtype)
    return q, pool_k, pool_v, bt, lens, D ** -0.5


def _reference_view(q, pool_k, pool_v, bt, lens):
    nb, Hkv, bs, D = pool_k.shape
    B = q.shape[0]
    heads = torch.arange(Hkv, dtype=torch.int32)
    bt3 = bt[:, None, :] * Hkv + heads[None, :, None]
    return (q[:, None], pool_k.reshape(nb * Hkv, bs, D), pool_v.reshape(nb * Hkv, bs, D),
            lens[:, None].expand(B, Hkv).contiguous(), bt3)


@pytest.mark.parametrize("layout", ["HND", "NHD"])
def test_pools_and_states(cuda_device, tc, layout):
    """vLLM-style pools (both layouts), and the partial-state form merged over
    a context split."""
    B, Hkv, G, D, bs = 3, 2, 32, 64, 8
    q, pk, pv, bt, lens, scale = _pool_case(B, Hkv, G, D, bs, [0, 77, 1300], torch.float16,
                                            seed=9)
    ref = run_oracle(*_reference_view(q, pk, pv, bt, lens), scale)[:, 0]
    dev = cuda_device
    if layout == "NHD":
        kc, vc = pk.permute(0, 2, 1, 3).contiguous(), pv.permute(0, 2, 1, 3).contiguous()
    else:
        kc, vc = pk, pv
    out = torch.full_like(q, float("nan")).to(dev)
    paged_attention(out, q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev), lens.to(dev), scale, bs,
                    kv_layout=layout)
    assert_close(out, ref, what=layout)
    ranks = 3
    starts, ends = context_ranges(lens, ranks, 64)
    states = torch.empty((ranks, state_numel(B, Hkv * G, D)), dtype=torch.float32, device=dev)
    for r in range(ranks):
        btl, ll = local_view(bt, lens, starts[r], ends[r], bs)
        paged_attention_states(q.to(dev), kc.to(dev), vc.to(dev), btl.to(dev), ll.to(dev), scale,
                               bs, kv_layout=layout, state=states[r])
    merged = merge_packed_states(states, B, Hkv * G, D, out_dtype=torch.float32)
    assert_close(merged, ref, what=f"{layout} states")


def test_status_and_empty_heads(cuda_device, tc):
    dev = cuda_device
    B, Hkv, G, D, bs = 2, 2, 32, 64, 16
    q, pk, pv, bt, lens, scale = _pool_case(B, Hkv, G, D, bs, [0, 400], torch.bfloat16, seed=4)
    out = torch.full_like(q, float("nan")).to(dev)
    args = [q.to(dev), pk.to(dev), pv.to(dev)]
    paged_attention(out, *args, bt.to(dev), lens.to(dev), scale, bs)
    assert read_status(dev) == 0
    assert torch.count_nonzero(out[0]) == 0
    bad = bt.clone()
    bad[1, 3] = pk.shape[0] + 1000
    paged_attention(out, *args, bad.to(dev), lens.to(dev), scale, bs)
    assert read_status(dev) & _lib.STATUS_BAD_PAGE_ID
    assert torch.isfinite(out.float()).all()


def test_mqa_small_page_workload(cuda_device, tc):
    """The full mqa_small_page workload (128 sequences, G 32, D 64, 8-token
    pages): sampled sequences against the oracle, bit-identical repeats."""
    inp = make_inputs(WORKLOADS["mqa_small_page"], device=cuda_device, gen_device=cuda_device)
    q, k, v, sl, bt = inp.reference_layout()
    bt = bt.contiguous()
    out = _decode(q, k, v, sl, bt, inp.scale)
    assert torch.equal(out, _decode(q, k, v, sl, bt, inp.scale))
    idx = [0, 41, 64, 127]
    sub_bt = bt[idx]
    pages = torch.unique(sub_bt.flatten().long())
    remap = torch.full((k.shape[0],), -1, dtype=torch.long, device=k.device)
    remap[pages] = torch.arange(pages.numel(), device=k.device)
    ref = run_oracle(q[idx].cpu(), k[pages].cpu(), v[pages].cpu(), sl[idx].cpu(),
                     remap[sub_bt.long()].to(torch.int32).cpu(), inp.scale, threads=8)
    assert_close(out[idx], ref, what="mqa_small_page")
