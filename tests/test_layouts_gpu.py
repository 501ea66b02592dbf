"""GPU: the in-place paged_attention form over vLLM-style pools (HND / NHD),
the partial-state path and its merge, and the device status bits.
Tolerance: atol = rtol = 2e-2 (scripts/benchmark.py:63-72)."""
import pytest
import torch

from pagedattention_b200 import (_lib, merge_packed_states, merge_states, paged_attention,
                                 paged_attention_states, read_status, state_numel)
from pagedattention_b200.distributed import context_ranges, local_view
from tests.util import assert_close, run_oracle

pytestmark = pytest.mark.gpu


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
    """The same problem in the reference layout (src/common.py:1-14)."""
    nb, Hkv, bs, D = pool_k.shape
    B = q.shape[0]
    heads = torch.arange(Hkv, dtype=torch.int32)
    bt3 = bt[:, None, :] * Hkv + heads[None, :, None]
    return (q[:, None], pool_k.reshape(nb * Hkv, bs, D), pool_v.reshape(nb * Hkv, bs, D),
            lens[:, None].expand(B, Hkv).contiguous(), bt3)


@pytest.mark.parametrize("layout", ["HND", "NHD"])
@pytest.mark.parametrize("G,D,bs,dtype", [(4, 128, 16, torch.bfloat16), (8, 128, 32, torch.bfloat16),
                                          (32, 64, 8, torch.float16), (1, 256, 16, torch.float16)])
def test_paged_attention_pools(cuda_device, layout, G, D, bs, dtype):
    B, Hkv = 3, 2
    q, pk, pv, bt, lens, scale = _pool_case(B, Hkv, G, D, bs, [0, 77, 300], dtype, seed=G + D)
    ref = run_oracle(*_reference_view(q, pk, pv, bt, lens), scale)[:, 0]
    dev = cuda_device
    if layout == "NHD":
        kc, vc = pk.permute(0, 2, 1, 3).contiguous(), pv.permute(0, 2, 1, 3).contiguous()
    else:
        kc, vc = pk, pv
    out = torch.full_like(q, float("nan")).to(dev)
    paged_attention(out, q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev), lens.to(dev), scale, bs,
                    kv_layout=layout)
    assert_close(out, ref, what=f"{layout} G{G} D{D} bs{bs}")


def test_paged_attention_per_head_lens(cuda_device):
    """context_lens of shape (num_seqs, num_kv_heads) over a reference page cache."""
    B, Hkv, G, D, bs = 2, 3, 4, 128, 16
    q, pk, pv, bt, lens, scale = _pool_case(B, Hkv, G, D, bs, [200, 90], torch.bfloat16, seed=3)
    q4, kp, vp, sl, bt3 = _reference_view(q, pk, pv, bt, lens)
    sl = sl.clone()
    sl[0, 1] = 17
    sl[1, 2] = 0
    ref = run_oracle(q4, kp, vp, sl, bt3, scale)[:, 0]
    dev = cuda_device
    out = torch.empty_like(q).to(dev)
    paged_attention(out, q.to(dev), kp.to(dev), vp.to(dev), bt3.to(dev), sl.to(dev), scale, bs)
    assert_close(out, ref)


@pytest.mark.parametrize("ranks", [2, 3, 8])
def test_context_split_states_merge(cuda_device, ranks):
    """Split every context into `ranks` token ranges (as the multi-GPU path
    does), decode each range to a packed (o, lse) state, merge on device."""
    B, Hkv, G, D, bs = 3, 2, 4, 128, 16
    lens = torch.tensor([1000, 64, 0], dtype=torch.int32)
    q, pk, pv, bt, lens, scale = _pool_case(B, Hkv, G, D, bs, lens, torch.bfloat16, seed=ranks)
    ref = run_oracle(*_reference_view(q, pk, pv, bt, lens), scale)[:, 0]
    dev = cuda_device
    starts, ends = context_ranges(lens, ranks, 64)
    S = state_numel(B, Hkv * G, D)
    states = torch.empty((ranks, S), dtype=torch.float32, device=dev)
    for r in range(ranks):
        btl, ll = local_view(bt, lens, starts[r], ends[r], bs)
        paged_attention_states(q.to(dev), pk.to(dev), pv.to(dev), btl.to(dev), ll.to(dev), scale,
                               bs, state=states[r])
    out = merge_packed_states(states, B, Hkv * G, D, out_dtype=torch.bfloat16)
    assert_close(out, ref, what=f"{ranks} ranges")
    # the unpacked form agrees
    rows = B * Hkv * G
    o = states[:, :rows * D].reshape(ranks, B, Hkv * G, D)
    l = states[:, rows * D:rows * D + rows].reshape(ranks, B, Hkv * G)
    out2 = merge_states(o, l, out_dtype=torch.float32)
    assert_close(out2, ref)


def test_states_of_empty_range(cuda_device):
    B, Hkv, G, D, bs = 2, 1, 8, 64, 16
    q, pk, pv, bt, lens, scale = _pool_case(B, Hkv, G, D, bs, [0, 40], torch.float16, seed=1)
    dev = cuda_device
    o, lse = paged_attention_states(q.to(dev), pk.to(dev), pv.to(dev), bt.to(dev), lens.to(dev),
                                    scale, bs)
    assert torch.count_nonzero(o[0]) == 0
    assert torch.isinf(lse[0]).all() and (lse[0] < 0).all()
    assert torch.isfinite(lse[1]).all()


def test_status_bits(cuda_device):
    """Out-of-range page ids and lengths are flagged, never faulted on: a bad
    page id reads a zero-filled box outside the tensor; lengths are clamped."""
    dev = cuda_device
    B, Hkv, G, D, bs = 2, 2, 4, 128, 16
    q, pk, pv, bt, lens, scale = _pool_case(B, Hkv, G, D, bs, [40, 40], torch.bfloat16, seed=4)
    out = torch.empty_like(q).to(dev)
    args = [q.to(dev), pk.to(dev), pv.to(dev)]
    paged_attention(out, *args, bt.to(dev), lens.to(dev), scale, bs)
    assert read_status(dev) == 0
    bad = bt.clone()
    bad[0, 1] = pk.shape[0] + 1000          # block id past the pool
    paged_attention(out, *args, bad.to(dev), lens.to(dev), scale, bs)
    assert read_status(dev) & _lib.STATUS_BAD_PAGE_ID
    assert torch.isfinite(out.float()).all()
    long = lens.clone()
    long[1] = bs * bt.shape[1] + 5           # past the block table's capacity
    paged_attention(out, *args, bt.to(dev), long.to(dev), scale, bs)
    assert read_status(dev) & _lib.STATUS_SEQLEN_CLAMP
    neg = lens.clone()
    neg[0] = -3
    paged_attention(out, *args, bt.to(dev), neg.to(dev), scale, bs)
    st = read_status(dev)
    assert st & _lib.STATUS_NEG_SEQLEN and not st & _lib.STATUS_SEQLEN_CLAMP
    assert torch.count_nonzero(out[0]) == 0


@pytest.mark.parametrize("core", ["0", "1"])
def test_states_merge_both_arithmetic_paths(cuda_device, monkeypatch, core):
    """Partial states written by the tensor-core and the CUDA-core variants
    merge to the oracle's output."""
    monkeypatch.setenv("PAB200_CORE", core)
    B, Hkv, G, D, bs = 2, 2, 2, 128, 16
    q, pk, pv, bt, lens, scale = _pool_case(B, Hkv, G, D, bs, [700, 90], torch.bfloat16, seed=9)
    ref = run_oracle(*_reference_view(q, pk, pv, bt, lens), scale)[:, 0]
    dev = cuda_device
    starts, ends = context_ranges(lens, 3, 64)
    S = state_numel(B, Hkv * G, D)
    states = torch.empty((3, S), dtype=torch.float32, device=dev)
    for r in range(3):
        btl, ll = local_view(bt, lens, starts[r], ends[r], bs)
        paged_attention_states(q.to(dev), pk.to(dev), pv.to(dev), btl.to(dev), ll.to(dev), scale,
                               bs, state=states[r])
    assert_close(merge_packed_states(states, B, Hkv * G, D), ref, what=f"core={core}")


@pytest.mark.parametrize("G,D", [(32, 64), (24, 128)])
def test_paired_warps_states_merge(cuda_device, monkeypatch, G, D):
    """Partial states of a group split over a pair of warps (each warp writes
    its 16 query heads' rows) merge to the oracle's output."""
    monkeypatch.setenv("PAB200_PAIR", "1")
    B, Hkv, bs = 2, 2, 16
    q, pk, pv, bt, lens, scale = _pool_case(B, Hkv, G, D, bs, [900, 130], torch.bfloat16,
                                            seed=G)
    ref = run_oracle(*_reference_view(q, pk, pv, bt, lens), scale)[:, 0]
    dev = cuda_device
    starts, ends = context_ranges(lens, 3, 64)
    S = state_numel(B, Hkv * G, D)
    states = torch.empty((3, S), dtype=torch.float32, device=dev)
    for r in range(3):
        btl, ll = local_view(bt, lens, starts[r], ends[r], bs)
        paged_attention_states(q.to(dev), pk.to(dev), pv.to(dev), btl.to(dev), ll.to(dev), scale,
                               bs, state=states[r])
    assert_close(merge_packed_states(states, B, Hkv * G, D), ref, what=f"paired G{G} D{D}")


@pytest.mark.parametrize("state_mode", [False, True])
def test_back_to_back_calls_reuse_outputs(cuda_device, state_mode):
    """Calls queued back to back on one stream into the same output: the
    next call's planner may overlap the previous call's reduce kernel, so a
    head that was split across warps in one call and is empty in the next
    must still end up zero (and an empty state: o = 0, lse = -inf), and
    every other head must hold the new call's result."""
    B, Hkv, G, D, bs = 4, 2, 4, 128, 16
    long_lens = [6000, 5000, 7000, 4000]
    q, pk, pv, bt, lens, scale = _pool_case(B, Hkv, G, D, bs, long_lens, torch.bfloat16, seed=21)
    dev = cuda_device
    qd, kd, vd, btd = q.to(dev), pk.to(dev), pv.to(dev), bt.to(dev)
    rounds = [long_lens, [0, 5000, 0, 4000], long_lens, [6000, 0, 7000, 0]]
    lens_d = [torch.tensor(x, dtype=torch.int32, device=dev) for x in rounds]
    if state_mode:
        state = torch.empty(state_numel(B, Hkv * G, D), dtype=torch.float32, device=dev)
        for ld in lens_d:  # no synchronisation between the calls
            paged_attention_states(qd, kd, vd, btd, ld, scale, bs, state=state)
        o = state[:B * Hkv * G * D].view(B, Hkv * G, D).cpu()
        lse = state[B * Hkv * G * D:B * Hkv * G * (D + 1)].view(B, Hkv * G).cpu()
        assert torch.count_nonzero(o[1]) == 0 and torch.count_nonzero(o[3]) == 0
        assert bool(torch.isneginf(lse[1]).all()) and bool(torch.isneginf(lse[3]).all())
        got = o[[0, 2]]
    else:
        out = torch.empty_like(qd)
        for ld in lens_d:  # no synchronisation between the calls
            paged_attention(out, qd, kd, vd, btd, ld, scale, bs)
        out = out.cpu()
        assert torch.count_nonzero(out[1]) == 0 and torch.count_nonzero(out[3]) == 0
        got = out[[0, 2]]
    last = torch.tensor(rounds[-1], dtype=torch.int32)
    q4, kp, vp, sl, bt3 = _reference_view(q, pk, pv, bt, last)
    ref = run_oracle(q4, kp, vp, sl, bt3, scale)[:, 0]
    assert_close(got.float(), ref[[0, 2]], what="back-to-back calls")
