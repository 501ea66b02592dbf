"""GPU: the five named workloads at full size.  The oracle checks sampled
sequences (all their kv heads); size-independent properties cover the whole
batch: relabelling the physical pages (and the block table with them) leaves
the output bit-identical, repeated calls are bit-identical, and every output
lies inside the range of its head's V values."""
import pytest
import torch

from pagedattention_b200 import flash_attn_with_kvcache_wrapper_b200 as decode
from pagedattention_b200.workloads import WORKLOADS, make_inputs
from tests.util import assert_close, run_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def workload_cache():
    return {}


def _inputs(name, dev, cache):
    if name not in cache:
        cache.clear()
        torch.cuda.empty_cache()
        inp = make_inputs(WORKLOADS[name], device=dev, gen_device=dev)
        q, k, v, sl, bt = inp.reference_layout()
        cache[name] = (inp, q, k, v, sl, bt.contiguous())
    return cache[name]


def _sampled_oracle(q, k, v, sl, bt, idx, scale):
    """Oracle on sequences `idx`, copying only the pages they use."""
    sub_bt = bt[idx]
    pages = torch.unique(sub_bt.flatten().long())
    remap = torch.full((k.shape[0],), -1, dtype=torch.long, device=k.device)
    remap[pages] = torch.arange(pages.numel(), device=k.device)
    return run_oracle(q[idx].cpu(), k[pages].cpu(), v[pages].cpu(), sl[idx].cpu(),
                      remap[sub_bt.long()].to(torch.int32).cpu(), scale, threads=8)


@pytest.mark.parametrize("name", list(WORKLOADS))
def test_full_size_sampled_parity(cuda_device, workload_cache, name):
    inp, q, k, v, sl, bt = _inputs(name, cuda_device, workload_cache)
    out = decode(q, k, v, sl, bt, inp.scale)
    B = q.shape[0]
    idx = sorted({0, B // 3, B // 2, B - 1})
    ref = _sampled_oracle(q, k, v, sl, bt, idx, inp.scale)
    assert_close(out[idx], ref, what=name)
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("name", list(WORKLOADS))
def test_full_size_properties(cuda_device, workload_cache, name):
    inp, q, k, v, sl, bt = _inputs(name, cuda_device, workload_cache)
    out = decode(q, k, v, sl, bt, inp.scale)
    again = decode(q, k, v, sl, bt, inp.scale)
    assert torch.equal(out, again), "repeated call differs"
    # page relabelling: page i of the new cache is page perm[i] of the old
    g = torch.Generator(device=k.device).manual_seed(7)
    perm = torch.randperm(k.shape[0], generator=g, device=k.device)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel(), device=k.device)
    k2, v2 = k[perm], v[perm]
    bt2 = inv[bt.long()].to(torch.int32)
    relabelled = decode(q, k2, v2, sl, bt2, inp.scale)
    del k2, v2
    assert torch.equal(out, relabelled), "page relabelling changed the output"
    # convexity: softmax weights are a probability vector, so each output
    # element lies within [min, max] of its head's V column (small slack for
    # the bf16/fp16 rounding of P and of the output)
    B, Hkv = sl.shape
    G = q.shape[2] // Hkv
    bs = k.shape[1]
    heads = torch.randperm(B * Hkv, generator=torch.Generator().manual_seed(1))[:64].tolist()
    for hd in heads:
        s, h = divmod(hd, Hkv)
        L = int(sl[s, h])
        if L == 0:
            continue
        n = (L + bs - 1) // bs
        V = v[bt[s, h, :n].long()].reshape(-1, v.shape[2])[:L].float()
        lo, hi = V.amin(0), V.amax(0)
        o = out[s, 0, h * G:(h + 1) * G].float()
        slack = 0.02 * (hi - lo) + 1e-3
        assert bool(((o >= lo - slack) & (o <= hi + slack)).all()), (name, s, h)
