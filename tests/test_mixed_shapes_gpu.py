"""GPU: decode calls of different shapes queued back to back on one stream,
with no synchronisation between them, all sharing the stream's workspace.

Each call's planner kernel is launched with programmatic dependent launch
and overlaps the previous call's reduce kernel.  When the previous call laid
the workspace out differently (another batch size, kv-head count, query
group or split count), the new planner must not write into the workspace
before that reduce has finished, or its segment table and head list would
land on partial states still being merged.  Every call's output is checked
against the oracle: as in the reference, whose wrapper allocates fresh
partial buffers per call (src/kernel_triton.py:232-243), a call's result
must not depend on the call before it.
Tolerance: atol = rtol = 2e-2 (scripts/benchmark.py:63-72).
"""
import os

import pytest
import torch

from pagedattention_b200 import flash_attn_with_kvcache_wrapper_b200, paged_attention
from tests.util import assert_close, random_case, run_oracle

pytestmark = pytest.mark.gpu

# few long heads: every head split over many warps, reduce kernel busy
LONG = dict(B=4, Hkv=2, G=4, D=128, bs=16, lens=[[6000, 5000], [7000, 4000], [6500, 3000],
                                                   [5500, 6100]], dtype=torch.bfloat16)
# many short heads: 16,384 heads of 1-64 tokens (a far larger workspace)
SHORT = dict(B=2048, Hkv=8, G=4, D=128, bs=16, lens=None, dtype=torch.bfloat16)
# another query group (another partial-state slot size)
LONG_G8 = dict(B=3, Hkv=2, G=8, D=128, bs=32, lens=[[9000, 100], [3000, 7000], [1, 8000]],
               dtype=torch.bfloat16)
MQA = dict(B=6, Hkv=1, G=32, D=64, bs=8, lens=[[4000], [77], [8000], [513], [2000], [6000]],
           dtype=torch.float16)


def _make(spec, seed, dev):
    lens = spec["lens"]
    if lens is None:
        g = torch.Generator().manual_seed(seed)
        lens = torch.randint(1, 65, (spec["B"], spec["Hkv"]), generator=g).tolist()
    q, k, v, sl, bt, scale = random_case(spec["B"], spec["Hkv"], spec["G"], spec["D"],
                                         spec["bs"], lens, spec["dtype"], seed=seed,
                                         k_scale=4.0 if spec["G"] == 32 else 1.0)
    cpu = (q, k, v, sl, bt)
    return cpu, tuple(t.to(dev) for t in cpu), scale


def _check(results):
    threads = os.cpu_count() or 1
    for i, (cpu, scale, out) in enumerate(results):
        ref = run_oracle(*cpu, scale, threads=threads)
        assert_close(out, ref, what=f"call {i + 1} of the queue")


def test_mixed_shapes_queued_without_sync(cuda_device):
    """short -> long -> short -> long (num_splits 2) -> long, G 8 -> MQA ->
    long: every change of layout in both directions, one stream, one sync."""
    dev = cuda_device
    plan = [(SHORT, 0), (LONG, 0), (SHORT, 0), (LONG, 2), (LONG_G8, 0), (MQA, 0), (LONG, 0),
            (LONG, 7)]
    inputs = [_make(spec, 900 + i, dev) + (splits,) for i, (spec, splits) in enumerate(plan)]
    torch.cuda.synchronize(dev)
    stream = torch.cuda.Stream(dev)  # a fresh stream: a fresh cached workspace
    outs = []
    with torch.cuda.stream(stream):
        for cpu, d, scale, splits in inputs:
            outs.append(flash_attn_with_kvcache_wrapper_b200(*d, scale, num_splits=splits))
    stream.synchronize()
    _check([(cpu, scale, out) for (cpu, _, scale, _), out in zip(inputs, outs)])


def test_mixed_shapes_in_place_outputs(cuda_device):
    """The in-place form, each call writing its own output buffer, shapes
    alternating between many short and few long heads."""
    dev = cuda_device
    plan = [LONG, SHORT, LONG_G8, SHORT, LONG]
    inputs = [_make(spec, 950 + i, dev) for i, spec in enumerate(plan)]
    outs = [torch.full_like(d[0][:, 0], float("nan")) for _, d, _ in inputs]
    torch.cuda.synchronize(dev)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for (cpu, d, scale), out in zip(inputs, outs):
            q, k, v, sl, bt = d
            paged_attention(out, q[:, 0], k, v, bt, sl, scale, k.shape[1])
    stream.synchronize()
    _check([(cpu, scale, out[:, None]) for (cpu, _, scale), out in zip(inputs, outs)])
