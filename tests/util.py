"""Shared helpers of the test suite (inputs, golden vectors, comparisons)."""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import torch

from oracle import eager as oracle

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"
ATOL = 2e-2   # tolerance of the reference's own parity check,
RTOL = 2e-2   # scripts/benchmark.py:63-72,161 (torch.isclose)

TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16}


def golden_names():
    return sorted(p.stem for p in GOLDEN_DIR.glob("*.npz"))


def load_golden(name):
    """Golden case as CPU torch tensors in their 16-bit dtype + fp32 outputs."""
    z = np.load(GOLDEN_DIR / f"{name}.npz")
    dt = TORCH_DT[str(z["dtype"])]

    def t16(a):
        return torch.from_numpy(a.astype(np.uint16).view(np.int16).copy()).view(dt)

    return dict(
        q=t16(z["q"]), k_cache=t16(z["k_cache"]), v_cache=t16(z["v_cache"]),
        cache_seqlens=torch.from_numpy(z["cache_seqlens"].copy()),
        block_table=torch.from_numpy(z["block_table"].copy()),
        softmax_scale=float(z["softmax_scale"]),
        out_fp32=torch.from_numpy(z["out_fp32"].copy()),
        out_native=torch.from_numpy(z["out_native"].copy()),
        dtype=dt,
    )


def run_oracle(q, k_cache, v_cache, cache_seqlens, block_table, scale, threads=1):
    """fp32 oracle on CPU copies of the inputs; returns a float32 torch tensor."""
    out = oracle.flash_attn_with_kvcache(
        q.float().cpu().numpy(), k_cache.float().cpu().numpy(), v_cache.float().cpu().numpy(),
        cache_seqlens.cpu().numpy(), block_table.cpu().numpy(), scale, threads=threads)
    return torch.from_numpy(out)


def assert_close(actual, expected, atol=ATOL, rtol=RTOL, what=""):
    a = actual.float().cpu()
    e = expected.float().cpu()
    assert a.shape == e.shape, (a.shape, e.shape)
    assert torch.isfinite(a).all(), f"{what}: non-finite output"
    ok = torch.isclose(a, e, atol=atol, rtol=rtol)
    if not bool(ok.all()):
        bad = (~ok).nonzero()[:5].tolist()
        diff = (a - e).abs().max().item()
        raise AssertionError(f"{what}: {int((~ok).sum())} mismatches, max |diff| {diff:.4g}, "
                             f"first at {bad}")


def random_case(B, Hkv, G, D, bs, lens, dtype, seed=0, k_scale=1.0, spare_pages=3,
                poison=True, extra_cols=1):
    """Random inputs in the reference's per-head page layout, CPU tensors.

    Unused block-table entries are -1; token slots the reference never reads
    (past each head's length, unused pages) hold NaN when ``poison``.
    ``lens`` is [B][Hkv] (or [B] broadcast over heads).
    """
    g = torch.Generator().manual_seed(seed)
    lens = torch.as_tensor(lens, dtype=torch.int32)
    if lens.dim() == 1:
        lens = lens[:, None].expand(B, Hkv).contiguous()
    nblk = (lens.to(torch.int64) + bs - 1) // bs
    maxb = int(nblk.max()) + extra_cols if lens.numel() else extra_cols
    maxb = max(maxb, 1)
    used = int(nblk.sum())
    P = used + spare_pages
    Hq = Hkv * G
    q = torch.randn((B, 1, Hq, D), generator=g).to(dtype)
    k = (torch.randn((P, bs, D), generator=g) * k_scale).to(dtype)
    v = torch.randn((P, bs, D), generator=g).to(dtype)
    perm = torch.randperm(P, generator=g)[:used].to(torch.int32)
    bt = torch.full((B, Hkv, maxb), -1, dtype=torch.int32)
    valid = torch.zeros((P, bs), dtype=torch.bool)
    off = 0
    for s in range(B):
        for h in range(Hkv):
            n = int(nblk[s, h])
            ids = perm[off:off + n]
            bt[s, h, :n] = ids
            L = int(lens[s, h])
            for i, pid in enumerate(ids.tolist()):
                valid[pid, :min(bs, L - i * bs)] = True
            off += n
    if poison:
        nan = torch.tensor(float("nan"), dtype=dtype)
        k = torch.where(valid[..., None], k, nan)
        v = torch.where(valid[..., None], v, nan)
    return q, k, v, lens, bt, 1.0 / math.sqrt(D)
