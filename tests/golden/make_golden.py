"""Generate the golden decode vectors in tests/golden/*.npz from the reference.

Run in a container that has the reference checkout (read-only is fine),
naming its root with --reference or the PAB200_REFERENCE environment
variable:

    python tests/golden/make_golden.py --reference <path of the reference checkout>

It imports the reference's own ``flash_attn_with_kvcache_wrapper_eager``
(src/kernel_eager.py:29-56) and runs it on CPU in float32 on seeded inputs in
the reference's batch==1 layout (src/common.py:1-14).  Inputs are rounded to
bf16 / fp16 first and stored as raw 16-bit patterns, so a GPU kernel fed the
same bits sees exactly the values the reference saw.  Every byte the reference
does not read is poisoned with NaN (token slots past a head's length in its
last page, and unused pages), and unused block-table entries are -1, so a
kernel that reads past the valid range fails the comparison.

Each file holds: q, k_cache, v_cache (uint16 bit patterns), dtype ("bf16" or
"f16"), cache_seqlens [1, Hkv] int32, block_table [1, Hkv, max_blocks] int32,
softmax_scale, out_fp32 (reference output in float32) and out_native (the
reference run in the 16-bit dtype itself, for information).
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# name: (Hkv, G, D, block_size, seqlens, dtype, k_scale)
CASES = {
    "g1_d128_bs16_edges": (6, 1, 128, 16, [1, 15, 16, 17, 40, 0], "f16", 1.0),
    "g4_d128_bs16": (4, 4, 128, 16, [33, 64, 100, 7], "bf16", 1.0),
    "g8_d128_bs32": (2, 8, 128, 32, [31, 97], "bf16", 1.0),
    "g32_d64_bs8_kx4": (2, 32, 64, 8, [9, 120], "f16", 4.0),
    "g2_d256_bs64": (2, 2, 256, 64, [65, 130], "bf16", 1.0),
    "g16_d128_bs8": (2, 16, 128, 8, [24, 57], "bf16", 1.0),
    "g4_d64_bs16_long": (1, 4, 64, 16, [300], "f16", 1.0),
}

TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16}


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def make_case(name, spec, seed):
    Hkv, G, D, bs, seqlens, dt, k_scale = spec
    tdt = TORCH_DT[dt]
    gen = torch.Generator().manual_seed(seed)
    Hq = Hkv * G
    nblk = [(L + bs - 1) // bs for L in seqlens]
    max_blocks = max(max(nblk), 1) + 1          # one spare column, left at -1
    used = sum(nblk)
    num_pages = used + 3                         # three never-referenced pages
    q = torch.randn((1, 1, Hq, D), generator=gen).to(tdt)
    k = (torch.randn((num_pages, bs, D), generator=gen) * k_scale).to(tdt)
    v = torch.randn((num_pages, bs, D), generator=gen).to(tdt)
    perm = torch.randperm(num_pages, generator=gen)[:used].to(torch.int32)
    block_table = torch.full((1, Hkv, max_blocks), -1, dtype=torch.int32)
    valid = torch.zeros((num_pages, bs), dtype=torch.bool)
    off = 0
    for h, (L, n) in enumerate(zip(seqlens, nblk)):
        ids = perm[off:off + n]
        block_table[0, h, :n] = ids
        for i, pid in enumerate(ids.tolist()):
            valid[pid, : min(bs, L - i * bs)] = True
        off += n
    nan = torch.tensor(float("nan"), dtype=tdt)
    k = torch.where(valid[..., None], k, nan)
    v = torch.where(valid[..., None], v, nan)
    cache_seqlens = torch.tensor([seqlens], dtype=torch.int32)
    scale = 1.0 / float(np.sqrt(D))
    return q, k, v, cache_seqlens, block_table, scale, dt


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PAB200_REFERENCE"),
                    help="root of the reference checkout (default: $PAB200_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or PAB200_REFERENCE")
    sys.path.insert(0, str(Path(args.reference) / "src"))
    from kernel_eager import flash_attn_with_kvcache_wrapper_eager  # the reference

    for i, (name, spec) in enumerate(CASES.items()):
        q, k, v, lens, bt, scale, dt = make_case(name, spec, seed=1000 + i)
        out32 = flash_attn_with_kvcache_wrapper_eager(
            q.float(), k.float(), v.float(), lens, bt, scale, num_splits=1)
        out_native = flash_attn_with_kvcache_wrapper_eager(q, k, v, lens, bt, scale, num_splits=1)
        assert torch.isfinite(out32).all(), name
        np.savez_compressed(
            HERE / f"{name}.npz",
            q=_bits(q), k_cache=_bits(k), v_cache=_bits(v), dtype=np.array(dt),
            cache_seqlens=lens.numpy(), block_table=bt.numpy(),
            softmax_scale=np.array(scale, dtype=np.float64),
            out_fp32=out32.numpy().astype(np.float32),
            out_native=out_native.float().numpy().astype(np.float32),
        )
        print(f"{name}: q{tuple(q.shape)} pages={k.shape[0]} lens={lens.tolist()[0]}")


if __name__ == "__main__":
    main()
