"""Named decode workloads and their seeded synthetic inputs.

The five configurations are the ones the paged decode path is measured on
(none comes from a public dataset; all inputs are seeded N(0, 1) tensors):

  mha_cpu        8 seqs, 32/32 heads, D 128, bs 16, lens ~ U[1, 1024], fp16,
                 1024-block pool (small enough for the CPU oracle)
  llama8b_gqa    64 seqs, 32/8 heads, D 128, bs 16, every len 4096, bf16,
                 pool 1.25x the needed blocks  (the headline workload)
  llama70b_mixed 256 seqs, 64/8 heads, D 128, bs 32,
                 lens ~ lognormal(median 2048, sigma 0.8) clipped to [16, 16384]
  long_context   4 seqs, 32/8 heads, D 128, bs 16, lens 32k/64k/96k/128k
  mqa_small_page 128 seqs, 32/1 heads, D 64, bs 8, lens ~ U[512, 8192], fp16,
                 K scaled by 4, 2x oversized pool

Pools are vLLM-style [num_blocks, num_kv_heads, block_size, head_size] ("HND");
``DecodeInputs.reference_layout()`` views one as the reference's per-head page
cache [num_blocks*num_kv_heads, block_size, head_size] with block_table
[B, Hkv, max_blocks] = block*Hkv + h, the layout of src/common.py:1-14.
Block ids are consecutive slices of one random permutation of the pool, as
scripts/benchmark.py:101-108 assigns them.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    num_seqs: int
    num_q_heads: int
    num_kv_heads: int
    head_size: int
    block_size: int
    dtype: torch.dtype
    lens: tuple            # ("uniform", lo, hi) | ("const", L) | ("lognormal", med, sigma, lo, hi) | ("list", ...)
    pool: tuple = ("needed",)  # ("blocks", n) | ("factor", f) | ("needed",)
    k_scale: float = 1.0
    partition_tokens: int = 0
    description: str = ""

    @property
    def group(self) -> int:
        return self.num_q_heads // self.num_kv_heads


WORKLOADS = {
    "mha_cpu": Workload(
        "mha_cpu", 8, 32, 32, 128, 16, torch.float16, ("uniform", 1, 1024),
        pool=("blocks", 1024),
        description="MHA decode, CPU-runnable: 8 seqs, 32/32 heads, D128, bs16, "
                    "lens U[1,1024], 1024-block pool"),
    "llama8b_gqa": Workload(
        "llama8b_gqa", 64, 32, 8, 128, 16, torch.bfloat16, ("const", 4096),
        pool=("factor", 1.25),
        description="Llama-3-8B GQA decode: 64 seqs x 4096 tokens, 32/8 heads, D128, bs16, "
                    "pool 1.25x needed"),
    "llama70b_mixed": Workload(
        "llama70b_mixed", 256, 64, 8, 128, 32, torch.bfloat16,
        ("lognormal", 2048, 0.8, 16, 16384), pool=("needed",),
        description="Llama-3-70B mixed lengths: 256 seqs, 64/8 heads, D128, bs32, "
                    "lens lognormal(2048, 0.8) in [16,16384]"),
    "long_context": Workload(
        "long_context", 4, 32, 8, 128, 16, torch.bfloat16,
        ("list", 32768, 65536, 98304, 131072), pool=("needed",), partition_tokens=512,
        description="Long-context split-KV: 4 seqs of 32k/64k/96k/128k, 32/8 heads, D128, bs16"),
    "mqa_small_page": Workload(
        "mqa_small_page", 128, 32, 1, 64, 8, torch.float16, ("uniform", 512, 8192),
        pool=("factor", 2.0), k_scale=4.0,
        description="Small-page MQA stress: 128 seqs, 32/1 heads, D64, bs8, lens U[512,8192], "
                    "K x4, 2x pool"),
}

HEADLINE = "llama8b_gqa"


def sample_lens(w: Workload, seed: int = 42) -> torch.Tensor:
    """Context lengths [num_seqs] int32, drawn on the CPU from ``seed``."""
    g = torch.Generator().manual_seed(seed)
    kind = w.lens[0]
    B = w.num_seqs
    if kind == "uniform":
        lo, hi = w.lens[1], w.lens[2]
        lens = torch.randint(lo, hi + 1, (B,), generator=g)
    elif kind == "const":
        lens = torch.full((B,), w.lens[1])
    elif kind == "lognormal":
        med, sigma, lo, hi = w.lens[1:]
        x = torch.exp(torch.randn(B, generator=g, dtype=torch.float64) * sigma + math.log(med))
        lens = torch.clamp(torch.round(x), lo, hi)
    elif kind == "list":
        vals = list(w.lens[1:])
        lens = torch.tensor([vals[i % len(vals)] for i in range(B)])
    else:
        raise ValueError(kind)
    return lens.to(torch.int32)


@dataclass
class DecodeInputs:
    workload: Workload
    q: torch.Tensor              # [B, Hq, D]
    k_pool: torch.Tensor         # [num_blocks, Hkv, bs, D]
    v_pool: torch.Tensor
    block_tables: torch.Tensor   # [B, max_blocks] int32 block ids
    context_lens: torch.Tensor   # [B] int32
    scale: float
    extra: dict = field(default_factory=dict)

    def reference_layout(self):
        """(q, k_cache, v_cache, cache_seqlens, block_table) in the shapes of
        src/common.py:1-14 (batch = num_seqs)."""
        B, Hq, D = self.q.shape
        nb, Hkv, bs, _ = self.k_pool.shape
        k_pages = self.k_pool.view(nb * Hkv, bs, D)
        v_pages = self.v_pool.view(nb * Hkv, bs, D)
        heads = torch.arange(Hkv, dtype=torch.int32, device=self.block_tables.device)
        bt = (self.block_tables[:, None, :] * Hkv + heads[None, :, None]).to(torch.int32)
        seqlens = self.context_lens[:, None].expand(B, Hkv).contiguous()
        return self.q[:, None], k_pages, v_pages, seqlens, bt

    def kv_bytes(self) -> int:
        w = self.workload
        elt = torch.finfo(self.q.dtype).bits // 8
        return int(self.context_lens.to(torch.int64).sum()) * w.num_kv_heads * w.head_size * elt * 2


def _randn(shape, gen, device, dtype, scale=1.0, chunk_elems=1 << 27):
    """N(0,1)*scale in ``dtype``, generated in chunks to bound fp32 temporaries."""
    out = torch.empty(shape, dtype=dtype, device=device)
    flat = out.view(-1)
    n = flat.numel()
    gdev = gen.device
    for i in range(0, n, chunk_elems):
        j = min(n, i + chunk_elems)
        x = torch.randn(j - i, generator=gen, device=gdev)
        if scale != 1.0:
            x.mul_(scale)
        flat[i:j].copy_(x.to(dtype))
    return out


def make_inputs(w: Workload, seed: int = 42, device="cpu", gen_device="cpu",
                lens: torch.Tensor | None = None, num_seqs: int | None = None) -> DecodeInputs:
    """Seeded inputs for workload ``w``.

    Lengths and block ids always come from a CPU generator; tensor values come
    from a generator on ``gen_device`` (CPU by default, so CPU and GPU copies
    are identical; "cuda" is much faster for the multi-GB workloads).
    ``num_seqs`` takes the first n sequences of the workload (a bounded sample).
    """
    if lens is None:
        lens = sample_lens(w, seed)
    if num_seqs is not None:
        lens = lens[:num_seqs]
    lens = lens.to(torch.int32)
    B = lens.numel()
    bs, Hkv, D = w.block_size, w.num_kv_heads, w.head_size
    nblk = (lens.to(torch.int64) + bs - 1) // bs
    needed = int(nblk.sum())
    maxb = max(int(nblk.max()) if B else 0, 1)
    kind = w.pool[0]
    if kind == "blocks":
        pool = max(int(w.pool[1]), needed)
    elif kind == "factor":
        pool = int(math.ceil(needed * w.pool[1]))
    else:
        pool = needed
    pool = max(pool, 1)
    g_cpu = torch.Generator().manual_seed(seed + 1)
    perm = torch.randperm(pool, generator=g_cpu)[:needed].to(torch.int32)
    bt = torch.zeros((B, maxb), dtype=torch.int32)
    off = 0
    for s in range(B):
        n = int(nblk[s])
        bt[s, :n] = perm[off:off + n]
        off += n
    gen = torch.Generator(device=gen_device).manual_seed(seed + 2)
    q = _randn((B, w.num_q_heads, D), gen, device, w.dtype)
    k = _randn((pool, Hkv, bs, D), gen, device, w.dtype, scale=w.k_scale)
    v = _randn((pool, Hkv, bs, D), gen, device, w.dtype)
    return DecodeInputs(w, q, k, v, bt.to(device), lens.to(device), 1.0 / math.sqrt(D))
