"""CPU oracle for the paged-attention decode path — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
import it.  The product path (``pagedattention_b200``) never calls it and fails
loudly when its CUDA library is missing.

It restates, in numpy float32, the reference's eager PyTorch implementation
(lashhw/pagedattention):

* ``materialize_kvcache``      follows src/kernel_eager.py:6-26
* ``flash_attn_with_kvcache``  follows src/kernel_eager.py:29-56
* ``split_state`` / ``merge_states`` restate the split-KV partial state of
  src/kernel_triton.py:8-117 and its log-sum-exp merge,
  src/kernel_triton.py:120-174, used to check the cross-device path.
* ``kv_append`` has no counterpart in the reference (which only reads the
  cache): it states the write that precedes a decode step — the new token's
  K and V go to row L % block_size of page block_table[L // block_size],
  L being the current length — in the page layout of src/common.py:6-7.

Parity is pinned: tests/golden/ holds vectors produced by importing the
reference's own ``flash_attn_with_kvcache_wrapper_eager`` (fp32, CPU), and
tests/test_oracle.py checks this restatement against every one of them.

Batch handling: the reference asserts batch == 1 (src/common.py:17-19) and
obtains batching by flattening (sequence, kv head) into its kv-head axis.  The
oracle accepts batch >= 1 and loops over sequences, which is the same
computation (q head (s*Hkv + h)*G + g of the flattened call is q head h*G + g
of sequence s).
"""
from __future__ import annotations

import math
from concurrent.futures import ThreadPoolExecutor

import numpy as np


def _ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


def materialize_kvcache(k_cache, v_cache, seqlens, block_table):
    """Gather every kv head's pages into contiguous [L, D] K and V.

    src/kernel_eager.py:6-26: for kv head h, take the first ceil(L/bs)
    entries of its block-table row, gather those pages, flatten
    (page, token) and truncate to L tokens.

    k_cache, v_cache: [num_pages, block_size, D]
    seqlens: [Hkv] ints; block_table: [Hkv, max_blocks] ints.
    """
    block_size = k_cache.shape[1]
    k_heads, v_heads = [], []
    for h in range(len(seqlens)):
        L = int(seqlens[h])
        nblk = _ceil_div(L, block_size)
        ids = np.asarray(block_table[h, :nblk], dtype=np.int64)
        k_heads.append(k_cache[ids].reshape(-1, k_cache.shape[2])[:L])
        v_heads.append(v_cache[ids].reshape(-1, v_cache.shape[2])[:L])
    return k_heads, v_heads


def _softmax_fp32(x):
    # torch.nn.functional.softmax(..., dtype=float32): max-subtracted exp / sum
    x = x.astype(np.float32, copy=False)
    if x.shape[-1] == 0:
        return x
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=-1, keepdims=True)


def _one_head(qg, K, V, scale):
    """softmax(qg K^T * scale) V for one kv head (src/kernel_eager.py:51-53)."""
    scores = (qg @ K.T) * np.float32(scale)
    p = _softmax_fp32(scores)
    return p @ V


def flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens, block_table,
                            softmax_scale, threads: int = 1):
    """Eager decode attention in float32.

    src/kernel_eager.py:29-56 with batch >= 1.

    q: [B, 1, Hq, D]; k_cache, v_cache: [num_pages, block_size, D];
    cache_seqlens: [B, Hkv]; block_table: [B, Hkv, max_blocks].
    Returns [B, 1, Hq, D] float32.
    """
    q = np.asarray(q, dtype=np.float32)
    B, q_len, Hq, D = q.shape
    assert q_len == 1
    Hkv = cache_seqlens.shape[1]
    assert Hq % Hkv == 0
    G = Hq // Hkv
    bs = k_cache.shape[1]
    out = np.zeros((B, 1, Hq, D), dtype=np.float32)

    def work(item):
        s, h = item
        L = int(cache_seqlens[s, h])
        nblk = _ceil_div(L, bs)
        ids = np.asarray(block_table[s, h, :nblk], dtype=np.int64)
        K = np.asarray(k_cache[ids], dtype=np.float32).reshape(-1, D)[:L]
        V = np.asarray(v_cache[ids], dtype=np.float32).reshape(-1, D)[:L]
        qg = q[s, 0, h * G:(h + 1) * G]
        out[s, 0, h * G:(h + 1) * G] = _one_head(qg, K, V, softmax_scale)

    items = [(s, h) for s in range(B) for h in range(Hkv)]
    if threads > 1:
        # one BLAS thread per worker: nested BLAS threads oversubscribe the cores
        from threadpoolctl import threadpool_limits
        with threadpool_limits(1), ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(work, items))
    else:
        for it in items:
            work(it)
    return out


def flash_attn_with_kvcache_flat(q, k_cache, v_cache, cache_seqlens, block_table,
                                 softmax_scale):
    """The reference's own batch==1 form (src/common.py:16-29 shapes)."""
    assert q.shape[0] == 1 and cache_seqlens.shape[0] == 1 and block_table.shape[0] == 1
    return flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens, block_table,
                                   softmax_scale)


def split_state(qg, K, V, scale):
    """Normalised output and log-sum-exp of one token range.

    Restates the partial state of src/kernel_triton.py:93-117 (running max m,
    exp-sum l, accumulator acc) in the (o = acc/l, lse = m + log l) form.
    Empty range: o = 0, lse = -inf.
    """
    G, D = qg.shape
    if K.shape[0] == 0:
        return np.zeros((G, D), np.float32), np.full((G,), -np.inf, np.float32)
    s = (qg.astype(np.float32) @ K.astype(np.float32).T) * np.float32(scale)
    m = s.max(axis=-1)
    e = np.exp(s - m[:, None])
    l = e.sum(axis=-1)
    o = (e @ V.astype(np.float32)) / l[:, None]
    return o.astype(np.float32), (m + np.log(l)).astype(np.float32)


def merge_states(os_, lses):
    """Log-sum-exp merge of partial states (src/kernel_triton.py:144-174).

    os_: [N, ..., D]; lses: [N, ...].  States with lse = -inf carry no weight
    (the has_partial guard of :157-163); all-empty rows give zeros (:172-174).
    """
    os_ = np.asarray(os_, dtype=np.float32)
    lses = np.asarray(lses, dtype=np.float32)
    M = lses.max(axis=0)
    Msafe = np.where(np.isfinite(M), M, 0.0)
    w = np.where(np.isfinite(lses), np.exp(lses - Msafe[None]), 0.0)
    L = w.sum(axis=0)
    acc = (w[..., None] * os_).sum(axis=0)
    return np.where(L[..., None] > 0, acc / np.where(L > 0, L, 1.0)[..., None], 0.0).astype(np.float32)


def kv_bytes(cache_seqlens, head_size: int, elt_bytes: int) -> int:
    """Algorithmic K+V bytes of one decode call: sum over heads of L*D*elt*2."""
    return int(np.asarray(cache_seqlens, dtype=np.int64).sum()) * head_size * elt_bytes * 2


def default_scale(head_size: int) -> float:
    return 1.0 / math.sqrt(head_size)


def kv_append(k_cache, v_cache, k_new, v_new, cache_seqlens, block_table, increment=True):
    """Write each (sequence, kv head)'s new token into its page (in place).

    k_cache/v_cache: [num_pages, block_size, D] (src/common.py:6-7); k_new,
    v_new: [B, Hkv, D]; cache_seqlens: [B, Hkv] (current lengths L);
    block_table: [B, Hkv, max_blocks].  Row L % block_size of page
    block_table[s, h, L // block_size] receives the token; with ``increment``
    the length becomes L + 1.  A (sequence, kv head) whose L is negative,
    whose page slot lies past max_blocks or whose page id is outside the cache
    is left untouched.  No counterpart in the reference.
    """
    k_cache, v_cache = np.asarray(k_cache), np.asarray(v_cache)
    k_new, v_new = np.asarray(k_new), np.asarray(v_new)
    lens = np.asarray(cache_seqlens).copy()
    bt = np.asarray(block_table)
    num_pages, bs, _ = k_cache.shape
    B, Hkv = lens.shape
    for s in range(B):
        for h in range(Hkv):
            L = int(lens[s, h])
            if L < 0 or L // bs >= bt.shape[2]:
                continue
            page = int(bt[s, h, L // bs])
            if not 0 <= page < num_pages:
                continue
            k_cache[page, L % bs] = k_new[s, h]
            v_cache[page, L % bs] = v_new[s, h]
            if increment:
                lens[s, h] = L + 1
    return lens
