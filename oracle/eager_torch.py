"""CPU restatement of the reference's eager decode in PyTorch — TEST AND
CPU-TIMING INFRASTRUCTURE ONLY (imported by ``tests/`` and by ``bench.py``'s
CPU timing / reference arm; never by the product path).

``oracle/eager.py`` restates src/kernel_eager.py:6-56 in numpy with a thread
pool over heads; it is the checker.  This module restates the same function
with the same PyTorch operations, in the same order and granularity, so that
its run time on the host is the reference's own CPU cost:

* per kv head, the lengths are read one by one and the head's pages are
  gathered by advanced indexing, flattened and truncated to its length
  (src/kernel_eager.py:6-26);
* per kv head, ``matmul(q_group, K^T) * scale``, softmax over keys in
  float32 cast back to the input dtype, ``matmul(P, V)`` (:43-54);
* the groups are concatenated along the head axis (:56).

Batch >= 1 is handled as the reference's own batch==1 call on the
flattened (sequence, kv head) axis, which is the same computation (query
head (s*Hkv + h)*G + g of the flattened call is query head h*G + g of
sequence s).  PyTorch's CPU kernels use every thread ``torch.set_num_threads``
allows, as the reference does when run on the host.
"""
from __future__ import annotations

import torch


def flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale):
    """Eager decode attention; q (B, 1, Hq, D), caches (pages, block_size,
    D), cache_seqlens (B, Hkv), block_table (B, Hkv, max_blocks) — CPU
    tensors of one floating dtype.  Returns (B, 1, Hq, D) in that dtype."""
    B, q_len, Hq, D = q.shape
    assert q_len == 1
    Hkv = cache_seqlens.shape[1]
    assert Hq % Hkv == 0
    G = Hq // Hkv
    bs = k_cache.shape[1]
    flat_lens = cache_seqlens.reshape(B * Hkv)
    flat_table = block_table.reshape(B * Hkv, -1)
    # (1, Hq', 1, D): the query heads of the flattened call, head-major
    qh = q.reshape(1, B * Hq, 1, D)
    # the gather pass: every head's K and V made contiguous first
    keys, values = [], []
    for hd in range(B * Hkv):
        L = int(flat_lens[hd].item())
        ids = flat_table[hd, :(L + bs - 1) // bs]
        keys.append(k_cache[ids].flatten(0, 1)[:L])
        values.append(v_cache[ids].flatten(0, 1)[:L])
    # the attention pass, one kv head (G query heads) at a time
    groups = []
    for hd in range(B * Hkv):
        qg = qh[:, hd * G:(hd + 1) * G]
        scores = torch.matmul(qg, keys[hd][None, None].transpose(-2, -1)) * softmax_scale
        p = torch.softmax(scores, dim=-1, dtype=torch.float32).to(q.dtype)
        groups.append(torch.matmul(p, values[hd][None, None]))
    return torch.cat(groups, dim=1).reshape(B, 1, Hq, D)
