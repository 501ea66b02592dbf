"""Interface contract of the decode wrappers.

Mirrors src/common.py of the reference (lashhw/pagedattention):

Interface for flash_attn_with_kvcache_wrapper_*

Args:
    q: Query tensor of shape (batch_size, 1, num_query_heads, head_size)
    k_cache: KV cache for keys of shape (num_blocks, block_size, head_size)
    v_cache: KV cache for values of shape (num_blocks, block_size, head_size)
    cache_seqlens: Sequence lengths of shape (batch_size, num_kv_heads)
    block_table: Block table mapping of shape
        (batch_size, num_kv_heads, max_num_blocks_per_head)
    softmax_scale: Scaling factor for attention scores

Returns:
    Output tensor of shape (batch_size, 1, num_query_heads, head_size)

One relaxation: the reference asserts batch_size == 1 (src/common.py:17-19)
and batches by flattening (sequence, kv head) into its kv-head axis; here any
batch_size >= 1 is accepted, and the flattened batch==1 form computes the same
thing.
"""
from __future__ import annotations


def _validate_decode_inputs(q, cache_seqlens, block_table):
    """Check the decode shapes; return (Hq, Hkv, G, D).

    Same checks and AssertionError behaviour as src/common.py:16-29, except
    that batch_size may exceed 1 (it must agree across the three inputs).
    """
    assert q.dim() == 4, "q must be (batch_size, 1, num_query_heads, head_size)"
    assert cache_seqlens.dim() == 2, "cache_seqlens must be (batch_size, num_kv_heads)"
    assert block_table.dim() == 3, \
        "block_table must be (batch_size, num_kv_heads, max_num_blocks_per_head)"
    assert q.shape[0] >= 1
    assert cache_seqlens.shape[0] == q.shape[0]
    assert block_table.shape[0] == q.shape[0]

    _, q_len, num_query_heads, head_size = q.shape
    _, num_kv_heads = cache_seqlens.shape

    assert q_len == 1
    assert block_table.shape[1] == num_kv_heads
    assert num_query_heads % num_kv_heads == 0

    num_kv_groups = num_query_heads // num_kv_heads

    return num_query_heads, num_kv_heads, num_kv_groups, head_size
