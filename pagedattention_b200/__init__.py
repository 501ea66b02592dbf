"""pagedattention_b200 — B200-native (sm_100a) paged-attention decode.

Drop-in for the decode path of lashhw/pagedattention: the same
``flash_attn_with_kvcache_wrapper_*`` signature (src/common.py:1-14) backed by
hand-written CUDA kernels in ``libpab200.so`` (C ABI: include/pab200.h).
"""
from .common import _validate_decode_inputs
from .kernel_b200 import (
    default_scale,
    flash_attn_with_kvcache_wrapper_b200,
    kv_append,
    kv_append_status,
    merge_packed_states,
    merge_states,
    paged_attention,
    paged_attention_exchange,
    paged_attention_states,
    read_status,
    state_numel,
)

__all__ = [
    "_validate_decode_inputs",
    "default_scale",
    "flash_attn_with_kvcache_wrapper_b200",
    "kv_append",
    "kv_append_status",
    "merge_packed_states",
    "merge_states",
    "paged_attention",
    "paged_attention_exchange",
    "paged_attention_states",
    "read_status",
    "state_numel",
]
