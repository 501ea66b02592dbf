"""The Python wrappers' argument handling (mirrors of the reference's error
behaviour) — everything here is refused before any device work."""
import pytest
import torch

from pagedattention_b200 import (_validate_decode_inputs, flash_attn_with_kvcache_wrapper_b200,
                                 paged_attention)


def _inputs(B=1, Hkv=2, G=4, D=64, dtype=torch.bfloat16):
    q = torch.zeros((B, 1, Hkv * G, D), dtype=dtype)
    k = torch.zeros((8, 16, D), dtype=dtype)
    sl = torch.zeros((B, Hkv), dtype=torch.int32)
    bt = torch.zeros((B, Hkv, 4), dtype=torch.int32)
    return q, k, k.clone(), sl, bt


def test_validate_returns_shape_tuple():
    q, k, v, sl, bt = _inputs(B=1, Hkv=2, G=4, D=64)
    assert _validate_decode_inputs(q, sl, bt) == (8, 2, 4, 64)


def test_validate_allows_batch_gt_1():
    q, k, v, sl, bt = _inputs(B=3)
    assert _validate_decode_inputs(q, sl, bt)[0] == 8


@pytest.mark.parametrize("bad", ["q_len", "group", "batch_mismatch", "table_heads"])
def test_validate_asserts_like_reference(bad):
    """AssertionError, as src/common.py:16-29 raises."""
    q, k, v, sl, bt = _inputs()
    if bad == "q_len":
        q = torch.zeros((1, 2, 8, 64))
    elif bad == "group":
        sl = torch.zeros((1, 3), dtype=torch.int32)
        bt = torch.zeros((1, 3, 4), dtype=torch.int32)
    elif bad == "batch_mismatch":
        sl = torch.zeros((2, 2), dtype=torch.int32)
    elif bad == "table_heads":
        bt = torch.zeros((1, 3, 4), dtype=torch.int32)
    with pytest.raises(AssertionError):
        _validate_decode_inputs(q, sl, bt)


def test_fp32_is_a_type_error():
    """TypeError on unsupported dtypes, as src/kernel_triton.py:195-196."""
    q, k, v, sl, bt = _inputs(dtype=torch.float32)
    with pytest.raises(TypeError):
        flash_attn_with_kvcache_wrapper_b200(q, k, v, sl, bt, 0.125)


def test_mixed_dtypes_is_a_type_error():
    q, k, v, sl, bt = _inputs()
    with pytest.raises(TypeError):
        flash_attn_with_kvcache_wrapper_b200(q, k.half(), v, sl, bt, 0.125)


def test_cpu_tensors_are_refused():
    """No CPU fallback: CPU tensors raise instead of computing."""
    q, k, v, sl, bt = _inputs()
    with pytest.raises(ValueError, match="CUDA"):
        flash_attn_with_kvcache_wrapper_b200(q, k, v, sl, bt, 0.125)


def test_paged_attention_checks_block_size():
    q = torch.zeros((2, 8, 64), dtype=torch.bfloat16)
    k = torch.zeros((4, 2, 16, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="block_size"):
        paged_attention(torch.empty_like(q), q, k, k, torch.zeros((2, 3), dtype=torch.int32),
                        torch.zeros(2, dtype=torch.int32), 0.1, 32)


def test_paged_attention_refuses_cpu():
    q = torch.zeros((2, 8, 64), dtype=torch.bfloat16)
    k = torch.zeros((4, 2, 16, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        paged_attention(torch.empty_like(q), q, k, k, torch.zeros((2, 3), dtype=torch.int32),
                        torch.zeros(2, dtype=torch.int32), 0.1, 16)
