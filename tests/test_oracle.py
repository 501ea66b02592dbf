"""The CPU oracle against the reference's own outputs (golden vectors) and the
algebraic facts the GPU path relies on.  No GPU needed."""
import numpy as np
import pytest
import torch

from oracle import eager as oracle
from oracle import eager_torch
from tests.util import ATOL, RTOL, golden_names, load_golden, random_case, run_oracle


def test_golden_files_present():
    assert len(golden_names()) >= 7


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_golden(name):
    """oracle/eager.py reproduces src/kernel_eager.py's fp32 output."""
    c = load_golden(name)
    out = oracle.flash_attn_with_kvcache_flat(
        c["q"].float().numpy(), c["k_cache"].float().numpy(), c["v_cache"].float().numpy(),
        c["cache_seqlens"].numpy(), c["block_table"].numpy(), c["softmax_scale"])
    np.testing.assert_allclose(out, c["out_fp32"].numpy(), atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("name", golden_names())
def test_torch_restatement_matches_reference_golden(name):
    """oracle/eager_torch.py (the CPU baseline's restatement, the reference's
    own torch operations) reproduces src/kernel_eager.py's fp32 output, and in
    the 16-bit dtype its native output."""
    c = load_golden(name)
    args = (c["k_cache"], c["v_cache"], c["cache_seqlens"], c["block_table"], c["softmax_scale"])
    out = eager_torch.flash_attn_with_kvcache(c["q"].float(), args[0].float(), args[1].float(),
                                             *args[2:])
    np.testing.assert_allclose(out.numpy(), c["out_fp32"].numpy(), atol=1e-5, rtol=1e-5)
    native = eager_torch.flash_attn_with_kvcache(c["q"], *args)
    assert native.dtype == c["q"].dtype
    assert torch.isclose(native.float(), c["out_native"], atol=1e-2, rtol=1e-2).all()


def test_torch_restatement_batched_equals_port():
    """Batch > 1 (flattened as the reference's batch==1 call) agrees with the
    numpy port on poisoned random inputs, empty heads included."""
    q, k, v, sl, bt, scale = random_case(3, 2, 4, 64, 16, [[40, 0], [100, 17], [1, 300]],
                                         torch.float32, seed=5)
    out = eager_torch.flash_attn_with_kvcache(q, k, v, sl, bt, scale)
    ref = run_oracle(q, k, v, sl, bt, scale)
    np.testing.assert_allclose(out.numpy(), ref.numpy(), atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("name", golden_names())
def test_golden_native_dtype_within_tolerance(name):
    """The reference's own bf16/fp16 eager output is within the parity bar of
    its fp32 output, so the bar is attainable by a 16-bit kernel."""
    c = load_golden(name)
    assert torch.isclose(c["out_native"], c["out_fp32"], atol=ATOL, rtol=RTOL).all()


def test_golden_poison_never_read():
    """Golden inputs carry NaN in every byte the reference does not read, yet
    the reference output is finite: the poison marks exactly the unread bytes."""
    c = load_golden("g1_d128_bs16_edges")
    assert torch.isnan(c["k_cache"].float()).any()
    assert torch.isfinite(c["out_fp32"]).all()
    assert (c["block_table"] == -1).any()


def test_materialize_matches_gather():
    q, k, v, sl, bt, scale = random_case(1, 3, 2, 64, 16, [[5, 16, 40]], torch.float16, seed=2,
                                         poison=False)
    ks, vs = oracle.materialize_kvcache(k.float().numpy(), v.float().numpy(), sl[0].numpy(),
                                        bt[0].numpy())
    assert [x.shape[0] for x in ks] == [5, 16, 40]
    page = int(bt[0, 2, 1])
    np.testing.assert_array_equal(ks[2][16:32], k[page].float().numpy())


def test_batched_equals_flattened():
    """Batch B == the reference's flattened batch==1 form (src/common.py:17-19)."""
    B, Hkv, G, D = 3, 2, 4, 64
    q, k, v, sl, bt, scale = random_case(B, Hkv, G, D, 16, [[9, 30], [0, 17], [64, 1]],
                                         torch.bfloat16, seed=5)
    out_b = run_oracle(q, k, v, sl, bt, scale)
    out_f = run_oracle(q.reshape(1, 1, B * Hkv * G, D), k, v, sl.reshape(1, -1),
                       bt.reshape(1, B * Hkv, -1), scale)
    torch.testing.assert_close(out_b.reshape(1, 1, -1, D), out_f)


def test_known_answers():
    q, k, v, sl, bt, scale = random_case(1, 2, 4, 128, 16, [[1, 0]], torch.float16, seed=9)
    out = run_oracle(q, k, v, sl, bt, scale)
    page = int(bt[0, 0, 0])
    for g in range(4):
        torch.testing.assert_close(out[0, 0, g], v[page, 0].float())
    assert torch.count_nonzero(out[0, 0, 4:]) == 0


def test_split_merge_equals_full():
    """LSE merge of any split of the tokens equals full attention
    (src/kernel_triton.py:120-174 algebra), including empty pieces."""
    rng = np.random.default_rng(0)
    G, D, L = 4, 64, 300
    qg = rng.standard_normal((G, D)).astype(np.float32)
    K = (rng.standard_normal((L, D)) * 3).astype(np.float32)
    V = rng.standard_normal((L, D)).astype(np.float32)
    full = oracle._one_head(qg, K, V, 0.125)
    for cuts in ([0, 300], [0, 1, 300], [0, 0, 150, 150, 300], [0, 7, 99, 200, 299, 300]):
        parts = [oracle.split_state(qg, K[a:b], V[a:b], 0.125) for a, b in zip(cuts, cuts[1:])]
        merged = oracle.merge_states([p[0] for p in parts], [p[1] for p in parts])
        np.testing.assert_allclose(merged, full, atol=1e-5, rtol=1e-5)


def test_merge_all_empty_is_zero():
    o = np.zeros((3, 2, 8), np.float32)
    lse = np.full((3, 2), -np.inf, np.float32)
    assert np.count_nonzero(oracle.merge_states(o, lse)) == 0


def test_kv_bytes():
    assert oracle.kv_bytes([[4096] * 8] * 64, 128, 2) == 1 << 30
