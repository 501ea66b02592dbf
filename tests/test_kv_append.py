"""KV append — the cache write before a decode step (no counterpart in the
reference, whose decode only reads the cache).  CPU: the oracle's semantics,
the C struct mirror and host-side argument checks.  GPU: bit-exact parity with
the oracle for the page cache and the HND / NHD pools, per-head and
per-sequence lengths, the status bits, and a decode after the append."""
import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import eager as oracle
from pagedattention_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def test_oracle_writes_the_row_at_the_current_length():
    bs, D = 4, 2
    k = np.zeros((5, bs, D), np.float32)
    v = np.zeros((5, bs, D), np.float32)
    lens = np.array([[5, 0]], np.int32)
    bt = np.array([[[3, 1], [2, 4]]], np.int32)
    kn = np.array([[[1, 2], [3, 4]]], np.float32)
    new = oracle.kv_append(k, v, kn, -kn, lens, bt)
    assert new.tolist() == [[6, 1]]
    assert k[1, 1].tolist() == [1, 2] and v[1, 1].tolist() == [-1, -2]  # L=5: page bt[1], row 1
    assert k[2, 0].tolist() == [3, 4]                                   # L=0: page bt[0], row 0
    assert np.count_nonzero(k) == 4


def test_oracle_leaves_full_and_invalid_entries_untouched():
    k = np.zeros((2, 2, 2), np.float32)
    v = np.zeros_like(k)
    lens = np.array([[4, 1]], np.int32)               # 4 = max_blocks * bs: full
    bt = np.array([[[0, 1], [7, 0]]], np.int32)       # page 7 is outside the cache
    new = oracle.kv_append(k, v, np.ones((1, 2, 2), np.float32), np.ones((1, 2, 2), np.float32),
                           lens, bt)
    assert new.tolist() == [[4, 1]] and np.count_nonzero(k) == 0


def test_struct_layout_matches_c(tmp_path):
    fields = [f for f, _ in _lib.KvAppendArgs._fields_]
    src = ['#include <stdio.h>', '#include <stddef.h>', '#include "pab200.h"', 'int main(void){',
           'printf("size %zu\\n", sizeof(pab200_kv_append_args));']
    src += [f'printf("{f} %zu\\n", offsetof(pab200_kv_append_args, {f}));' for f in fields]
    src += ['return 0;}']
    c = tmp_path / "layout.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", str(ROOT / "include"), str(c), "-o", str(exe)],
                   check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True,
                                                       text=True, check=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(_lib.KvAppendArgs)
    for f in fields:
        assert int(out[f]) == getattr(_lib.KvAppendArgs, f).offset, f


def test_host_argument_checks():
    lib = _lib.load()
    assert lib.pab200_kv_append(None, None) == _lib.ERR_INVALID_ARGUMENT
    a = _lib.KvAppendArgs()
    a.dtype, a.layout = 9, _lib.LAYOUT_PAGES
    assert lib.pab200_kv_append(ctypes.byref(a), None) == _lib.ERR_UNSUPPORTED
    a.dtype = _lib.DTYPE_BF16
    a.num_seqs, a.num_kv_heads, a.head_size, a.block_size, a.max_blocks = 2, 2, 127, 16, 4
    assert lib.pab200_kv_append(ctypes.byref(a), None) == _lib.ERR_INVALID_ARGUMENT  # odd D
    a.head_size = 128
    assert lib.pab200_kv_append(ctypes.byref(a), None) == _lib.ERR_INVALID_ARGUMENT  # nulls
    a.num_seqs = 0
    assert lib.pab200_kv_append(ctypes.byref(a), None) == _lib.OK                    # nothing to do


# ----------------------------------------------------------------------- GPU
def _case(B, Hkv, D, bs, maxb, num_pages, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn((num_pages, bs, D), generator=g).to(dtype)
    v = torch.randn((num_pages, bs, D), generator=g).to(dtype)
    bt = torch.randperm(num_pages, generator=g)[:B * Hkv * maxb].to(torch.int32).reshape(B, Hkv, maxb)
    lens = torch.randint(0, maxb * bs, (B, Hkv), generator=g, dtype=torch.int32)
    kn = torch.randn((B, Hkv, D), generator=g).to(dtype)
    vn = torch.randn((B, Hkv, D), generator=g).to(dtype)
    return k, v, kn, vn, lens, bt


def _oracle(k, v, kn, vn, lens, bt):
    """The oracle on raw 16-bit patterns (a copy is exact in any dtype)."""
    k2, v2 = k.view(torch.int16).numpy().copy(), v.view(torch.int16).numpy().copy()
    new = oracle.kv_append(k2, v2, kn.view(torch.int16).numpy(), vn.view(torch.int16).numpy(),
                           lens.numpy(), bt.numpy())
    return torch.from_numpy(k2).view(k.dtype), torch.from_numpy(v2).view(v.dtype), torch.from_numpy(new)


@pytest.mark.gpu
@pytest.mark.parametrize("D,bs,dtype", [(128, 16, torch.bfloat16), (64, 8, torch.float16),
                                        (256, 32, torch.bfloat16)])
def test_page_cache_parity(cuda_device, D, bs, dtype):
    from pagedattention_b200 import kv_append, kv_append_status
    k, v, kn, vn, lens, bt = _case(6, 3, D, bs, 5, 120, dtype, seed=D + bs)
    ek, ev, elens = _oracle(k, v, kn, vn, lens, bt)
    dev = cuda_device
    kd, vd, ld = k.to(dev), v.to(dev), lens.to(dev)
    kv_append(kd, vd, kn.to(dev), vn.to(dev), ld, bt.to(dev))
    assert torch.equal(kd.cpu(), ek) and torch.equal(vd.cpu(), ev)
    assert torch.equal(ld.cpu(), elens)
    assert kv_append_status(dev) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["HND", "NHD"])
def test_pool_layouts_parity(cuda_device, layout):
    """Per-sequence lengths over a vLLM-style pool: every kv head of a
    sequence writes at the shared length, which then moves once."""
    from pagedattention_b200 import kv_append
    B, Hkv, D, bs, maxb, nb = 5, 4, 128, 16, 6, 40
    g = torch.Generator().manual_seed(4)
    shape = (nb, Hkv, bs, D) if layout == "HND" else (nb, bs, Hkv, D)
    pk = torch.randn(shape, generator=g).to(torch.bfloat16)
    pv = torch.randn(shape, generator=g).to(torch.bfloat16)
    bt = torch.randperm(nb, generator=g)[:B * maxb].to(torch.int32).reshape(B, maxb)
    lens = torch.randint(0, maxb * bs, (B,), generator=g, dtype=torch.int32)
    kn = torch.randn((B, Hkv, D), generator=g).to(torch.bfloat16)
    vn = torch.randn((B, Hkv, D), generator=g).to(torch.bfloat16)
    # the same write in the reference page layout
    heads = torch.arange(Hkv, dtype=torch.int32)
    if layout == "HND":
        kp, vp = pk.reshape(nb * Hkv, bs, D), pv.reshape(nb * Hkv, bs, D)
        bt3 = bt[:, None, :] * Hkv + heads[None, :, None]
    else:  # one page per (block, head) after moving the head axis forward
        kp = pk.permute(0, 2, 1, 3).reshape(nb * Hkv, bs, D)
        vp = pv.permute(0, 2, 1, 3).reshape(nb * Hkv, bs, D)
        bt3 = bt[:, None, :] * Hkv + heads[None, :, None]
    ek, ev, _ = _oracle(kp, vp, kn, vn, lens[:, None].expand(B, Hkv).contiguous(), bt3)
    dev = cuda_device
    kd, vd, ld = pk.to(dev), pv.to(dev), lens.to(dev)
    kv_append(kd, vd, kn.to(dev), vn.to(dev), ld, bt.to(dev), kv_layout=layout)
    got_k, got_v = kd.cpu(), vd.cpu()
    if layout == "HND":
        got_k, got_v = got_k.reshape(nb * Hkv, bs, D), got_v.reshape(nb * Hkv, bs, D)
    else:
        got_k = got_k.permute(0, 2, 1, 3).reshape(nb * Hkv, bs, D)
        got_v = got_v.permute(0, 2, 1, 3).reshape(nb * Hkv, bs, D)
    assert torch.equal(got_k, ek) and torch.equal(got_v, ev)
    assert torch.equal(ld.cpu(), lens + 1)


@pytest.mark.gpu
def test_full_table_and_bad_page_set_status(cuda_device):
    from pagedattention_b200 import kv_append, kv_append_status
    k, v, kn, vn, lens, bt = _case(2, 2, 128, 16, 2, 20, torch.bfloat16, seed=9)
    lens[0, 0] = 2 * 16          # no page slot left
    bt[1, 1, :] = 1000           # page id outside the cache
    lens[1, 1] = 3
    ek, ev, elens = _oracle(k, v, kn, vn, lens, bt)
    dev = cuda_device
    kv_append_status(dev)        # clear bits of earlier tests
    kd, vd, ld = k.to(dev), v.to(dev), lens.to(dev)
    kv_append(kd, vd, kn.to(dev), vn.to(dev), ld, bt.to(dev))
    assert torch.equal(kd.cpu(), ek) and torch.equal(vd.cpu(), ev)
    assert torch.equal(ld.cpu(), elens)
    bits = kv_append_status(dev)
    assert bits & _lib.STATUS_APPEND_FULL and bits & _lib.STATUS_BAD_PAGE_ID


@pytest.mark.gpu
def test_decode_after_append(cuda_device):
    """Three decode steps, each appending its token first: the decode output
    of every step matches the oracle on the oracle-appended cache."""
    from pagedattention_b200 import flash_attn_with_kvcache_wrapper_b200 as decode, kv_append
    from tests.util import assert_close, run_oracle
    B, Hkv, G, D, bs, maxb = 3, 2, 4, 128, 16, 40
    k, v, _, _, lens, bt = _case(B, Hkv, D, bs, maxb, 300, torch.bfloat16, seed=13)
    lens = torch.tensor([[100, 5], [600, 17], [0, 333]], dtype=torch.int32)
    dev = cuda_device
    kd, vd, ld, btd = k.to(dev), v.to(dev), lens.to(dev), bt.to(dev)
    g = torch.Generator().manual_seed(2)
    for step in range(3):
        kn = torch.randn((B, Hkv, D), generator=g).to(torch.bfloat16)
        vn = torch.randn((B, Hkv, D), generator=g).to(torch.bfloat16)
        q = torch.randn((B, 1, Hkv * G, D), generator=g).to(torch.bfloat16)
        k, v, lens = _oracle(k, v, kn, vn, lens, bt)
        kv_append(kd, vd, kn.to(dev), vn.to(dev), ld, btd)
        out = decode(q.to(dev), kd, vd, ld, btd, D ** -0.5)
        assert_close(out, run_oracle(q, k, v, lens, bt, D ** -0.5), what=f"step {step}")


def test_decode_append_refuses_mismatched_arguments():
    """pab200_decode_append checks on the host that the append addresses
    the decode call's own caches, block table and lengths."""
    lib = _lib.load()
    a = _lib.DecodeArgs()
    a.k_cache = a.v_cache = a.q = a.out = a.seqlens = a.block_table = 4096
    app = _lib.KvAppendArgs()
    app.k_cache = app.v_cache = app.k_new = app.v_new = app.seqlens = app.block_table = 4096
    app.dtype, app.layout = _lib.DTYPE_BF16, _lib.LAYOUT_PAGES
    app.num_seqs, app.num_kv_heads, app.head_size, app.block_size, app.max_blocks = 2, 2, 128, 16, 4
    app.num_pages = 64
    a.num_seqs = 3  # differs
    assert lib.pab200_decode_append(ctypes.byref(a), ctypes.byref(app), None, 0, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert lib.pab200_decode_append(None, ctypes.byref(app), None, 0, None) == \
        _lib.ERR_INVALID_ARGUMENT


@pytest.mark.gpu
def test_fused_append_decode_matches_separate_calls(cuda_device):
    """Three steps of the wrapper with k=, v= (append done by the decode
    call's planner) against kv_append followed by a plain decode: outputs,
    caches and lengths are bit-identical, and every step matches the oracle
    on the appended cache."""
    from pagedattention_b200 import flash_attn_with_kvcache_wrapper_b200 as decode, kv_append
    from tests.util import assert_close, run_oracle
    B, Hkv, G, D, bs, maxb = 4, 2, 4, 128, 16, 40
    k, v, _, _, _, bt = _case(B, Hkv, D, bs, maxb, 330, torch.bfloat16, seed=31)
    lens = torch.tensor([[100, 5], [600, 17], [0, 333], [31, 32]], dtype=torch.int32)
    dev = cuda_device
    k1, v1, l1 = k.to(dev), v.to(dev), lens.to(dev)   # fused
    k2, v2, l2 = k.to(dev), v.to(dev), lens.to(dev)   # separate
    btd = bt.to(dev)
    g = torch.Generator().manual_seed(3)
    for step in range(3):
        kn = torch.randn((B, 1, Hkv, D), generator=g).to(torch.bfloat16)
        vn = torch.randn((B, 1, Hkv, D), generator=g).to(torch.bfloat16)
        q = torch.randn((B, 1, Hkv * G, D), generator=g).to(torch.bfloat16)
        k, v, lens = _oracle(k, v, kn[:, 0], vn[:, 0], lens, bt)
        fused = decode(q.to(dev), k1, v1, l1, btd, D ** -0.5, k=kn.to(dev), v=vn.to(dev))
        kv_append(k2, v2, kn[:, 0].to(dev), vn[:, 0].to(dev), l2, btd)
        sep = decode(q.to(dev), k2, v2, l2, btd, D ** -0.5)
        assert torch.equal(fused, sep), f"step {step}"
        assert torch.equal(k1, k2) and torch.equal(v1, v2) and torch.equal(l1, l2)
        assert torch.equal(l1.cpu(), lens)
        assert_close(fused, run_oracle(q, k, v, lens, bt, D ** -0.5), what=f"fused step {step}")


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["HND", "NHD"])
def test_fused_append_paged_attention_pools(cuda_device, layout):
    """paged_attention(..., k_new=, v_new=) over a vLLM-style pool with
    per-sequence lengths equals kv_append followed by paged_attention."""
    from pagedattention_b200 import kv_append, paged_attention
    B, Hkv, G, D, bs, maxb, nb = 5, 4, 4, 128, 16, 6, 40
    g = torch.Generator().manual_seed(8)
    shape = (nb, Hkv, bs, D) if layout == "HND" else (nb, bs, Hkv, D)
    pk = torch.randn(shape, generator=g).to(torch.bfloat16)
    pv = torch.randn(shape, generator=g).to(torch.bfloat16)
    bt = torch.randperm(nb, generator=g)[:B * maxb].to(torch.int32).reshape(B, maxb)
    lens = torch.randint(0, maxb * bs - 2, (B,), generator=g, dtype=torch.int32)
    dev = cuda_device
    k1, v1, l1 = pk.to(dev), pv.to(dev), lens.to(dev)
    k2, v2, l2 = pk.to(dev), pv.to(dev), lens.to(dev)
    btd = bt.to(dev)
    for step in range(2):
        kn = torch.randn((B, Hkv, D), generator=g).to(torch.bfloat16).to(dev)
        vn = torch.randn((B, Hkv, D), generator=g).to(torch.bfloat16).to(dev)
        q = torch.randn((B, Hkv * G, D), generator=g).to(torch.bfloat16).to(dev)
        o1, o2 = torch.empty_like(q), torch.empty_like(q)
        paged_attention(o1, q, k1, v1, btd, l1, D ** -0.5, bs, kv_layout=layout, k_new=kn, v_new=vn)
        kv_append(k2, v2, kn, vn, l2, btd, kv_layout=layout)
        paged_attention(o2, q, k2, v2, btd, l2, D ** -0.5, bs, kv_layout=layout)
        assert torch.equal(o1, o2) and torch.equal(k1, k2) and torch.equal(v1, v2)
        assert torch.equal(l1, l2) and torch.equal(l1.cpu(), lens + step + 1)
