"""pab200_decode_noalloc: the decode entry point for callers that cannot
allocate device memory (a binding with no device allocator of its own, or an
engine whose memory pool already holds all free device memory).  It runs the
same planner and decode kernels as pab200_decode, with the scratch taken from
a fixed 16 MiB array inside the library instead of a caller workspace.

Both entry points are called through the C ABI (ctypes); the no-alloc output
must match the workspace entry point's within the suite's tolerance on two
calls in a row with different inputs (the shared scratch keeps the previous
call's contents), and a call whose scratch need exceeds the fixed size must be
refused with PAB200_ERR_WORKSPACE.  This file sorts last so that a failure here
does not hide the rest of the suite.
"""
import ctypes

import pytest
import torch

from pagedattention_b200 import _lib
from tests.util import assert_close, random_case

pytestmark = pytest.mark.gpu


def _args(q, k, v, sl, bt, out, scale):
    a = _lib.DecodeArgs()
    B, _, Hq, D = q.shape
    a.out, a.q = out.data_ptr(), q.data_ptr()
    a.k_cache, a.v_cache = k.data_ptr(), v.data_ptr()
    a.seqlens, a.block_table = sl.data_ptr(), bt.data_ptr()
    a.dtype = _lib.DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.DTYPE_F16
    a.layout = _lib.LAYOUT_PAGES
    a.num_seqs, a.num_q_heads, a.num_kv_heads = B, Hq, sl.shape[1]
    a.head_size, a.block_size = D, k.shape[1]
    a.max_blocks, a.num_pages = bt.shape[2], k.shape[0]
    a.q_stride_b, a.q_stride_h = q.stride(0), q.stride(2)
    a.out_stride_b, a.out_stride_h = out.stride(0), out.stride(2)
    a.seqlens_stride_b, a.seqlens_stride_h = sl.stride(0), sl.stride(1)
    a.bt_stride_b, a.bt_stride_h, a.bt_stride_i = bt.stride(0), bt.stride(1), bt.stride(2)
    a.bt_page_mul, a.bt_page_add = 1, 0
    a.softmax_scale = scale
    a.num_splits = 0
    return a


def _with_workspace(lib, a, dev, stream):
    need = lib.pab200_decode_workspace_size(ctypes.byref(a))
    assert 0 < need <= _lib.NOALLOC_SCRATCH_BYTES
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    rc = lib.pab200_decode(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), need,
                           ctypes.c_void_p(stream))
    assert rc == 0, _lib.error_text(lib, rc)
    return ws


CASES = [
    # B, Hkv, G, D, bs, lens, dtype
    (3, 4, 4, 128, 16, [[700, 5, 64, 0], [1, 333, 1024, 17], [16, 2000, 48, 129]], torch.bfloat16),
    (2, 1, 32, 64, 8, [[4000], [77]], torch.float16),
]


def test_noalloc_matches_workspace_entry_point(cuda_device):
    lib = _lib.load()
    dev = cuda_device
    stream = torch.cuda.current_stream(dev).cuda_stream
    for i, (B, Hkv, G, D, bs, lens, dtype) in enumerate(CASES):
        q, k, v, sl, bt, scale = random_case(B, Hkv, G, D, bs, lens, dtype, seed=50 + i)
        q, k, v, sl, bt = (t.to(dev) for t in (q, k, v, sl, bt))
        expected = torch.empty_like(q)
        ws = _with_workspace(lib, _args(q, k, v, sl, bt, expected, scale), dev, stream)
        got = torch.full_like(q, float("nan"))
        rc = lib.pab200_decode_noalloc(ctypes.byref(_args(q, k, v, sl, bt, got, scale)),
                                       ctypes.c_void_p(stream))
        assert rc == 0, _lib.error_text(lib, rc)
        torch.cuda.synchronize(dev)
        del ws
        assert_close(got, expected.float(), what=f"no-alloc call {i + 1}")


def test_noalloc_refuses_oversized_scratch(cuda_device):
    lib = _lib.load()
    dev = cuda_device
    # 4000 x 8 heads: the partial-state slots alone exceed 16 MiB.  Every
    # sequence is empty, so even an accepted call would only write zeros.
    B, Hkv, G, D = 4000, 2, 8, 128
    q = torch.zeros((B, 1, Hkv * G, D), dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(q)
    k = torch.zeros((1, 16, D), dtype=torch.bfloat16, device=dev)
    sl = torch.zeros((B, Hkv), dtype=torch.int32, device=dev)
    bt = torch.zeros((B, Hkv, 1), dtype=torch.int32, device=dev)
    a = _args(q, k, k, sl, bt, out, 0.1)
    assert lib.pab200_decode_workspace_size(ctypes.byref(a)) > _lib.NOALLOC_SCRATCH_BYTES
    rc = lib.pab200_decode_noalloc(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert rc == _lib.ERR_WORKSPACE
    assert b"no-alloc scratch" in lib.pab200_last_error()
