"""pab200_decode_noalloc: the decode entry point for callers that cannot
allocate device memory — a foreign-language binding with no device
allocator of its own, or an engine whose memory pool already holds all free
device memory, so that handing the library a workspace is not possible.  It
runs the same planner and decode kernels as pab200_decode, with the scratch
taken from a fixed 16 MiB array inside the library instead of a caller
workspace.

Both entry points are called through the C ABI (ctypes).  The expected
outputs come from pab200_decode, one workspace per call, computed first;
then the no-alloc calls are queued back to back on one stream with shapes
that change from call to call and no synchronisation in between (they share
the one scratch array, which keeps the previous call's contents, and each
call's planner overlaps the previous call's reduce).  Every no-alloc output
must equal the workspace entry point's bit for bit (same kernels, same plan)
and match the oracle at the suite's tolerance.  A call whose scratch need
exceeds the fixed size must be refused with PAB200_ERR_WORKSPACE.  This file
sorts last so that a failure here does not hide the rest of the suite.
"""
import ctypes

import pytest
import torch

from pagedattention_b200 import _lib
from tests.util import assert_close, random_case, run_oracle

pytestmark = pytest.mark.gpu


def _args(q, k, v, sl, bt, out, scale, num_splits=0):
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
    a.num_splits = num_splits
    return a


def _short_lens(B, Hkv, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(1, 200, (B, Hkv), generator=g).tolist()


# B, Hkv, G, D, bs, lens, dtype, num_splits — each call's workspace fits the
# 16 MiB scratch without trimming its plan, so outputs must be bit-identical.
CASES = [
    (256, 8, 4, 128, 16, _short_lens(256, 8, 1), torch.bfloat16, 0),       # many short heads
    (3, 4, 4, 128, 16, [[7000, 5, 64, 0], [1, 333, 6024, 17], [16, 2000, 48, 129]],
     torch.bfloat16, 0),                                                    # few long heads
    (2, 1, 32, 64, 8, [[4000], [77]], torch.float16, 64),                   # 32-head group
    (256, 8, 4, 128, 16, _short_lens(256, 8, 2), torch.bfloat16, 0),       # many short again
    (3, 4, 4, 128, 16, [[6000, 900, 64, 3], [1, 5000, 600, 17], [4000, 20, 48, 129]],
     torch.bfloat16, 2),                                                    # split count 2
]


def test_noalloc_matches_workspace_entry_point(cuda_device):
    lib = _lib.load()
    dev = cuda_device
    stream = torch.cuda.current_stream(dev).cuda_stream
    calls = []
    for i, (B, Hkv, G, D, bs, lens, dtype, splits) in enumerate(CASES):
        cpu = random_case(B, Hkv, G, D, bs, lens, dtype, seed=50 + i,
                          k_scale=4.0 if G == 32 else 1.0)
        q, k, v, sl, bt = (t.to(dev) for t in cpu[:5])
        scale = cpu[5]
        expected = torch.empty_like(q)
        a = _args(q, k, v, sl, bt, expected, scale, splits)
        need = lib.pab200_decode_workspace_size(ctypes.byref(a))
        assert 0 < need <= _lib.NOALLOC_SCRATCH_BYTES, need
        ws = torch.empty(need, dtype=torch.uint8, device=dev)  # a workspace of its own
        rc = lib.pab200_decode(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), need,
                               ctypes.c_void_p(stream))
        assert rc == 0, _lib.error_text(lib, rc)
        torch.cuda.synchronize(dev)
        del ws
        calls.append((cpu, (q, k, v, sl, bt), scale, splits, expected))
    # The no-alloc calls, queued back to back with no synchronisation.
    outs = []
    for cpu, (q, k, v, sl, bt), scale, splits, _ in calls:
        got = torch.full_like(q, float("nan"))
        rc = lib.pab200_decode_noalloc(ctypes.byref(_args(q, k, v, sl, bt, got, scale, splits)),
                                       ctypes.c_void_p(stream))
        assert rc == 0, _lib.error_text(lib, rc)
        outs.append(got)
    torch.cuda.synchronize(dev)
    for i, ((cpu, _, scale, _, expected), got) in enumerate(zip(calls, outs)):
        assert torch.equal(got, expected), f"no-alloc call {i + 1} differs from pab200_decode"
        assert_close(got, run_oracle(*cpu[:5], scale), what=f"no-alloc call {i + 1}")


def test_noalloc_refuses_oversized_scratch(cuda_device):
    lib = _lib.load()
    dev = cuda_device
    # 4000 x 8 heads: the partial-state slots alone exceed 16 MiB even with
    # no tail chunks.  Every sequence is empty, so even an accepted call would
    # only write zeros.
    B, Hkv, G, D = 4000, 2, 8, 128
    q = torch.zeros((B, 1, Hkv * G, D), dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(q)
    k = torch.zeros((1, 16, D), dtype=torch.bfloat16, device=dev)
    sl = torch.zeros((B, Hkv), dtype=torch.int32, device=dev)
    bt = torch.zeros((B, Hkv, 1), dtype=torch.int32, device=dev)
    a = _args(q, k, k, sl, bt, out, 0.1)
    assert lib.pab200_decode_workspace_size(ctypes.byref(a)) > _lib.NOALLOC_SCRATCH_BYTES
    rc = lib.pab200_decode_noalloc(ctypes.byref(a),
                                   ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert rc == _lib.ERR_WORKSPACE
    assert b"no-alloc scratch" in lib.pab200_last_error()
