"""B200 paged-attention decode: the Python face of libpab200.so.

Public entry points:

* ``flash_attn_with_kvcache_wrapper_b200(q, k_cache, v_cache, cache_seqlens,
  block_table, softmax_scale, num_splits=1)`` — drop-in beside the reference's
  ``flash_attn_with_kvcache_wrapper_{eager,triton,vllm}``
  (src/kernel_eager.py:29, src/kernel_triton.py:181, src/kernel_vllm.py:4),
  same keywords, shapes (src/common.py:1-14) and error types.
* ``paged_attention(out, query, key_cache, value_cache, block_tables,
  context_lens, scale, block_size)`` — the in-place form, which also accepts
  vLLM-style [num_blocks, num_kv_heads, block_size, head_size] pools.
* ``paged_attention_states`` / ``merge_states`` — the partial (o, lse) form and
  its log-sum-exp merge, for contexts split across devices.

Every call launches CUDA kernels from libpab200.so on the current stream of
the tensors' device; there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import math
import threading
from contextlib import contextmanager

import torch

from . import _lib
from .common import _validate_decode_inputs

_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}

_tls = threading.local()
_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], torch.Tensor] = {}
_last_ws: dict[int, tuple[torch.Tensor, int]] = {}


def _check_dtypes(q, k_cache, v_cache):
    # The reference Triton wrapper raises TypeError on unsupported dtypes
    # (src/kernel_triton.py:195-196); this kernel takes bf16 or fp16.
    if q.dtype not in _DTYPES:
        raise TypeError(f"q must be bfloat16 or float16, got {q.dtype}")
    if k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise TypeError("q, k_cache and v_cache must share one dtype "
                        f"(got {q.dtype}, {k_cache.dtype}, {v_cache.dtype})")


def _check_device(*tensors):
    dev = tensors[0].device
    if dev.type != "cuda":
        raise ValueError("pagedattention_b200 runs on CUDA tensors only (no CPU fallback)")
    for t in tensors[1:]:
        if t.device != dev:
            raise ValueError(f"all tensors must be on {dev}, got {t.device}")
    return dev


def _as_int32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype == torch.int32:
        return t
    if t.dtype in (torch.int64, torch.int16, torch.uint8, torch.int8):
        return t.to(torch.int32)
    raise TypeError(f"{name} must be an integer tensor, got {t.dtype}")


_ws_sizes: dict[tuple, int] = {}


def _workspace(lib, args, device, stream_handle) -> torch.Tensor:
    # The size depends only on shapes and the device, so it is cached per
    # shape key (the C call re-plans the launch geometry).
    skey = (device.index, args.num_seqs, args.num_q_heads, args.num_kv_heads, args.head_size,
            args.block_size, args.dtype, args.num_splits, args.max_blocks)
    need = _ws_sizes.get(skey)
    if need is None:
        need = lib.pab200_decode_workspace_size(ctypes.byref(args))
        if need == 0:
            raise ValueError(f"pab200_decode_workspace_size: {lib.pab200_last_error().decode()}")
        _ws_sizes[skey] = need
    key = (device.index, stream_handle)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < need:
        with _ws_lock:
            ws = _workspaces.get(key)
            if ws is None or ws.numel() < need:
                ws = torch.empty(need, dtype=torch.uint8, device=device)
                _workspaces[key] = ws
    _last_ws[device.index] = (ws, stream_handle)
    return ws


def launches_per_call(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale,
                      num_splits=1) -> int:
    """Kernel launches one flash_attn_with_kvcache_wrapper_b200 call with these
    arguments makes (2, or 3 when a separate reduce kernel merges split heads)."""
    Hq, Hkv, G, D = _validate_decode_inputs(q, cache_seqlens, block_table)
    args = _lib.DecodeArgs()
    lens = _as_int32(cache_seqlens, "cache_seqlens")
    bt = _as_int32(block_table, "block_table")
    _fill_common(args, q=q, k_cache=k_cache, v_cache=v_cache, lens=lens, bt=bt, dtype=q.dtype,
                 B=q.shape[0], Hq=Hq, Hkv=Hkv, D=D, bs=k_cache.shape[1],
                 num_pages=k_cache.shape[0], scale=softmax_scale, num_splits=num_splits)
    args.out, args.layout, args.max_blocks = q.data_ptr(), _lib.LAYOUT_PAGES, bt.shape[2]
    args.q_stride_b, args.q_stride_h = q.stride(0), q.stride(2)
    args.out_stride_b, args.out_stride_h = q.stride(0), q.stride(2)
    args.seqlens_stride_b, args.seqlens_stride_h = lens.stride(0), lens.stride(1)
    args.bt_stride_b, args.bt_stride_h, args.bt_stride_i = bt.stride(0), bt.stride(1), bt.stride(2)
    args.bt_page_mul = 1
    lib = _lib.load()
    with torch.cuda.device(q.device):
        n = lib.pab200_decode_launch_count(ctypes.byref(args))
    if n == 0:
        raise ValueError(f"pab200_decode_launch_count: {lib.pab200_last_error().decode()}")
    return n


@contextmanager
def kernel_events(before: torch.cuda.Event, after: torch.cuda.Event):
    """Record ``before``/``after`` around the main decode kernel of every
    decode call made inside the block (kernel-only timing; both events must
    already exist, i.e. have been recorded once)."""
    prev = getattr(_tls, "events", None)
    _tls.events = (before, after)
    try:
        yield
    finally:
        _tls.events = prev


def _run_decode(args: _lib.DecodeArgs, device: torch.device, append=None, exchange=None) -> None:
    lib = _lib.load()
    ev = getattr(_tls, "events", None)
    if ev is not None:
        args.event_before = ev[0].cuda_event
        args.event_after = ev[1].cuda_event
    if torch.cuda.current_device() == device.index:
        rc = _launch(lib, args, device, append, exchange)
    else:
        with torch.cuda.device(device):
            rc = _launch(lib, args, device, append, exchange)
    if rc == _lib.ERR_INVALID_ARGUMENT or rc == _lib.ERR_UNSUPPORTED:
        raise ValueError(f"pab200_decode: {_lib.error_text(lib, rc)}")
    _lib.check(lib, rc, "pab200_decode")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _current_stream_handle(device) -> int:
    if _raw_stream is not None:  # cudaStream_t of the current stream, cheaply
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def _call(lib, args, append, ws, stream_handle, exchange=None) -> int:
    if exchange is not None:
        ex, out, code = exchange
        return lib.pab200_decode_exchange(
            ctypes.byref(args), ws.data_ptr(), ws.numel(), ex.bufs.data_ptr(), ex.rank, ex.world,
            out.data_ptr(), out.stride(1), code, ex.wait_limit_ns, ex.status.data_ptr(),
            stream_handle)
    if append is None:
        return lib.pab200_decode(ctypes.byref(args), ws.data_ptr(), ws.numel(), stream_handle)
    return lib.pab200_decode_append(ctypes.byref(args), ctypes.byref(append), ws.data_ptr(),
                                    ws.numel(), stream_handle)


def _launch(lib, args, device, append=None, exchange=None) -> int:
    stream_handle = _current_stream_handle(device)
    rc = _call(lib, args, append, _workspace(lib, args, device, stream_handle), stream_handle,
               exchange)
    if rc == _lib.ERR_WORKSPACE:
        # launch geometry changed (e.g. a tuning variable): re-size once
        _ws_sizes.clear()
        rc = _call(lib, args, append, _workspace(lib, args, device, stream_handle),
                   stream_handle, exchange)
    return rc


def _fill_common(args, *, q, k_cache, v_cache, lens, bt, dtype, B, Hq, Hkv, D, bs,
                 num_pages, scale, num_splits):
    args.q = q.data_ptr()
    args.k_cache = k_cache.data_ptr()
    args.v_cache = v_cache.data_ptr()
    args.seqlens = lens.data_ptr()
    args.block_table = bt.data_ptr()
    args.dtype = _DTYPES[dtype]
    args.num_seqs = B
    args.num_q_heads = Hq
    args.num_kv_heads = Hkv
    args.head_size = D
    args.block_size = bs
    args.num_pages = num_pages
    args.softmax_scale = float(scale)
    args.num_splits = int(num_splits)


def flash_attn_with_kvcache_wrapper_b200(q, k_cache, v_cache, cache_seqlens, block_table,
                                         softmax_scale, num_splits=1, k=None, v=None):
    """Paged decode attention; returns a new (batch, 1, Hq, head_size) tensor.

    Arguments as in src/common.py:1-14: q (B, 1, Hq, D); k_cache, v_cache
    (num_blocks, block_size, D), one page per (sequence, kv head); cache_seqlens
    (B, Hkv); block_table (B, Hkv, max_num_blocks_per_head).  ``num_splits``
    keeps the reference's meaning (src/kernel_triton.py:206-209, chunks per kv
    head): 0 or 1 lets the kernel size the split to the device, n > 1 caps the
    number of chunks at B*Hkv*n.

    ``k``, ``v`` (optional, not in the reference): the step's new token,
    (B, 1, Hkv, D) or (B, Hkv, D), written into the cache at cache_seqlens
    before attending (flash-attn's ``flash_attn_with_kvcache`` semantics);
    cache_seqlens must then be int32 and is advanced in place.  One call,
    the append done by the decode's planner.
    """
    Hq, Hkv, G, D = _validate_decode_inputs(q, cache_seqlens, block_table)
    _check_dtypes(q, k_cache, v_cache)
    device = _check_device(q, k_cache, v_cache, cache_seqlens, block_table)
    if k_cache.dim() != 3 or tuple(v_cache.shape) != tuple(k_cache.shape):
        raise ValueError("k_cache and v_cache must both be (num_blocks, block_size, head_size)")
    if k_cache.shape[2] != D:
        raise ValueError(f"cache head_size {k_cache.shape[2]} != q head_size {D}")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("k_cache and v_cache must be contiguous")
    qs = q.stride()
    if qs[3] != 1:
        raise ValueError("q must be contiguous in head_size")
    if num_splits < 0:
        raise ValueError("num_splits must be >= 0")
    B = q.shape[0]
    lens = _as_int32(cache_seqlens, "cache_seqlens")
    bt = _as_int32(block_table, "block_table")
    out = torch.empty((B, 1, Hq, D), dtype=q.dtype, device=device)
    args = _lib.DecodeArgs()
    _fill_common(args, q=q, k_cache=k_cache, v_cache=v_cache, lens=lens, bt=bt, dtype=q.dtype,
                 B=B, Hq=Hq, Hkv=Hkv, D=D, bs=k_cache.shape[1], num_pages=k_cache.shape[0],
                 scale=softmax_scale, num_splits=num_splits)
    args.out = out.data_ptr()
    args.layout = _lib.LAYOUT_PAGES
    args.max_blocks = bt.shape[2]
    args.q_stride_b, args.q_stride_h = qs[0], qs[2]
    args.out_stride_b, args.out_stride_h = Hq * D, D   # fresh contiguous output
    args.seqlens_stride_b, args.seqlens_stride_h = lens.stride()
    args.bt_stride_b, args.bt_stride_h, args.bt_stride_i = bt.stride()
    args.bt_page_mul, args.bt_page_add = 1, 0
    append = None
    if k is not None or v is not None:
        if k is None or v is None:
            raise ValueError("k and v must be given together")
        if cache_seqlens.dtype != torch.int32:
            raise TypeError("cache_seqlens must be int32 to be advanced in place")
        kn = k.reshape(B, Hkv, D) if k.dim() == 4 else k
        vn = v.reshape(B, Hkv, D) if v.dim() == 4 else v
        if tuple(kn.shape) != (B, Hkv, D) or tuple(vn.shape) != (B, Hkv, D):
            raise ValueError("k and v must be (batch, 1, Hkv, head_size) or (batch, Hkv, head_size)")
        if kn.dtype != k_cache.dtype or vn.dtype != k_cache.dtype:
            raise TypeError("k and v must have the caches' dtype")
        if kn.stride(2) != 1 or vn.stride(2) != 1 or kn.stride() != vn.stride():
            raise ValueError("k and v must share strides, contiguous in head_size")
        _check_device(q, kn, vn)
        append = _lib.KvAppendArgs()
        append.k_cache, append.v_cache = args.k_cache, args.v_cache
        append.k_new, append.v_new = kn.data_ptr(), vn.data_ptr()
        append.seqlens, append.block_table = args.seqlens, args.block_table
        append.dtype, append.layout = args.dtype, args.layout
        append.num_seqs, append.num_kv_heads = B, Hkv
        append.head_size, append.block_size = D, args.block_size
        append.max_blocks, append.num_pages = args.max_blocks, args.num_pages
        append.new_stride_b, append.new_stride_h = kn.stride(0), kn.stride(1)
        append.seqlens_stride_b = args.seqlens_stride_b
        append.seqlens_stride_h = args.seqlens_stride_h
        append.bt_stride_b, append.bt_stride_h = args.bt_stride_b, args.bt_stride_h
        append.bt_stride_i = args.bt_stride_i
        append.bt_page_mul, append.bt_page_add = 1, 0
        append.increment = 1
    _run_decode(args, device, append)
    return out


def _paged_args(query, key_cache, value_cache, block_tables, context_lens, scale, block_size,
                kv_layout, num_splits):
    """Shared argument handling of paged_attention / paged_attention_states."""
    if query.dim() != 3:
        raise ValueError("query must be (num_seqs, num_q_heads, head_size)")
    _check_dtypes(query, key_cache, value_cache)
    if tuple(key_cache.shape) != tuple(value_cache.shape):
        raise ValueError("key_cache and value_cache shapes differ")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("key_cache and value_cache must be contiguous")
    if query.stride(2) != 1:
        raise ValueError("query must be contiguous in head_size")
    B, Hq, D = query.shape
    bt = _as_int32(block_tables, "block_tables")
    lens = _as_int32(context_lens, "context_lens")
    args = _lib.DecodeArgs()
    if key_cache.dim() == 3:                       # reference page layout
        if kv_layout not in ("HND", "pages"):
            raise ValueError("a 3-D cache is (num_pages, block_size, head_size)")
        if bt.dim() != 3:
            raise ValueError("a 3-D (per-head page) cache needs block_tables "
                             "(num_seqs, num_kv_heads, max_blocks)")
        Hkv = bt.shape[1]
        num_pages, bs, Dc = key_cache.shape
        layout, mul, add = _lib.LAYOUT_PAGES, 1, 0
    elif key_cache.dim() == 4 and kv_layout == "HND":  # [nb, Hkv, bs, D]
        nb, Hkv, bs, Dc = key_cache.shape
        num_pages = nb * Hkv
        layout, mul, add = _lib.LAYOUT_PAGES, Hkv, 1
    elif key_cache.dim() == 4 and kv_layout == "NHD":  # [nb, bs, Hkv, D]
        nb, bs, Hkv, Dc = key_cache.shape
        num_pages = nb
        layout, mul, add = _lib.LAYOUT_NHD, 1, 0
    else:
        raise ValueError(f"unsupported cache rank {key_cache.dim()} / kv_layout {kv_layout!r}")
    if Dc != D:
        raise ValueError(f"cache head_size {Dc} != query head_size {D}")
    if bs != block_size:
        raise ValueError(f"block_size {block_size} != cache block size {bs}")
    if Hq % Hkv != 0:
        raise ValueError(f"num_q_heads {Hq} is not a multiple of num_kv_heads {Hkv}")
    if bt.dim() == 3:
        if bt.shape[0] != B or bt.shape[1] != Hkv:
            raise ValueError("block_tables must be (num_seqs, num_kv_heads, max_blocks)")
        sb, sh, si, maxb = bt.stride(0), bt.stride(1), bt.stride(2), bt.shape[2]
    elif bt.dim() == 2:
        if bt.shape[0] != B:
            raise ValueError("block_tables must be (num_seqs, max_blocks)")
        sb, sh, si, maxb = bt.stride(0), 0, bt.stride(1), bt.shape[1]
    else:
        raise ValueError("block_tables must be 2-D or 3-D")
    if lens.dim() == 1 and lens.shape[0] == B:
        lsb, lsh = lens.stride(0), 0
    elif lens.dim() == 2 and tuple(lens.shape) == (B, Hkv):
        lsb, lsh = lens.stride(0), lens.stride(1)
    else:
        raise ValueError("context_lens must be (num_seqs,) or (num_seqs, num_kv_heads)")
    device = _check_device(query, key_cache, value_cache, bt, lens)
    _fill_common(args, q=query, k_cache=key_cache, v_cache=value_cache, lens=lens, bt=bt,
                 dtype=query.dtype, B=B, Hq=Hq, Hkv=Hkv, D=D, bs=bs, num_pages=num_pages,
                 scale=scale, num_splits=num_splits)
    args.layout = layout
    args.max_blocks = maxb
    args.q_stride_b, args.q_stride_h = query.stride(0), query.stride(1)
    args.seqlens_stride_b, args.seqlens_stride_h = lsb, lsh
    args.bt_stride_b, args.bt_stride_h, args.bt_stride_i = sb, sh, si
    args.bt_page_mul, args.bt_page_add = mul, add
    # keep converted tensors alive until the launch is enqueued
    return args, device, (bt, lens)


def _append_args_like(args, k_new, v_new, lens):
    """KvAppendArgs addressing the caches, table and lengths of ``args``."""
    B, Hkv, D = args.num_seqs, args.num_kv_heads, args.head_size
    if tuple(k_new.shape) != (B, Hkv, D) or tuple(v_new.shape) != (B, Hkv, D):
        raise ValueError("k_new and v_new must be (num_seqs, num_kv_heads, head_size)")
    if k_new.stride(2) != 1 or v_new.stride(2) != 1 or k_new.stride() != v_new.stride():
        raise ValueError("k_new and v_new must share strides, contiguous in head_size")
    if lens.dtype != torch.int32:
        raise TypeError("context_lens must be int32 to be advanced in place")
    a = _lib.KvAppendArgs()
    a.k_cache, a.v_cache = args.k_cache, args.v_cache
    a.k_new, a.v_new = k_new.data_ptr(), v_new.data_ptr()
    a.seqlens, a.block_table = args.seqlens, args.block_table
    a.dtype, a.layout = args.dtype, args.layout
    a.num_seqs, a.num_kv_heads, a.head_size = B, Hkv, D
    a.block_size, a.max_blocks, a.num_pages = args.block_size, args.max_blocks, args.num_pages
    a.new_stride_b, a.new_stride_h = k_new.stride(0), k_new.stride(1)
    a.seqlens_stride_b, a.seqlens_stride_h = args.seqlens_stride_b, args.seqlens_stride_h
    a.bt_stride_b, a.bt_stride_h, a.bt_stride_i = args.bt_stride_b, args.bt_stride_h, args.bt_stride_i
    a.bt_page_mul, a.bt_page_add = args.bt_page_mul, args.bt_page_add
    a.increment = 1
    return a


def paged_attention(out, query, key_cache, value_cache, block_tables, context_lens, scale,
                    block_size, kv_layout="HND", num_splits=0, k_new=None, v_new=None):
    """In-place paged decode: writes ``out`` (num_seqs, num_q_heads, head_size).

    Caches: (num_pages, block_size, head_size) with block_tables
    (num_seqs, num_kv_heads, max_blocks) — the reference layout; or a 4-D pool
    (num_blocks, num_kv_heads, block_size, head_size) ("HND", default) or
    (num_blocks, block_size, num_kv_heads, head_size) ("NHD") with block_tables
    (num_seqs, max_blocks) of block ids shared by all kv heads.  context_lens:
    (num_seqs,) or (num_seqs, num_kv_heads).  With ``k_new``, ``v_new``
    (num_seqs, num_kv_heads, head_size) the step's tokens are first written
    at the current lengths, which advance in place (int32 context_lens),
    inside the same call.
    """
    args, device, keep = _paged_args(query, key_cache, value_cache, block_tables, context_lens,
                                     scale, block_size, kv_layout, num_splits)
    if out.shape != query.shape or out.dtype != query.dtype or out.device != device:
        raise ValueError("out must match query in shape, dtype and device")
    if out.stride(2) != 1:
        raise ValueError("out must be contiguous in head_size")
    args.out = out.data_ptr()
    args.out_stride_b, args.out_stride_h = out.stride(0), out.stride(1)
    append = None
    if k_new is not None or v_new is not None:
        if k_new is None or v_new is None:
            raise ValueError("k_new and v_new must be given together")
        if k_new.dtype != key_cache.dtype or v_new.dtype != key_cache.dtype:
            raise TypeError("k_new and v_new must have the caches' dtype")
        _check_device(query, k_new, v_new)
        append = _append_args_like(args, k_new, v_new, context_lens)
    _run_decode(args, device, append)
    del keep


def state_numel(num_seqs: int, num_q_heads: int, head_size: int) -> int:
    """Floats in one packed partial state: o [rows, D] then lse [rows], the lse
    part padded to a multiple of 4 floats (rows = num_seqs * num_q_heads)."""
    rows = num_seqs * num_q_heads
    return rows * head_size + ((rows + 3) // 4) * 4


def paged_attention_states(query, key_cache, value_cache, block_tables, context_lens, scale,
                           block_size, kv_layout="HND", num_splits=0, state=None):
    """Like paged_attention, but return the partial state of the given KV range.

    Returns (o, lse): o (num_seqs, num_q_heads, head_size) float32, the
    attention output over just these tokens, and lse (num_seqs, num_q_heads)
    float32, the natural log of the sum of exp(scaled score); empty ranges give
    o = 0, lse = -inf.  ``state``, if given, is a float32 tensor of
    ``state_numel(...)`` elements that receives the packed (o, lse) (the layout
    ``merge_packed_states`` reads).  ``merge_states`` combines states of
    disjoint ranges.
    """
    args, device, keep = _paged_args(query, key_cache, value_cache, block_tables, context_lens,
                                     scale, block_size, kv_layout, num_splits)
    B, Hq, D = query.shape
    rows = B * Hq
    if state is None:
        state = torch.empty(state_numel(B, Hq, D), dtype=torch.float32, device=device)
    if (state.dtype != torch.float32 or state.numel() < state_numel(B, Hq, D)
            or not state.is_contiguous() or state.device != device):
        raise ValueError("state must be a contiguous float32 tensor of state_numel() elements")
    o = state[:rows * D].view(B, Hq, D)
    lse = state[rows * D:rows * D + rows].view(B, Hq)
    args.state_o = o.data_ptr()
    args.state_lse = lse.data_ptr()
    _run_decode(args, device)
    del keep
    return o, lse


def paged_attention_exchange(query, key_cache, value_cache, block_tables, context_lens, scale,
                             block_size, exchange, out=None, kv_layout="HND", num_splits=0):
    """Decode this rank's token ranges and merge every rank's result (a
    context split across the GPUs of one node), in one call.

    Arguments as for ``paged_attention_states``; ``exchange`` is a
    ``PeerExchange`` of this shape.  The decode writes this rank's (o, lse)
    state into ``exchange.state`` and the exchange kernel, which also folds
    the partial states of heads the decode split, stores it into every
    peer's buffer and merges the world's states into ``out`` (num_seqs,
    num_q_heads, head_size) in query's dtype, identical on every rank.  The
    log-sum-exp merge is the reduce of src/kernel_triton.py:120-174 applied
    across devices.
    """
    args, device, keep = _paged_args(query, key_cache, value_cache, block_tables, context_lens,
                                     scale, block_size, kv_layout, num_splits)
    B, Hq, D = query.shape
    if (B, Hq, D) != tuple(exchange.shape):
        raise ValueError(f"query shape {(B, Hq, D)} != exchange shape {tuple(exchange.shape)}")
    if out is None:
        out = torch.empty((B, Hq, D), dtype=query.dtype, device=device)
    code = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16,
            torch.float32: _lib.DTYPE_F32}.get(out.dtype)
    if code is None:
        raise TypeError(f"unsupported out dtype {out.dtype}")
    if tuple(out.shape) != (B, Hq, D) or not out.is_contiguous() or out.device != device:
        raise ValueError(f"out must be a contiguous {(B, Hq, D)} tensor on {device}")
    rows = B * Hq
    state = exchange.state
    args.state_o = state.data_ptr()
    args.state_lse = state.data_ptr() + rows * D * 4
    _run_decode(args, device, exchange=(exchange, out, code))
    del keep
    return out


def _merge(lib, device, o_ptr, o_stride, lse_ptr, lse_stride, n, rows, D, out):
    code = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16,
            torch.float32: _lib.DTYPE_F32}.get(out.dtype)
    if code is None:
        raise TypeError(f"unsupported out dtype {out.dtype}")
    if not out.is_contiguous():
        raise ValueError("out must be contiguous")
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        rc = lib.pab200_merge_states(ctypes.c_void_p(o_ptr), o_stride, ctypes.c_void_p(lse_ptr),
                                     lse_stride, n, rows, D, ctypes.c_void_p(out.data_ptr()), D,
                                     code, ctypes.c_void_p(stream.cuda_stream))
    _lib.check(lib, rc, "pab200_merge_states")
    return out


def merge_states(state_o, state_lse, out=None, out_dtype=torch.bfloat16):
    """Log-sum-exp merge of N partial states (the reduce of
    src/kernel_triton.py:120-174, across devices).

    state_o: (N, ..., head_size) float32; state_lse: (N, ...) float32.
    Returns (or fills) out of shape (..., head_size).
    """
    if state_o.dtype != torch.float32 or state_lse.dtype != torch.float32:
        raise TypeError("states must be float32")
    device = _check_device(state_o, state_lse)
    N, D = state_o.shape[0], state_o.shape[-1]
    if tuple(state_lse.shape) != tuple(state_o.shape[:-1]):
        raise ValueError("state_lse must be state_o.shape[:-1]")
    rows = state_lse[0].numel()
    so = state_o.contiguous()
    sl = state_lse.contiguous()
    if out is None:
        out = torch.empty(tuple(state_o.shape[1:]), dtype=out_dtype, device=device)
    return _merge(_lib.load(), device, so.data_ptr(), rows * D, sl.data_ptr(), rows, N, rows, D,
                  out)


def merge_packed_states(states, num_seqs, num_q_heads, head_size, out=None,
                        out_dtype=torch.bfloat16):
    """Merge N packed states (rows of a (N, S) float32 tensor, S >=
    state_numel(...), as written by ``paged_attention_states(state=...)`` and
    gathered across devices) into out (num_seqs, num_q_heads, head_size)."""
    if states.dtype != torch.float32 or states.dim() != 2 or not states.is_contiguous():
        raise ValueError("states must be a contiguous float32 (N, S) tensor")
    device = _check_device(states)
    N, S = states.shape
    rows = num_seqs * num_q_heads
    if S < state_numel(num_seqs, num_q_heads, head_size) or S % 4:
        raise ValueError("state row too short or not a multiple of 4 floats")
    if out is None:
        out = torch.empty((num_seqs, num_q_heads, head_size), dtype=out_dtype, device=device)
    base = states.data_ptr()
    return _merge(_lib.load(), device, base, S, base + rows * head_size * 4, S, N, rows,
                  head_size, out)


def read_status(device=None) -> int:
    """PAB200_STATUS_* bits raised by the last decode call on ``device``
    (synchronises that call's stream)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       torch.device(device).index or 0)
    entry = _last_ws.get(dev.index)
    if entry is None:
        return 0
    ws, stream_handle = entry
    lib = _lib.load()
    val = ctypes.c_uint32(0)
    with torch.cuda.device(dev):
        rc = lib.pab200_read_status(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(val),
                                    ctypes.c_void_p(stream_handle))
    _lib.check(lib, rc, "pab200_read_status")
    return int(val.value)


def default_scale(head_size: int) -> float:
    return 1.0 / math.sqrt(head_size)


_append_status: dict[int, torch.Tensor] = {}


def _append_status_word(device) -> torch.Tensor:
    w = _append_status.get(device.index)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=device)
        _append_status[device.index] = w
    return w


def kv_append(key_cache, value_cache, k_new, v_new, cache_seqlens, block_table, increment=True,
              kv_layout="HND"):
    """Write each (sequence, kv head)'s new token into its page, in place.

    The step before a decode call; the reference has no counterpart (its
    cache is filled once by its benchmark).  Caches and tables as for
    ``paged_attention``: a 3-D reference page cache (num_pages, block_size,
    head_size) with block_table (num_seqs, num_kv_heads, max_blocks), or a
    4-D pool ("HND" (num_blocks, num_kv_heads, block_size, head_size) or
    "NHD" (num_blocks, block_size, num_kv_heads, head_size)) with
    block_table (num_seqs, max_blocks).  k_new, v_new: (num_seqs,
    num_kv_heads, head_size).  cache_seqlens: int32 (num_seqs,) or
    (num_seqs, num_kv_heads), the current lengths L; the token goes to row
    L % block_size of page block_table[..., L // block_size] and, with
    ``increment``, L becomes L + 1 (in place).  A full table or an invalid
    page id leaves that entry untouched and sets a bit read by
    ``kv_append_status``.
    """
    if tuple(key_cache.shape) != tuple(value_cache.shape):
        raise ValueError("key_cache and value_cache shapes differ")
    if key_cache.dtype not in _DTYPES or value_cache.dtype != key_cache.dtype:
        raise TypeError("caches must share one dtype, bfloat16 or float16")
    if k_new.dtype != key_cache.dtype or v_new.dtype != key_cache.dtype:
        raise TypeError("k_new and v_new must have the caches' dtype")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("key_cache and value_cache must be contiguous")
    if k_new.dim() != 3 or tuple(k_new.shape) != tuple(v_new.shape):
        raise ValueError("k_new and v_new must be (num_seqs, num_kv_heads, head_size)")
    if k_new.stride(2) != 1 or v_new.stride(2) != 1 or k_new.stride() != v_new.stride():
        raise ValueError("k_new and v_new must share strides, contiguous in head_size")
    if cache_seqlens.dtype != torch.int32:
        raise TypeError("cache_seqlens must be int32 (it is updated in place)")
    bt = _as_int32(block_table, "block_table")
    B, Hkv, D = k_new.shape
    a = _lib.KvAppendArgs()
    if key_cache.dim() == 3:
        if bt.dim() != 3 or tuple(bt.shape[:2]) != (B, Hkv):
            raise ValueError("a 3-D cache needs block_table (num_seqs, num_kv_heads, max_blocks)")
        num_pages, bs, Dc = key_cache.shape
        layout, mul, add = _lib.LAYOUT_PAGES, 1, 0
        sb, sh, si, maxb = bt.stride(0), bt.stride(1), bt.stride(2), bt.shape[2]
    elif key_cache.dim() == 4 and kv_layout in ("HND", "NHD"):
        if bt.dim() != 2 or bt.shape[0] != B:
            raise ValueError("a 4-D pool needs block_table (num_seqs, max_blocks)")
        if kv_layout == "HND":
            nb, Hc, bs, Dc = key_cache.shape
            num_pages, layout, mul, add = nb * Hc, _lib.LAYOUT_PAGES, Hc, 1
        else:
            nb, bs, Hc, Dc = key_cache.shape
            num_pages, layout, mul, add = nb, _lib.LAYOUT_NHD, 1, 0
        if Hc != Hkv:
            raise ValueError(f"cache has {Hc} kv heads, k_new {Hkv}")
        sb, sh, si, maxb = bt.stride(0), 0, bt.stride(1), bt.shape[1]
    else:
        raise ValueError(f"unsupported cache rank {key_cache.dim()} / kv_layout {kv_layout!r}")
    if Dc != D:
        raise ValueError(f"cache head_size {Dc} != k_new head_size {D}")
    lens = cache_seqlens
    if lens.dim() == 1 and lens.shape[0] == B:
        lsb, lsh = lens.stride(0), 0
    elif lens.dim() == 2 and tuple(lens.shape) == (B, Hkv):
        lsb, lsh = lens.stride(0), lens.stride(1)
    else:
        raise ValueError("cache_seqlens must be (num_seqs,) or (num_seqs, num_kv_heads)")
    device = _check_device(key_cache, value_cache, k_new, v_new, lens, bt)
    status = _append_status_word(device)
    a.k_cache, a.v_cache = key_cache.data_ptr(), value_cache.data_ptr()
    a.k_new, a.v_new = k_new.data_ptr(), v_new.data_ptr()
    a.seqlens, a.block_table, a.status = lens.data_ptr(), bt.data_ptr(), status.data_ptr()
    a.dtype, a.layout = _DTYPES[key_cache.dtype], layout
    a.num_seqs, a.num_kv_heads, a.head_size, a.block_size = B, Hkv, D, bs
    a.max_blocks, a.num_pages = maxb, num_pages
    a.new_stride_b, a.new_stride_h = k_new.stride(0), k_new.stride(1)
    a.seqlens_stride_b, a.seqlens_stride_h = lsb, lsh
    a.bt_stride_b, a.bt_stride_h, a.bt_stride_i = sb, sh, si
    a.bt_page_mul, a.bt_page_add = mul, add
    a.increment = 1 if increment else 0
    lib = _lib.load()
    with torch.cuda.device(device):
        rc = lib.pab200_kv_append(ctypes.byref(a), ctypes.c_void_p(_current_stream_handle(device)))
    _lib.check(lib, rc, "pab200_kv_append")
    del bt


def kv_append_status(device=None, reset=True) -> int:
    """PAB200_STATUS_* bits raised by kv_append calls on ``device`` since the
    last reset (synchronises the device)."""
    device = torch.device("cuda", torch.cuda.current_device() if device is None else
                          torch.device(device).index)
    w = _append_status_word(device)
    bits = int(w.item())
    if reset:
        w.zero_()
    return bits
