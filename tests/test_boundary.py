"""The C ABI boundary without a GPU: the library loads, exports every function
include/pab200.h declares, its struct layout matches the ctypes mirror, and
host-side argument validation returns the documented codes."""
import ctypes
import re
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from pagedattention_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "pab200.h"


def header_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(pab200_\w+)\s*\(", text)))


def test_header_declares_expected_api():
    assert set(header_functions()) == set(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in header_functions():
        assert hasattr(lib, name), name
    nm = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)],
                        capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in nm.splitlines() if " T " in line}
    assert exported == set(header_functions())


def test_abi_version_and_strerror():
    lib = _lib.load()
    assert lib.pab200_abi_version() == _lib.ABI_VERSION
    assert lib.pab200_strerror(0) == b"ok"
    assert lib.pab200_strerror(_lib.ERR_WORKSPACE) == b"workspace missing or too small"


def test_struct_layout_matches_c(tmp_path):
    """Compile a C program against the header and compare sizeof/offsetof with
    the ctypes mirror field by field."""
    fields = [f for f, _ in _lib.DecodeArgs._fields_]
    src = ['#include <stdio.h>', '#include <stddef.h>', '#include "pab200.h"', 'int main(void){',
           'printf("size %zu\\n", sizeof(pab200_decode_args));']
    src += [f'printf("{f} %zu\\n", offsetof(pab200_decode_args, {f}));' for f in fields]
    src += ['return 0;}']
    c = tmp_path / "layout.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", str(ROOT / "include"), str(c), "-o", str(exe)],
                   check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True,
                                                       text=True, check=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(_lib.DecodeArgs)
    for f in fields:
        assert int(out[f]) == getattr(_lib.DecodeArgs, f).offset, f


def _valid_args():
    a = _lib.DecodeArgs()
    a.out = a.q = a.k_cache = a.v_cache = a.seqlens = a.block_table = 4096
    a.dtype, a.layout = _lib.DTYPE_BF16, _lib.LAYOUT_PAGES
    a.num_seqs, a.num_q_heads, a.num_kv_heads = 2, 8, 2
    a.head_size, a.block_size, a.max_blocks, a.num_pages = 128, 16, 4, 16
    a.q_stride_b, a.q_stride_h = 8 * 128, 128
    a.out_stride_b, a.out_stride_h = 8 * 128, 128
    a.seqlens_stride_b, a.seqlens_stride_h = 2, 1
    a.bt_stride_b, a.bt_stride_h, a.bt_stride_i = 8, 4, 1
    a.bt_page_mul = 1
    a.softmax_scale = 0.1
    return a


@pytest.mark.parametrize("field,value,code", [
    ("dtype", 7, _lib.ERR_UNSUPPORTED),
    ("head_size", 96, _lib.ERR_UNSUPPORTED),
    ("block_size", 12, _lib.ERR_UNSUPPORTED),
    ("num_q_heads", 7, _lib.ERR_INVALID_ARGUMENT),     # not a multiple of Hkv
    ("num_q_heads", 2 * 64, _lib.ERR_UNSUPPORTED),     # G = 64: above a warp pair's tile
    ("num_seqs", 0, _lib.ERR_INVALID_ARGUMENT),
    ("layout", 5, _lib.ERR_INVALID_ARGUMENT),
    ("q", 4098, _lib.ERR_ALIGNMENT),
    ("k_cache", 4104, _lib.ERR_ALIGNMENT),
    ("num_splits", -1, _lib.ERR_INVALID_ARGUMENT),
    ("q", 0, _lib.ERR_INVALID_ARGUMENT),
])
def test_host_validation_codes(field, value, code):
    """Bad arguments are refused on the host with the documented code before
    any device work (these calls never reach CUDA)."""
    lib = _lib.load()
    a = _valid_args()
    setattr(a, field, value)
    assert lib.pab200_decode_workspace_size(ctypes.byref(a)) == 0
    rc = lib.pab200_decode(ctypes.byref(a), ctypes.c_void_p(1 << 20), 1 << 20, None)
    assert rc == code, lib.pab200_last_error()
    assert lib.pab200_last_error() != b""


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_no_device_is_a_clean_error():
    lib = _lib.load()
    a = _valid_args()
    rc = lib.pab200_decode(ctypes.byref(a), ctypes.c_void_p(1 << 20), 1 << 20, None)
    assert rc == _lib.ERR_CUDA


def test_merge_states_argument_checks():
    lib = _lib.load()
    assert lib.pab200_merge_states(None, 0, None, 0, 0, 1, 128, None, 128, 0, None) == \
        _lib.ERR_INVALID_ARGUMENT
    assert lib.pab200_merge_states(None, 0, None, 0, 2, 0, 128, None, 128, 0, None) == _lib.OK
    assert lib.pab200_merge_states(16, 4, 16, 1, 2, 8, 128, 16, 128, 0, None) == \
        _lib.ERR_INVALID_ARGUMENT   # strides smaller than one state


def test_missing_library_fails_loudly(tmp_path):
    """No CPU fallback: without libpab200.so the package raises."""
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "from pathlib import Path\n"
        "import pagedattention_b200._lib as L\n"
        "L.LIB_PATH = Path(%r)\n"
        "try:\n"
        "    L.load()\n"
        "except L.LibraryNotBuilt as e:\n"
        "    print('raised', e)\n"
    ) % (str(ROOT), str(tmp_path / "missing.so"))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True)
    assert "raised" in out.stdout, out.stderr


def test_exchange_argument_checks():
    """Host-side checks of the multi-GPU exchange entry points (no device
    work): buffer sizing, and refusals before any launch."""
    lib = _lib.load()
    assert lib.pab200_exchange_buffer_bytes(0, 8, 128) == 0
    assert lib.pab200_exchange_buffer_bytes(2, 0, 128) == 0
    assert lib.pab200_exchange_buffer_bytes(2, 8, 130) == 0
    rows, D, world = 8, 128, 2
    S = rows * D + ((rows + 3) // 4) * 4
    nb = min((rows + 7) // 8, 128)
    want = 2 * world * S * 8 + ((nb + 3) // 4) * 4 * 4
    assert lib.pab200_exchange_buffer_bytes(world, rows, D) == want
    # rank outside [0, world), zero wait limit, null pointers, misalignment
    args = (16, 16, 2, 2, rows, D, 16, D, _lib.DTYPE_BF16, 10**9, 16, None)
    assert lib.pab200_exchange_merge(*args) == _lib.ERR_INVALID_ARGUMENT
    args = (16, 16, 0, 2, rows, D, 16, D, _lib.DTYPE_BF16, 0, 16, None)
    assert lib.pab200_exchange_merge(*args) == _lib.ERR_INVALID_ARGUMENT
    args = (None, 16, 0, 2, rows, D, 16, D, _lib.DTYPE_BF16, 10**9, 16, None)
    assert lib.pab200_exchange_merge(*args) == _lib.ERR_INVALID_ARGUMENT
    args = (8, 16, 0, 2, rows, D, 16, D, _lib.DTYPE_BF16, 10**9, 16, None)
    assert lib.pab200_exchange_merge(*args) == _lib.ERR_ALIGNMENT
    # the fused decode + exchange: args and the packed state are checked first
    assert lib.pab200_decode_exchange(None, 0, 0, 16, 0, 2, 16, D, _lib.DTYPE_BF16, 10**9, 16,
                                      None) == _lib.ERR_INVALID_ARGUMENT
    a = _lib.DecodeArgs()
    a.num_seqs, a.num_q_heads, a.head_size = 2, 4, D
    a.state_o, a.state_lse = 256, 256 + 4            # lse not right after o
    assert lib.pab200_decode_exchange(ctypes.byref(a), 0, 0, 16, 0, 2, 16, D, _lib.DTYPE_BF16,
                                      10**9, 16, None) == _lib.ERR_INVALID_ARGUMENT
    a.state_lse = 256 + 2 * 4 * D * 4                # packed, but rank outside [0, world)
    assert lib.pab200_decode_exchange(ctypes.byref(a), 0, 0, 16, 2, 2, 16, D, _lib.DTYPE_BF16,
                                      10**9, 16, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.pab200_exchange_buffer_close(None) == _lib.OK
    assert lib.pab200_exchange_buffer_destroy(None) == _lib.OK
    assert lib.pab200_exchange_buffer_create(0, ctypes.byref(ctypes.c_void_p()), None) == \
        _lib.ERR_INVALID_ARGUMENT
