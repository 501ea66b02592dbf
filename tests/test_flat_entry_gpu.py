"""GPU: the flat north-star C entry point, pab200_paged_attention, called
through the ctypes binding that INTEGRATION.md section 3 gives a maintainer
of the reference (read from that file and run as written, with only the
library path filled in).

Contract: src/common.py:1-14 (q (B, 1, Hq, D), caches (pages, block_size, D),
cache_seqlens (B, Hkv), block_table (B, Hkv, max_blocks)).  Checked against
the fp32 oracle at the reference's tolerance, atol = rtol = 2e-2
(scripts/benchmark.py:63-72), and bit for bit against the package wrapper,
which runs the same kernels with the same plan.
"""
import os
import re
from pathlib import Path

import pytest
import torch

from pagedattention_b200 import flash_attn_with_kvcache_wrapper_b200
from pagedattention_b200.workloads import WORKLOADS, make_inputs
from tests.util import assert_close, run_oracle

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def _documented_binding():
    """The python block of INTEGRATION.md section 3, executed as written."""
    text = (ROOT / "INTEGRATION.md").read_text()
    sec = text[text.index("## 3."):text.index("## 4.")]
    code = re.search(r"```python\n(.*?)```", sec, re.S).group(1)
    assert "pab200_paged_attention(" in code
    code = code.replace("/path/to/this/repo", str(ROOT))
    ns = {}
    exec(compile(code, "INTEGRATION.md#3", "exec"), ns)
    return ns["flash_attn_with_kvcache_wrapper_b200"]


@pytest.mark.parametrize("workload,num_seqs", [("llama8b_gqa", None), ("llama70b_mixed", 24)])
def test_flat_entry_point_matches_oracle(cuda_device, workload, num_seqs):
    """The headline batch (64 x 4096 tokens, 32/8 heads, D 128, bs 16, bf16)
    and a mixed-length batch (lognormal lengths, 64/8 heads, bs 32)."""
    dev = cuda_device
    flat = _documented_binding()
    w = WORKLOADS[workload]
    inp = make_inputs(w, seed=17, device=dev, gen_device=dev, num_seqs=num_seqs)
    q, k, v, sl, bt = inp.reference_layout()
    q, sl, bt = q.contiguous(), sl.contiguous(), bt.contiguous()
    out = flat(q=q, k_cache=k, v_cache=v, cache_seqlens=sl, block_table=bt,
               softmax_scale=inp.scale, num_splits=1)
    pkg = flash_attn_with_kvcache_wrapper_b200(q, k, v, sl, bt, inp.scale, num_splits=1)
    torch.cuda.synchronize(dev)
    assert out.shape == q.shape and out.dtype == q.dtype
    assert torch.equal(out, pkg), "flat entry point and package wrapper differ"
    ref = run_oracle(q.cpu(), k.cpu(), v.cpu(), sl.cpu(), bt.cpu(), inp.scale,
                     threads=os.cpu_count() or 1)
    assert_close(out, ref, what=f"flat entry point, {workload}")


def test_flat_entry_point_reports_errors(cuda_device):
    """An unsupported head size is refused with the library's message."""
    dev = cuda_device
    flat = _documented_binding()
    q = torch.zeros((1, 1, 4, 96), dtype=torch.bfloat16, device=dev)
    k = torch.zeros((2, 16, 96), dtype=torch.bfloat16, device=dev)
    sl = torch.ones((1, 1), dtype=torch.int32, device=dev)
    bt = torch.zeros((1, 1, 1), dtype=torch.int32, device=dev)
    with pytest.raises(ValueError, match="head_size 96"):
        flat(q=q, k_cache=k, v_cache=k, cache_seqlens=sl, block_table=bt, softmax_scale=0.1)
