"""The first backward of a process runs on autograd's worker thread, which may have no current
CUDA context yet.  It must still get the copy-engine (TMA) kernels, not the generic loader that
serves layouts the copy engine cannot stage.  Checked in a fresh child process (kernel names
through torch.profiler), since later calls in this process would find a context already bound.
"""

from __future__ import annotations

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys
sys.path.insert(0, sys.argv[1])
import torch
from torch.profiler import ProfilerActivity, profile
import sbda_b200
base = [torch.randn(1, 3000, 4, 64, device="cuda").to(torch.bfloat16) for _ in range(4)]
q, k, v = (t.permute(0, 2, 1, 3).requires_grad_() for t in base[:3])
with profile(activities=[ProfilerActivity.CUDA]) as prof:
    out = sbda_b200.fused_sbda_key_backward(q, k, v, (0, 1))
    out.backward(base[3].permute(0, 2, 1, 3))
    torch.cuda.synchronize()
for e in prof.events():
    if "sbda_" in e.name and e.device_type.name == "CUDA":
        print("KERNEL", e.name.split("(")[0])
"""


def test_first_backward_on_the_autograd_thread_uses_the_copy_engine():
    result = subprocess.run([sys.executable, "-c", CHILD, ROOT], capture_output=True, text=True, timeout=600)
    assert result.returncode == 0, result.stderr[-2000:]
    kernels = [line.split(" ", 1)[1] for line in result.stdout.splitlines() if line.startswith("KERNEL ")]
    bwd = [name for name in kernels if "sbda_bwd_v2_kernel" in name]
    fwd = [name for name in kernels if "sbda_fwd_v2_kernel" in name]
    assert len(bwd) == 1 and len(fwd) == 1, kernels
    # template arguments <element, lanes per row, copy engine, source-set shape, maps>
    assert ", true," in bwd[0] and ", true," in fwd[0], kernels
