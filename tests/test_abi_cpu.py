"""C-ABI library: builds, loads, exports every declared symbol, validates arguments.

No test here launches device work: each call returns from host-side argument
validation before any CUDA call, so the suite runs without a GPU.
"""

from __future__ import annotations

import ctypes
import os
import re

import pytest
import torch

import sbda_b200
from sbda_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "sbda_b200.h")


@pytest.fixture(scope="module")
def lib():
    build.build_library()
    return _lib.load()


def declared_symbols() -> list[str]:
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(sbda_b200_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert "sbda_b200_forward" in names and "sbda_b200_backward" in names
    for name in names:
        assert hasattr(lib, name), name


def test_abi_version_matches_header(lib):
    version = int(re.search(r"#define SBDA_B200_ABI_VERSION (\d+)", open(HEADER).read()).group(1))
    assert lib.sbda_b200_abi_version() == version


def test_kernel_family_is_an_argument(lib):
    """The family is a per-call argument: unknown families are rejected before any device work,
    and the library exports no process-wide switch."""
    assert not hasattr(lib, "sbda_b200_set_kernel_path")
    t = _lib.SbdaTensor(16, 1 << 20, 1 << 14, 64, 1)
    s = _lib.SbdaShape(1, 2, 2, 64, 64)
    offs = _lib.offsets_array((0, 1, 2, 4))
    for bad in (-1, 3, 7):
        assert lib.sbda_b200_forward_ex(bad, 2, s, offs, 4, 0.1, t, t, t, t, 16, None) == _lib.SBDA_ERR_INVALID
        assert lib.sbda_b200_backward_ex(bad, 2, s, offs, 4, 0.1, t, t, t, t, 16, t, t, t, None) \
            == _lib.SBDA_ERR_INVALID
    # Valid families on an empty problem: a successful no-op.
    empty = _lib.SbdaShape(0, 2, 2, 64, 64)
    for family in (0, 1, 2):
        assert lib.sbda_b200_forward_ex(family, 2, empty, offs, 4, 0.1, t, t, t, t, 16, None) == _lib.SBDA_OK


def test_status_strings(lib):
    for code in range(6):
        assert _lib.status_string(code)
    assert "dtype" in _lib.status_string(_lib.SBDA_ERR_DTYPE)


def _call_forward(lib, *, dtype=_lib.SBDA_DTYPE_BF16, shape=(1, 2, 2, 64, 64), offsets=(0, 1, 2, 4), n=None,
                  ptr=16):
    t = _lib.SbdaTensor(ptr, 1 << 20, 1 << 14, 64, 1)
    s = _lib.SbdaShape(*shape)
    return lib.sbda_b200_forward(dtype, s, _lib.offsets_array(offsets), len(offsets) if n is None else n,
                                 0.125, t, t, t, t, ptr, None)


def test_forward_validation_codes(lib):
    assert _call_forward(lib, dtype=7) == _lib.SBDA_ERR_DTYPE
    assert _call_forward(lib, n=5) == _lib.SBDA_ERR_INVALID
    assert _call_forward(lib, n=0) == _lib.SBDA_ERR_INVALID
    assert _call_forward(lib, offsets=(0, 1, 1, 4)) == _lib.SBDA_ERR_INVALID
    assert _call_forward(lib, offsets=(0, -1)) == _lib.SBDA_ERR_INVALID
    assert _call_forward(lib, shape=(1, 2, 2, 64, 129)) == _lib.SBDA_ERR_INVALID
    assert _call_forward(lib, shape=(1, 3, 2, 64, 64)) == _lib.SBDA_ERR_INVALID
    assert _call_forward(lib, shape=(1, 2, 2, 64, 0)) == _lib.SBDA_ERR_INVALID
    assert _call_forward(lib, ptr=0) == _lib.SBDA_ERR_INVALID
    # Sequences beyond 2^30 positions are outside the envelope.
    assert _call_forward(lib, shape=(1, 2, 2, (1 << 30) + 1, 64)) == _lib.SBDA_ERR_UNSUPPORTED
    # Empty problems are a successful no-op (no device work).
    assert _call_forward(lib, shape=(0, 2, 2, 64, 64)) == _lib.SBDA_OK
    assert _call_forward(lib, shape=(1, 2, 2, 0, 64)) == _lib.SBDA_OK


def test_kernel_family_context_is_local():
    """``kernel_family`` pins the family in this context only; another thread sees ``auto``."""
    import threading

    import sbda_b200

    assert sbda_b200.current_family() == 0
    seen = []
    with sbda_b200.kernel_family("uniform") as code:
        assert code == 2 and sbda_b200.current_family() == 2
        worker = threading.Thread(target=lambda: seen.append(sbda_b200.current_family()))
        worker.start()
        worker.join()
        with sbda_b200.kernel_family("general"):
            assert sbda_b200.current_family() == 1
        assert sbda_b200.current_family() == 2
    assert sbda_b200.current_family() == 0 and seen == [0]
    with pytest.raises(ValueError):
        with sbda_b200.kernel_family("fast"):
            pass


def test_backward_validation_codes(lib):
    t = _lib.SbdaTensor(16, 1 << 20, 1 << 14, 64, 1)
    s = _lib.SbdaShape(1, 2, 2, 64, 64)
    offs = _lib.offsets_array((0, 1, 2, 4))
    assert lib.sbda_b200_backward(9, s, offs, 4, 0.1, t, t, t, t, 16, t, t, t, None) == _lib.SBDA_ERR_DTYPE
    assert lib.sbda_b200_backward(2, s, offs, 4, 0.1, t, t, t, t, None, t, t, t, None) == _lib.SBDA_ERR_INVALID


def test_python_errors_follow_reference_types():
    q = torch.randn(1, 2, 8, 16)
    with pytest.raises(RuntimeError):
        sbda_b200.fused_sbda_key_backward(q, q, q, (0, 1))
    assert sbda_b200.host_offsets(torch.tensor([0, 1, 2, 8], dtype=torch.int32)) == (0, 1, 2, 8)
    assert sbda_b200.host_offsets([0, 2]) == (0, 2)
    module = sbda_b200.SBDAttention(16, 2, 3)
    with pytest.raises(RuntimeError):
        module(torch.randn(1, 4, 16))
    with pytest.raises(ValueError):
        sbda_b200.SBDAttention(16, 2, 3, use_fused=False)
    assert set(module.state_dict()) == {"q.weight", "k.weight", "v.weight", "out.weight",
                                        "q_norm.weight", "k_norm.weight"}


def test_norm_rope_validation_codes(lib):
    t = _lib.SbdaTensor(16, 1 << 20, 64, 256, 1)
    s = _lib.SbdaShape(1, 4, 4, 1000, 64)
    fwd = lib.sbda_b200_norm_rope_forward
    assert fwd(9, s, t, t, 16, 1e-6, 16, 16, 0, None) == _lib.SBDA_ERR_DTYPE
    assert fwd(2, _lib.SbdaShape(1, 4, 4, 1000, 129), t, t, 16, 1e-6, 16, 16, 0, None) == _lib.SBDA_ERR_INVALID
    assert fwd(2, s, t, t, 16, -1.0, 16, 16, 0, None) == _lib.SBDA_ERR_INVALID
    assert fwd(2, s, t, t, None, 1e-6, 16, 16, 0, None) == _lib.SBDA_ERR_INVALID
    assert fwd(2, s, t, t, 16, 1e-6, None, 16, 0, None) == _lib.SBDA_ERR_INVALID  # even D needs tables
    assert fwd(2, _lib.SbdaShape(1, 4, 4, 0, 64), t, t, 16, 1e-6, 16, 16, 0, None) == _lib.SBDA_OK
    # one partial row of fp32 per CTA of 128 rows, capped at 1024 CTAs
    assert lib.sbda_b200_norm_rope_workspace_floats(s) == 32 * 64
    # Backward grid cap: 2048 CTAs at head_dim <= 64, 1024 above; the partials always fit the
    # allocation-free entry point's 1024 x 128-float array.
    assert lib.sbda_b200_norm_rope_workspace_floats(_lib.SbdaShape(8, 8, 8, 1 << 20, 64)) == 2048 * 64
    assert lib.sbda_b200_norm_rope_workspace_floats(_lib.SbdaShape(8, 8, 8, 1 << 20, 128)) == 1024 * 128
    bwd = lib.sbda_b200_norm_rope_backward
    assert bwd(2, s, t, t, 16, 1e-6, 16, 16, 0, t, 16, 16, 2047, None) == _lib.SBDA_ERR_INVALID  # workspace
    assert bwd(2, s, t, t, 16, 1e-6, 16, 16, 0, t, None, 16, 2048, None) == _lib.SBDA_ERR_INVALID
