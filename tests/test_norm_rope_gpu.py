"""Per-head RMSNorm + RoPE kernels against the CPU oracle (attention_common.py restated).

Forward: the oracle runs the reference's op sequence in the same dtype on the CPU (bf16/fp16
roundings included); bf16/fp16 outputs agree within 2e-2 max-abs, fp32 within 1e-5.
Backward: against fp64 autograd of the oracle on the same inputs (the casts have identity
derivatives there, as in the kernel); the norm-weight gradient is a sum over every row, so it
is compared with a relative bound.
"""

from __future__ import annotations

import pytest
import torch

from oracle import sbda_oracle as orc

import sbda_b200

pytestmark = pytest.mark.gpu

TOL = {torch.float32: dict(rtol=1e-5, atol=1e-5),
       torch.bfloat16: dict(rtol=0.0, atol=2e-2),
       torch.float16: dict(rtol=0.0, atol=2e-2)}


def _table(x: torch.Tensor, theta: float, offset: int):
    """The cos/sin rows the kernel used (built on the device like the reference's)."""
    length, head_dim = x.shape[1], x.shape[-1]
    if head_dim % 2:
        return None, None
    cos, sin = sbda_b200.rope_table(offset + length, head_dim, theta, x.dtype, x.device)
    return cos[offset:].cpu(), sin[offset:].cpu()


def _oracle_forward(x: torch.Tensor, w: torch.Tensor, theta: float, offset: int) -> torch.Tensor:
    cos, sin = _table(x, theta, offset)
    y = orc.head_rms_norm(x.cpu(), w.cpu())
    return y if cos is None else orc.apply_rope_table(y, cos, sin)


def _oracle_grads(x, w, dy, theta, offset, dtype):
    cos, sin = _table(x.to(dtype), theta, offset)
    xd = x.detach().cpu().double().requires_grad_()
    wd = w.detach().cpu().double().requires_grad_()
    y = orc.head_rms_norm(xd, wd)
    rq = y if cos is None else orc.apply_rope_table(y, cos.double(), sin.double())
    rq.backward(dy.detach().cpu().double())
    return xd.grad, wd.grad


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("head_dim", [8, 16, 40, 64, 96, 128, 7])
def test_norm_rope_matches_oracle(dtype, head_dim):
    g = torch.Generator(device="cuda").manual_seed(head_dim)
    x = (torch.randn(2, 300, 3, head_dim, device="cuda", generator=g) * 1.7).to(dtype)
    w = (torch.rand(head_dim, device="cuda", generator=g) + 0.5).requires_grad_()
    xg = x.clone().requires_grad_()
    y = sbda_b200.norm_rope(xg, w, theta=1e6)
    expected = _oracle_forward(x, w.detach(), 1e6, 0)
    torch.testing.assert_close(y.float().cpu(), expected.float(), **TOL[dtype])
    dy = torch.randn(y.shape, device="cuda", generator=g).to(dtype)
    y.backward(dy)
    rdx, rdw = _oracle_grads(x.float(), w.detach(), dy.float(), 1e6, 0, dtype)
    torch.testing.assert_close(xg.grad.float().cpu(), rdx.float(), **TOL[dtype])
    torch.testing.assert_close(w.grad.cpu(), rdw.float(), rtol=1e-3 if dtype == torch.float32 else 2e-2,
                               atol=1e-3 if dtype == torch.float32 else 5e-2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rope_table_follows_reference_formula(dtype):
    """The device table equals attention_common.py:13-22 evaluated on the CPU, up to the last
    bit of fp32 pow/cos (angles up to 1e4 rad here) and one rounding step of the dtype."""
    cos, sin = sbda_b200.rope_table(10000, 64, 1e6, dtype, torch.device("cuda"))
    rc, rs = orc.rope_cos_sin(torch.arange(10000), 64, 1e6, dtype)
    rc, rs = rc[0, :, 0, :32], rs[0, :, 0, :32]
    tol = dict(rtol=0, atol=2e-3) if dtype == torch.float32 else dict(rtol=0, atol=8e-3)
    torch.testing.assert_close(cos.cpu().float(), rc.float(), **tol)
    torch.testing.assert_close(sin.cpu().float(), rs.float(), **tol)
    # and exactly torch's own expression on the device
    inv = 1e6 ** (-torch.arange(0, 64, 2, device="cuda", dtype=torch.float32) / 64)
    ang = torch.outer(torch.arange(10000, device="cuda").to(torch.float32), inv)
    assert torch.equal(cos, ang.cos().to(dtype)) and torch.equal(sin, ang.sin().to(dtype))


def test_norm_rope_strided_input_and_position_offset():
    g = torch.Generator(device="cuda").manual_seed(5)
    base = torch.randn(1, 700, 4, 96, device="cuda", generator=g).to(torch.bfloat16)
    x = base[..., 16:80]  # a strided [B, L, H, 64] view
    w = torch.rand(64, device="cuda", generator=g) + 0.5
    full = sbda_b200.norm_rope(x, w, theta=1e4)
    part = sbda_b200.norm_rope(x[:, 500:].contiguous(), w, theta=1e4, position_offset=500)
    assert torch.equal(full[:, 500:], part)
    torch.testing.assert_close(full.float().cpu(), _oracle_forward(x, w, 1e4, 0).float(), rtol=0, atol=2e-2)


def test_norm_rope_backward_is_deterministic():
    g = torch.Generator(device="cuda").manual_seed(6)
    x = torch.randn(4, 20000, 4, 64, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.rand(64, device="cuda", generator=g) + 0.5)
    dy = torch.randn(x.shape, device="cuda", generator=g).to(torch.bfloat16)
    grads = []
    for _ in range(2):
        xg, wg = x.clone().requires_grad_(), w.clone().requires_grad_()
        sbda_b200.norm_rope(xg, wg).backward(dy)
        grads.append((xg.grad, wg.grad))
    assert torch.equal(grads[0][0], grads[1][0])
    assert torch.equal(grads[0][1], grads[1][1])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 4099, 3), (2, 20000, 4), (3, 1, 5), (1, 300000, 4)])
def test_norm_rope_contiguous_and_strided_paths_agree(dtype, shape):
    """head_dim 64: contiguous [B, L, H, 64] rows take the kernels that stream rows through a
    shared-memory ring, other vector layouts the kernels that load rows into registers.  Both run
    the same rows, lanes and operations, so y, dx and the weight gradient agree bit for bit.  The
    shapes cover a partial last chunk, a single partial chunk and many chunks per CTA."""
    B, L, H = shape
    g = torch.Generator(device="cuda").manual_seed(L + H)
    x = (torch.randn(B, L, H, 64, device="cuda", generator=g) * 1.7).to(dtype)
    dy = torch.randn(B, L, H, 64, device="cuda", generator=g).to(dtype)
    w = torch.rand(64, device="cuda", generator=g) + 0.5
    wide = torch.zeros(B, L, H, 128, device="cuda", dtype=dtype)
    wide[..., 32:96] = x
    results = []
    for leaf in (x.clone().requires_grad_(), wide.clone().requires_grad_()):
        xs = leaf if leaf.shape[-1] == 64 else leaf[..., 32:96]  # contiguous rows, then a strided view
        wg = w.clone().requires_grad_()
        y = sbda_b200.norm_rope(xs, wg, theta=1e6)
        y.backward(dy)
        dx = leaf.grad if leaf.shape[-1] == 64 else leaf.grad[..., 32:96]
        results.append((y, dx, wg.grad))
    (y1, dx1, dw1), (y2, dx2, dw2) = results
    assert torch.equal(y1, y2)
    assert torch.equal(dx1, dx2)
    assert torch.equal(dw1, dw2)
    assert sbda_b200.device_status(reset=True) == 0


def test_norm_rope_fault_word_clean():
    assert sbda_b200.device_status(reset=True) == 0
