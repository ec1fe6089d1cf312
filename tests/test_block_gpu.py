"""The block around the attention op (BiAttn/model.py:248-335) on the fused kernels.

* Whole ``BiAttnBlock`` layers against golden vectors the reference's own block wrote on the
  CPU (tests/golden/make_golden.py): output, input gradient and every parameter gradient.
* The fused residual + mask + RMSNorm and SwiGLU-gate kernels against a plain PyTorch fp32
  computation of the same ops over head widths 8..2048, with and without residual and mask.
"""

from __future__ import annotations

import types

import pytest
import torch
import torch.nn.functional as F

import sbda_b200

pytestmark = pytest.mark.gpu


def test_blocks_match_reference_golden(block_golden):
    for case in block_golden.cases:
        name = case["name"]
        block = sbda_b200.BiAttnBlock(types.SimpleNamespace(**case["config"]), case["layer_index"]).cuda()
        state = {k: block_golden.get(name, "param." + k) for k in block.state_dict()}
        block.load_state_dict(state)
        x = block_golden.get(name, "x").cuda().requires_grad_()
        valid_mask = block_golden.get(name, "valid_mask").cuda().bool() if case["valid_mask"] else None
        seam_reset = block_golden.get(name, "seam_reset").cuda().bool() if case["seam_reset"] else None
        y = block(x, valid_mask, seam_reset)
        y.backward(block_golden.get(name, "grad_y").cuda())
        tol = dict(rtol=3e-5, atol=3e-5)
        torch.testing.assert_close(y.detach().cpu(), block_golden.get(name, "y"), **tol, msg=name)
        torch.testing.assert_close(x.grad.cpu(), block_golden.get(name, "dx"), **tol, msg=name)
        for pname, param in block.named_parameters():
            torch.testing.assert_close(param.grad.cpu(), block_golden.get(name, "grad." + pname), **tol,
                                       msg=f"{name} {pname}")


def _torch_add_norm(x, a, mask, w, eps, dtype):
    """fp32 torch composite; x1 is rounded to ``dtype`` where the module forms it in ``dtype``
    (the rounding passes gradients straight through)."""
    x1 = x if a is None else x + (a * mask[..., None].to(a.dtype) if mask is not None else a)
    if a is not None and dtype != torch.float32:
        x1 = x1 + (x1.detach().to(dtype).float() - x1.detach())
    return x1, F.rms_norm(x1.float(), (x.shape[-1],), w.float(), eps)


@pytest.mark.parametrize("dim", [8, 64, 136, 256, 320, 1024, 2048])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_add_rms_norm_matches_torch(dim, dtype):
    g = torch.Generator(device="cuda").manual_seed(dim)
    rows = (3, 701)
    x = torch.randn(*rows, dim, device="cuda", generator=g).to(dtype)
    a = torch.randn(*rows, dim, device="cuda", generator=g).to(dtype)
    w = torch.rand(dim, device="cuda", generator=g) + 0.5
    mask = torch.rand(*rows, device="cuda", generator=g) > 0.2
    dy = torch.randn(*rows, dim, device="cuda", generator=g).to(dtype)
    dx1e = torch.randn(*rows, dim, device="cuda", generator=g).to(dtype)
    # bf16: 2e-2 max-abs plus one bf16 ulp relative (2^-7): the kernel rounds x1 = x + m*a to
    # bf16 before the norm and stores bf16 gradients, as the reference's bf16 module does; the
    # comparison here runs unrounded in fp32.
    tol = dict(rtol=1e-5, atol=1e-5) if dtype == torch.float32 else dict(rtol=2.0 ** -7, atol=2e-2)
    for with_add in (False, True):
        for m in ((None, mask) if with_add else (None,)):
            xs, as_, ws = (t.detach().clone().requires_grad_() for t in (x, a, w))
            xr, ar, wr = (t.detach().clone().float().requires_grad_() for t in (x, a, w))
            if with_add:
                x1, y = sbda_b200.add_rms_norm(xs, as_, ws, 1e-6, m)
                (y.float() * dy.float()).sum().backward(retain_graph=True)
                (x1.float() * dx1e.float()).sum().backward()
                rx1, ry = _torch_add_norm(xr, ar, m, wr, 1e-6, dtype)
                (ry * dy.float()).sum().backward(retain_graph=True)
                (rx1 * dx1e.float()).sum().backward()
                torch.testing.assert_close(x1.float(), rx1.detach(), **tol)
                torch.testing.assert_close(as_.grad.float(), ar.grad, **tol)
            else:
                y = sbda_b200.rms_norm(xs, ws, 1e-6)
                (y.float() * dy.float()).sum().backward()
                _, ry = _torch_add_norm(xr, None, None, wr, 1e-6, dtype)
                (ry * dy.float()).sum().backward()
            torch.testing.assert_close(y.float(), ry.detach(), **tol)
            torch.testing.assert_close(xs.grad.float(), xr.grad, **tol)
            wtol = dict(rtol=1e-4, atol=1e-4) if dtype == torch.float32 else dict(rtol=2e-2, atol=1e-1)
            torch.testing.assert_close(ws.grad.float(), wr.grad, **wtol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_silu_mul_matches_torch(dtype):
    g = torch.Generator(device="cuda").manual_seed(1)
    gate = (torch.randn(5, 333, 64, device="cuda", generator=g) * 3).to(dtype).requires_grad_()
    up = torch.randn(5, 333, 64, device="cuda", generator=g).to(dtype).requires_grad_()
    dh = torch.randn(5, 333, 64, device="cuda", generator=g).to(dtype)
    h = sbda_b200.silu_mul(gate, up)
    h.backward(dh)
    gr, ur = (t.detach().clone().requires_grad_() for t in (gate, up))
    hr = F.silu(gr) * ur
    hr.backward(dh)
    tol = dict(rtol=1e-5, atol=1e-5) if dtype == torch.float32 else dict(rtol=0, atol=3e-2)
    torch.testing.assert_close(h.float(), hr.float(), **tol)
    torch.testing.assert_close(gate.grad.float(), gr.grad.float(), **tol)
    torch.testing.assert_close(up.grad.float(), ur.grad.float(), **tol)


def test_norm_weight_gradient_is_deterministic():
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(4, 50_000, 256, device="cuda", generator=g).to(torch.bfloat16)
    w = torch.rand(256, device="cuda", generator=g) + 0.5
    dy = torch.randn_like(x)
    grads = []
    for _ in range(2):
        ws = w.detach().clone().requires_grad_()
        sbda_b200.rms_norm(x, ws).backward(dy)
        grads.append(ws.grad)
    assert torch.equal(grads[0], grads[1])
