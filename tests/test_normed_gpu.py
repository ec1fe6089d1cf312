"""Attention with the per-head RMSNorm + RoPE fused into the windowed kernels.

``normed_attention(q_raw, k_raw, v, wq, wk, offsets)`` must compute
``attention(rope(norm(q_raw)), rope(norm(k_raw)), v)`` (``BiAttn/attention_common.py:13-76``
then ``BiAttn/left_v2.py:335-405``) and its gradients with respect to ``q_raw``, ``k_raw``, ``v``
and both norm weights.  Checked on every walk mode of the backward (layers 1, 2, 3, 6, 7, 9, 12:
the {0,1} and {0,2} sets, local, local-carry and chain walks) and every dtype, against

* an fp64 oracle of the same function (the reference's norm and RoPE values -- fp32 norm cast
  to the dtype, RoPE in dtype ops with the device's cos/sin table -- then exact gather attention
  in fp64; gradients of the unrounded norm and RoPE), within the stated tolerances: fp32 1e-5
  relative (rtol = atol = 1e-5 on O(1) values), bf16/fp16 2e-2 max-abs on O, dQ, dK, dV, with
  2^-7 relative added for the raw-input gradients dQ, dK, dV (see ``GRAD_RTOL_16``); the weight
  gradients, sums over every row, within 1e-4 (fp32) or 3e-2 (16-bit) of their largest entry;
* the separate route (norm + RoPE kernels, then the attention kernels), in the same dtype.
"""

from __future__ import annotations

import pytest
import torch

from oracle import sbda_oracle as orc

import sbda_b200

pytestmark = pytest.mark.gpu

TOL = {torch.float32: dict(rtol=1e-5, atol=1e-5), torch.bfloat16: dict(rtol=0.0, atol=2e-2),
       torch.float16: dict(rtol=0.0, atol=2e-2)}
# Gradients with respect to the raw projections pass through the RMSNorm Jacobian (a factor
# 1 / rms(x) and the weights), so they reach magnitudes of ~30 here, where half an ulp of the
# stored 16-bit value alone is 0.06.  For them the 2e-2 bound is widened by 2^-7 relative (two
# bf16 ulps: the storage rounding plus the rounding of the attention's inputs).
GRAD_RTOL_16 = 2.0 ** -7
W_TOL = {torch.float32: 1e-4, torch.bfloat16: 3e-2, torch.float16: 3e-2}


def _inputs(batch, heads, length, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)

    def proj():  # [B, L, H, 64] projections, viewed as [B, H, L, 64]
        return (torch.randn(batch, length, heads, 64, device="cuda", generator=g) * 1.7).to(dtype).permute(0, 2, 1, 3)

    q, k, v, do = proj(), proj(), proj(), proj()
    wq = (torch.rand(64, device="cuda", generator=g) + 0.5)
    wk = (torch.rand(64, device="cuda", generator=g) + 0.5)
    return q, k, v, do, wq, wk


def _fused(q, k, v, do, wq, wk, offsets):
    q, k, v = (t.detach().requires_grad_() for t in (q, k, v))
    wq, wk = wq.detach().requires_grad_(), wk.detach().requires_grad_()
    out = sbda_b200.normed_attention(q, k, v, wq, wk, offsets)
    out.backward(do)
    return out.detach(), q.grad, k.grad, v.grad, wq.grad, wk.grad


def _separate(q, k, v, do, wq, wk, offsets):
    q, k, v = (t.detach().requires_grad_() for t in (q, k, v))
    wq, wk = wq.detach().requires_grad_(), wk.detach().requires_grad_()
    qn = sbda_b200.norm_rope(q.permute(0, 2, 1, 3), wq).permute(0, 2, 1, 3)
    kn = sbda_b200.norm_rope(k.permute(0, 2, 1, 3), wk).permute(0, 2, 1, 3)
    out = sbda_b200.fused_sbda_key_backward(qn, kn, v, offsets)
    out.backward(do)
    return out.detach(), q.grad, k.grad, v.grad, wq.grad, wk.grad


def _oracle(q, k, v, do, wq, wk, offsets, eps=1e-6, theta=1e6):
    """fp64 attention on the reference's normalised, rotated q and k.

    Forward values follow the reference's roundings exactly: the fp32 RMSNorm cast to the dtype
    (``attention_common.py:72-76``) and the RoPE run as dtype ops with the device table
    (``:44-49``), on the CPU.  Gradients are those of the unrounded norm and RoPE (each rounding
    passes its gradient straight through), in fp64: the function the kernels differentiate.
    """
    length = q.shape[2]
    cos, sin = sbda_b200.rope_table(length, 64, theta, q.dtype, q.device)
    cos, sin = cos.cpu(), sin.cpu()
    c = torch.cat((cos, cos), -1).double()[None, None]
    s = torch.cat((sin, sin), -1).double()[None, None]
    qr, kr, vr, dr = (t.detach().double().cpu().requires_grad_() for t in (q, k, v, do))
    wq64, wk64 = (w.detach().double().cpu().requires_grad_() for w in (wq, wk))

    def nr(x, w, x_dtype):
        y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w
        exact = y * c + orc.rotate_half(y) * s
        # The reference's values: norm in fp32 cast to the dtype, RoPE in dtype ops ([B,L,H,D] layout).
        ref = orc.head_rms_norm(x_dtype.permute(0, 2, 1, 3), w.detach().float())
        ref = orc.apply_rope_table(ref, cos, sin).permute(0, 2, 1, 3).double()
        return exact + (ref - exact).detach()

    qn = nr(qr, wq64, q.detach().cpu())
    kn = nr(kr, wk64, k.detach().cpu())
    out = orc.exact_attention(qn, kn, vr, offsets)
    out.backward(dr)
    return out.detach(), qr.grad, kr.grad, vr.grad, wq64.grad, wk64.grad


def _compare(got, ref, dtype, tag, widen=1.0):
    names = ("O", "dQ", "dK", "dV")
    errs = [float((a.double().cpu() - b.double().cpu()).abs().max()) for a, b in zip(got, ref)]
    print(tag, " ".join(f"{n}={e:.2e}" for n, e in zip(names + ("dWq", "dWk"), errs)))
    for name, a, b in zip(names, got[:4], ref[:4]):
        tol = dict(TOL[dtype])
        if name != "O" and dtype != torch.float32:
            tol["rtol"] = GRAD_RTOL_16
        tol = {key: value * widen for key, value in tol.items()}
        torch.testing.assert_close(a.float().cpu(), b.float().cpu(), **tol, msg=lambda m: f"{tag} {name}: {m}")
    for name, a, b in zip(("dWq", "dWk"), got[4:], ref[4:]):
        scale = float(b.abs().max())
        err = float((a.double().cpu() - b.double().cpu()).abs().max())
        assert err <= widen * W_TOL[dtype] * max(scale, 1.0), \
            f"{tag} {name}: max error {err:.3e} (largest entry {scale:.3e})"


LAYERS = (1, 2, 3, 6, 7, 9, 12)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_normed_attention_matches_fp64_oracle(dtype):
    for layer in LAYERS:
        offsets = sbda_b200.topology_offsets(layer, topology="sbda")
        for length in (3000, 1000):
            q, k, v, do, wq, wk = _inputs(2, 4, length, dtype, seed=layer * 10 + length)
            if max(offsets) >= length:
                # The far source never exists: the set is {0, 1, 2}, served by the separate route.
                assert not sbda_b200.normed_supported(q, k, v, offsets), (layer, length)
                continue
            assert sbda_b200.normed_supported(q, k, v, offsets), (layer, length)
            got = _fused(q, k, v, do, wq, wk, offsets)
            ref = _oracle(q, k, v, do, wq, wk, offsets)
            _compare(got, ref, dtype, f"layer {layer} L {length} {dtype}")
    assert sbda_b200.device_status(reset=True) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_normed_attention_matches_separate_route(dtype):
    """Fused and separate routes agree, including long segmented chain walks.  Each route is an
    approximation of the same function; the separate one rounds dQ and dK of the normalised rows
    to the dtype before the norm's Jacobian, whose cancellation can amplify that rounding.  Two
    results each within the oracle bound of the truth differ by at most twice it, which is the
    bound used here (the fused route itself is held to the single bound above)."""
    for layer, length in ((8, 20000), (11, 20000), (14, 40000), (5, 20000)):
        offsets = sbda_b200.topology_offsets(layer, topology="sbda")
        q, k, v, do, wq, wk = _inputs(1, 4, length, dtype, seed=layer)
        got = _fused(q, k, v, do, wq, wk, offsets)
        ref = _separate(q, k, v, do, wq, wk, offsets)
        _compare(got, ref, dtype, f"layer {layer} L {length} {dtype} vs separate", widen=2.0)
    assert sbda_b200.device_status(reset=True) == 0


def test_normed_attention_is_deterministic():
    offsets = sbda_b200.topology_offsets(10, topology="sbda")
    q, k, v, do, wq, wk = _inputs(2, 4, 9000, torch.bfloat16, seed=3)
    first = _fused(q, k, v, do, wq, wk, offsets)
    second = _fused(q, k, v, do, wq, wk, offsets)
    for a, b in zip(first, second):
        assert torch.equal(a, b)


def test_normed_support_envelope():
    q, k, v, _, _, _ = _inputs(1, 4, 512, torch.bfloat16, seed=1)
    assert sbda_b200.normed_supported(q, k, v, (0, 1, 2, 8))
    assert not sbda_b200.normed_supported(q, k, v, (0, 3))  # near offset outside {0, 1, 2}
    assert not sbda_b200.normed_supported(q[..., :32], k[..., :32], v[..., :32], (0, 1))  # head_dim 32
    assert not sbda_b200.normed_supported(q, k[:, :2], v[:, :2], (0, 1))  # GQA
    with pytest.raises(ValueError):
        sbda_b200.normed_attention(q, k, v, torch.ones(64, device="cuda"), torch.ones(64, device="cuda"), (0, 3))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_module_fused_route_matches_separate_route(dtype):
    """``SBDAttention`` with head_dim 64 takes the fused route; its output and every parameter
    gradient match the same module on the separate norm kernels."""
    for layer in (2, 5, 9):
        torch.manual_seed(layer)
        module = sbda_b200.SBDAttention(256, 4, layer, total_layers=12).cuda().to(dtype)
        with torch.no_grad():
            module.q_norm.weight.uniform_(0.5, 1.5)
            module.k_norm.weight.uniform_(0.5, 1.5)
        x = torch.randn(2, 700, 256, device="cuda").to(dtype)
        dy = torch.randn(2, 700, 256, device="cuda").to(dtype)
        results = []
        for fused in (True, False):
            module.fused_norm_rope = fused
            module.zero_grad()
            xi = x.detach().requires_grad_()
            y = module(xi)
            y.backward(dy)
            results.append((y.detach(), xi.grad, {n: p.grad.clone() for n, p in module.named_parameters()}))
        (y1, dx1, g1), (y2, dx2, g2) = results
        tol = dict(rtol=2e-5, atol=2e-5) if dtype == torch.float32 else dict(rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(y1.float(), y2.float(), **tol)
        torch.testing.assert_close(dx1.float(), dx2.float(), **tol)
        for name in g1:
            scale = max(1.0, float(g2[name].abs().max()))
            torch.testing.assert_close(g1[name].float() / scale, g2[name].float() / scale, **tol, msg=name)
    assert sbda_b200.device_status(reset=True) == 0
