"""Parity of the B200 kernels (through the C ABI) with the CPU oracle.

Tolerances (stated by the task): fp32 within 1e-5 relative (checked as
``rtol=atol=1e-5`` on O(1) values, against an fp64 oracle); bf16/fp16 within
2e-2 max-abs on O, dQ, dK and dV (against the fp32 oracle on the same
bf16-rounded inputs).  Index/mask logic is exercised at every offset and
boundary; results must also be bitwise deterministic.
"""

from __future__ import annotations

import pytest
import torch

from oracle import sbda_oracle as orc

import sbda_b200
from sbda_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["auto", "general", "uniform"])
def kernel_path(request):
    """Runs a test through the windowed kernels (auto), the general ones and the uniform ones."""
    with sbda_b200.kernel_family(request.param):
        yield request.param

TOL = {torch.float32: dict(rtol=1e-5, atol=1e-5),
       torch.bfloat16: dict(rtol=0.0, atol=2e-2),
       torch.float16: dict(rtol=0.0, atol=2e-2)}


def _close(actual: torch.Tensor, expected: torch.Tensor, dtype: torch.dtype, msg: str, *,
           rtol: float | None = None) -> None:
    tol = dict(TOL[dtype])
    if rtol is not None:
        tol["rtol"] = rtol
    torch.testing.assert_close(actual.detach().float().cpu(), expected.float().cpu(), **tol,
                               msg=lambda detail: f"{msg}: {detail}")


def _inputs(batch, heads, length, dim, dtype, *, kv_heads=None, layout="blhd", seed=0):
    """q/k/v/dO as [B,H,L,D] views; ``blhd`` = permuted projections (the reference layout)."""
    kv_heads = heads if kv_heads is None else kv_heads
    g = torch.Generator(device="cuda").manual_seed(seed)

    def randn(*shape):
        return torch.randn(*shape, device="cuda", generator=g).to(dtype)

    def make(h):
        if layout == "blhd":
            return randn(batch, length, h, dim).permute(0, 2, 1, 3)
        if layout == "bhld":
            return randn(batch, h, length, dim)
        if layout == "misaligned":  # 2-byte shifted start and padded rows: the generic staging path
            return randn(batch, h, length, dim + 3)[..., 1:dim + 1]
        raise ValueError(layout)

    return make(heads), make(kv_heads), make(kv_heads), make(heads)


def _oracle(q, k, v, do, offsets, kv_heads=None):
    """fp64 oracle (fp32 module semantics are checked against fp64 within tolerance)."""
    heads = q.shape[1]
    group = heads // k.shape[1]
    qc, kc, vc, doc = (t.detach().cpu().double() for t in (q, k, v, do))
    if group > 1:  # the reference expands K/V per query head (left_v2.py:288-293)
        kc = kc.repeat_interleave(group, 1)
        vc = vc.repeat_interleave(group, 1)
    kc.requires_grad_()
    vc.requires_grad_()
    qc.requires_grad_()
    out = orc.exact_attention(qc, kc, vc, offsets)
    out.backward(doc)
    dk, dv = kc.grad, vc.grad
    if group > 1:
        b, _, l, d = dk.shape
        dk = dk.view(b, -1, group, l, d).sum(2)
        dv = dv.view(b, -1, group, l, d).sum(2)
    lse = orc.exact_lse(qc.detach(), kc.detach(), offsets)
    return out.detach(), qc.grad, dk, dv, lse


def _run(q, k, v, do, offsets, *, gqa=False):
    q, k, v = (t.detach().requires_grad_() for t in (q, k, v))
    if len(offsets) in (2, 4):
        fn = sbda_b200.fused_sbda_gqa_key_backward if gqa else sbda_b200.fused_sbda_key_backward
    else:
        fn = sbda_b200.sbda_attention
    out = fn(q, k, v, torch.tensor(offsets, dtype=torch.int32, device="cuda"))
    out.backward(do)
    return out, q.grad, k.grad, v.grad


def _check(batch, heads, length, dim, dtype, offsets, *, layout="blhd", kv_heads=None, seed=0):
    q, k, v, do = _inputs(batch, heads, length, dim, dtype, kv_heads=kv_heads, layout=layout, seed=seed)
    gqa = kv_heads is not None and kv_heads != heads
    out, dq, dk, dv = _run(q, k, v, do, offsets, gqa=gqa)
    ro, rdq, rdk, rdv, rlse = _oracle(q, k, v, do, offsets)
    tag = f"B{batch} H{heads} L{length} D{dim} {dtype} {offsets} {layout}"
    # GQA dK/dV sum H/kv_heads query heads, so their magnitude grows with the
    # group; the bf16 rounding of the stored result (half an ulp, 2^-9 relative)
    # is added to the 2e-2 max-abs bound for them.
    grad_rtol = 2.0 ** -8 if gqa and dtype != torch.float32 else None
    assert out.stride() == torch.empty_like(q).stride(), "output is allocated like the reference (empty_like)"
    _close(out, ro, dtype, "O " + tag)
    _close(dq, rdq, dtype, "dQ " + tag)
    _close(dk, rdk, dtype, "dK " + tag, rtol=grad_rtol)
    _close(dv, rdv, dtype, "dV " + tag, rtol=grad_rtol)
    _, lse = sbda_b200.sbda_forward(q, k, v, offsets)
    torch.testing.assert_close(lse.cpu().double(), rlse, rtol=1e-5, atol=1e-5 if dtype == torch.float32 else 1e-4)


@pytest.fixture(autouse=True, scope="module")
def _clean_fault_word():
    sbda_b200.device_status(reset=True)
    yield
    assert sbda_b200.device_status(reset=True) == 0, "a kernel reported a device-side fault"


def test_reference_golden_vectors(golden):
    """The kernels reproduce the reference module's own q/k/v -> O and gradients (fp32)."""
    for case in golden.cases:
        name = case["name"]
        q, k, v, do = (golden.get(name, key) for key in ("q", "k", "v", "do"))

        def blhd(t):  # the reference's memory layout: permuted [B,L,H,D]
            return t.permute(0, 2, 1, 3).contiguous().cuda().permute(0, 2, 1, 3)

        out, dq, dk, dv = _run(blhd(q), blhd(k), blhd(v), blhd(do), case["offsets"])
        for label, got in (("o", out), ("dq", dq), ("dk", dk), ("dv", dv)):
            _close(got, golden.get(name, label), torch.float32, f"{name} {label}")


@pytest.mark.parametrize("layer", list(range(1, 13)))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_every_layer_schedule(layer, dtype, kernel_path):
    offsets = sbda_b200.topology_offsets(layer, topology="sbda")
    _check(2, 2, 1000, 64, dtype, offsets, seed=layer)


@pytest.mark.parametrize("length", [1, 2, 3, 7, 63, 64, 65, 129, 4099, 20000])
def test_ragged_lengths(length, kernel_path):
    for layer in (1, 3, 8, 13):
        _check(1, 3, length, 64, torch.bfloat16, sbda_b200.topology_offsets(layer, topology="sbda"), seed=length + layer)


@pytest.mark.parametrize("dim", [8, 16, 24, 40, 64, 96, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_head_dims_and_dtypes(dim, dtype, kernel_path):
    for layer in (3, 9):
        _check(1, 2, 300, dim, dtype, sbda_b200.topology_offsets(layer, topology="sbda"), seed=dim)


@pytest.mark.parametrize("layout", ["bhld", "blhd", "misaligned"])
def test_layouts(layout, kernel_path):
    for layer in (2, 7, 10):
        _check(2, 2, 700, 64, torch.bfloat16, sbda_b200.topology_offsets(layer, topology="sbda"), layout=layout)
    _check(1, 2, 200, 6, torch.float32, (0, 1, 2, 16), layout="bhld")  # 12-byte rows: generic path


def test_gqa_reference_protocol():
    """tests/test_model.py:44-68 of the reference: H=4, Hkv=2, D=40, three (L, offsets)."""
    for length, offsets in ((1, (0, 1)), (7, (0, 1, 2, 1024)), (129, (0, 1, 2, 4))):
        _check(1, 4, length, 40, torch.bfloat16, offsets, kv_heads=2, layout="bhld", seed=42)


@pytest.mark.parametrize("kv_heads", [1, 2, 4])
def test_gqa_groups(kv_heads):
    for layer in (4, 11):
        _check(2, 8, 500, 64, torch.bfloat16, sbda_b200.topology_offsets(layer, topology="sbda"), kv_heads=kv_heads)
        _check(1, 8, 257, 32, torch.float32, sbda_b200.topology_offsets(layer, topology="sbda"), kv_heads=kv_heads)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_gqa_windowed_every_walk_mode(dtype):
    """Grouped-query attention on the windowed kernels (forward from kv head h / G; backward with
    fp32 per-query-head dK/dV partials and a fixed-order group sum), on every walk mode of the
    backward and groups of 2, 4 and 8, against the fp64 oracle."""
    for layer in (1, 2, 3, 6, 7, 9, 12):
        offsets = sbda_b200.topology_offsets(layer, topology="sbda")
        for heads, kv_heads in ((4, 2), (8, 2), (8, 1)):
            _check(1, heads, 3000, 64, dtype, offsets, kv_heads=kv_heads, seed=layer * 7 + heads)


def test_gqa_windowed_deterministic_and_matches_general_family():
    q, k, v, do = _inputs(2, 8, 5000, 64, torch.bfloat16, kv_heads=2, seed=21)
    offsets = sbda_b200.topology_offsets(10, topology="sbda")
    first = _run(q, k, v, do, offsets, gqa=True)
    second = _run(q, k, v, do, offsets, gqa=True)
    for a, b in zip(first, second):
        assert torch.equal(a, b)
    with sbda_b200.kernel_family("general"):
        general = _run(q, k, v, do, offsets, gqa=True)
    for a, b in zip(first, general):
        torch.testing.assert_close(a.float(), b.float(), rtol=2.0 ** -7, atol=2e-2)


def test_other_offset_sets(kernel_path):
    for offsets in ((0,), (0, 3), (0, 1, 2), (0, 1, 2, 3), (0, 5, 64), (0, 2, 100), (0, 1, 64, 200),
                    (4, 0), (0, 1, 2, 65), (2, 0, 1, 128), (0, 1, 2, 32), (0, 1, 2, 63), (0, 1, 2, 399),
                    (0, 1, 2, 400), (0, 1, 2, 5000)):
        _check(1, 2, 400, 32, torch.float32, offsets)


@pytest.mark.parametrize("layer", [1, 2, 3, 6, 7, 8, 12, 15])
def test_chain_walk_segments(layer, kernel_path):
    """Long sequences split the backward's chain walks into segments with a carry-only first tile."""
    _check(1, 4, 65536, 64, torch.bfloat16, sbda_b200.topology_offsets(layer, topology="sbda"), seed=100 + layer)


def test_kernel_families_agree():
    """The windowed and the general kernels give the same results on the same inputs."""
    q, k, v, do = _inputs(2, 4, 3000, 64, torch.bfloat16, seed=11)
    for layer in (2, 5, 7, 9, 11):
        offsets = sbda_b200.topology_offsets(layer, topology="sbda")
        with sbda_b200.kernel_family("auto"):
            auto = _run(q, k, v, do, offsets)
        with sbda_b200.kernel_family("general"):
            general = _run(q, k, v, do, offsets)
        for a, b in zip(auto, general):
            torch.testing.assert_close(a.float(), b.float(), rtol=0, atol=1.6e-2)


def test_backward_uses_the_forwards_family():
    """The autograd op records the kernel family at forward time: a backward run after the
    context has changed (or on autograd's worker thread) still uses the forward's family."""
    q, k, v, do = _inputs(1, 4, 3000, 64, torch.bfloat16, seed=12)
    offsets = sbda_b200.topology_offsets(9, topology="sbda")
    ref = {}
    for family in ("auto", "general"):
        with sbda_b200.kernel_family(family):
            ref[family] = _run(q, k, v, do, offsets)
    qs, ks, vs = (t.detach().requires_grad_() for t in (q, k, v))
    with sbda_b200.kernel_family("general"):
        out = sbda_b200.fused_sbda_key_backward(qs, ks, vs, offsets)
    out.backward(do)  # outside the context: still the general family
    for a, b in zip((out, qs.grad, ks.grad, vs.grad), ref["general"]):
        assert torch.equal(a, b)


def test_offsets_without_self_source(kernel_path):
    """Rows with no valid source give zero output and zero gradients (left_v2.py:392-393)."""
    _check(1, 2, 50, 16, torch.float32, (3, 7))


def test_deterministic(kernel_path):
    q, k, v, do = _inputs(2, 4, 5000, 64, torch.bfloat16, seed=9)
    first = _run(q, k, v, do, sbda_b200.topology_offsets(9, topology="sbda"))
    second = _run(q, k, v, do, sbda_b200.topology_offsets(9, topology="sbda"))
    for a, b in zip(first, second):
        assert torch.equal(a, b)


def test_full_size_sampled_rows(kernel_path):
    """1M positions at layer 20 (dyadic 2^19): sampled rows against the fp64 row oracle."""
    length = 1 << 20
    offsets = sbda_b200.topology_offsets(20, topology="sbda")
    q, k, v, do = _inputs(1, 4, length, 64, torch.bfloat16, seed=20)
    out, dq, dk, dv = _run(q, k, v, do, offsets)
    g = torch.Generator().manual_seed(1)
    rows = torch.cat([torch.tensor([0, 1, 2, 63, 64, (1 << 19) - 1, 1 << 19, (1 << 19) + 1, length - 1]),
                      torch.randint(0, length, (200,), generator=g)])
    qc, kc, vc, doc = (t.detach().cpu() for t in (q, k, v, do))
    ro, rdq = orc.query_rows(qc, kc, vc, doc, offsets, rows)
    rdk, rdv = orc.key_rows(qc, kc, vc, doc, offsets, rows)
    dev_rows = rows.cuda()
    _close(out[:, :, dev_rows], ro, torch.bfloat16, "O rows")
    _close(dq[:, :, dev_rows], rdq, torch.bfloat16, "dQ rows")
    _close(dk[:, :, dev_rows], rdk, torch.bfloat16, "dK rows")
    _close(dv[:, :, dev_rows], rdv, torch.bfloat16, "dV rows")
    assert torch.isfinite(out).all() and torch.isfinite(dq).all()
    assert torch.isfinite(dk).all() and torch.isfinite(dv).all()


def test_module_matches_reference_golden(golden):
    """SBDAttention (drop-in) reproduces the reference module: output, dx and parameter grads."""
    for case in golden.cases:
        name = case["name"]
        module = sbda_b200.SBDAttention(case["dim"], case["heads"], case["layer"], total_layers=12).cuda()
        state = {key[len("param."):]: golden.get(name, key) for key in
                 ("param.q.weight", "param.k.weight", "param.v.weight", "param.out.weight",
                  "param.q_norm.weight", "param.k_norm.weight")}
        module.load_state_dict(state)
        x = golden.get(name, "x").cuda().requires_grad_()
        y = module(x)
        y.backward(golden.get(name, "grad_y").cuda())
        tol = dict(rtol=2e-5, atol=2e-5)
        torch.testing.assert_close(y.detach().cpu(), golden.get(name, "y"), **tol, msg=name)
        torch.testing.assert_close(x.grad.cpu(), golden.get(name, "dx"), **tol, msg=name)
        for pname, param in module.named_parameters():
            torch.testing.assert_close(param.grad.cpu(), golden.get(name, "grad." + pname), **tol,
                                       msg=f"{name} {pname}")


def test_config2_full_parity():
    """Config 2: B 4, 8 heads x 64, L 32768, layer 10 (offsets 0, 1, 2, 512), bf16, vs the fp32 oracle."""
    q, k, v, do = _inputs(4, 8, 32768, 64, torch.bfloat16, seed=2)
    offsets = sbda_b200.topology_offsets(10, topology="sbda")
    out, dq, dk, dv = _run(q, k, v, do, offsets)
    ro, rdq, rdk, rdv = orc.exact_attention_grads(q, k, v, offsets, do)
    for name, got, ref in (("O", out, ro), ("dQ", dq, rdq), ("dK", dk, rdk), ("dV", dv, rdv)):
        _close(got, ref, torch.bfloat16, f"config 2 {name}")


def test_config3_stack_sampled_rows():
    """Config 3: B 8, 8 heads x 64, L 32768, all 15 SBDA layers, bf16.

    The kernels run on the whole batch; sampled rows of the first and last batch entries are
    checked against the fp64 row oracle (the rest of the batch shares the same code path).
    """
    g = torch.Generator().manual_seed(3)
    rows = torch.cat([torch.tensor([0, 1, 2, 3, 63, 64, 65, 16383, 16384, 32767]),
                      torch.randint(0, 32768, (60,), generator=g)])
    batches = torch.tensor([0, 7])
    dev_rows, dev_batches = rows.cuda(), batches.cuda()
    for layer in range(1, 16):
        offsets = sbda_b200.topology_offsets(layer, topology="sbda", total_layers=15)
        q, k, v, do = _inputs(8, 8, 32768, 64, torch.bfloat16, seed=300 + layer)
        out, dq, dk, dv = _run(q, k, v, do, offsets)
        qc, kc, vc, doc = (t.detach()[dev_batches].cpu() for t in (q, k, v, do))
        ro, rdq = orc.query_rows(qc, kc, vc, doc, offsets, rows)
        rdk, rdv = orc.key_rows(qc, kc, vc, doc, offsets, rows)
        for name, got, ref in (("O", out, ro), ("dQ", dq, rdq), ("dK", dk, rdk), ("dV", dv, rdv)):
            _close(got[dev_batches][:, :, dev_rows], ref, torch.bfloat16, f"config 3 layer {layer} {name}")


@pytest.mark.parametrize("length", [64, 65, 4099, 20000])
def test_local_carry_offsets(length, kernel_path):
    """Far offsets below the tile height: the local walk (small d, or d not a multiple of 4)
    and the carried local walk (d % 4 == 0 with d large enough that local staging would
    lower occupancy), with and without near offsets, across segment boundaries and ragged ends."""
    for offsets in ((0, 1, 2, 4), (0, 1, 2, 12), (0, 1, 2, 32), (0, 1, 2, 60), (0, 2, 48), (0, 8), (0, 1, 2, 6)):
        _check(1, 4, length, 64, torch.bfloat16, offsets, seed=length + offsets[-1])


@pytest.mark.parametrize("length", [1, 65, 700, 3000])
def test_several_far_offsets(length):
    """Offset sets with more than one source beyond the tile (butterfly, radix-4, mesh and h2/h6
    shapes at large strides, topology.py:102-145) and sets without a self source."""
    for offsets in ((0, 64, 128, 192), (0, 1, 300, 301), (0, 129, 259), (50, 150), (0, 3, 9, 27),
                    (64, 0, 128), (0, 256, 512, 768)):
        _check(1, 2, length, 64, torch.bfloat16, offsets, seed=length + offsets[-1])
    _check(1, 4, length, 40, torch.float32, (0, 100, 300, 301), kv_heads=2, layout="bhld", seed=length)
    _check(2, 4, length, 128, torch.float16, (0, 65, 130), kv_heads=1, seed=length + 1)


def test_path_topology_modules_match_reference_golden(path_golden):
    """BinaryPathAttention over other topologies (butterfly, radix4, mesh, h2, h8a, binary, the
    three-source h5 layer, GQA), modules with padding holes and segment resets, and modules given
    caller path tables (the reference's eager routes) reproduce the reference module: output, dx
    and parameter grads."""
    for case in path_golden.cases:
        name = case["name"]
        module = sbda_b200.BinaryPathAttention(case["dim"], case["heads"], case["layer"],
                                               kv_heads=case["kv_heads"], topology=case["topology"],
                                               total_layers=12).cuda()
        assert list(module.offsets) == case["offsets"]
        state = {key[len("param."):]: path_golden.get(name, key) for key in
                 ("param.q.weight", "param.k.weight", "param.v.weight", "param.out.weight",
                  "param.q_norm.weight", "param.k_norm.weight")}
        module.load_state_dict(state)
        x = path_golden.get(name, "x").cuda().requires_grad_()
        valid_mask = path_golden.get(name, "valid_mask").cuda().bool() if case.get("valid_mask") else None
        seam_reset = path_golden.get(name, "seam_reset").cuda().bool() if case.get("seam_reset") else None
        tables = {}
        if case.get("path_table"):
            tables = dict(path_indices=path_golden.get(name, "path_indices").cuda().long(),
                          path_valid=path_golden.get(name, "path_valid").cuda().bool())
        y = module(x, valid_mask=valid_mask, seam_reset=seam_reset, **tables)
        y.backward(path_golden.get(name, "grad_y").cuda())
        tol = dict(rtol=2e-5, atol=2e-5)
        torch.testing.assert_close(y.detach().cpu(), path_golden.get(name, "y"), **tol, msg=name)
        torch.testing.assert_close(x.grad.cpu(), path_golden.get(name, "dx"), **tol, msg=name)
        for pname, param in module.named_parameters():
            torch.testing.assert_close(param.grad.cpu(), path_golden.get(name, "grad." + pname), **tol,
                                       msg=f"{name} {pname}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_source_masks_match_oracle(dtype):
    """Per-row source masks (padding holes, segment resets) through sbda_b200_forward_masked /
    sbda_b200_backward_masked against the oracle's masked route (left_v2.py:349-396)."""
    g = torch.Generator().manual_seed(5)
    for layer, length, kv_heads in ((3, 300, 4), (7, 700, 4), (10, 1500, 2), (2, 130, 4)):
        offsets = sbda_b200.topology_offsets(layer, topology="sbda")
        q, k, v, do = _inputs(2, 4, length, 64, dtype, kv_heads=kv_heads, seed=layer)
        valid_mask = torch.rand(2, length, generator=g) > 0.1
        valid_mask[1, length - 17:] = False
        seam_reset = torch.rand(2, length, generator=g) < 0.03
        module = sbda_b200.BinaryPathAttention(32, 2, layer, topology="sbda")
        for vm, sr in ((valid_mask, None), (None, seam_reset), (valid_mask, seam_reset)):
            bits = module.source_mask(vm.cuda() if vm is not None else None,
                                      sr.cuda() if sr is not None else None)
            qq, kk, vv = (t.detach().requires_grad_() for t in (q, k, v))
            out = sbda_b200.ops._SBDAFunction.apply(qq, kk, vv, offsets, bits)
            out.backward(do)
            usable = orc.source_usable(length, offsets, vm, sr)
            group = 4 // kv_heads
            qc, kc, vc, doc = (t.detach().cpu().double() for t in (q, k, v, do))
            kc, vc = kc.repeat_interleave(group, 1), vc.repeat_interleave(group, 1)
            qc, kc, vc = (t.requires_grad_() for t in (qc, kc, vc))
            ref = orc.exact_attention(qc, kc, vc, offsets, usable=usable)
            ref.backward(doc)
            rdk = kc.grad.view(2, kv_heads, group, length, 64).sum(2)
            rdv = vc.grad.view(2, kv_heads, group, length, 64).sum(2)
            rows = usable.any(-1)  # rows with a usable source (others: zero output in both)
            tag = f"layer {layer} {dtype} holes={vm is not None} seams={sr is not None}"
            _close(out, ref.detach(), dtype, "O " + tag)
            _close(qq.grad, qc.grad, dtype, "dQ " + tag)
            _close(kk.grad, rdk, dtype, "dK " + tag, rtol=2.0 ** -8 if dtype != torch.float32 else None)
            _close(vv.grad, rdv, dtype, "dV " + tag, rtol=2.0 ** -8 if dtype != torch.float32 else None)
            assert bool(rows.any())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_path_tables_match_oracle(dtype):
    """Caller path tables through sbda_b200_{forward,backward}_paths against the oracle's
    gather route (left_v2.py:323-396): random causal tables, path_valid, holes, seams, GQA."""
    g = torch.Generator().manual_seed(8)
    for length, sources, kv_heads in ((257, 3, 4), (1000, 4, 2), (64, 1, 4), (3000, 2, 1)):
        q, k, v, do = _inputs(2, 4, length, 64, dtype, kv_heads=kv_heads, seed=length)
        positions = torch.arange(length)
        jumps = torch.randint(0, 400, (2, length, sources), generator=g)
        indices = (positions[None, :, None] - jumps).clamp_min(0)
        indices[0, 5:, -1] = torch.randint(0, length, (length - 5,), generator=g)  # some future sources
        path_valid = torch.rand(2, length, sources, generator=g) > 0.15
        valid_mask = torch.rand(2, length, generator=g) > 0.1
        seam_reset = torch.rand(2, length, generator=g) < 0.02
        module = sbda_b200.BinaryPathAttention(32, 2, 1, topology="h4_greedy")
        bits = module.path_source_mask(indices.cuda(), path_valid.cuda(), valid_mask.cuda(), seam_reset.cuda())
        qq, kk, vv = (t.detach().requires_grad_() for t in (q, k, v))
        out = sbda_b200.ops._SBDAPathFunction.apply(qq, kk, vv, indices.cuda().to(torch.int32).contiguous(), bits)
        out.backward(do)
        usable = orc.path_usable(indices, path_valid, valid_mask, seam_reset)
        group = 4 // kv_heads
        qc, kc, vc, doc = (t.detach().cpu().double() for t in (q, k, v, do))
        kc, vc = kc.repeat_interleave(group, 1), vc.repeat_interleave(group, 1)
        qc, kc, vc = (t.requires_grad_() for t in (qc, kc, vc))
        ref = orc.exact_attention(qc, kc, vc, (), usable=usable, indices=indices)
        ref.backward(doc)
        rdk = kc.grad.view(2, kv_heads, group, length, 64).sum(2)
        rdv = vc.grad.view(2, kv_heads, group, length, 64).sum(2)
        tag = f"L {length} S {sources} kv {kv_heads} {dtype}"
        grad_rtol = 2.0 ** -8 if dtype != torch.float32 else None
        _close(out, ref.detach(), dtype, "O " + tag)
        _close(qq.grad, qc.grad, dtype, "dQ " + tag)
        _close(kk.grad, rdk, dtype, "dK " + tag, rtol=grad_rtol)
        _close(vv.grad, rdv, dtype, "dV " + tag, rtol=grad_rtol)
