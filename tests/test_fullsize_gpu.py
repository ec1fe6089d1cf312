"""Parity at the benchmark sizes themselves.

1. Config 4, the metric: every one of the 20 SBDA layers at 1,048,576 positions x 4 heads x 64,
   bf16, on the kernels the benchmark runs (automatic family: the windowed kernels).  The walk
   mode and the segment split of the backward change with the layer (local, local-carry and
   chain walks; per-layer segment counts), so each layer is checked on its own rows: the first
   and last rows, tile and chain boundaries of its far offset, and random rows, against the fp64
   row oracle (the restatement of ``BiAttn/left_v2.py:335-405``), within the bf16 bound of
   2e-2 max-abs.
2. Config 5: 4,194,304 positions, layers 19-22 (far offsets 2^18 .. 2^21, the last two longer
   than a shard at 8 ranks), emulated 2-, 4- and 8-rank sequence shards on one GPU must equal the
   unsharded call bit for bit.
"""

from __future__ import annotations

import pytest
import torch

from oracle import sbda_oracle as orc

import sbda_b200
from test_ops_gpu import _close, _inputs, _run
from test_sharded_gpu import _emulated, _whole

pytestmark = pytest.mark.gpu


def _layer_rows(length: int, d: int, seed: int, n_random: int = 200) -> torch.Tensor:
    """Rows to check for a layer with far offset ``d``: edges, tile and chain boundaries, random."""
    fixed = {0, 1, 2, 3, 31, 32, 63, 64, 65, 127, 128, length - 1, length - 2, length - 3, length - 64,
             length - 65, length // 2 - 1, length // 2}
    for base in (d, 2 * d, length - d):
        for delta in (-65, -64, -2, -1, 0, 1, 2, 63, 64):
            fixed.add(base + delta)
    g = torch.Generator().manual_seed(seed)
    rows = torch.tensor(sorted(r for r in fixed if 0 <= r < length))
    return torch.cat([rows, torch.randint(0, length, (n_random,), generator=g)])


def test_metric_every_layer_full_size():
    length, heads, layers = 1 << 20, 4, 20
    q, k, v, do = _inputs(1, heads, length, 64, torch.bfloat16, seed=2024)
    # fp64 host copies once: the row oracle then gathers rows without converting whole tensors.
    qc, kc, vc, doc = (t.detach().cpu().double() for t in (q, k, v, do))
    for layer, offsets in enumerate(sbda_b200.sbda_layer_offsets(layers), start=1):
        with sbda_b200.kernel_family("auto"):
            out, dq, dk, dv = _run(q, k, v, do, offsets)
        rows = _layer_rows(length, max(offsets), seed=layer)
        ro, rdq = orc.query_rows(qc, kc, vc, doc, offsets, rows)
        rdk, rdv = orc.key_rows(qc, kc, vc, doc, offsets, rows)
        dev_rows = rows.cuda()
        tag = f"layer {layer} {offsets}"
        _close(out[:, :, dev_rows], ro, torch.bfloat16, "O " + tag)
        _close(dq[:, :, dev_rows], rdq, torch.bfloat16, "dQ " + tag)
        _close(dk[:, :, dev_rows], rdk, torch.bfloat16, "dK " + tag)
        _close(dv[:, :, dev_rows], rdv, torch.bfloat16, "dV " + tag)
        for name, t in (("O", out), ("dQ", dq), ("dK", dk), ("dV", dv)):
            assert torch.isfinite(t).all(), f"{name} {tag} has non-finite values"
        del out, dq, dk, dv
    assert sbda_b200.device_status(reset=True) == 0


def test_config5_emulated_shards_at_full_size():
    total = 1 << 22
    g = torch.Generator(device="cuda").manual_seed(5)

    def make():
        return torch.randn(1, total, 4, 64, device="cuda", generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)

    q, k, v, do = make(), make(), make(), make()
    offsets_by_layer = sbda_b200.sbda_layer_offsets(22)
    for layer in (19, 20, 21, 22):
        offsets = offsets_by_layer[layer - 1]
        ref = _whole(q, k, v, do, offsets, 0)
        for world in (2, 4, 8):
            with sbda_b200.kernel_family("auto"):
                got = _emulated(q, k, v, do, offsets, world)
            for name, a, b in zip(("O", "dQ", "dK", "dV"), got, ref):
                assert torch.equal(a, b), f"layer {layer} world {world}: {name} differs"
            del got
        del ref
    assert sbda_b200.device_status(reset=True) == 0
