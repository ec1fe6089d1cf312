"""The CPU oracle against vectors produced by the reference's own code (CPU)."""

from __future__ import annotations

import pytest
import torch

from oracle import sbda_oracle as orc

import sbda_b200


def test_schedules_match_reference(golden):
    for topology, layers in golden.schedules.items():
        for layer, expected in enumerate(layers, start=1):
            assert list(orc.schedule_offsets(layer, topology, golden.total_layers)) == expected, (topology, layer)
            got = sbda_b200.topology_offsets(layer, topology=topology, total_layers=golden.total_layers)
            assert list(got) == expected, (topology, layer)


def test_schedule_known_answers():
    # BiAttn/topology.py:141-142 and tests/test_model.py:110-134 of the reference.
    assert orc.schedule_offsets(1) == (0, 1)
    assert orc.schedule_offsets(2) == (0, 2)
    assert orc.schedule_offsets(3) == (0, 1, 2, 4)
    assert orc.schedule_offsets(10) == (0, 1, 2, 512)
    assert orc.schedule_offsets(20) == (0, 1, 2, 524288)
    assert orc.schedule_offsets(22) == (0, 1, 2, 2097152)
    for layer in range(1, 7):
        offsets = sbda_b200.topology_offsets(layer, topology="sbda", total_layers=6)
        assert offsets[0] == 0 and all(o >= 0 for o in offsets)
        assert len(offsets) == (2 if layer <= 2 else 4)
    assert [sbda_b200.sbda_stage(layer) for layer in (1, 2, 3)] == ["binary", "binary", "local_diffusion"]
    with pytest.raises(ValueError):
        sbda_b200.topology_offsets(0)


def _case_tensors(golden, case):
    return {key: golden.get(case["name"], key) for key in ("q", "k", "v", "o", "do", "dq", "dk", "dv")}


def test_oracle_forward_matches_reference(golden):
    for case in golden.cases:
        t = _case_tensors(golden, case)
        for use_sdpa in (True, False):
            out = orc.exact_attention(t["q"], t["k"], t["v"], case["offsets"], use_sdpa=use_sdpa)
            torch.testing.assert_close(out, t["o"], rtol=1e-5, atol=1e-6, msg=case["name"])


def test_oracle_gradients_match_reference(golden):
    for case in golden.cases:
        t = _case_tensors(golden, case)
        out, dq, dk, dv = orc.exact_attention_grads(t["q"], t["k"], t["v"], case["offsets"], t["do"])
        torch.testing.assert_close(out, t["o"], rtol=1e-5, atol=1e-6)
        for name, got in (("dq", dq), ("dk", dk), ("dv", dv)):
            torch.testing.assert_close(got, t[name], rtol=1e-5, atol=1e-6, msg=f"{case['name']} {name}")


def test_oracle_norm_rope_and_module_match_reference(golden):
    for case in golden.cases:
        name, heads = case["name"], case["heads"]
        params = {key: golden.get(name, "param." + key) for key in
                  ("q.weight", "k.weight", "v.weight", "out.weight", "q_norm.weight", "k_norm.weight")}
        x = golden.get(name, "x")
        batch, length, dim = x.shape
        hd = dim // heads
        q_raw = torch.nn.functional.linear(x, params["q.weight"]).view(batch, length, heads, hd)
        k_raw = torch.nn.functional.linear(x, params["k.weight"]).view(batch, length, heads, hd)
        q, k = orc.norm_rope(q_raw, k_raw, params["q_norm.weight"], params["k_norm.weight"])
        torch.testing.assert_close(q.permute(0, 2, 1, 3), golden.get(name, "q"), rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(k.permute(0, 2, 1, 3), golden.get(name, "k"), rtol=1e-5, atol=1e-6)
        y = orc.module_forward(x, params, heads=heads, layer=case["layer"])
        torch.testing.assert_close(y, golden.get(name, "y"), rtol=1e-5, atol=1e-6)


def test_oracle_lse_normalises_the_softmax(golden):
    case = golden.cases[-1]
    t = _case_tensors(golden, case)
    lse = orc.exact_lse(t["q"], t["k"], case["offsets"])
    idx, valid = orc.path_tensors(t["q"].shape[2], case["offsets"])
    hd = t["q"].shape[-1]
    keys = t["k"].double()[:, :, idx]  # [B,H,L,S,D]
    scores = (t["q"].double().unsqueeze(3) * keys).sum(-1) * hd ** -0.5
    weights = torch.exp(scores - lse.unsqueeze(-1)).masked_fill(~valid, 0.0)
    torch.testing.assert_close(weights.sum(-1), torch.ones_like(lse), rtol=0, atol=1e-12)


def test_oracle_is_causal():
    # Changing future positions never changes earlier outputs (tests/test_model.py:19-32).
    torch.manual_seed(3)
    q, k, v = (torch.randn(1, 2, 40, 8) for _ in range(3))
    offsets = orc.schedule_offsets(5)
    base = orc.exact_attention(q, k, v, offsets)
    k2, v2 = k.clone(), v.clone()
    k2[:, :, 25:] += 10
    v2[:, :, 25:] -= 7
    torch.testing.assert_close(orc.exact_attention(q, k2, v2, offsets)[:, :, :25], base[:, :, :25])


def test_sampled_row_oracle_agrees_with_full_oracle():
    torch.manual_seed(5)
    q, k, v, do = (torch.randn(2, 2, 300, 16) for _ in range(4))
    offsets = orc.schedule_offsets(8)
    out, dq, dk, dv = orc.exact_attention_grads(q, k, v, offsets, do, dtype=torch.float64)
    rows = torch.tensor([0, 1, 2, 127, 128, 129, 255, 299])
    o_rows, dq_rows = orc.query_rows(q, k, v, do, offsets, rows)
    dk_rows, dv_rows = orc.key_rows(q, k, v, do, offsets, rows)
    torch.testing.assert_close(o_rows, out[:, :, rows])
    torch.testing.assert_close(dq_rows, dq[:, :, rows])
    torch.testing.assert_close(dk_rows, dk[:, :, rows])
    torch.testing.assert_close(dv_rows, dv[:, :, rows])


def test_every_topology_matches_reference_table():
    """All 31 path topologies against the reference's own schedules (tests/golden/topology_table.json,
    written by tests/golden/make_topology_table.py from BiAttn/topology.py)."""
    import json
    import os

    with open(os.path.join(os.path.dirname(__file__), "golden", "topology_table.json")) as handle:
        table = json.load(handle)
    assert tuple(table["topologies"]) == sbda_b200.PATH_TOPOLOGIES
    checked = 0
    for name, by_total in table["offsets"].items():
        for total, rows in by_total.items():
            for layer, expected in zip(table["layers"], rows):
                if expected is None:  # more than 64 offsets (h3 at large layers)
                    continue
                got = sbda_b200.topology_offsets(layer, topology=name, total_layers=int(total))
                assert list(got) == expected, (name, total, layer)
                checked += 1
    assert checked > 1900  # 31 topologies x 22 layers x 3 stack depths, less the capped h3 rows


def test_topology_default_is_the_references():
    """With no ``topology=`` the drop-in returns the reference's default schedule, ``binary``
    (``BiAttn/topology.py:24-28``), for every layer and stack depth the reference table holds."""
    import json
    import os

    with open(os.path.join(os.path.dirname(__file__), "golden", "topology_table.json")) as handle:
        table = json.load(handle)
    assert sbda_b200.topology_offsets(5) == (0, 16)
    assert sbda_b200.topology_offsets(1) == (0, 1)
    for total, rows in table["offsets"]["binary"].items():
        for layer, expected in zip(table["layers"], rows):
            assert list(sbda_b200.topology_offsets(layer, total_layers=int(total))) == expected, (total, layer)
            if int(total) == 12:
                assert list(sbda_b200.topology_offsets(layer)) == expected, layer


def test_path_golden_offsets_match_topologies(path_golden):
    for case in path_golden.cases:
        assert list(sbda_b200.topology_offsets(case["layer"], topology=case["topology"], total_layers=12)) \
            == case["offsets"], case["name"]
