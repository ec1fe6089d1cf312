"""The dense-causal LM evaluation of the oracle against whole-LM steps the reference ran itself
(``tests/golden/make_lm_golden.py``): logits, loss and every parameter gradient."""

from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle import sbda_oracle as orc


def lm_step(golden, case, device="cpu", model=None):
    """One step of the golden case: the oracle's dense LM (``model=None``) or ``model``.
    Returns ``(logits, loss, grads by parameter name)``."""
    name, cfg = case["name"], case["config"]
    ids = golden.get(name, "ids").to(device)
    valid = golden.get(name, "valid").to(device) if case["loss"] == "triangle" else None
    if model is None:
        params = {key: golden.get(name, "param." + key).to(device).requires_grad_()
                  for key in case["state"]}
        if cfg.get("tie_embeddings", True):
            params["lm_head.weight"] = params["embedding.weight"]
        logits_all = orc.lm_forward_dense(ids, params, cfg, valid)
        named = {key: params[key] for key in case["params"]}
    else:
        logits_all = model(ids, valid) if valid is not None else model(ids)
        named = dict(model.named_parameters())
    if case["loss"] == "triangle":
        rows = torch.arange(ids.shape[0], device=device)
        logits = logits_all[rows, valid.sum(dim=1) - 1]
        loss = F.cross_entropy(logits, golden.get(name, "targets").to(device))
    else:
        logits = logits_all
        loss = F.cross_entropy(logits[:, :-1].reshape(-1, cfg["vocab_size"]), ids[:, 1:].reshape(-1))
    loss.backward()
    return logits.detach(), loss.detach(), {key: named[key].grad for key in case["params"]}


def test_dense_oracle_lm_matches_reference_steps(lm_golden):
    for case in lm_golden.cases:
        name = case["name"]
        logits, loss, grads = lm_step(lm_golden, case)
        tol = dict(rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(logits, lm_golden.get(name, "logits"), **tol, msg=name)
        torch.testing.assert_close(loss, lm_golden.get(name, "loss"), **tol, msg=name)
        for key, grad in grads.items():
            torch.testing.assert_close(grad, lm_golden.get(name, "grad." + key), **tol, msg=f"{name} {key}")


def test_lm_state_dict_keys_and_shapes_match_reference(lm_golden):
    """``sbda_b200.BiAttnLM`` holds the reference model's parameters under the same names and shapes,
    so a reference checkpoint loads as is."""
    import sbda_b200

    for case in lm_golden.cases:
        model = sbda_b200.BiAttnLM(sbda_b200.BiAttnConfig(**case["config"]))
        state = model.state_dict()
        assert sorted(state) == sorted(case["state"]), case["name"]
        for key in case["state"]:
            assert tuple(state[key].shape) == tuple(lm_golden.get(case["name"], "param." + key).shape), key
        assert [name for name, _ in model.named_parameters()] == case["params"], case["name"]
