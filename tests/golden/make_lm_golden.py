"""Golden vectors for whole ``BiAttnLM`` steps, produced by the reference's own model on the CPU.

Run from the repository root with the reference checkout available::

    python tests/golden/make_lm_golden.py --reference <path to the reference checkout>

For each case it builds the reference's ``BiAttnLM(BiAttnConfig(...))`` (``BiAttn/model.py``) with
seeded weights (the model's own ``_init_weights``: N(0, 0.02)), runs one forward + backward step
on seeded token ids and records the parameters (state dict), the ids, the logits, the loss and
the gradient of every parameter.  On the CPU the reference's attention takes its exact eager
path.  Cases:

* ``cfg1``: the config-1 smoke shape -- 96-symbol vocabulary, d_model 16, 3 SBDA layers (offsets
  (0,1), (0,2), (0,1,2,4)), 2 heads x 8, FFN hidden 32, batch 1, sequence 32; next-token
  cross-entropy over the sequence;
* ``triangle``: the reference test's prefix-triangle batch (``tests/test_model.py:72-79``) through
  ``triangle_loss``, 2 SBDA layers, 4 heads;
* ``left_v2_binary``: the ``left_v2`` backend (binary paths), 5 layers, batch 2 x 40.

Output: ``tests/golden/lm_golden.npz`` (float32).  The GPU tests only read the ``.npz``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

CASES = [
    # name, config kwargs, batch, length, loss kind, seed
    ("cfg1", dict(vocab_size=96, dim=16, layers=3, heads=2, ff_hidden=32, attention_backend="sbda"), 1, 32, "next",
     1),
    ("triangle", dict(vocab_size=32, dim=32, layers=2, heads=4, attention_backend="sbda"), 3, 4, "triangle", 2),
    ("left_v2_binary", dict(vocab_size=32, dim=32, layers=5, heads=4, attention_backend="left_v2"), 2, 40, "next",
     3),
]


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True)
    parser.add_argument("--out", default=os.path.join(os.path.dirname(__file__), "lm_golden.npz"))
    args = parser.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from BiAttn.model import BiAttnConfig, BiAttnLM  # noqa: E402  (reference code)

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    arrays: dict[str, np.ndarray] = {}
    manifest = []
    for name, kwargs, batch, length, loss_kind, seed in CASES:
        torch.manual_seed(seed)
        model = BiAttnLM(BiAttnConfig(**kwargs))
        gen = torch.Generator().manual_seed(100 + seed)
        if loss_kind == "triangle":
            ids = torch.tensor([[1, 0, 0, 0], [1, 2, 0, 0], [1, 2, 3, 0]])
            valid = torch.tensor([[1, 0, 0, 0], [1, 1, 0, 0], [1, 1, 1, 0]], dtype=torch.bool)
            targets = torch.tensor([2, 3, 4])
            logits = model.next_logits(ids, valid)
            loss = model.triangle_loss(ids, valid, targets)
            arrays[f"{name}/valid"] = valid.numpy()
            arrays[f"{name}/targets"] = targets.numpy()
        else:
            ids = torch.randint(0, kwargs["vocab_size"], (batch, length), generator=gen)
            logits = model(ids)
            loss = F.cross_entropy(logits[:, :-1].reshape(-1, kwargs["vocab_size"]), ids[:, 1:].reshape(-1))
        loss.backward()
        arrays[f"{name}/ids"] = ids.numpy()
        arrays[f"{name}/logits"] = logits.detach().numpy()
        arrays[f"{name}/loss"] = loss.detach().numpy()
        params = []
        for pname, tensor in model.state_dict().items():
            arrays[f"{name}/param.{pname}"] = tensor.detach().numpy()
        for pname, param in model.named_parameters():
            arrays[f"{name}/grad.{pname}"] = param.grad.detach().numpy()
            params.append(pname)
        manifest.append({"name": name, "config": kwargs, "loss": loss_kind, "params": params,
                         "state": list(model.state_dict().keys())})
        print(name, float(loss))
    arrays["manifest"] = np.frombuffer(json.dumps({"cases": manifest}).encode(), dtype=np.uint8)
    np.savez_compressed(args.out, **arrays)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
