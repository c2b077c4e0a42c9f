"""Golden vectors of the reference's route predictor (ExpertStore.record_route /
prefetch_predictions / snapshot()["frequent_experts"], streaming.py:400-453),
made by running the reference's own ExpertStore.

    python tests/golden/make_predictor_golden.py <reference checkout> tests/golden/predictor.json

Only ExpertStore's bookkeeping runs: mlx (absent here) and the native row
reader are replaced by empty stub modules, the package's __init__ (which loads
the MLX model) is skipped,
the safetensors index is a stand-in exposing the expert tensor metadata the
constructor validates, and request() is replaced by a recorder of the
(layer, expert) prefetch requests. Every input is seeded."""
import importlib
import json
import os
import sys
import types
from types import SimpleNamespace

import numpy as np


def load_reference(root):
    for name in ("mlx", "mlx.core", "mlx.nn"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["mlx"].core = sys.modules["mlx.core"]
    sys.modules["mlx"].nn = sys.modules["mlx.nn"]
    pkg = types.ModuleType("colibri_runtime")
    pkg.__path__ = [os.path.join(root, "src", "colibri_runtime")]
    sys.modules["colibri_runtime"] = pkg
    # the native row reader is not built here, and no rows are read
    sys.modules["colibri_runtime._rowio"] = types.ModuleType("colibri_runtime._rowio")
    return importlib.import_module("colibri_runtime.streaming")


def make_store(streaming, L, E, depth):
    tensors = {}
    for layer in range(L):
        for proj in ("gate", "up", "down"):
            tensors[f"model.layers.{layer}.mlp.switch_mlp.{proj}_proj.weight"] = \
                SimpleNamespace(shape=(E, 4, 4), row_bytes=64)
    index = SimpleNamespace(tensors=tensors, executor=SimpleNamespace(_max_workers=2))
    store = streaming.ExpertStore(index, budget_bytes=64 * 3 * E * L, num_layers=L, num_experts=E,
                                  prefetch=depth)
    calls = []
    store.request = lambda layer, expert, prefetch=False: calls.append([int(layer), int(expert)])
    return store, calls


def routed_step(rng, E, k, tokens, skew):
    """tokens x k distinct experts per token, drawn with a Zipf-like skew over a
    random permutation (many equal counts, so ties are exercised)."""
    p = 1.0 / np.arange(1, E + 1) ** skew
    p /= p.sum()
    perm = rng.permutation(E)
    out = []
    for _ in range(tokens):
        out.extend(int(perm[i]) for i in rng.choice(E, size=k, replace=False, p=p))
    return out


def main():
    ref, dst = sys.argv[1], sys.argv[2]
    streaming = load_reference(ref)
    cases = []
    for ci, (L, E, k, depth, steps, skew, max_tok) in enumerate(
            [(3, 8, 2, 2, 24, 0.0, 3), (4, 16, 4, 2, 40, 1.1, 4), (2, 32, 4, 3, 30, 0.6, 8),
             (5, 64, 8, 2, 50, 1.1, 2), (3, 12, 3, 0, 10, 0.5, 2), (1, 16, 2, 4, 12, 1.0, 3),
             # the workload's shape: 512 experts, top-10, Zipf(1.1); max_tok -1 = one token a step
             (4, 512, 10, 2, 160, 1.1, -1), (2, 512, 10, 2, 12, 1.1, 48)]):
        rng = np.random.default_rng(20261206 + ci)
        store, calls = make_store(streaming, L, E, depth)
        rec = []
        for s in range(steps):
            layer = s % L
            ntok = 1 if max_tok < 0 else int(rng.integers(0, max_tok + 1))
            routed = routed_step(rng, E, k, ntok, skew)
            selected = sorted(set(routed))
            store.record_route(layer, routed)
            del calls[:]
            store.prefetch_predictions(layer, selected)
            rec.append({"layer": layer, "routed": routed, "selected": selected,
                        "requests": [list(c) for c in calls]})
        snap = store.snapshot()
        cases.append({"num_layers": L, "num_experts": E, "depth": depth, "steps": rec,
                      "routes": snap["routes"],
                      "frequent": [[f["layer"], f["expert"], f["count"]] for f in snap["frequent_experts"]],
                      "counts": [[int(store._freq[l][e]) for e in range(E)] for l in range(L)]})
    with open(dst, "w") as f:
        json.dump({"source": "streaming.py ExpertStore (record_route, prefetch_predictions, snapshot)",
                   "cases": cases}, f, separators=(",", ":"))


if __name__ == "__main__":
    main()
