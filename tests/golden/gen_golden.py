"""Generates the committed golden fixtures for the MoE layer.

Run in a checkout that has the reference sources (oracle/_ref builds from
them): `python tests/golden/gen_golden.py`. Writes:

- moe_cfg0.npz: configuration 0 (32 tokens, hidden 256, 16 experts, top-4,
  intermediate 128, group 64) run through the reference's own moe_forward
  (c/src/model.c:1281-1405, compiled unmodified into oracle/_ref): the
  output, the routing as sorted sets, the renormalised weights in that sorted
  order, plus SHA-256 digests of every synthetic input tensor so the input
  generator is pinned too.
- moe_cfg1_tokens.npz: configuration-1 shapes (hidden 2048, 512 experts,
  top-10, intermediate 512) for 4 decode tokens, same content.
- moe_cfg2_route.npz: configuration-2 routing (Zipf(1.1) logit bias) for 64
  tokens: sorted top-10 sets and per-expert counts, from the restatement's
  router (identical arithmetic to the reference harness's router).
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "qwen3.8-flash-next_b200"))

import oracle  # noqa: E402
import qmoe  # noqa: E402

SEED = 20261201


def digests(s: "qmoe.SynthLayer") -> dict:
    out = {"router": hashlib.sha256(s.router.tobytes()).hexdigest(),
           "shared_gate": hashlib.sha256(s.shared_gate.tobytes()).hexdigest()}
    for name, arrs in sorted(s.t.items()):
        h = hashlib.sha256()
        for a in arrs:
            h.update(a.tobytes())
        out[name] = h.hexdigest()
    if s.logit_bias is not None:
        out["logit_bias"] = hashlib.sha256(s.logit_bias.tobytes()).hexdigest()
    return out


def sorted_routing(idx, w):
    order = np.argsort(idx, axis=1, kind="stable")
    return np.take_along_axis(idx, order, 1), np.take_along_axis(w, order, 1)


def case(name, d, E, k, I, n, stream, zipf=None):
    cfg = qmoe.make_config(d, E, k, I, max_tokens=n)
    s = qmoe.SynthLayer(cfg, SEED, 0, zipf_s=zipf)
    x = qmoe.synth_tokens(SEED, stream, n, d)
    ref = oracle.reference()
    out, idx, w = ref.forward(s, x)
    si, sw = sorted_routing(idx, w)
    dg = digests(s)
    np.savez_compressed(os.path.join(HERE, name), out=out, idx_sorted=si, w_sorted=sw,
                        x_sha=hashlib.sha256(x.tobytes()).hexdigest(),
                        **{f"sha_{k_}": v for k_, v in dg.items()},
                        shape=np.array([d, E, k, I, 64, n, stream]), seed=SEED)
    ref.lib.ref_reset_cache()


def route_case(name, d, E, k, I, n, stream, zipf, weights=True):
    cfg = qmoe.make_config(d, E, k, I, max_tokens=n)
    s = qmoe.SynthLayer(cfg, SEED, 0, zipf_s=zipf)
    x = qmoe.synth_tokens(SEED, stream, n, d)
    idx, w, lg = oracle.restatement().route(s, x)
    si, sw = sorted_routing(idx, w)
    counts = np.bincount(idx.ravel(), minlength=E).astype(np.int32)
    extra = {"w_sorted": sw} if weights else {}
    np.savez_compressed(os.path.join(HERE, name), idx_sorted=si.astype(np.int16), counts=counts,
                        x_sha=hashlib.sha256(x.tobytes()).hexdigest(),
                        shape=np.array([d, E, k, I, 64, n, stream]), seed=SEED, **extra)


if __name__ == "__main__":
    oracle.build()
    if oracle.reference() is None:
        sys.exit("oracle/_ref is not built: the reference sources are needed")
    case("moe_cfg0.npz", 256, 16, 4, 128, 32, 0)
    case("moe_cfg1_tokens.npz", 2048, 512, 10, 512, 4, 1)
    route_case("moe_cfg2_route.npz", 2048, 512, 10, 512, 64, 2, 1.1)
    # every token of configuration 2 (4096 tokens): sets and counts
    route_case("moe_cfg2_full_route.npz", 2048, 512, 10, 512, 4096, 3, 1.1, weights=False)
    print("golden fixtures written to", HERE)
