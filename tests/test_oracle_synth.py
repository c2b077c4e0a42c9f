"""The checkers' own restatement of the seeded workload generator
(oracle/synth_oracle.c): the CPU baselines and the benchmark's reference arm
build their layers and tokens with it, so that they need nothing from the
product library. Pinned to the SHA-256 digests of every input tensor that the
reference's own moe_forward consumed when it wrote the golden fixtures, and
checked bit for bit against the product library's generator."""
import hashlib
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _digest(arrs):
    h = hashlib.sha256()
    for a in arrs:
        h.update(a.tobytes())
    return h.hexdigest()


@pytest.mark.parametrize("name", ["moe_cfg0.npz", "moe_cfg1_tokens.npz"])
def test_checker_generator_matches_golden_digests(built, name):
    import oracle
    g = np.load(os.path.join(GOLD, name))
    d, E, k, I, gs, n, stream = (int(v) for v in g["shape"])
    seed = int(g["seed"])
    s = oracle.SynthLayer(d, E, k, I, gs, seed)
    x = oracle.synth_tokens(seed, stream, n, d)
    assert hashlib.sha256(x.tobytes()).hexdigest() == str(g["x_sha"])
    assert _digest([s.router]) == str(g["sha_router"])
    assert _digest([s.shared_gate]) == str(g["sha_shared_gate"])
    for t in ("gate", "up", "down", "sh_gate", "sh_up", "sh_down"):
        assert _digest(s.t[t]) == str(g[f"sha_{t}"]), t


def test_checker_generator_reproduces_reference_golden_output(built):
    """configs[0] end to end from checker code only: the reference's output
    recorded in the fixture is reproduced by the restatement on inputs the
    checkers generated themselves."""
    import oracle
    g = np.load(os.path.join(GOLD, "moe_cfg0.npz"))
    d, E, k, I, gs, n, stream = (int(v) for v in g["shape"])
    seed = int(g["seed"])
    s = oracle.SynthLayer(d, E, k, I, gs, seed)
    x = oracle.synth_tokens(seed, stream, n, d)
    out, idx, _ = oracle.restatement().forward(s, x)
    assert np.array_equal(np.sort(idx, 1), g["idx_sorted"])
    assert np.linalg.norm(out - g["out"]) / np.linalg.norm(g["out"]) < 1e-5


@pytest.mark.parametrize("shape,layer,zipf,experts", [
    ((256, 16, 4, 128, 64), 0, None, None),
    ((256, 16, 4, 128, 32), 3, 1.1, None),
    ((512, 64, 6, 256, 64), 7, 1.1, (5, 17)),    # an expert slice
    ((2048, 512, 10, 512, 64), 75, 1.1, (500, 512)),
])
def test_checker_generator_equals_library_generator(built, shape, layer, zipf, experts):
    import oracle
    import qmoe
    d, E, k, I, g = shape
    a = oracle.SynthLayer(d, E, k, I, g, 4242, layer, zipf_s=zipf, experts=experts)
    cfg = qmoe.make_config(d, E, k, I, g, max_tokens=1)
    b = qmoe.SynthLayer(cfg, 4242, layer, zipf_s=zipf)
    assert np.array_equal(a.router, b.router)
    assert np.array_equal(a.shared_gate, b.shared_gate)
    if zipf is not None:
        assert np.array_equal(a.logit_bias, b.logit_bias)
    for name in a.t:
        for u, v in zip(a.t[name], b.t[name]):
            if experts is not None and not name.startswith("sh_"):
                per = u.size // E
                lo, hi = experts[0] * per, experts[1] * per
                assert np.array_equal(u[lo:hi], v[lo:hi]), name
                assert not u[:lo].any() and not u[hi:].any(), name
            else:
                assert np.array_equal(u, v), name
    assert np.array_equal(oracle.synth_tokens(4242, 9, 5, d), qmoe.synth_tokens(4242, 9, 5, d))


def test_checker_rmsnorm_matches_reference_kernel(built):
    import oracle
    x = oracle.synth_tokens(7, 1, 6, 2048) * np.float32(3.0)
    y = oracle.rmsnorm(x, 1e-6)
    r = 1.0 / np.sqrt((x.astype(np.float64) ** 2).mean(1) + 1e-6)
    np.testing.assert_allclose(y, x * r[:, None], rtol=2e-6, atol=0)


@pytest.mark.parametrize("q4,biases", [(True, True), (True, False), (False, True)])
def test_checker_hc_weights_equal_library_hc_weights(built, q4, biases):
    """The bench's hyper-connection leg builds its GPU weights with
    qmoe.SynthHC and its CPU baseline with oracle.SynthHC: both are the same
    bytes for the same seed."""
    import oracle
    import qmoe
    a = oracle.SynthHC(256, 4, 64, 20261213, q4=q4, biases=biases)
    b = qmoe.SynthHC(256, 4, 64, 20261213, q4=q4, biases=biases)
    assert np.array_equal(a.norm.view(np.uint32), b.norm.view(np.uint32))
    assert np.array_equal(a.inject, b.inject)
    for part in ("down", "up"):
        for x, y in zip(a.parts[part], b.parts[part]):
            assert (x is None) == (y is None)
            if x is not None:
                assert x.dtype == y.dtype and np.array_equal(x, y), part
