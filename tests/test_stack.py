"""MoE-only layer stack (the 76-layer batched-decode configuration's
arithmetic) and the device-side synthetic layers it is benchmarked on.

The stack is h <- h + MoE_l(RMSNorm(h)) per layer, RMSNorm with unit weight
and eps 1e-6 as kernel_rmsnorm (c/src/kernel.c:10-20); the checker composes
the C restatement of moe_forward (c/src/model.c:1281-1405) with a numpy
RMSNorm and an fp32 residual, layer by layer."""
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EPS = 1e-6


def rmsnorm(h):
    """kernel_rmsnorm with unit weight: r = 1 / sqrt(ss / n + eps) in fp32,
    y = x * r (the sum of squares in fp64, as the device kernel takes it)."""
    h = h.astype(np.float32)
    ss = (h.astype(np.float64) ** 2).sum(1).astype(np.float32)
    r = np.float32(1.0) / np.sqrt(ss / np.float32(h.shape[1]) + np.float32(EPS))
    return (h * r[:, None]).astype(np.float32)


def compose(layers, h):
    """Oracle stack: returns the final h and every layer's routing."""
    import oracle
    routes = []
    for s in layers:
        y, idx, _ = oracle.restatement().forward(s, rmsnorm(h))
        routes.append(idx)
        h = (h + y).astype(np.float32)
    return h, routes


def _run_stack(shape, n_layers, n, seed):
    import torch

    import qmoe
    d, E, k, I = shape
    cfg = qmoe.make_config(d, E, k, I, layers=n_layers, max_tokens=n)
    layers = [qmoe.SynthLayer(cfg, seed, l) for l in range(n_layers)]
    ctx = qmoe.Context(cfg)
    for l, s in enumerate(layers):
        ctx.upload(l, s)
    h0 = qmoe.synth_tokens(seed, 9, n, d)
    h = torch.from_numpy(h0).cuda()
    # layer by layer, collecting the routing, then the whole stack at once
    routes = []
    for l in range(n_layers):
        ctx.forward_stack(l, l + 1, h.data_ptr(), n, EPS, None)
        ctx.sync()
        routes.append(ctx.routing(n)[0])
    h_steps = h.cpu().numpy()
    h.copy_(torch.from_numpy(h0))
    ctx.forward_stack(0, n_layers, h.data_ptr(), n, EPS, None)
    ctx.sync()
    h_all = h.cpu().numpy()
    ctx.close()
    return layers, h0, h_steps, h_all, routes


def _check(layers, h0, h_steps, h_all, routes):
    ref, ref_routes = compose(layers, h0)
    assert np.array_equal(h_steps, h_all), "one call per layer differs from one call per stack"
    for l, (a, b) in enumerate(zip(routes, ref_routes)):
        assert np.array_equal(np.sort(a, 1), np.sort(b, 1)), f"layer {l} routing"
    delta, rdelta = h_all - h0, ref - h0      # the stack's contribution
    mab = float(np.abs(delta - rdelta).max())
    rr = float(np.linalg.norm(delta - rdelta) / np.linalg.norm(rdelta))
    assert mab <= 2e-2 and rr <= 1e-3, (mab, rr)


@pytest.mark.gpu
def test_stack_small_shape_matches_composition(built):
    """Four config-0-shaped layers, 32 tokens."""
    _check(*_run_stack((256, 16, 4, 128), 4, 32, 31))


@pytest.mark.gpu
def test_stack_full_shape_matches_composition(built):
    """Two full-size layers (hidden 2048, 512 experts, top-10) at the stack
    configuration's batch of 64 tokens: routing bit-exact per layer, the
    stack's contribution to h within the layer tolerance."""
    _check(*_run_stack((2048, 512, 10, 512), 2, 64, 33))


@pytest.mark.gpu
@pytest.mark.parametrize("shape,zipf", [((256, 16, 4, 128), 0.0), ((2048, 512, 10, 512), 1.1)])
def test_device_synth_layer_equals_host(built, shape, zipf):
    """A layer generated on the device gives the same routing and outputs as
    the same seeded layer built on the host and uploaded."""
    import qmoe
    d, E, k, I = shape
    n = 24
    cfg = qmoe.make_config(d, E, k, I, layers=2, max_tokens=n)
    a, b = qmoe.Context(cfg), qmoe.Context(cfg)
    a.upload(1, qmoe.SynthLayer(cfg, 77, 1, zipf_s=zipf if zipf else None))
    b.synth_layer_dev(1, 77, zipf)
    x = qmoe.synth_tokens(77, 2, n, d)
    oa, ob = a.forward(1, x), b.forward(1, x)
    ra, rb = a.routing(n)[0], b.routing(n)[0]
    a.close()
    b.close()
    assert np.array_equal(ra, rb)
    assert np.array_equal(oa, ob)


def test_rmsnorm_checker_matches_reference_formula():
    """The checker's RMSNorm against a direct fp32 restatement of
    kernel_rmsnorm's sequential loop (c/src/kernel.c:10-20) on a few rows."""
    rng = np.random.default_rng(3)
    h = rng.standard_normal((3, 256)).astype(np.float32)
    got = rmsnorm(h)
    for t in range(3):
        ss = np.float32(0)
        for v in h[t]:
            ss = np.float32(ss + v * v)
        r = np.float32(1.0) / np.sqrt(ss / np.float32(256) + np.float32(EPS))
        want = (h[t] * r).astype(np.float32)
        assert np.allclose(got[t], want, rtol=1e-6, atol=0)
