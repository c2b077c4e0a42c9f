"""CPU tests of the checkers themselves: the C restatement (oracle/moe_oracle.c)
against the reference's own moe_forward (oracle/_ref), against the committed
golden fixtures, and against the reference's known-answer vectors."""
import hashlib
import math
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _setup(built):
    import oracle
    import qmoe
    return oracle, qmoe


def test_dequant_known_answer_vectors(built):
    """MLX q4 packing, c/tests/test_kernel.c:122-141 (vectors checked there
    against mx.quantize/dequantize of mlx 0.32.2)."""
    oracle, _ = _setup(built)
    o = oracle.restatement()
    q = np.array([0x43322110, 0, 0, 0], np.uint32)
    out = o.dequant(q, np.array([2.0], np.float32), np.array([-16.0], np.float32), 1, 32, 32)
    assert out[0, :8].tolist() == [-16, -14, -14, -12, -12, -10, -10, -8]
    q2 = np.array([0x76543210, 0, 0, 0], np.uint32)
    out2 = o.dequant(q2, np.array([2.0], np.float32), np.array([-16.0], np.float32), 1, 32, 32)
    assert out2[0, 0] == -16 and out2[0, 1] == -14 and out2[0, 2] == -12
    assert out2[0, 6] == -4 and out2[0, 7] == -2


def test_dequant_matches_mlx_style_quantiser(built):
    """Round trip of an MLX-style affine quantiser, as c/tests/test_kernel.c:143-187."""
    oracle, _ = _setup(built)
    rng = np.random.default_rng(23)
    w = (rng.random(128, dtype=np.float32) - 0.5) * 8
    q = np.zeros(16, np.uint32)
    scales, biases, ref = np.zeros(2, np.float32), np.zeros(2, np.float32), np.zeros(128, np.float32)
    for g in range(2):
        wg = w[g * 64:(g + 1) * 64]
        mn, mx = float(wg.min()), float(wg.max())
        scale = np.float32(max((mx - mn) / 15.0, 1e-7))
        side = abs(mn) > abs(mx)
        scale = scale if side else -scale
        edge = np.float32(mn if side else mx)
        q0 = np.float32(round(float(edge / scale)))
        if q0 != 0:
            scale = np.float32(edge / q0)
        bias = np.float32(0.0 if q0 == 0 else edge)
        scales[g], biases[g] = scale, bias
        for i in range(64):
            v = int(min(round(float((wg[i] - bias) / scale)), 15))
            v = max(v, 0)
            q[g * 8 + i // 8] |= np.uint32(v << (4 * (i % 8)))
            ref[g * 64 + i] = np.float32(v) * scale + bias
    out = oracle.restatement().dequant(q, scales, biases, 2, 64, 64)
    assert np.array_equal(out.reshape(-1), ref)


def test_router_dot_is_correctly_rounded_in_practice(built):
    """The canonical router dot (fp64 sums of exact products in a fixed order,
    one rounding) agrees with the exactly rounded dot product (math.fsum) to
    within one fp32 ulp, and exactly on almost every row."""
    oracle, qmoe = _setup(built)
    o = oracle.restatement()
    rng = np.random.default_rng(5)
    exact_hits = 0
    for trial in range(200):
        K = int(rng.choice([256, 512, 2048]))
        x = rng.standard_normal(K).astype(np.float32)
        wf = (rng.standard_normal(K) * 0.02).astype(np.float32)
        w = (wf.view(np.uint32) >> 16).astype(np.uint16)
        wv = (w.astype(np.uint32) << 16).view(np.float32)
        got = o.router_dot(x, w)
        ex = np.float32(math.fsum(float(a) * float(b) for a, b in zip(x, wv)))
        assert abs(float(got) - float(ex)) <= float(np.spacing(np.float32(abs(ex)))), trial
        exact_hits += got == ex
    assert exact_hits >= 195


def test_topk_property(built):
    """Selection property of c/tests/test_kernel.c:95-120 on the restatement's
    routing: min(chosen) >= max(unchosen), distinct, (value desc, index asc)."""
    oracle, qmoe = _setup(built)
    cfg = qmoe.make_config(256, 64, 10, 128, max_tokens=48)
    s = qmoe.SynthLayer(cfg, 17)
    x = qmoe.synth_tokens(17, 3, 48, 256)
    idx, w, lg = oracle.restatement().route(s, x)
    for t in range(48):
        sel = idx[t]
        assert len(set(sel.tolist())) == 10
        chosen = lg[t, sel]
        rest = np.delete(lg[t], sel)
        assert chosen.min() >= rest.max()
        assert all(chosen[i] >= chosen[i + 1] for i in range(9))
        assert abs(float(w[t].sum()) - 1.0) < 1e-5


def _sorted(idx, w):
    o = np.argsort(idx, 1, kind="stable")
    return np.take_along_axis(idx, o, 1), np.take_along_axis(w, o, 1)


@pytest.mark.parametrize("name", ["moe_cfg0.npz", "moe_cfg1_tokens.npz"])
def test_restatement_matches_golden(built, name):
    """Golden outputs come from the reference's own moe_forward (gen_golden.py);
    the input digests pin the synthetic generator as well."""
    oracle, qmoe = _setup(built)
    g = np.load(os.path.join(GOLD, name))
    d, E, k, I, gs, n, stream = (int(v) for v in g["shape"])
    seed = int(g["seed"])
    s = qmoe.SynthLayer(qmoe.make_config(d, E, k, I, gs, max_tokens=n), seed)
    x = qmoe.synth_tokens(seed, stream, n, d)
    assert hashlib.sha256(x.tobytes()).hexdigest() == str(g["x_sha"])
    assert hashlib.sha256(s.router.tobytes()).hexdigest() == str(g["sha_router"])
    for t in ("gate", "up", "down", "sh_gate", "sh_up", "sh_down"):
        h = hashlib.sha256()
        for a in s.t[t]:
            h.update(a.tobytes())
        assert h.hexdigest() == str(g[f"sha_{t}"]), t
    out, idx, w = oracle.restatement().forward(s, x)
    si, sw = _sorted(idx, w)
    assert np.array_equal(si, g["idx_sorted"])
    np.testing.assert_allclose(sw, g["w_sorted"], rtol=1e-5, atol=1e-7)
    ref = g["out"]
    assert np.abs(out - ref).max() <= 1e-4 * max(1.0, float(np.abs(ref).max()))
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 1e-5


def test_restatement_route_matches_golden_zipf(built):
    oracle, qmoe = _setup(built)
    g = np.load(os.path.join(GOLD, "moe_cfg2_route.npz"))
    d, E, k, I, gs, n, stream = (int(v) for v in g["shape"])
    seed = int(g["seed"])
    s = qmoe.SynthLayer(qmoe.make_config(d, E, k, I, gs, max_tokens=n), seed, zipf_s=1.1)
    x = qmoe.synth_tokens(seed, stream, n, d)
    idx, w, _ = oracle.restatement().route(s, x)
    si, sw = _sorted(idx, w)
    assert np.array_equal(si, g["idx_sorted"])
    assert np.array_equal(np.bincount(idx.ravel(), minlength=E), g["counts"])


def test_restatement_matches_reference_build(built):
    """Restatement vs the reference compiled unmodified (only where built)."""
    oracle, qmoe = _setup(built)
    ref = oracle.reference()
    if ref is None:
        pytest.skip("oracle/_ref not built (reference sources absent)")
    for (d, E, k, I, g, n, zipf) in ((256, 16, 4, 128, 64, 32, None), (512, 64, 6, 256, 64, 12, 1.1),
                                     (256, 8, 1, 128, 64, 7, None),       # top-1
                                     (256, 32, 8, 128, 32, 16, None),     # group 32
                                     (1024, 128, 10, 256, 64, 5, 1.1),
                                     (2048, 512, 10, 512, 64, 2, None)):  # configs[1]
        s = qmoe.SynthLayer(qmoe.make_config(d, E, k, I, g=g, max_tokens=n), 99, zipf_s=zipf)
        x = qmoe.synth_tokens(99, 5, n, d)
        a, ia, wa = oracle.restatement().forward(s, x)
        b, ib, wb = ref.forward(s, x)
        ref.lib.ref_reset_cache()
        sa, swa = _sorted(ia, wa)
        sb, swb = _sorted(ib, wb)
        assert np.array_equal(sa, sb)
        np.testing.assert_allclose(swa, swb, rtol=1e-5, atol=1e-7)
        if g != 64:
            # the reference runs the shared expert with group 64 whatever the
            # checkpoint's group (model.c:1391-1395); the restatement uses the
            # checkpoint's. Routing is unaffected; outputs agree at g = 64.
            continue
        assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-5
