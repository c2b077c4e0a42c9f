"""A CPU model (numpy, no GPU) of the numerics of the small-group CUDA-core
path (k_sb_xq, k_sb_gu, k_sb_dn in qmoe_prefill.cu) against the C
restatement of moe_forward: x as 16-bit block fixed point with one
power-of-two scale per 64 values, h as 24-bit with one scale per 32 values
(quant_word's rules: the largest magnitude of a block below 2^15, or 2^22, after
scaling; round to nearest even), the q4 weights applied as s * sum(q v) +
b * sum(v) per scale group. The model computes in fp64 apart from the two
quantisations, so what it measures is their error. It must take at most half
of the GPU tests' tight bars (3e-3 max-abs, 3e-5 relative RMS), leaving the
rest for the kernels' fp32 sums. Measured: 4.6e-5 / 6.7e-6 at config-0
shapes and 5.7e-4 / 5.7e-6 at config-1 shapes, where the GPU's small-group
path gives 6.4e-4 / 4.4e-6."""
import numpy as np

TIGHT = (3e-3, 3e-5)


def _f32_of_bf16(u16):
    return (np.asarray(u16, np.uint32) << 16).view(np.float32).astype(np.float64)


def _nibbles(words, rows, cols):
    """q4 words of [rows, cols] values, low nibble first -> int array."""
    w = np.asarray(words, np.uint64).reshape(rows, cols // 8)
    out = np.stack([(w >> np.uint64(4 * j)) & np.uint64(0xF) for j in range(8)], axis=-1)
    return out.reshape(rows, cols).astype(np.int64)


def _quant(v, block, kbits):
    """quant_word: per block of `block` values, e = kbits - exponent(max|v|)
    (max = f 2^ex, f in [0.5, 1)), q = min(rint(v 2^e), 2^(8 nb - 1) - 1);
    returns the integers and the per-block scale 2^-e."""
    vb = v.reshape(-1, block)
    m = np.abs(vb).max(axis=1)
    _, ex = np.frexp(m)
    e = np.where(m > 0, kbits - ex, 0)
    e = np.clip(e, -126, 126)
    qmax = (1 << (16 if kbits == 15 else 24) - 1) - 1
    q = np.minimum(np.rint(vb * np.ldexp(1.0, e)[:, None]), qmax).astype(np.int64)
    return q.reshape(v.shape), np.ldexp(1.0, -e)


def _expert_model(x, gq, gs, gb, uq, us, ub, dq, ds, db, d, I, g):
    """One expert on one token through the small-group arithmetic."""
    xq, xsc = _quant(x, 64, 15)                      # 16-bit x, a scale per 64
    xg = xq.reshape(-1, g)
    xsum = (xg * xsc.reshape(-1, 1)).sum(1)          # the scaled-back group sums
    def gu(q, s, b):
        qg = q.reshape(I, d // g, g)
        dots = (qg * xg[None]).sum(-1) * xsc[None]   # sum q x per group, scaled
        return (s * dots + b * xsum[None]).sum(1)
    gate = gu(gq, gs, gb)
    up = gu(uq, us, ub)
    h = gate / (1.0 + np.exp(-gate)) * up
    hq, hsc = _quant(h, 32, 22)                      # 24-bit h, a scale per 32
    hu = hq.reshape(-1, 32)
    hsum = (hu * hsc.reshape(-1, 1)).sum(1)
    qd = dq.reshape(d, I // 32, 32)
    dots = (qd * hu[None]).sum(-1) * hsc[None]       # per 32-value unit
    sd = np.repeat(ds, g // 32, axis=1)
    bd = np.repeat(db, g // 32, axis=1)
    return (sd * dots + bd * hsum[None]).sum(1)


def _model_forward(s, x, idx, wts, sg):
    d, E, I, g = s.d, s.E, s.I, s.g
    t = s.t
    def expert(name_g, name_u, name_d, e):
        gq = _nibbles(t[name_g][0], (E if e is not None else 1) * I, d)
        uq = _nibbles(t[name_u][0], (E if e is not None else 1) * I, d)
        dq = _nibbles(t[name_d][0], (E if e is not None else 1) * d, I)
        gs = _f32_of_bf16(t[name_g][1]).reshape(-1, d // g)
        gb = _f32_of_bf16(t[name_g][2]).reshape(-1, d // g)
        us = _f32_of_bf16(t[name_u][1]).reshape(-1, d // g)
        ub = _f32_of_bf16(t[name_u][2]).reshape(-1, d // g)
        ds = _f32_of_bf16(t[name_d][1]).reshape(-1, I // g)
        db = _f32_of_bf16(t[name_d][2]).reshape(-1, I // g)
        r = slice(0, I) if e is None else slice(e * I, (e + 1) * I)
        rd = slice(0, d) if e is None else slice(e * d, (e + 1) * d)
        return gq[r], gs[r], gb[r], uq[r], us[r], ub[r], dq[rd], ds[rd], db[rd]
    shared = expert("sh_gate", "sh_up", "sh_down", None)
    cache = {}
    out = np.zeros((x.shape[0], d))
    for ti in range(x.shape[0]):
        xt = x[ti].astype(np.float64)
        acc = np.zeros(d)
        for sl in range(s.k):
            e = int(idx[ti, sl])
            if e not in cache:
                cache[e] = expert("gate", "up", "down", e)
            acc += wts[ti, sl] * _expert_model(xt, *cache[e], d, I, g)
        acc += sg[ti] * _expert_model(xt, *shared, d, I, g)
        out[ti] = acc
    return out


def _case(built, d, E, k, I, n, seed):
    import oracle
    s = oracle.SynthLayer(d, E, k, I, 64, seed)
    x = oracle.synth_tokens(seed, 7, n, d)
    o = oracle.restatement()
    ref, idx, wts = o.forward(s, x)
    # the shared expert's sigmoid gate (its logit is the canonical router dot)
    sg = np.array([1.0 / (1.0 + np.exp(-float(o.router_dot(x[i], s.shared_gate)))) for i in range(n)])
    got = _model_forward(s, x, idx, wts.astype(np.float64), sg)
    mab = float(np.abs(got - ref).max())
    rr = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    assert mab <= TIGHT[0] / 2 and rr <= TIGHT[1] / 2, (mab, rr)
    return mab, rr


def test_small_group_numerics_cfg0_shapes(built):
    """Config-0 shapes (hidden 256, 16 experts, top-4, I 128), 16 tokens."""
    _case(built, 256, 16, 4, 128, 16, 11)


def test_small_group_numerics_cfg1_shapes(built):
    """Config-1 row shapes (hidden 2048, I 512, top-10) over 16 experts, 4 tokens."""
    _case(built, 2048, 16, 10, 512, 4, 12)
