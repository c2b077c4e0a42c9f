"""The approximate router logits of small calls (k_route_approx,
qmoe_prefill.cu) against the bound the exact re-ranking (k_route_exact) uses
to choose its candidates: beta = 2^-10 |x| max_e |w_e| + 2^-20 max_e |a_e|.
If |a - logit| <= beta for every expert, the candidates (a >= a_(k) - 3 beta)
hold the exact top-k and everything tied with it, so the selection is exact.

A CPU model of the kernel's fp32 arithmetic (no GPU): lane l of 32 sums
x_k w_k for k = 4l + 128i + j (i over d / 128 steps, j = 0..3) with one
fused multiply-add at a time, then the 32 lane sums are added in a balanced
tree (the halving butterfly's shape). fma is modelled as the fp64 sum of the
exact product and the fp32 accumulator, rounded to fp32 (the product of an
fp32 and a bf16 value is exact in fp64). The exact logit is the fp64 sum of
the exact products, far closer to the true value than beta."""
import numpy as np

RNG = np.random.default_rng(20261203)


def _bf16(a):
    """fp32 -> bf16 values (round to nearest even), as fp32."""
    u = np.asarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def _kernel_logits(x, w):
    """x [T, d] fp32, w [E, d] bf16-valued fp32 -> [T, E] in the kernel's order."""
    T, d = x.shape
    E = w.shape[0]
    xd = x.astype(np.float64)
    wd = w.astype(np.float64)
    lanes = np.zeros((32, T, E), dtype=np.float32)
    for l in range(32):
        acc = np.zeros((T, E), dtype=np.float32)
        for k0 in range(4 * l, d, 128):
            for j in range(4):
                k = k0 + j
                prod = np.outer(xd[:, k], wd[:, k])  # exact
                acc = (acc.astype(np.float64) + prod).astype(np.float32)
        lanes[l] = acc
    vals = list(lanes)
    while len(vals) > 1:  # balanced tree of fp32 additions
        vals = [(vals[2 * i].astype(np.float64) + vals[2 * i + 1]).astype(np.float32)
                for i in range(len(vals) // 2)]
    return vals[0]


def _bound(x, w, a):
    xnorm = np.sqrt((x.astype(np.float64) ** 2).sum(1))
    wmax = np.sqrt((w.astype(np.float64) ** 2).sum(1)).max()
    return 2.0**-10 * xnorm[:, None] * wmax + 2.0**-20 * np.abs(a).max(1, keepdims=True)


def _case(x, w):
    a = _kernel_logits(x, w).astype(np.float64)
    exact = x.astype(np.float64) @ w.astype(np.float64).T
    err = np.abs(a - exact)
    beta = _bound(x, w, a)
    assert np.all(err <= beta), float((err / beta).max())
    return float((err / beta).max())


def test_small_router_within_rerank_bound():
    """Config-1 shapes in miniature (d = 2048, 64 experts, 8 tokens): RMSNorm-
    scaled tokens and N(0, 0.02) bf16 router rows, plus tokens scaled by 2^10
    and 2^-10 and one with a few large entries. The error stays far inside
    the bound (under 1% of it)."""
    d, E = 2048, 64
    w = _bf16(RNG.normal(0.0, 0.02, size=(E, d)).astype(np.float32))
    x = RNG.normal(0.0, 1.0, size=(8, d)).astype(np.float32)
    x[1] *= 1024.0
    x[2] *= 1.0 / 1024.0
    x[3, :16] *= 300.0
    worst = _case(x, w)
    assert worst < 1e-2, worst


def test_small_router_cancellation_within_bound():
    """Rows built to cancel (w and -w halves against a token of equal halves):
    the logits are near zero while |x| |w| is large; the error still stays
    within the bound."""
    d, E = 2048, 8
    half = _bf16(RNG.normal(0.0, 0.05, size=(E, d // 2)).astype(np.float32))
    w = np.concatenate([half, -half], axis=1)
    xh = RNG.normal(0.0, 1.0, size=(4, d // 2)).astype(np.float32)
    x = np.concatenate([xh, xh], axis=1)
    _case(x, w)
