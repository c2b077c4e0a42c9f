"""The hyper-connection step around the MoE block (the next fusion target):
the restatement (oracle/moe_oracle.c) against the reference's own
gated_residual and layer wiring (c/src/model.c:728-796, :1708-1731), compiled
unmodified into oracle/_ref."""
import numpy as np
import pytest


def _impls():
    import oracle
    ref = oracle.reference()
    if ref is None:
        pytest.skip("reference build (oracle/_ref) absent")
    return oracle, oracle.restatement(), ref


@pytest.mark.parametrize("q4,biases", [(True, True), (True, False), (False, True)],
                         ids=["q4", "q4-no-biases", "bf16"])
@pytest.mark.parametrize("d,hc,lr,n", [(256, 4, 32, 1), (256, 4, 32, 33), (2048, 4, 64, 5)])
def test_gated_residual_equals_reference(built, q4, biases, d, hc, lr, n):
    oracle, o, r = _impls()
    H = oracle.SynthHC(d, hc, lr, 20261207 + d + n, q4=q4, biases=biases)
    h = np.random.default_rng(n).standard_normal((n, hc * d)).astype(np.float32)
    mo, io = o.gated_residual(H, h)
    mr, ir = r.gated_residual(H, h)
    assert np.array_equal(mo, mr) and np.array_equal(io, ir)
    assert np.all(np.isfinite(mo)) and np.all((io > 0) & (io < 2))


def test_hc_moe_step_equals_reference(built):
    """configs[0]'s MoE layer inside the hyper-connection wiring, 32 tokens."""
    import qmoe
    oracle, o, r = _impls()
    d, E, k, I, hc = 256, 16, 4, 128, 4
    s = qmoe.SynthLayer(qmoe.make_config(d, E, k, I, max_tokens=32), 20261208)
    H = oracle.SynthHC(d, hc, 32, 20261209)
    h = np.random.default_rng(3).standard_normal((32, hc * d)).astype(np.float32)
    ho, hr = o.hc_moe_step(H, s, h), r.hc_moe_step(H, s, h)
    assert not np.array_equal(ho, h)
    rr = float(np.linalg.norm(ho - hr) / np.linalg.norm(hr - h))
    assert rr <= 1e-5, rr
