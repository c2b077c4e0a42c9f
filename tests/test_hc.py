"""The hyper-connection step around the MoE block on the GPU
(qmoe_upload_hc / qmoe_forward_hc): gated_residual (c/src/model.c:728-796),
the MoE block on its mixed rows and the inject-add after it (:1708-1731),
against the C restatement (oracle_hc_moe_step) and the reference's own
compiled code (ref_hc_moe_step). Bars: the step's contribution h' - h within
2e-2 max-abs and 1e-3 relative RMS of the checker's,
and within the measured precision of the path (TIGHT)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS, REL_RMS = 2e-2, 1e-3
# measured precision with headroom: the block's input (mixed) is fp32, not
# bf16, so the decode kernel's 16-bit blocks of x round it (about 6e-5
# relative on the step's contribution; bf16 inputs are held exactly)
TIGHT = (3e-3, 3e-4)


def _check(got, want, h0, case):
    from conftest import record_margin
    dg, dw = got.astype(np.float64) - h0, want.astype(np.float64) - h0
    mab = float(np.abs(dg - dw).max())
    rr = float(np.linalg.norm(dg - dw) / np.linalg.norm(dw))
    record_margin(case, mab, rr, {"north_star": [MAX_ABS, REL_RMS], "tight": TIGHT})
    assert mab <= MAX_ABS and rr <= REL_RMS, (case, mab, rr)
    assert mab <= TIGHT[0] and rr <= TIGHT[1], (case, mab, rr)


def _run(ctx, layer, h0):
    import torch
    h = torch.from_numpy(h0).cuda()
    ctx.forward_hc(layer, h.data_ptr(), h0.shape[0])
    ctx.sync()
    return h.cpu().numpy()


@pytest.mark.parametrize("q4,biases", [(True, True), (True, False), (False, True)],
                         ids=["q4", "q4-no-biases", "bf16"])
def test_hc_step_small_shape(built, q4, biases):
    """configs[0]'s MoE layer (d 256, 16 experts, top-4) inside the hyper
    connection (hc 4, lowrank 64), one token and 32 tokens."""
    import oracle
    import qmoe
    d, E, k, I, hc, lr = 256, 16, 4, 128, 4, 64
    cfg = qmoe.make_config(d, E, k, I, max_tokens=32)
    s = qmoe.SynthLayer(cfg, 20261210)
    H = oracle.SynthHC(d, hc, lr, 20261211, q4=q4, biases=biases)
    ctx = qmoe.Context(cfg)
    ctx.upload(0, s)
    ctx.upload_hc(0, H)
    ref = oracle.reference()
    for n in (1, 32):
        h0 = np.random.default_rng(n).standard_normal((n, hc * d)).astype(np.float32)
        got = _run(ctx, 0, h0)
        _check(got, oracle.restatement().hc_moe_step(H, s, h0), h0, f"hc small n={n} vs restatement")
        if ref is not None:
            _check(got, ref.hc_moe_step(H, s, h0), h0, f"hc small n={n} vs reference build")
            ref.lib.ref_reset_cache()
    ctx.close()


def test_hc_step_full_shape(built):
    """The config-1 layer (d 2048, 512 experts, top-10) inside the hyper
    connection (hc 4, lowrank 64, q4 mixers): the decode kernel for one token,
    the grouped path for eight."""
    import oracle
    import qmoe
    d, E, k, I, hc, lr = 2048, 512, 10, 512, 4, 64
    cfg = qmoe.make_config(d, E, k, I, max_tokens=8)
    s = qmoe.SynthLayer(cfg, 20261212)
    H = oracle.SynthHC(d, hc, lr, 20261213)
    ctx = qmoe.Context(cfg)
    ctx.upload(0, s)
    ctx.upload_hc(0, H)
    for n in (1, 8):
        h0 = np.random.default_rng(100 + n).standard_normal((n, hc * d)).astype(np.float32)
        got = _run(ctx, 0, h0)
        _check(got, oracle.restatement().hc_moe_step(H, s, h0), h0, f"hc full n={n} vs restatement")
    ctx.close()


def test_hc_upload_refuses_uncovered_shapes(built):
    import oracle
    import qmoe
    d, E, k, I = 256, 16, 4, 128
    ctx = qmoe.Context(qmoe.make_config(d, E, k, I, max_tokens=4))
    with pytest.raises(qmoe.QmoeError, match="lowrank"):
        ctx.upload_hc(0, oracle.SynthHC(d, 4, 32, 1))  # q4 up mixer with lowrank 32
    H = oracle.SynthHC(d, 4, 64, 1)
    H.hc = 9
    with pytest.raises(qmoe.QmoeError, match="hc <= 8"):
        ctx.upload_hc(0, H)
    import torch
    h = torch.zeros((1, 4 * d), dtype=torch.float32, device="cuda")
    with pytest.raises(qmoe.QmoeError, match="no hyper connection"):
        ctx.forward_hc(0, h.data_ptr(), 1)
    ctx.close()
