"""qmoe_forward_token_noalloc: one decode token for callers that cannot call
cudaMalloc (code confined to someone else's device-memory arena or running
where an allocation may block or is not allowed). The entry point allocates
nothing; its intermediates live in the library's fixed device array.

This file is collected last on purpose. The test packs the experts into the
documented slot layout itself (numpy), places them in device memory that the
test owns, calls the entry point several times in a row through the C ABI
(fp32 and bf16 tokens), and checks each output against the context path
(qmoe_forward / qmoe_forward_dev) within the parity tests' tolerance, and bit
for bit, since both run the same single-launch kernel."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS, REL_RMS = 2e-2, 1e-3
SEED = 20261201


def _bytes(a, rows):
    return np.ascontiguousarray(a).view(np.uint8).reshape(rows, -1)


def pack_slots(s, slot_bytes):
    """Experts and shared expert in the slot layout documented in qmoe.h."""
    d, E, I, g = s.d, s.E, s.I, s.g
    G, Gd = d // g, I // g
    d_row = ((I // 2 + Gd * 4) + 15) // 16 * 16

    def one(gq, gs, gb, uq, us, ub, dq, ds, db):
        gu = np.concatenate([_bytes(gq, I), _bytes(uq, I),
                             _bytes(np.stack([gs.reshape(I, G), gb.reshape(I, G),
                                              us.reshape(I, G), ub.reshape(I, G)], -1), I)], 1)
        dn = np.zeros((d, d_row), np.uint8)
        dn[:, :I // 2] = _bytes(dq, d)
        dn[:, I // 2:I // 2 + Gd * 4] = _bytes(np.stack([ds.reshape(d, Gd), db.reshape(d, Gd)], -1), d)
        slot = np.zeros(slot_bytes, np.uint8)
        body = np.concatenate([gu.ravel(), dn.ravel()])
        slot[:body.size] = body
        return slot

    t = s.t
    qg, qu, qd = (t[n][0].reshape(E, -1) for n in ("gate", "up", "down"))
    sg, su, sd = (t[n][1].reshape(E, -1) for n in ("gate", "up", "down"))
    bg, bu, bd = (t[n][2].reshape(E, -1) for n in ("gate", "up", "down"))
    pool = np.stack([one(qg[e], sg[e], bg[e], qu[e], su[e], bu[e], qd[e], sd[e], bd[e])
                     for e in range(E)])
    sh = one(t["sh_gate"][0], t["sh_gate"][1], t["sh_gate"][2], t["sh_up"][0], t["sh_up"][1],
             t["sh_up"][2], t["sh_down"][0], t["sh_down"][1], t["sh_down"][2])
    return pool, sh


def _args(qmoe, d, E, k, I, x_ptr, x_dtype, out_ptr, router_d, sgate_d, pool_d, slots_d, sh_d):
    return qmoe.TokenArgs(d, E, k, I, 64, x_ptr, x_dtype, out_ptr, router_d.data_ptr(),
                          sgate_d.data_ptr(), None, pool_d.data_ptr(), slots_d.data_ptr(),
                          sh_d.data_ptr())


def _call(qmoe, a):
    err = qmoe.Err()
    rc = qmoe.lib().qmoe_forward_token_noalloc(C.byref(a), None, C.byref(err))
    return rc, err.text()


def _margins(out, ref):
    return float(np.abs(out - ref).max()), float(np.linalg.norm(out - ref) / np.linalg.norm(ref))


def test_noalloc_token_matches_context_path(built):
    """Two fp32 calls in a row, then two bf16 calls, each checked against the
    context path on the same token (qmoe_forward for fp32 host x,
    qmoe_forward_dev for bf16 device x); device memory in use is the same
    before and after the calls (the entry point allocates nothing)."""
    import torch

    import qmoe

    d, E, k, I = 2048, 512, 10, 512
    cfg = qmoe.make_config(d, E, k, I, max_tokens=1)
    s = qmoe.SynthLayer(cfg, SEED)
    slot_bytes = qmoe.lib().qmoe_slot_bytes(cfg)
    pool, sh = pack_slots(s, slot_bytes)

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    pool_d = torch.from_numpy(pool).to(dev)
    sh_d = torch.from_numpy(sh).to(dev)
    slots_d = torch.arange(E, dtype=torch.int32, device=dev)
    router_d = torch.from_numpy(s.router.view(np.int16)).to(dev)
    sgate_d = torch.from_numpy(s.shared_gate.view(np.int16)).to(dev)
    x = qmoe.synth_tokens(SEED, 21, 4, d)
    x_d = torch.from_numpy(x).to(dev)
    xb_d = x_d.to(torch.bfloat16).contiguous()  # the tokens are bf16 values: exact
    out_d = torch.zeros((4, d), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()

    outs = []
    free0 = None
    for t in range(4):  # calls in a row share the scratch array
        if t == 1:
            torch.cuda.synchronize()
            free0 = torch.cuda.mem_get_info(0)[0]
        if t < 2:
            a = _args(qmoe, d, E, k, I, x_d[t].data_ptr(), qmoe.QMOE_F32, out_d[t].data_ptr(),
                      router_d, sgate_d, pool_d, slots_d, sh_d)
        else:
            a = _args(qmoe, d, E, k, I, xb_d[t].data_ptr(), qmoe.QMOE_BF16, out_d[t].data_ptr(),
                      router_d, sgate_d, pool_d, slots_d, sh_d)
        rc, msg = _call(qmoe, a)
        assert rc == 0, msg
        outs.append(out_d[t].cpu().numpy())
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(0)[0] == free0  # nothing allocated by calls 2-4

    ctx = qmoe.Context(cfg)
    ctx.upload(0, s)
    for t in range(4):
        if t < 2:
            ref = ctx.forward(0, x[t:t + 1])[0]
        else:
            o = torch.empty((1, d), dtype=torch.float32, device=dev)
            ctx.forward_dev(0, xb_d[t].data_ptr(), qmoe.QMOE_BF16, 1, o.data_ptr(), None)
            ctx.sync()
            ref = o[0].cpu().numpy()
        mab, rr = _margins(outs[t], ref)
        assert mab <= MAX_ABS and rr <= REL_RMS, (t, mab, rr)
        # the same single-launch kernel on the same values: the same bits
        assert np.array_equal(outs[t], ref), (t, mab, rr)
    assert not np.array_equal(outs[0], outs[1])
    ctx.close()


def test_noalloc_reports_the_device_error_word(built):
    """A slot table naming no resident expert: the kernel issues no copy,
    sets its error word, and the call returns -1 with the word's code; the
    next good call on the same array succeeds (each call clears the word)."""
    import torch

    import qmoe

    d, E, k, I = 256, 16, 4, 128
    cfg = qmoe.make_config(d, E, k, I, max_tokens=1)
    s = qmoe.SynthLayer(cfg, SEED)
    pool, sh = pack_slots(s, qmoe.lib().qmoe_slot_bytes(cfg))
    dev = torch.device("cuda", 0)
    pool_d = torch.from_numpy(pool).to(dev)
    sh_d = torch.from_numpy(sh).to(dev)
    router_d = torch.from_numpy(s.router.view(np.int16)).to(dev)
    sgate_d = torch.from_numpy(s.shared_gate.view(np.int16)).to(dev)
    x_d = torch.from_numpy(qmoe.synth_tokens(SEED, 22, 1, d)).to(dev)
    out_d = torch.zeros((1, d), dtype=torch.float32, device=dev)
    none_d = torch.full((E,), -1, dtype=torch.int32, device=dev)
    slots_d = torch.arange(E, dtype=torch.int32, device=dev)
    rc, msg = _call(qmoe, _args(qmoe, d, E, k, I, x_d.data_ptr(), qmoe.QMOE_F32, out_d.data_ptr(),
                                router_d, sgate_d, pool_d, none_d, sh_d))
    assert rc == -1 and "device reported error" in msg, msg
    rc, msg = _call(qmoe, _args(qmoe, d, E, k, I, x_d.data_ptr(), qmoe.QMOE_F32, out_d.data_ptr(),
                                router_d, sgate_d, pool_d, slots_d, sh_d))
    assert rc == 0, msg
    ctx = qmoe.Context(cfg)
    ctx.upload(0, s)
    ref = ctx.forward(0, x_d.cpu().numpy())[0]
    ctx.close()
    assert np.array_equal(out_d[0].cpu().numpy(), ref)


def test_noalloc_rejects_shapes_beyond_its_scratch(built):
    import qmoe

    # k=32, I=1024 needs ~135 KB of scratch, more than the library's 64 KB
    a = qmoe.TokenArgs(2048, 64, 32, 1024, 64, 16, qmoe.QMOE_F32, 16, 16, 16, None, 16, 16, 16)
    err = qmoe.Err()
    assert qmoe.lib().qmoe_forward_token_noalloc(C.byref(a), None, C.byref(err)) == -1
    assert "QMOE_NOALLOC_SCRATCH_BYTES" in err.text()
