"""qmoe_forward_token_noalloc: one decode token for callers that cannot call
cudaMalloc (code confined to someone else's device-memory arena or running
where an allocation may block or is not allowed). The entry point allocates
nothing; its intermediates live in the library's fixed device array.

This file is collected last on purpose. The test packs the experts into the
documented slot layout itself (numpy), places them in device memory that the
test owns, calls the entry point twice in a row through the C ABI, and checks
each output against the context path (qmoe_forward) within the parity tests'
tolerance."""
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


def test_noalloc_token_matches_context_path(built):
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
    x = qmoe.synth_tokens(SEED, 21, 2, d)
    x_d = torch.from_numpy(x).to(dev)
    out_d = torch.zeros((2, d), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()

    outs = []
    for t in range(2):  # two calls in a row share the scratch array
        a = qmoe.TokenArgs(d, E, k, I, 64, x_d[t].data_ptr(), qmoe.QMOE_F32, out_d[t].data_ptr(),
                           router_d.data_ptr(), sgate_d.data_ptr(), None, pool_d.data_ptr(),
                           slots_d.data_ptr(), sh_d.data_ptr())
        err = qmoe.Err()
        rc = qmoe.lib().qmoe_forward_token_noalloc(C.byref(a), None, C.byref(err))
        assert rc == 0, err.text()
        outs.append(out_d[t].cpu().numpy())

    ctx = qmoe.Context(cfg)
    ctx.upload(0, s)
    for t in range(2):
        ref = ctx.forward(0, x[t:t + 1])[0]
        mab = float(np.abs(outs[t] - ref).max())
        rr = float(np.linalg.norm(outs[t] - ref) / np.linalg.norm(ref))
        assert mab <= MAX_ABS and rr <= REL_RMS, (t, mab, rr)
    assert not np.array_equal(outs[0], outs[1])
    ctx.close()


def test_noalloc_rejects_shapes_beyond_its_scratch(built):
    import qmoe

    # k=32, I=1024 needs ~135 KB of scratch, more than the library's 64 KB
    a = qmoe.TokenArgs(2048, 64, 32, 1024, 64, 16, qmoe.QMOE_F32, 16, 16, 16, None, 16, 16, 16)
    err = qmoe.Err()
    assert qmoe.lib().qmoe_forward_token_noalloc(C.byref(a), None, C.byref(err)) == -1
    assert "QMOE_NOALLOC_SCRATCH_BYTES" in err.text()
