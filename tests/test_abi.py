"""The C ABI without a GPU: libqmoe.so loads, exports every symbol that
include/qmoe.h declares, and its host-only parts (layout, synthetic data)
behave. No CUDA call is made."""
import os
import re
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    txt = open(os.path.join(ROOT, "include", "qmoe.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(qmoe_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_declared_symbol(built):
    import qmoe
    lib = qmoe.lib()
    names = _declared()
    assert len(names) > 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the binding covers the same set
    assert set(names) == set(qmoe.SIGNATURES), set(names) ^ set(qmoe.SIGNATURES)
    nm = subprocess.run(["nm", "-D", "--defined-only", qmoe.LIB_PATH], capture_output=True,
                        text=True, check=True).stdout
    exported = set(re.findall(r" T (qmoe_[a-z0-9_]+)$", nm, flags=re.M))
    assert set(names) <= exported


def test_library_holds_sm100a_code(built):
    import qmoe
    out = subprocess.run(["cuobjdump", "--list-elf", qmoe.LIB_PATH], capture_output=True,
                         text=True).stdout
    assert "sm_100a" in out


def test_slot_bytes(built):
    import qmoe
    lib = qmoe.lib()
    cfg1 = qmoe.make_config(2048, 512, 10, 512)
    assert lib.qmoe_slot_bytes(cfg1) == 1769472  # the packed q4 expert, no padding
    cfg0 = qmoe.make_config(256, 16, 4, 128)
    assert lib.qmoe_slot_bytes(cfg0) == 128 * 288 + 256 * 80  # down rows padded to 16 B
    bad = qmoe.make_config(2048, 512, 10, 500)
    assert lib.qmoe_slot_bytes(bad) == 0


def test_synth_is_seeded_and_sliceable(built):
    import ctypes as C
    import qmoe
    cfg = qmoe.make_config(256, 16, 4, 128)
    a = qmoe.SynthLayer(cfg, 7)
    b = qmoe.SynthLayer(cfg, 7)
    c = qmoe.SynthLayer(cfg, 8)
    assert np.array_equal(a.t["gate"][0], b.t["gate"][0])
    assert not np.array_equal(a.t["gate"][0], c.t["gate"][0])
    # experts [5, 9) generated alone equal the full generation's slice
    part = qmoe.SynthLayer(cfg, 9)
    for arrs in part.t.values():
        for arr in arrs:
            arr[:] = 0
    w = part.weights()
    assert qmoe.lib().qmoe_synth_layer(C.byref(cfg), 7, 0, C.byref(w), 5, 9) == 0
    per = 128 * 256 // 8
    assert np.array_equal(part.t["gate"][0][5 * per:9 * per], a.t["gate"][0][5 * per:9 * per])
    assert not part.t["gate"][0][:5 * per].any()


def test_synth_distributions(built):
    import qmoe
    cfg = qmoe.make_config(2048, 64, 10, 512)
    s = qmoe.SynthLayer(cfg, 3)
    q = s.t["gate"][0]
    nib = np.stack([(q >> (4 * i)) & 0xF for i in range(8)]).ravel()
    counts = np.bincount(nib, minlength=16) / nib.size
    assert np.all(np.abs(counts - 1 / 16) < 2e-3)
    sc = (s.t["gate"][1].astype(np.uint32) << 16).view(np.float32)
    bi = (s.t["gate"][2].astype(np.uint32) << 16).view(np.float32)
    assert np.all(sc >= 0)
    assert np.array_equal(bi, -8 * sc)  # weight = (q - 8) * scale exactly
    assert abs(np.sqrt(np.mean(sc.astype(np.float64) ** 2)) - 0.02) < 1e-3
    r = (s.router.astype(np.uint32) << 16).view(np.float32)
    assert abs(r.std() - 0.02) < 1e-3 and abs(r.mean()) < 1e-3
    x = qmoe.synth_tokens(3, 0, 64, 2048)
    assert abs(x.std() - 1) < 0.02
    xb = (x.view(np.uint32) & 0xFFFF)
    assert not xb.any()  # bf16-representable


def test_zipf_bias(built):
    import qmoe
    cfg = qmoe.make_config(2048, 512, 10, 512)
    s = qmoe.SynthLayer(cfg, 3, zipf_s=1.1)
    b = s.logit_bias
    ranks = np.rint(np.exp(-b.astype(np.float64) / 1.1)).astype(int)
    assert sorted(ranks.tolist()) == list(range(1, 513))


def _arity():
    """{name: number of parameters} of every function declared in qmoe.h."""
    txt = open(os.path.join(ROOT, "include", "qmoe.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    txt = re.sub(r"#[^\n]*", "", txt)
    out = {}
    for m in re.finditer(r"\b(qmoe_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", txt, flags=re.S):
        params, depth, n = m.group(2).strip(), 0, 1
        if params in ("", "void"):
            out[m.group(1)] = 0
            continue
        for ch in params:
            depth += ch in "([" and 1 or ch in ")]" and -1 or 0
            n += ch == "," and depth == 0
        out[m.group(1)] = n
    return out


def test_binding_arity_matches_the_header(built):
    """Every ctypes signature in qmoe.py takes as many arguments as the C
    declaration it binds."""
    import qmoe
    ar = _arity()
    assert set(ar) == set(qmoe.SIGNATURES), set(ar) ^ set(qmoe.SIGNATURES)
    bad = {n: (len(qmoe.SIGNATURES[n][1]), k) for n, k in ar.items() if len(qmoe.SIGNATURES[n][1]) != k}
    assert not bad, bad


def test_noalloc_refuses_bad_arguments_before_any_launch(built):
    """qmoe_forward_token_noalloc checks its arguments on the host before any
    CUDA call: a misaligned pointer (the kernel moves its inputs with 16-byte
    vector loads and bulk copies) and a shape beyond the library's scratch
    array are refused with a message. No GPU is needed for either."""
    import ctypes as C

    import qmoe
    lib = qmoe.lib()
    base = dict(x=16, out=16, router=16, shared_gate=16, pool=16, slot_of=16, shared_slot=16)
    for name in base:
        p = dict(base, **{name: base[name] + 4})
        a = qmoe.TokenArgs(2048, 512, 10, 512, 64, p["x"], qmoe.QMOE_F32, p["out"], p["router"],
                           p["shared_gate"], None, p["pool"], p["slot_of"], p["shared_slot"])
        err = qmoe.Err()
        assert lib.qmoe_forward_token_noalloc(C.byref(a), None, C.byref(err)) == -1
        assert f"{name} (" in err.text() and "16-byte aligned" in err.text(), err.text()
    a = qmoe.TokenArgs(2048, 512, 10, 512, 64, 16, qmoe.QMOE_F32, 16, 16, 16, 18, 16, 16, 16)
    err = qmoe.Err()
    assert lib.qmoe_forward_token_noalloc(C.byref(a), None, C.byref(err)) == -1
    assert "logit_bias" in err.text()
    # k=32, I=1024 needs ~135 KB of scratch, more than the library's 64 KB
    a = qmoe.TokenArgs(2048, 64, 32, 1024, 64, 16, qmoe.QMOE_F32, 16, 16, 16, None, 16, 16, 16)
    err = qmoe.Err()
    assert lib.qmoe_forward_token_noalloc(C.byref(a), None, C.byref(err)) == -1
    assert "QMOE_NOALLOC_SCRATCH_BYTES" in err.text()
