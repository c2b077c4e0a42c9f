"""The drop-in at the source level: tests/c/port_dropin.c includes the
reference's own c/src/model.c with qmoe.h, writes the C port's integration
(err_t passed as qmoe_err, qmoe_config from qcfg, layers uploaded from the
checkpoint, model_forward's MoE call through qmoe_forward), and is compiled and
linked against the reference's other units and libqmoe.so. Skipped where the
reference sources are absent."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "qwen3.8-flash-next_b200")
OBJ = os.path.join(ROOT, "oracle", "_ref", "obj")


def test_port_links_against_libqmoe(built, tmp_path):
    import oracle
    if not os.path.isdir(oracle.REF_SRC) or not os.path.isdir(OBJ):
        pytest.skip("reference sources or their build absent")
    units = [os.path.join(OBJ, f"{u}.o") for u in
             ("kernel", "cache", "reader", "safetensors", "json", "ngram", "accel_shim", "moe_oracle")]
    exe = tmp_path / "port_dropin"
    # no -w: it would also silence the diagnostics promoted to errors here
    cmd = ["gcc", "-std=c11", "-O1", "-D_GNU_SOURCE",
           "-Werror=implicit-function-declaration", "-Werror=incompatible-pointer-types",
           "-Werror=int-conversion",
           "-I", oracle.REF_SRC, "-I", os.path.join(ROOT, "oracle", "shim"),
           "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "c", "port_dropin.c"), *units,
           "-L", PKG, "-lqmoe", f"-Wl,-rpath,{PKG}", "-lm", "-ldl", "-lpthread", "-o", str(exe)]
    p = subprocess.run(cmd, capture_output=True, text=True)
    assert p.returncode == 0, p.stderr[-3000:]
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "drop-in resolved: 1" in r.stdout, r.stdout + r.stderr
