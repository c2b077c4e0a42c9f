"""include/qmoe.h from C: tests/c/host_abi.c compiled as C11 and as C++17
(pedantic, warnings as errors), linked against libqmoe.so and run; it exercises the
host-only objects (expert cache, route predictor, checkpoint index) through the
C ABI without a GPU."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "qwen3.8-flash-next_b200")


@pytest.mark.parametrize("lang", ["c", "c++"])
def test_host_abi_from_c(built, tmp_path, lang):
    exe = tmp_path / f"host_abi_{lang}"
    cc = ["gcc", "-std=c11"] if lang == "c" else ["g++", "-std=c++17", "-x", "c++"]
    src = os.path.join(ROOT, "tests", "c", "host_abi.c")
    cmd = cc + ["-Wall", "-Wextra", "-Wpedantic", "-Werror", "-I", os.path.join(ROOT, "include"), src]
    if lang == "c++":
        cmd += ["-x", "none"]
    cmd += ["-L", PKG, "-lqmoe", f"-Wl,-rpath,{PKG}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    d = tmp_path / "ck"
    d.mkdir()
    p = subprocess.run([str(exe), str(d)], capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "0 failure(s)" in p.stdout


def test_struct_layouts_match_the_bindings(built, tmp_path):
    """Each struct of qmoe.h has the size and field offsets of its ctypes
    mirror in qmoe.py (a mismatch would corrupt arguments silently)."""
    import ctypes as C

    import qmoe
    exe = tmp_path / "layouts"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c", "layouts.c"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    mirror = {"qmoe_err": qmoe.Err, "qmoe_config": qmoe.Config, "qmoe_q4": qmoe.Q4,
              "qmoe_layer_weights": qmoe.LayerWeights, "qmoe_cache_stats": qmoe.CacheStats,
              "qmoe_stats": qmoe.Stats, "qmoe_token_args": qmoe.TokenArgs,
              "qmoe_synth_size": qmoe.SynthSize, "qmoe_tensor_info": qmoe.TensorInfo,
              "qmoe_io_stats": qmoe.IOStats, "qmoe_hc_weights": qmoe.HCWeights}
    n = 0
    for line in out.splitlines():
        name, field, value = line.split()
        T = mirror[name]
        if field == "-":
            assert C.sizeof(T) == int(value), (name, C.sizeof(T), value)
        else:
            assert getattr(T, field).offset == int(value), (name, field)
        n += 1
    assert n > 25
