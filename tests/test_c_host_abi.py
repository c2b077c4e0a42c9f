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
