"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU checkers.

- `restatement()`  -> _build/liboracle.so, the C restatement of the reference
  runtime's moe_forward (moe_oracle.c).
- `reference()`    -> _ref/libmoe_ref.so, the reference's own moe_forward built
  unmodified from its sources (None when that build is absent, e.g. on a
  machine without the reference sources and without a prebuilt copy).

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline legs use this
module, always as the checker or the timed CPU baseline, never as a product
path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmoe_ref.so")
REF_SRC = "/root/reference/c/src"


class OracleLayer(C.Structure):
    _fields_ = [("d", C.c_int), ("E", C.c_int), ("k", C.c_int), ("I", C.c_int), ("g", C.c_int),
                ("router", C.c_void_p), ("shared_gate", C.c_void_p), ("logit_bias", C.c_void_p)] + \
               [(n, C.c_void_p) for n in ("gq", "uq", "dq", "gs", "gb", "us", "ub", "ds", "db",
                                          "sgq", "suq", "sdq", "sgs", "sgb", "sus", "sub", "sds",
                                          "sdb")]


def build(ref: bool = True) -> None:
    """Builds the restatement, and the reference harness when its sources exist."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref and os.path.isdir(REF_SRC):
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


def _p(a):
    return None if a is None else a.ctypes.data


def layer_struct(s) -> OracleLayer:
    """OracleLayer view of a qmoe.SynthLayer (same numpy buffers)."""
    t = s.t
    return OracleLayer(
        s.d, s.E, s.k, s.I, s.g, _p(s.router), _p(s.shared_gate), _p(s.logit_bias),
        _p(t["gate"][0]), _p(t["up"][0]), _p(t["down"][0]),
        _p(t["gate"][1]), _p(t["gate"][2]), _p(t["up"][1]), _p(t["up"][2]),
        _p(t["down"][1]), _p(t["down"][2]),
        _p(t["sh_gate"][0]), _p(t["sh_up"][0]), _p(t["sh_down"][0]),
        _p(t["sh_gate"][1]), _p(t["sh_gate"][2]), _p(t["sh_up"][1]), _p(t["sh_up"][2]),
        _p(t["sh_down"][1]), _p(t["sh_down"][2]))


_V, _I = C.c_void_p, C.c_int
_SIGS = {
    "oracle_moe_forward": (_I, [C.POINTER(OracleLayer), _V, _I, _V, _V, _V, _V]),
    "oracle_route": (_I, [C.POINTER(OracleLayer), _V, _I, _V, _V, _V]),
    "oracle_router_dot": (C.c_float, [_V, _V, _I]),
    "oracle_dequant_q4": (None, [_V, _V, _V, _I, _I, _I, _V]),
    "ref_moe_forward": (_I, [C.POINTER(OracleLayer), _V, _I, _V, _V, _V]),
    "ref_set_threads": (None, [_I]),
    "ref_reset_cache": (None, []),
    "ref_blas_available": (_I, []),
}


class _Impl:
    def __init__(self, path: str, fn: str):
        self.lib = C.CDLL(path)
        for name, (res, args) in _SIGS.items():
            f = getattr(self.lib, name, None)
            if f is not None:
                f.restype = res
                f.argtypes = args
        self.fn = getattr(self.lib, fn)
        self.kind = fn

    def forward(self, s, x: np.ndarray):
        """Returns (out [n,d] fp32, idx [n,k] int32, weights [n,k] fp32)."""
        x = np.ascontiguousarray(x, np.float32)
        n = x.shape[0]
        out = np.empty((n, s.d), np.float32)
        idx = np.empty((n, s.k), np.int32)
        w = np.empty((n, s.k), np.float32)
        L = layer_struct(s)
        if self.kind == "oracle_moe_forward":
            rc = self.fn(C.byref(L), _p(x), n, _p(out), _p(idx), _p(w), None)
        else:
            rc = self.fn(C.byref(L), _p(x), n, _p(out), _p(idx), _p(w))
        if rc != 0:
            raise RuntimeError(f"{self.kind} failed")
        return out, idx, w

    def route(self, s, x: np.ndarray):
        """Routing only (restatement): (idx, weights, logits [n, E])."""
        x = np.ascontiguousarray(x, np.float32)
        n = x.shape[0]
        idx = np.empty((n, s.k), np.int32)
        w = np.empty((n, s.k), np.float32)
        lg = np.empty((n, s.E), np.float32)
        L = layer_struct(s)
        if self.lib.oracle_route(C.byref(L), _p(x), n, _p(idx), _p(w), _p(lg)) != 0:
            raise RuntimeError("oracle_route failed")
        return idx, w, lg

    def router_dot(self, x: np.ndarray, w: np.ndarray) -> float:
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.uint16)
        return self.lib.oracle_router_dot(_p(x), _p(w), x.size)

    def dequant(self, q, scales, biases, rows, cols, group):
        out = np.empty((rows, cols), np.float32)
        q = np.ascontiguousarray(q, np.uint32)
        scales = np.ascontiguousarray(scales, np.float32)
        biases = np.ascontiguousarray(biases, np.float32)
        self.lib.oracle_dequant_q4(_p(q), _p(scales), _p(biases), rows, cols, group, _p(out))
        return out


_cache = {}


def restatement() -> _Impl:
    if "o" not in _cache:
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"{ORACLE_SO} missing: run `make -C {HERE}`")
        _cache["o"] = _Impl(ORACLE_SO, "oracle_moe_forward")
    return _cache["o"]


def reference():
    """The reference's own moe_forward, or None when its build is absent."""
    if "r" not in _cache:
        _cache["r"] = _Impl(REF_SO, "ref_moe_forward") if os.path.exists(REF_SO) else None
    return _cache["r"]
