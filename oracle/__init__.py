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


class OracleHC(C.Structure):
    """oracle_hc: one layer's MoE-side hyper connection."""
    _fields_ = [("d", C.c_int), ("hc", C.c_int), ("lowrank", C.c_int), ("norm", C.c_void_p),
                ("down_q", C.c_void_p), ("down_s", C.c_void_p), ("down_b", C.c_void_p),
                ("down_bf16", C.c_void_p), ("up_q", C.c_void_p), ("up_s", C.c_void_p),
                ("up_b", C.c_void_p), ("up_bf16", C.c_void_p), ("inject", C.c_void_p)]


def _bf16(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even (c/src/util.h:63-71)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


class SynthHC:
    """Seeded hyper-connection weights of one layer (test inputs): hc_norm
    near 1, the two mixer weights q4 (nibbles uniform, scales |N(0, 0.02)|,
    biases -8 scales; `biases=False` leaves them absent) or dense bf16
    N(0, 0.02), block_inject bf16 N(0, 0.02)."""

    def __init__(self, d: int, hc: int, lowrank: int, seed: int, q4: bool = True, biases: bool = True):
        rng = np.random.default_rng(seed)
        self.d, self.hc, self.lowrank, hd = d, hc, lowrank, hc * d
        self.norm = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
        self.norm = (_bf16(self.norm).astype(np.uint32) << 16).view(np.float32)   # bf16 on disk
        self.inject = _bf16(0.02 * rng.standard_normal((hc, hd)))
        self.parts = {}
        for name, rows, cols in (("down", lowrank, hd), ("up", hd, lowrank)):
            if q4:
                q = rng.integers(0, 2 ** 32, size=(rows, cols // 8), dtype=np.uint32)
                sc = _bf16(np.abs(0.02 * rng.standard_normal((rows, cols // 64))))
                bi = _bf16(-8.0 * (sc.astype(np.uint32) << 16).view(np.float32)) if biases else None
                self.parts[name] = (q, sc, bi, None)
            else:
                self.parts[name] = (None, None, None, _bf16(0.02 * rng.standard_normal((rows, cols))))

    def struct(self) -> OracleHC:
        dq, ds, db, dbf = self.parts["down"]
        uq, us, ub, ubf = self.parts["up"]
        return OracleHC(self.d, self.hc, self.lowrank, _p(self.norm), _p(dq), _p(ds), _p(db), _p(dbf),
                        _p(uq), _p(us), _p(ub), _p(ubf), _p(self.inject))


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
    "oracle_gated_residual": (_I, [C.POINTER(OracleHC), _V, _I, _V, _V]),
    "oracle_hc_moe_step": (_I, [C.POINTER(OracleHC), C.POINTER(OracleLayer), _V, _I]),
    "ref_gated_residual": (_I, [C.POINTER(OracleHC), _V, _I, _V, _V]),
    "ref_hc_moe_step": (_I, [C.POINTER(OracleHC), C.POINTER(OracleLayer), _V, _I]),
    "ref_set_threads": (None, [_I]),
    "ref_st_open": (_V, [C.c_char_p, _I, C.c_char_p, _I]),
    "ref_st_close": (None, [_V]),
    "ref_st_count": (_I, [_V]),
    "ref_st_name": (C.c_char_p, [_V, _I]),
    "ref_st_info": (_I, [_V, C.c_char_p, C.POINTER(_I), C.POINTER(_I), _V, C.POINTER(C.c_uint64),
                         C.POINTER(C.c_uint64)]),
    "ref_st_read_rows": (_I, [_V, C.c_char_p, _V, C.c_size_t, _V]),
    "ref_st_rows_read": (C.c_uint64, [_V]),
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

    def _hc(self, name):
        prefix = "oracle_" if self.kind == "oracle_moe_forward" else "ref_"
        return getattr(self.lib, prefix + name)

    def gated_residual(self, H: "SynthHC", h: np.ndarray):
        """(mixed [n, d], inject [n, hc]) of hyper states h [n, hc*d]."""
        h = np.ascontiguousarray(h, np.float32)
        n = h.shape[0]
        mixed = np.empty((n, H.d), np.float32)
        inj = np.empty((n, H.hc), np.float32)
        st = H.struct()
        if self._hc("gated_residual")(C.byref(st), _p(h), n, _p(mixed), _p(inj)) != 0:
            raise RuntimeError("gated_residual failed")
        return mixed, inj

    def hc_moe_step(self, H: "SynthHC", s, h: np.ndarray) -> np.ndarray:
        """h after one layer's gated_residual -> MoE -> inject-add."""
        h = np.array(h, np.float32, order="C", copy=True)
        st, L = H.struct(), layer_struct(s)
        if self._hc("hc_moe_step")(C.byref(st), C.byref(L), _p(h), h.shape[0]) != 0:
            raise RuntimeError("hc_moe_step failed")
        return h

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


class RefIndex:
    """The reference's own safetensors index (c/src/safetensors.c) over a
    directory, through the harness; raises ValueError with its message."""
    DT = ["BOOL", "U8", "I8", "U16", "I16", "U32", "I32", "U64", "I64", "F16", "BF16", "F32", "F64"]

    def __init__(self, lib, path: str, workers: int = 2):
        self.lib = lib
        msg = C.create_string_buffer(512)
        self.h = lib.ref_st_open(os.fsencode(path), workers, msg, 512)
        if not self.h:
            raise ValueError(msg.value.decode("utf-8", "surrogateescape"))

    def close(self):
        if self.h:
            self.lib.ref_st_close(self.h)
            self.h = None

    def table(self):
        out = []
        for i in range(self.lib.ref_st_count(self.h)):
            raw = self.lib.ref_st_name(self.h, i)
            dt, nd = C.c_int(), C.c_int()
            shape = (C.c_int64 * 8)()
            off, nb = C.c_uint64(), C.c_uint64()
            self.lib.ref_st_info(self.h, raw, C.byref(dt), C.byref(nd), shape, C.byref(off), C.byref(nb))
            out.append([raw.decode("utf-8", "surrogatepass"), self.DT[dt.value], list(shape[:nd.value]),
                        off.value, nb.value])
        return sorted(out)

    def read_rows(self, name: str, rows, row_bytes: int) -> np.ndarray:
        r = np.ascontiguousarray(np.asarray(list(rows), np.int64))
        out = np.empty(len(r) * row_bytes + 1, np.uint8)
        if self.lib.ref_st_read_rows(self.h, name.encode(), _p(r), len(r), _p(out)) != 0:
            raise ValueError(f"row read refused for {name}")
        return out[:len(r) * row_bytes]

    def rows_read(self) -> int:
        return self.lib.ref_st_rows_read(self.h)


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
