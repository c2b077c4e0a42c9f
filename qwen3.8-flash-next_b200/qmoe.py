"""ctypes binding of libqmoe.so (include/qmoe.h) for Python callers.

The product is the C library; this module only marshals arguments. It is what
the tests and bench.py use to reach the C ABI, and it is the binding a Python
host of the reference runtime would add. Loading fails
loudly when libqmoe.so has not been built; there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqmoe.so")

QMOE_POLICY_LRU, QMOE_POLICY_LFU, QMOE_POLICY_ADAPTIVE = 0, 1, 2
QMOE_F32, QMOE_BF16 = 0, 1


class Err(C.Structure):
    _fields_ = [("msg", C.c_char * 512)]

    def text(self) -> str:
        return self.msg.decode(errors="replace")


class Config(C.Structure):
    _fields_ = [
        ("hidden", C.c_int), ("num_experts", C.c_int), ("top_k", C.c_int),
        ("moe_inter", C.c_int), ("group_size", C.c_int), ("bits", C.c_int),
        ("num_layers", C.c_int), ("max_tokens", C.c_int), ("pool_bytes", C.c_uint64),
        ("policy", C.c_int), ("prefetch_depth", C.c_int), ("device", C.c_int),
        ("ep_rank", C.c_int), ("ep_world", C.c_int),
    ]


class Q4(C.Structure):
    _fields_ = [("q", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p)]


class LayerWeights(C.Structure):
    _fields_ = [
        ("router", C.c_void_p), ("shared_gate", C.c_void_p), ("logit_bias", C.c_void_p),
        ("gate", Q4), ("up", Q4), ("down", Q4),
        ("sh_gate", Q4), ("sh_up", Q4), ("sh_down", Q4),
    ]


class CacheStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in
                ("hits", "misses", "evictions", "rejected", "pinned",
                 "bytes", "peak_bytes", "size", "hot")]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


class Stats(C.Structure):
    _fields_ = [
        ("expert_loads", C.c_uint64), ("expert_bytes", C.c_uint64),
        ("expert_wait_seconds", C.c_double), ("prefill_calls", C.c_uint64),
        ("decode_calls", C.c_uint64), ("forward_seconds", C.c_double),
        ("prefetch_issued", C.c_uint64), ("prefetch_hits", C.c_uint64),
        ("routed_lookups", C.c_uint64), ("routed_hits", C.c_uint64),
        ("prefetch_wasted", C.c_uint64), ("expert_waves", C.c_uint64),
    ]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


class SynthSize(C.Structure):
    _fields_ = [(n, C.c_size_t) for n in
                ("router", "shared_gate", "expert_q", "expert_sb", "down_q", "down_sb",
                 "sh_q", "sh_sb", "sh_down_q", "sh_down_sb")]


class HCWeights(C.Structure):
    """qmoe_hc_weights: one layer's hyper connection around the MoE block."""
    _fields_ = [
        ("hc", C.c_int), ("lowrank", C.c_int), ("norm", C.c_void_p),
        ("down", Q4), ("down_bf16", C.c_void_p), ("up", Q4), ("up_bf16", C.c_void_p),
        ("inject", C.c_void_p),
    ]


class TokenArgs(C.Structure):
    """qmoe_token_args: one decode token for qmoe_forward_token_noalloc."""
    _fields_ = [
        ("hidden", C.c_int), ("num_experts", C.c_int), ("top_k", C.c_int),
        ("moe_inter", C.c_int), ("group_size", C.c_int),
        ("x", C.c_void_p), ("x_dtype", C.c_int), ("out", C.c_void_p),
        ("router", C.c_void_p), ("shared_gate", C.c_void_p), ("logit_bias", C.c_void_p),
        ("pool", C.c_void_p), ("slot_of", C.c_void_p), ("shared_slot", C.c_void_p),
    ]


NOALLOC_SCRATCH_BYTES = 64 * 1024

# safetensors dtypes (QMOE_ST_*): name, numpy type
ST_DTYPES = [("BOOL", np.bool_), ("U8", np.uint8), ("I8", np.int8), ("U16", np.uint16),
             ("I16", np.int16), ("U32", np.uint32), ("I32", np.int32), ("U64", np.uint64),
             ("I64", np.int64), ("F16", np.float16), ("BF16", np.uint16), ("F32", np.float32),
             ("F64", np.float64)]


class TensorInfo(C.Structure):
    _fields_ = [("dtype", C.c_int), ("ndim", C.c_int), ("shape", C.c_int64 * 8),
                ("nbytes", C.c_uint64), ("row_bytes", C.c_uint64), ("file", C.c_int),
                ("offset", C.c_uint64)]


class IOStats(C.Structure):
    _fields_ = [("pread_calls", C.c_uint64), ("bytes_read", C.c_uint64),
                ("rows_read", C.c_uint64), ("tensors_read", C.c_uint64),
                ("read_seconds", C.c_double)]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


# every symbol include/qmoe.h declares, with (restype, argtypes)
_P = C.c_void_p
SIGNATURES = {
    "qmoe_create": (_P, [C.POINTER(Config), C.POINTER(Err)]),
    "qmoe_destroy": (None, [_P]),
    "qmoe_slot_bytes": (C.c_size_t, [C.POINTER(Config)]),
    "qmoe_upload_layer": (C.c_int, [_P, C.c_int, C.POINTER(LayerWeights), C.POINTER(Err)]),
    "qmoe_forward": (C.c_int, [_P, C.c_int, _P, C.c_int, _P, C.POINTER(Err)]),
    "qmoe_forward_dev": (C.c_int, [_P, C.c_int, _P, C.c_int, C.c_int, _P, _P, C.POINTER(Err)]),
    "qmoe_ep_unique_id": (C.c_int, [_P, C.POINTER(Err)]),
    "qmoe_ep_plan_host": (C.c_int, [_P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P, _P]),
    "qmoe_ep_connect": (C.c_int, [_P, _P, C.POINTER(Err)]),
    "qmoe_forward_ep": (C.c_int, [_P, C.c_int, _P, C.c_int, C.c_int, _P, _P, C.POINTER(Err)]),
    "qmoe_sync": (C.c_int, [_P, C.POINTER(Err)]),
    "qmoe_forward_stack": (C.c_int, [_P, C.c_int, C.c_int, _P, C.c_int, C.c_float, _P,
                                     C.POINTER(Err)]),
    "qmoe_synth_layer_dev": (C.c_int, [_P, C.c_int, C.c_uint64, C.c_double, C.POINTER(Err)]),
    "qmoe_last_routing": (C.c_int, [_P, _P, _P, _P, C.POINTER(Err)]),
    "qmoe_forward_token_noalloc": (C.c_int, [C.POINTER(TokenArgs), _P, C.POINTER(Err)]),
    "qmoe_upload_hc": (C.c_int, [_P, C.c_int, C.POINTER(HCWeights), C.POINTER(Err)]),
    "qmoe_forward_hc": (C.c_int, [_P, C.c_int, _P, C.c_int, _P, C.POINTER(Err)]),
    "qmoe_capture_begin": (C.c_int, [_P, _P, C.POINTER(Err)]),
    "qmoe_capture_end": (_P, [_P, _P, C.POINTER(Err)]),
    "qmoe_graph_launch": (C.c_int, [_P, _P, C.POINTER(Err)]),
    "qmoe_graph_free": (None, [_P]),
    "qmoe_profile_forward": (C.c_int, [_P, C.c_int, _P, C.c_int, C.c_int, _P, C.c_int,
                                       C.POINTER(C.c_double), C.c_int, C.POINTER(C.c_int),
                                       C.POINTER(Err)]),
    "qmoe_expert_peek": (C.c_int, [_P, C.c_int, C.c_int]),
    "qmoe_expert_get": (C.c_int, [_P, C.c_int, C.c_int]),
    "qmoe_experts_load": (C.c_int, [_P, C.c_int, _P, C.c_size_t, C.POINTER(Err)]),
    "qmoe_expert_pin": (C.c_int, [_P, C.c_int, C.c_int]),
    "qmoe_expert_unpin": (C.c_int, [_P, C.c_int, C.c_int]),
    "qmoe_expert_mark_hot": (C.c_int, [_P, C.c_int, C.c_int, C.c_int]),
    "qmoe_cache_snapshot": (C.c_int, [_P, C.POINTER(CacheStats)]),
    "qmoe_stats_get": (C.c_int, [_P, C.POINTER(Stats)]),
    "qmoe_prefetch": (C.c_int, [_P, C.c_int, _P, C.c_size_t]),
    "qmoe_record_route": (None, [_P, C.c_int, _P, C.c_size_t]),
    "qmoe_prefetch_predictions": (C.c_int, [_P, C.c_int, _P, C.c_size_t]),
    "qmoe_cache_new": (_P, [C.c_uint64, C.c_int, C.c_int]),
    "qmoe_cache_free": (None, [_P]),
    "qmoe_cache_peek": (C.c_int, [_P, C.c_uint64, C.POINTER(C.c_uint64)]),
    "qmoe_cache_get": (C.c_int, [_P, C.c_uint64, C.POINTER(C.c_uint64)]),
    "qmoe_cache_put": (C.c_int, [_P, C.c_uint64, C.c_uint64, C.c_uint64, C.c_int, C.c_int,
                                 _P, C.c_size_t, C.POINTER(C.c_size_t)]),
    "qmoe_cache_pin": (C.c_int, [_P, C.c_uint64]),
    "qmoe_cache_unpin": (C.c_int, [_P, C.c_uint64]),
    "qmoe_cache_mark_hot": (C.c_int, [_P, C.c_uint64, C.c_int]),
    "qmoe_cache_erase": (C.c_int, [_P, C.c_uint64, C.POINTER(C.c_uint64)]),
    "qmoe_cache_stats_get": (CacheStats, [_P]),
    "qmoe_synth_sizes": (C.c_int, [C.POINTER(Config), C.POINTER(SynthSize)]),
    "qmoe_synth_layer": (C.c_int, [C.POINTER(Config), C.c_uint64, C.c_int,
                                   C.POINTER(LayerWeights), C.c_int, C.c_int]),
    "qmoe_synth_tokens": (None, [C.c_uint64, C.c_uint64, C.c_int, C.c_int, _P]),
    "qmoe_synth_zipf_bias": (None, [C.c_uint64, C.c_int, C.c_int, C.c_double, _P]),
    "qmoe_ckpt_open": (_P, [C.c_char_p, C.c_int, C.POINTER(Err)]),
    "qmoe_ckpt_close": (None, [_P]),
    "qmoe_ckpt_count": (C.c_size_t, [_P]),
    "qmoe_ckpt_name": (C.c_char_p, [_P, C.c_size_t]),
    "qmoe_ckpt_find": (C.c_int, [_P, C.c_char_p, C.POINTER(TensorInfo)]),
    "qmoe_ckpt_read_tensor": (C.c_int, [_P, C.c_char_p, _P, C.c_size_t, C.POINTER(Err)]),
    "qmoe_ckpt_read_rows": (C.c_int, [_P, C.c_char_p, _P, C.c_size_t, _P, C.c_size_t,
                                      C.POINTER(Err)]),
    "qmoe_ckpt_io_stats": (C.c_int, [_P, C.POINTER(IOStats)]),
    "qmoe_ckpt_layer_bytes": (C.c_size_t, [C.POINTER(Config)]),
    "qmoe_ckpt_read_layer": (C.c_int, [_P, C.POINTER(Config), C.c_int, _P, C.c_size_t,
                                       C.POINTER(LayerWeights), C.POINTER(Err)]),
    "qmoe_ckpt_pack_experts": (C.c_int, [_P, C.POINTER(Config), C.c_int, _P, C.c_size_t, _P,
                                         C.c_size_t, C.POINTER(Err)]),
    "qmoe_pack_expert": (C.c_int, [C.POINTER(Config), C.POINTER(LayerWeights), C.c_int, _P]),
    "qmoe_upload_layer_ckpt": (C.c_int, [_P, C.c_int, _P, C.c_int, C.POINTER(Err)]),
    "qmoe_predictor_new": (_P, [C.c_int, C.c_int]),
    "qmoe_predictor_free": (None, [_P]),
    "qmoe_predictor_record": (C.c_int, [_P, _P, C.c_int, _P, C.c_size_t, _P]),
    "qmoe_predictor_predict": (C.c_int, [_P, C.c_int, _P, C.c_size_t, C.c_int, _P,
                                         C.POINTER(C.c_int), _P, C.POINTER(C.c_int)]),
    "qmoe_predictor_count": (C.c_uint64, [_P, C.c_int, C.c_int]),
    "qmoe_predictor_routes": (C.c_uint64, [_P]),
    "qmoe_predictor_frequent": (C.c_int, [_P, C.c_int, _P, _P, _P]),
    "qmoe_ctx_predictor": (_P, [_P]),
    "qmoe_version": (C.c_char_p, []),
}

_lib = None


def lib() -> C.CDLL:
    """Loads libqmoe.so once; raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} missing: run `make -C {HERE}` first")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def ptr(a) -> int | None:
    return None if a is None else a.ctypes.data


def ep_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for qmoe_ep_connect; made on one rank
    and handed to the others by the caller."""
    buf = C.create_string_buffer(128)
    err = Err()
    if lib().qmoe_ep_unique_id(buf, C.byref(err)) != 0:
        raise QmoeError(err.text())
    return buf.raw


def make_config(d, E, k, I, g=64, layers=1, max_tokens=1, pool_bytes=0,
                policy=QMOE_POLICY_ADAPTIVE, prefetch=2, device=0, ep_rank=0, ep_world=0) -> Config:
    return Config(d, E, k, I, g, 4, layers, max_tokens, pool_bytes, policy, prefetch, device,
                  ep_rank, ep_world)


class SynthLayer:
    """One seeded synthetic layer in the reference checkpoint layout (numpy)."""

    def __init__(self, cfg: Config, seed: int, layer: int = 0, zipf_s: float | None = None):
        L = lib()
        sz = SynthSize()
        if L.qmoe_synth_sizes(C.byref(cfg), C.byref(sz)) != 0:
            raise ValueError("unsupported synthetic shape")
        self.cfg = cfg
        self.d, self.E, self.k = cfg.hidden, cfg.num_experts, cfg.top_k
        self.I, self.g = cfg.moe_inter, cfg.group_size
        u16, u32 = np.uint16, np.uint32
        self.router = np.empty(sz.router, u16)
        self.shared_gate = np.empty(sz.shared_gate, u16)
        self.t = {}
        for name, nq, nsb in (("gate", sz.expert_q, sz.expert_sb), ("up", sz.expert_q, sz.expert_sb),
                              ("down", sz.down_q, sz.down_sb), ("sh_gate", sz.sh_q, sz.sh_sb),
                              ("sh_up", sz.sh_q, sz.sh_sb), ("sh_down", sz.sh_down_q, sz.sh_down_sb)):
            self.t[name] = (np.empty(nq, u32), np.empty(nsb, u16), np.empty(nsb, u16))
        self.logit_bias = None
        if zipf_s is not None:
            self.logit_bias = np.empty(self.E, np.float32)
            L.qmoe_synth_zipf_bias(seed, layer, self.E, zipf_s, ptr(self.logit_bias))
        w = self.weights()
        if L.qmoe_synth_layer(C.byref(cfg), seed, layer, C.byref(w), 0, 0) != 0:
            raise ValueError("qmoe_synth_layer failed")

    def weights(self) -> LayerWeights:
        def q4(n):
            q, s, b = self.t[n]
            return Q4(ptr(q), ptr(s), ptr(b))
        return LayerWeights(ptr(self.router), ptr(self.shared_gate), ptr(self.logit_bias),
                            q4("gate"), q4("up"), q4("down"), q4("sh_gate"), q4("sh_up"),
                            q4("sh_down"))


def _bf16_bits(a) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


class SynthHC:
    """Seeded synthetic hyper-connection weights of one layer (numpy, in the
    layout qmoe_upload_hc takes): hc_norm near 1 (bf16-valued fp32), the two
    low-rank mixers q4 (nibbles uniform, scales |N(0, 0.02)|, biases -8 x
    scale; biases=False leaves them absent) or dense bf16 N(0, 0.02), and
    block_inject bf16 N(0, 0.02) [hc, hc*d]. Draws come from numpy's
    default_rng(seed) in that order."""

    def __init__(self, d: int, hc: int, lowrank: int, seed: int, q4: bool = True, biases: bool = True):
        rng = np.random.default_rng(seed)
        self.d, self.hc, self.lowrank, hd = d, hc, lowrank, hc * d
        norm = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
        self.norm = (_bf16_bits(norm).astype(np.uint32) << 16).view(np.float32)
        self.inject = _bf16_bits(0.02 * rng.standard_normal((hc, hd)))
        self.parts = {}
        for name, rows, cols in (("down", lowrank, hd), ("up", hd, lowrank)):
            if q4:
                q = rng.integers(0, 2 ** 32, size=(rows, cols // 8), dtype=np.uint32)
                sc = _bf16_bits(np.abs(0.02 * rng.standard_normal((rows, cols // 64))))
                bi = (_bf16_bits(-8.0 * (sc.astype(np.uint32) << 16).view(np.float32))
                      if biases else None)
                self.parts[name] = (q, sc, bi, None)
            else:
                self.parts[name] = (None, None, None,
                                    _bf16_bits(0.02 * rng.standard_normal((rows, cols))))


def synth_tokens(seed: int, stream: int, n: int, d: int) -> np.ndarray:
    x = np.empty((n, d), np.float32)
    lib().qmoe_synth_tokens(seed, stream, n, d, ptr(x))
    return x


class QmoeError(RuntimeError):
    pass


def pack_expert(cfg: Config, w: LayerWeights, expert: int) -> np.ndarray:
    """One expert of host weights in the HBM slot layout (expert -1: the
    shared expert)."""
    L = lib()
    out = np.empty(L.qmoe_slot_bytes(C.byref(cfg)), np.uint8)
    if L.qmoe_pack_expert(C.byref(cfg), C.byref(w), expert, ptr(out)) != 0:
        raise QmoeError(f"qmoe_pack_expert failed for expert {expert}")
    return out


class Predictor:
    """A host-side route predictor (qmoe_predictor_*): ExpertStore's route
    statistics and prefetch prediction. `cache` is an optional qmoe_cache
    handle whose hot marks record() sets."""

    def __init__(self, num_layers: int, num_experts: int, depth: int = 2):
        self.h = lib().qmoe_predictor_new(num_layers, num_experts)
        if not self.h:
            raise QmoeError("qmoe_predictor_new failed")
        self.L, self.E, self.depth = num_layers, num_experts, depth

    def close(self):
        if self.h:
            lib().qmoe_predictor_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def record(self, layer: int, routed, cache=None) -> list[int]:
        r = np.ascontiguousarray(np.asarray(list(routed), np.int32))
        sel = np.empty(self.E, np.int32)
        ns = lib().qmoe_predictor_record(self.h, cache, layer, ptr(r), len(r), ptr(sel))
        if ns < 0:
            raise ValueError("qmoe_predictor_record refused the routing")
        return sel[:ns].tolist()

    def predict(self, layer: int, selected) -> list[tuple[int, int]]:
        """The (layer, expert) prefetch requests, in the order issued."""
        s = np.ascontiguousarray(np.asarray(list(selected), np.int32))
        pick, nxt = np.empty(64, np.int64), np.empty(64, np.int64)
        npick, nnext = C.c_int(), C.c_int()
        if lib().qmoe_predictor_predict(self.h, layer, ptr(s), len(s), self.depth, ptr(pick),
                                        C.byref(npick), ptr(nxt), C.byref(nnext)):
            raise ValueError("qmoe_predictor_predict refused the selection")
        return [(layer, int(e)) for e in pick[:npick.value]] + \
               [(layer + 1, int(e)) for e in nxt[:nnext.value]]

    def count(self, layer: int, expert: int) -> int:
        return lib().qmoe_predictor_count(self.h, layer, expert)

    def routes(self) -> int:
        return lib().qmoe_predictor_routes(self.h)

    def frequent(self, n: int = 20) -> list[tuple[int, int, int]]:
        lay, ex, cnt = np.empty(n, np.int32), np.empty(n, np.int32), np.empty(n, np.uint64)
        got = lib().qmoe_predictor_frequent(self.h, n, ptr(lay), ptr(ex), ptr(cnt))
        return [(int(lay[i]), int(ex[i]), int(cnt[i])) for i in range(got)]


class Checkpoint:
    """A directory of safetensors files (qmoe_ckpt_*): the index, whole-tensor
    and row reads, and the MoE layer / expert-slot readers."""

    def __init__(self, path, io_workers: int = 4):
        err = Err()
        self.h = lib().qmoe_ckpt_open(os.fsencode(path), io_workers, C.byref(err))
        if not self.h:
            raise QmoeError(err.text())

    def close(self):
        if self.h:
            lib().qmoe_ckpt_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *_):
        self.close()

    def __getattribute__(self, name):
        # every reader method needs an open index (storage.py:265-268)
        if name in ("names", "find", "read_tensor", "read_rows", "stats", "read_layer",
                    "pack_experts") and object.__getattribute__(self, "h") is None:
            raise QmoeError("checkpoint index is closed")
        return object.__getattribute__(self, name)

    def names(self) -> list[str]:
        L = lib()
        return [L.qmoe_ckpt_name(self.h, i).decode("utf-8", "surrogatepass")
                for i in range(L.qmoe_ckpt_count(self.h))]

    def find(self, name: str) -> dict | None:
        t = TensorInfo()
        if lib().qmoe_ckpt_find(self.h, name.encode("utf-8", "surrogatepass"), C.byref(t)) != 0:
            return None
        return {"dtype": ST_DTYPES[t.dtype][0], "shape": tuple(t.shape[:t.ndim]),
                "nbytes": t.nbytes, "row_bytes": t.row_bytes, "file": t.file, "offset": t.offset}

    def _info(self, name):
        t = TensorInfo()
        if lib().qmoe_ckpt_find(self.h, name.encode(), C.byref(t)) != 0:
            raise KeyError(name)
        return t, ST_DTYPES[t.dtype][1], tuple(t.shape[:t.ndim])

    def read_tensor(self, name: str) -> np.ndarray:
        t, dt, shape = self._info(name)
        out = np.empty(t.nbytes, np.uint8)
        err = Err()
        if lib().qmoe_ckpt_read_tensor(self.h, name.encode(), ptr(out), out.nbytes, C.byref(err)):
            raise QmoeError(err.text())
        return out.view(dt).reshape(shape)

    def read_rows(self, name: str, rows) -> np.ndarray:
        t, dt, shape = self._info(name)
        r = np.ascontiguousarray(np.asarray(list(rows), np.int64))
        out = np.empty(len(r) * t.row_bytes, np.uint8)
        err = Err()
        if lib().qmoe_ckpt_read_rows(self.h, name.encode(), ptr(r), len(r), ptr(out), out.nbytes,
                                     C.byref(err)):
            raise QmoeError(err.text())
        return out.view(dt).reshape((len(r),) + shape[1:])

    def stats(self) -> dict:
        s = IOStats()
        lib().qmoe_ckpt_io_stats(self.h, C.byref(s))
        return s.as_dict()

    def read_layer(self, cfg: Config, layer: int):
        """(buffer, LayerWeights pointing into it) for qmoe_upload_layer."""
        L = lib()
        buf = np.empty(L.qmoe_ckpt_layer_bytes(C.byref(cfg)), np.uint8)
        w = LayerWeights()
        err = Err()
        if L.qmoe_ckpt_read_layer(self.h, C.byref(cfg), layer, ptr(buf), buf.nbytes, C.byref(w),
                                  C.byref(err)):
            raise QmoeError(err.text())
        return buf, w

    def pack_experts(self, cfg: Config, layer: int, ids) -> np.ndarray:
        L = lib()
        r = np.ascontiguousarray(np.asarray(list(ids), np.int64))
        sb = L.qmoe_slot_bytes(C.byref(cfg))
        out = np.empty((len(r), sb), np.uint8)
        err = Err()
        if L.qmoe_ckpt_pack_experts(self.h, C.byref(cfg), layer, ptr(r), len(r), ptr(out),
                                    out.nbytes, C.byref(err)):
            raise QmoeError(err.text())
        return out


class Context:
    """Owns one qmoe_ctx (one GPU)."""

    def __init__(self, cfg: Config):
        self.cfg = cfg
        err = Err()
        self.h = lib().qmoe_create(C.byref(cfg), C.byref(err))
        if not self.h:
            raise QmoeError(err.text())

    def close(self):
        if self.h:
            lib().qmoe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _chk(self, rc, err):
        if rc != 0:
            raise QmoeError(err.text())

    def upload(self, layer: int, s: SynthLayer):
        err = Err()
        w = s.weights()
        self._chk(lib().qmoe_upload_layer(self.h, layer, C.byref(w), C.byref(err)), err)

    def upload_ckpt(self, layer: int, ck: Checkpoint, ckpt_layer: int | None = None):
        """Checkpoint layer ckpt_layer (default: layer) into this context's layer."""
        err = Err()
        rc = lib().qmoe_upload_layer_ckpt(self.h, layer, ck.h, layer if ckpt_layer is None else ckpt_layer,
                                          C.byref(err))
        self._chk(rc, err)

    def forward(self, layer: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        n = x.shape[0]
        out = np.empty((n, self.cfg.hidden), np.float32)
        err = Err()
        self._chk(lib().qmoe_forward(self.h, layer, ptr(x), n, ptr(out), C.byref(err)), err)
        return out

    def forward_dev(self, layer: int, x_ptr: int, x_dtype: int, n: int, out_ptr: int,
                    stream: int | None = None):
        err = Err()
        self._chk(lib().qmoe_forward_dev(self.h, layer, x_ptr, x_dtype, n, out_ptr, stream,
                                         C.byref(err)), err)

    def ep_connect(self, uid: bytes):
        """Joins the expert-parallel group (collective over the ep_world ranks)."""
        err = Err()
        buf = C.create_string_buffer(bytes(uid), 128)
        self._chk(lib().qmoe_ep_connect(self.h, buf, C.byref(err)), err)

    def forward_ep(self, layer: int, x_ptr: int, x_dtype: int, n: int, out_ptr: int,
                   stream: int | None = None):
        """Collective forward of this rank's n tokens (device pointers)."""
        err = Err()
        self._chk(lib().qmoe_forward_ep(self.h, layer, x_ptr, x_dtype, n, out_ptr, stream,
                                        C.byref(err)), err)

    def upload_hc(self, layer: int, hcw):
        """A layer's hyper-connection weights: an object with hc, lowrank, norm
        (fp32 [hc*d]), inject (bf16 bits [hc, hc*d]) and parts["down"] /
        parts["up"] = (q, scales, biases, dense_bf16), q4 or dense."""
        def ptr_(a):
            return None if a is None else a.ctypes.data
        dq, ds, db, dbf = hcw.parts["down"]
        uq, us, ub, ubf = hcw.parts["up"]
        w = HCWeights(hcw.hc, hcw.lowrank, ptr_(hcw.norm), Q4(ptr_(dq), ptr_(ds), ptr_(db)), ptr_(dbf),
                      Q4(ptr_(uq), ptr_(us), ptr_(ub)), ptr_(ubf), ptr_(hcw.inject))
        err = Err()
        self._chk(lib().qmoe_upload_hc(self.h, layer, C.byref(w), C.byref(err)), err)

    def forward_hc(self, layer: int, h_ptr: int, n: int, stream: int | None = None):
        """gated_residual, the MoE block and the inject-add; h: device fp32
        [n, hc*d], updated in place."""
        err = Err()
        self._chk(lib().qmoe_forward_hc(self.h, layer, h_ptr, n, stream, C.byref(err)), err)

    def synth_layer_dev(self, layer: int, seed: int, zipf_s: float = 0.0):
        """The seeded synthetic layer generated on the device (resident contexts)."""
        err = Err()
        self._chk(lib().qmoe_synth_layer_dev(self.h, layer, seed, zipf_s, C.byref(err)), err)

    def forward_stack(self, l0: int, l1: int, h_ptr: int, n: int, eps: float = 1e-6,
                      stream: int | None = None):
        """h <- h + MoE_l(RMSNorm(h)) for layers [l0, l1); h: device fp32 [n, d]."""
        err = Err()
        self._chk(lib().qmoe_forward_stack(self.h, l0, l1, h_ptr, n, eps, stream, C.byref(err)),
                  err)

    def sync(self):
        err = Err()
        self._chk(lib().qmoe_sync(self.h, C.byref(err)), err)

    def routing(self, n: int):
        k = self.cfg.top_k
        idx = np.empty((n, k), np.int32)
        w = np.empty((n, k), np.float32)
        g = np.empty(n, np.float32)
        err = Err()
        self._chk(lib().qmoe_last_routing(self.h, ptr(idx), ptr(w), ptr(g), C.byref(err)), err)
        return idx, w, g

    def experts_load(self, layer: int, ids):
        ids = np.ascontiguousarray(ids, np.int64)
        err = Err()
        self._chk(lib().qmoe_experts_load(self.h, layer, ptr(ids), ids.size, C.byref(err)), err)

    def cache_stats(self) -> dict:
        s = CacheStats()
        lib().qmoe_cache_snapshot(self.h, C.byref(s))
        return s.as_dict()

    def stats(self) -> dict:
        s = Stats()
        lib().qmoe_stats_get(self.h, C.byref(s))
        return s.as_dict()

    def capture_begin(self, stream=None):
        err = Err()
        self._chk(lib().qmoe_capture_begin(self.h, stream, C.byref(err)), err)

    def capture_end(self, stream=None) -> "Graph":
        err = Err()
        g = lib().qmoe_capture_end(self.h, stream, C.byref(err))
        if not g:
            raise QmoeError(err.text())
        return Graph(g)

    def profile_forward(self, layer, x_ptr, x_dtype, n, out_ptr, reps):
        """Mean device microseconds per kernel launch [router, topk, gateup, down]."""
        us = (C.c_double * 8)()
        nk = C.c_int()
        err = Err()
        self._chk(lib().qmoe_profile_forward(self.h, layer, x_ptr, x_dtype, n, out_ptr, reps,
                                             us, 8, C.byref(nk), C.byref(err)), err)
        return [us[i] for i in range(nk.value)]


class Graph:
    """An instantiated CUDA graph of captured forward calls."""

    def __init__(self, h):
        self.h = h

    def launch(self, stream=None):
        err = Err()
        if lib().qmoe_graph_launch(self.h, stream, C.byref(err)) != 0:
            raise QmoeError(err.text())

    def close(self):
        if self.h:
            lib().qmoe_graph_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
