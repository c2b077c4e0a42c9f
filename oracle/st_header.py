"""TEST INFRASTRUCTURE ONLY: a pure-Python restatement of the reference's
safetensors header validation (SafeTensorIndex._parse, src/colibri_runtime/
storage.py:92-152), the checker of the library's qmoe_ckpt_open.

parse(raw, prefix_name) takes a whole file's bytes and returns
{name: (dtype, shape, absolute offset, nbytes)} or raises ValueError with the
reference's message. Pinned against the reference's own SafeTensorIndex by the
corpus in tests/golden/st_headers.json (tests/golden/make_st_golden.py).
"""
from __future__ import annotations

import json
import math
import struct

DTYPE_SIZES = {"BOOL": 1, "U8": 1, "I8": 1, "U16": 2, "I16": 2, "U32": 4, "I32": 4, "U64": 8,
               "I64": 8, "F16": 2, "BF16": 2, "F32": 4, "F64": 8}


def _is_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


def parse(raw: bytes, path: str = "file") -> dict:
    if len(raw) < 8:
        raise ValueError(f"truncated safetensors header: {path}")
    header_len = struct.unpack("<Q", raw[:8])[0]
    file_size = len(raw)
    if header_len > file_size - 8:
        raise ValueError(f"truncated safetensors JSON: {path}")
    header = json.loads(raw[8:8 + header_len])
    if not isinstance(header, dict):
        raise ValueError(f"safetensors header must be an object: {path}")
    base = 8 + header_len
    tensors, ranges = {}, []
    for stored, meta in header.items():
        if stored == "__metadata__":
            continue
        if not isinstance(meta, dict):
            raise ValueError(f"invalid safetensors entry in {path}")
        name = stored.removeprefix("language_model.")
        dtype = meta.get("dtype")
        if not isinstance(dtype, str) or dtype not in DTYPE_SIZES:
            raise ValueError(f"unsupported safetensors dtype {dtype} for {name}")
        offsets, shape = meta.get("data_offsets"), meta.get("shape")
        if not isinstance(offsets, list) or len(offsets) != 2 or not isinstance(shape, list):
            raise ValueError(f"invalid safetensors metadata for {name}")
        if not all(_is_int(v) for v in offsets):
            raise ValueError(f"invalid data offsets for {name}")
        if not all(_is_int(v) and v >= 0 for v in shape):
            raise ValueError(f"invalid tensor shape for {name}")
        lo, hi = offsets
        expected = math.prod(shape) * DTYPE_SIZES[dtype]
        if lo < 0 or hi < lo or hi - lo != expected or hi > file_size - base:
            raise ValueError(f"invalid safetensors range for {name}")
        if name in tensors:
            raise ValueError(f"duplicate tensor {name}")
        tensors[name] = (dtype, tuple(shape), base + lo, hi - lo)
        ranges.append((lo, hi, name))
    end = 0
    for lo, hi, name in sorted(ranges):
        if lo < end:
            raise ValueError(f"overlapping safetensors ranges for {name}")
        end = hi
    return tensors
