"""Golden accept/reject vectors for safetensors headers, made by running the
reference's own index (SafeTensorIndex, src/colibri_runtime/storage.py:69-152)
over a seeded corpus of valid and mutated files.

    python tests/golden/make_st_golden.py <reference checkout> tests/golden/st_headers.json

mlx and the native row reader (absent here, and not used by the header parse)
are replaced by empty stub modules; the package's __init__ is skipped. Each
record keeps the whole file (base64), whether the index opened, the exception
type and message otherwise, and the tensor table (name, dtype, shape, absolute
offset, bytes) when it did."""
import base64
import importlib
import json
import os
import struct
import sys
import tempfile
import types

import numpy as np

DTYPES = {"BOOL": 1, "U8": 1, "I8": 1, "U16": 2, "I16": 2, "U32": 4, "I32": 4, "U64": 8, "I64": 8,
          "F16": 2, "BF16": 2, "F32": 4, "F64": 8}
NAMES = ["model.layers.0.mlp.gate.weight", "language_model.model.layers.1.mlp.switch_mlp.up_proj.scales",
         "wéight", "a/b", "x y", "中文", "tab\tname", "q\"uote", "back\\slash", "e"]
SIG = b'{}[]",:0123456789.eE+-tfnul\\ \t\n'


def load_reference(root):
    for name in ("mlx", "mlx.core", "mlx.nn"):
        sys.modules.setdefault(name, types.ModuleType(name))
    pkg = types.ModuleType("colibri_runtime")
    pkg.__path__ = [os.path.join(root, "src", "colibri_runtime")]
    sys.modules["colibri_runtime"] = pkg
    sys.modules["colibri_runtime._rowio"] = types.ModuleType("colibri_runtime._rowio")
    return importlib.import_module("colibri_runtime.storage")


def valid_file(rng):
    """A random well-formed file: 0-5 tensors laid out back to back (with
    gaps sometimes), optional __metadata__, random key order and spacing."""
    n = int(rng.integers(0, 6))
    names = list(rng.choice(NAMES, size=n, replace=False))
    meta, off = {}, 0
    for nm in names:
        dt = str(rng.choice(list(DTYPES)))
        shape = [int(v) for v in rng.integers(0, 4, size=int(rng.integers(0, 4)))]
        nb = int(np.prod(shape)) * DTYPES[dt] if shape else DTYPES[dt]
        off += int(rng.integers(0, 3)) if rng.random() < 0.3 else 0
        meta[nm] = {"dtype": dt, "shape": shape, "data_offsets": [off, off + nb]}
        off += nb
    if rng.random() < 0.5:
        meta["__metadata__"] = {"format": "mlx", "nested": [1, {"k": None}, True, -2.5e3]}
    items = list(meta.items())
    rng.shuffle(items)
    text = json.dumps(dict(items), ensure_ascii=bool(rng.random() < 0.5),
                      indent=int(rng.integers(0, 3)) if rng.random() < 0.3 else None)
    hdr = text.encode()
    return struct.pack("<Q", len(hdr)) + hdr + bytes(int(v) for v in rng.integers(0, 256, off))


def mutate(rng, raw):
    hlen = struct.unpack("<Q", raw[:8])[0]
    hdr, data = bytearray(raw[8:8 + hlen]), raw[8 + hlen:]
    kind = int(rng.integers(0, 8))
    if kind == 0 and hdr:                      # truncate the JSON
        hdr = hdr[:int(rng.integers(0, len(hdr)))]
    elif kind == 1 and hdr:                    # a JSON-significant byte replaced
        hdr[int(rng.integers(0, len(hdr)))] = SIG[int(rng.integers(0, len(SIG)))]
    elif kind == 2 and hdr:                    # any byte replaced
        hdr[int(rng.integers(0, len(hdr)))] = int(rng.integers(1, 256))
    elif kind == 3 and hdr:                    # a byte deleted
        del hdr[int(rng.integers(0, len(hdr)))]
    elif kind == 4:                            # a byte inserted
        hdr.insert(int(rng.integers(0, len(hdr) + 1)), SIG[int(rng.integers(0, len(SIG)))])
    elif kind == 5:                            # the data cut short or grown
        data = data[:int(rng.integers(0, len(data) + 1))] if rng.random() < 0.5 else data + b"\0" * 3
    elif kind == 6:                            # a wrong header length
        return struct.pack("<Q", max(0, hlen + int(rng.integers(-3, 4)))) + bytes(hdr) + data
    else:                                      # a field rewritten
        try:
            meta = json.loads(bytes(hdr))
        except ValueError:
            return raw
        keys = [k for k in meta if k != "__metadata__"]
        if not keys:
            return raw
        k = keys[int(rng.integers(0, len(keys)))]
        f = ["dtype", "shape", "data_offsets"][int(rng.integers(0, 3))]
        repl = [None, 3, "F8", [1.0], [-1], [True], [1, 2, 3], [2 ** 70], "BF16", [0, 0], {}][
            int(rng.integers(0, 11))]
        if isinstance(meta[k], dict):
            meta[k][f] = repl
        hdr = bytearray(json.dumps(meta).encode())
    return struct.pack("<Q", len(hdr)) + bytes(hdr) + data


def fixed_cases():
    out = []

    def f(header, data=b"\0" * 32):
        h = header.encode() if isinstance(header, str) else header
        out.append(struct.pack("<Q", len(h)) + h + data)

    f('{"t":{"dtype":"F32","shape":[4],"data_offsets":[0,16]}}')
    f(b'\xef\xbb\xbf{"t":{"dtype":"F32","shape":[4],"data_offsets":[0,16]}}')        # UTF-8 BOM
    f('{"t\\ud800x":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}')               # lone surrogate escape
    f(b'{"\xed\xa0\x80":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}')           # encoded surrogate
    f(b'{"\xc3\x28":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}')               # invalid UTF-8
    f(b'{"\xe0\x80\xaf":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}')           # overlong
    f(b'{"\xf4\x90\x80\x80":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}')       # above U+10FFFF
    f('{"a":{"dtype":"U8","shape":[0],"data_offsets":[4,4]},"b":{"dtype":"U8","shape":[8],"data_offsets":[0,8]}}')
    f('{"a":{"dtype":"U8","shape":[0],"data_offsets":[0,0]},"b":{"dtype":"U8","shape":[8],"data_offsets":[0,8]}}')
    f('{"a":{"dtype":"U8","shape":[2],"data_offsets":[0,2],"extra":[1,{"x":[]}]}}')
    f('{"a":{"dtype":"U8","shape":[2],"data_offsets":[-0,2]}}')
    f('{"a":{"dtype":"U8","shape":[2],"data_offsets":[0,02]}}')
    f('{"a":{"dtype":"U8","shape":[2],"data_offsets":[0,2e0]}}')
    f('{"a":{"dtype":"U8","shape":[99999999999999999999],"data_offsets":[0,2]}}')
    f('{"a":{"dtype":"U8","shape":[2],"data_offsets":[0,2]}}   \n ')
    f('  {}  ')
    f('{"__metadata__":{"a":"b"}}')
    f('{"__metadata__":3}')
    f('"just a string"')
    f('{"a":{"dtype":"U8","shape":[2],"data_offsets":[0,2]},}')
    f('{"a":{"dtype":"U8","shape":[2],"data_offsets":[0,2]}')
    f('{"a":{"dtype":"U8","shape":[2,],"data_offsets":[0,2]}}')
    f('{"a":{"dtype":"U8","shape":[2],"data_offsets":[0,2]},"language_model.a":'
      '{"dtype":"U8","shape":[2],"data_offsets":[2,4]}}')
    f('{"a":{"dtype":"U8","shape":[1,1,1,1,1,1,1,1],"data_offsets":[0,1]}}')
    f('{"a":{"dtype":"U8","shape":[2],"data_offsets":[0,2]},"b":{"dtype":"U8","shape":[2],'
      '"data_offsets":[1,3]}}')
    out.append(b"\x01\x02\x03")                                                     # shorter than 8
    return out


def main():
    ref, dst = sys.argv[1], sys.argv[2]
    storage = load_reference(ref)
    rng = np.random.default_rng(20261210)
    files = fixed_cases()
    for _ in range(120):
        files.append(valid_file(rng))
    for _ in range(360):
        base = valid_file(rng)
        for _ in range(int(rng.integers(1, 3))):
            base = mutate(rng, base)
        files.append(base)
    records = []
    with tempfile.TemporaryDirectory() as tmp:
        for i, raw in enumerate(files):
            d = os.path.join(tmp, str(i))
            os.mkdir(d)
            path = os.path.join(d, "m.safetensors")
            with open(path, "wb") as f:
                f.write(raw)
            rec = {"raw": base64.b64encode(raw).decode()}
            try:
                ix = storage.SafeTensorIndex(d, workers=1)
                rec["ok"] = True
                rec["tensors"] = sorted([n, t.dtype, list(t.shape), t.offset, t.nbytes]
                                        for n, t in ix.tensors.items())
                ix.close()
            except Exception as e:                 # the reference's own exception
                rec["ok"] = False
                rec["type"] = type(e).__name__
                rec["msg"] = str(e).replace(path, "<path>")
            records.append(rec)
    with open(dst, "w") as f:
        json.dump({"source": "storage.py SafeTensorIndex", "records": records}, f, separators=(",", ":"))
    print(len(records), "records,", sum(r["ok"] for r in records), "accepted")


if __name__ == "__main__":
    main()
