"""The checkpoint reader against the reference's own C index and row reader
(c/src/safetensors.c, c/src/reader.c, compiled unmodified into oracle/_ref):
row reads return the same bytes and count the same rows for random requests,
the cases of c/tests/test_reader.c:31-80 hold, and on the recorded header
corpus the library differs from the C index only where the C index and the
Python runtime's index differ from each other (there it follows the Python
one, whose json.loads is strict JSON)."""
import base64
import json
import os
import struct

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _ref():
    import oracle
    r = oracle.reference()
    if r is None:
        pytest.skip("reference build (oracle/_ref) absent")
    return oracle, r


def _write(path, tensors):
    meta, blobs, off = {}, [], 0
    for name, (dt, a) in tensors.items():
        raw = np.ascontiguousarray(a).tobytes()
        meta[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    text = json.dumps(meta).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)) + text + b"".join(blobs))


def test_reader_cases_of_the_reference(built, tmp_path):
    """c/tests/test_reader.c:31-80: a 1000 x 32 tensor whose row r holds the
    byte r mod 256; out-of-order and repeated rows, a single row, a block,
    rows out of range; rows_read counts every requested row."""
    import qmoe
    oracle, r = _ref()
    rows = (np.arange(1000, dtype=np.uint32)[:, None] % 256).astype(np.uint8).repeat(32, 1)
    _write(tmp_path / "m.safetensors", {"rows": ("U8", rows)})
    ck, ri = qmoe.Checkpoint(str(tmp_path), 4), oracle.RefIndex(r.lib, str(tmp_path), 4)
    for req in ([999, 0, 5, 5, 100, 3, 999, 42], [777], [10, 11, 12, 13]):
        got = ck.read_rows("rows", req)
        assert np.array_equal(got, rows[req])
        assert np.array_equal(got.ravel(), ri.read_rows("rows", req, 32))
        if req == [777]:
            assert got[0, 0] == 9 and got[0, 31] == 9    # the byte value wraps
    for bad in ([1000], [-1]):
        with pytest.raises(qmoe.QmoeError):
            ck.read_rows("rows", bad)
        with pytest.raises(ValueError):
            ri.read_rows("rows", bad, 32)
    assert ck.stats()["rows_read"] == ri.rows_read() == 8 + 1 + 4
    ri.close()
    ck.close()


def test_row_reads_match_the_reference_reader(built, tmp_path):
    import qmoe
    oracle, r = _ref()
    rng = np.random.default_rng(20261211)
    tensors = {
        "model.layers.0.mlp.switch_mlp.gate_proj.weight":
            ("U32", rng.integers(0, 2 ** 32, size=(64, 8, 16), dtype=np.uint32)),
        "model.layers.0.mlp.switch_mlp.gate_proj.scales": ("BF16", rng.integers(0, 2 ** 16, size=(64, 8, 2), dtype=np.uint16)),
        "wide": ("U8", rng.integers(0, 256, size=(40, 4099), dtype=np.uint8)),
        "one": ("F32", rng.standard_normal((1, 3)).astype(np.float32)),
    }
    _write(tmp_path / "model.safetensors", tensors)
    ck, ri = qmoe.Checkpoint(str(tmp_path), 3), oracle.RefIndex(r.lib, str(tmp_path), 3)
    assert ri.table() == sorted([n, t["dtype"], list(t["shape"]), t["offset"], t["nbytes"]]
                                for n, t in ((n, ck.find(n)) for n in ck.names()))
    total = 0
    for name, (_, a) in tensors.items():
        rb = ck.find(name)["row_bytes"]
        for _ in range(25):
            n = int(rng.integers(0, 12))
            kind = rng.integers(0, 3)
            if kind == 0:      # scattered, repeated, unsorted
                req = rng.integers(0, a.shape[0], size=n)
            elif kind == 1:    # a run, shuffled, with repeats
                s = int(rng.integers(0, a.shape[0]))
                req = rng.permutation(np.minimum(np.arange(s, s + n), a.shape[0] - 1))
            else:              # strictly increasing
                req = np.unique(rng.integers(0, a.shape[0], size=n))
            req = [int(v) for v in req]
            got = ck.read_rows(name, req)
            assert np.array_equal(np.ascontiguousarray(got).view(np.uint8).ravel(),
                                  ri.read_rows(name, req, rb)), (name, req)
            assert np.array_equal(got, a[req]) if req else got.shape[0] == 0
            total += len(req)
    assert ck.stats()["rows_read"] == ri.rows_read() == total
    ri.close()
    ck.close()


def test_index_against_both_references_on_the_corpus(built, tmp_path):
    """Where the C index and the Python runtime's index agree, the library
    agrees with both; where they disagree (a UTF-8 byte-order mark, numbers
    with leading zeros or an exponent, invalid UTF-8, raw control characters
    in strings), it agrees with the Python runtime."""
    import qmoe
    oracle, r = _ref()
    with open(os.path.join(HERE, "golden", "st_headers.json")) as f:
        recs = json.load(f)["records"]
    split = 0
    for i, rec in enumerate(recs):
        raw = base64.b64decode(rec["raw"])
        d = tmp_path / str(i)
        d.mkdir()
        (d / "m.safetensors").write_bytes(raw)
        try:
            ix = oracle.RefIndex(r.lib, str(d), 1)
            c_ok, c_table = True, ix.table()
            ix.close()
        except ValueError:
            c_ok, c_table = False, None
        try:
            ck = qmoe.Checkpoint(str(d), 1)
            ours = sorted([n, t["dtype"], list(t["shape"]), t["offset"], t["nbytes"]]
                          for n, t in ((n, ck.find(n)) for n in ck.names()))
            ck.close()
        except qmoe.QmoeError:
            ours = None
        assert (ours is not None) == rec["ok"], i
        if c_ok == rec["ok"]:
            assert (ours is not None) == c_ok, i
            if c_ok:
                assert ours == c_table == rec["tensors"], i
        else:
            split += 1
    assert split == 5
