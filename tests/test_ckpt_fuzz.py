"""The checkpoint index on untrusted headers: qmoe_ckpt_open accepts exactly
the files the reference's SafeTensorIndex accepts, with the same tensor table,
and refuses the others (with the reference's message where the reference's
index, not its JSON decoder, refused them).

tests/golden/st_headers.json holds 506 files (valid, systematically broken and
randomly mutated) with the outcome of the reference's own index on each
(tests/golden/make_st_golden.py); oracle/st_header.py restates the same checks
and is pinned to that corpus first, then serves as the checker for random
mutations (hypothesis). Two documented differences are kept out of the
random part: duplicate keys inside one JSON object (json.loads keeps the last
one; the C port, and this library, refuse a duplicate name) and the
non-standard NaN/Infinity literals, which json.loads accepts."""
import base64
import json
import os
import struct

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _records():
    with open(os.path.join(HERE, "golden", "st_headers.json")) as f:
        return json.load(f)["records"]


def _dup_keys(raw):
    """True when some JSON object of the header repeats a key."""
    if len(raw) < 8:
        return False
    hlen = struct.unpack("<Q", raw[:8])[0]
    seen_dup = []

    def hook(pairs):
        keys = [k for k, _ in pairs]
        if len(keys) != len(set(keys)):
            seen_dup.append(True)
        return dict(pairs)
    try:
        json.loads(raw[8:8 + hlen], object_pairs_hook=hook)
    except ValueError:
        return False
    return bool(seen_dup)


def _ours(tmp_path, raw, i):
    """(ok, table or message) of libqmoe's index on one file."""
    import qmoe
    d = tmp_path / f"c{i}"
    d.mkdir()
    path = d / "m.safetensors"
    path.write_bytes(raw)
    try:
        ck = qmoe.Checkpoint(str(d), 1)
    except qmoe.QmoeError as e:
        return False, str(e).replace(str(path), "<path>")
    table = sorted([n, t["dtype"], list(t["shape"]), t["offset"], t["nbytes"]]
                   for n, t in ((n, ck.find(n)) for n in ck.names()))
    ck.close()
    return True, table


def test_restatement_matches_reference_corpus():
    from oracle import st_header
    for i, r in enumerate(_records()):
        raw = base64.b64decode(r["raw"])
        try:
            t = st_header.parse(raw, "<path>")
            got_ok = True
        except ValueError as e:
            got_ok, msg = False, str(e)
        assert got_ok == r["ok"], (i, r)
        if got_ok:
            assert sorted([n, v[0], list(v[1]), v[2], v[3]] for n, v in t.items()) == r["tensors"], i
        elif r["type"] == "ValueError":
            assert msg == r["msg"], (i, msg, r["msg"])


def test_library_index_matches_reference_corpus(built, tmp_path):
    n_ok = n_msg = 0
    for i, r in enumerate(_records()):
        raw = base64.b64decode(r["raw"])
        if _dup_keys(raw):
            continue
        ok, got = _ours(tmp_path, raw, i)
        assert ok == r["ok"], (i, got, r)
        if ok:
            assert got == r["tensors"], (i, got, r["tensors"])
            n_ok += 1
        elif r["type"] == "ValueError":
            assert got == r["msg"], (i, got, r["msg"])
            n_msg += 1
    assert n_ok > 150 and n_msg > 60


hypothesis = pytest.importorskip("hypothesis")
from hypothesis import HealthCheck, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

SIG = b'{}[]",:0123456789.eE+-tfnul\\ \t\n'


@st.composite
def mutated_files(draw):
    """A corpus file (valid or not) with up to three byte-level edits of its
    header: replace (a JSON-significant byte or any byte), delete, insert, or
    a header length off by a little."""
    recs = _records()
    raw = bytearray(base64.b64decode(recs[draw(st.integers(0, len(recs) - 1))]["raw"]))
    if len(raw) < 8:
        return bytes(raw)
    hlen = struct.unpack("<Q", raw[:8])[0]
    hdr, data = bytearray(raw[8:8 + hlen]), bytes(raw[8 + hlen:])
    for _ in range(draw(st.integers(0, 3))):
        kind = draw(st.integers(0, 3))
        pos = draw(st.integers(0, max(0, len(hdr))))
        if kind == 0 and pos < len(hdr):
            hdr[pos] = draw(st.sampled_from(list(SIG)))
        elif kind == 1 and pos < len(hdr):
            hdr[pos] = draw(st.integers(1, 255))
        elif kind == 2 and pos < len(hdr):
            del hdr[pos]
        else:
            hdr.insert(pos, draw(st.sampled_from(list(SIG))))
    skew = draw(st.sampled_from([0, 0, 0, -1, 1, 5]))
    return struct.pack("<Q", max(0, len(hdr) + skew)) + bytes(hdr) + data


@settings(max_examples=400, deadline=None, suppress_health_check=list(HealthCheck))
@given(raw=mutated_files())
def test_library_index_agrees_with_restatement_on_mutations(built, tmp_path_factory, raw):
    from oracle import st_header
    hdr = raw[8:]
    if _dup_keys(raw) or b"NaN" in hdr or b"Infinity" in hdr:
        return
    try:
        want = st_header.parse(raw, "<path>")
        want_ok = True
    except ValueError:
        want_ok = False
    ok, got = _ours(tmp_path_factory.mktemp("fz"), raw, 0)
    assert ok == want_ok, (raw, got)
    if ok:
        assert got == sorted([n, v[0], list(v[1]), v[2], v[3]] for n, v in want.items())
