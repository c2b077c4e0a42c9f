"""The safetensors checkpoint reader (qmoe_ckpt_*), on the CPU, and one GPU
test of a context uploaded from checkpoint files.

Index validation follows c/tests/test_safetensors.c:63-166 and the storage
cases of tests/test_streaming.py:43-127 (the reference's own tests); row reads
follow c/src/reader.c:11-112 (sorted unique rows, one pread per contiguous
run, request order restored, duplicates read once); the MoE layer reader is
checked byte for byte against the arrays the files were written from, and its
packed slots against an independent numpy packing of the slot layout."""
import json
import os
import struct
import threading

import numpy as np
import pytest

D, E, K, I, G = 256, 16, 4, 128, 64   # configs[0]


def write_st(path, tensors, header=None, prefix=""):
    """A safetensors file of {name: (dtype, array)}; `header` replaces the
    JSON text when given (for malformed files)."""
    meta, blobs, off = {}, [], 0
    for name, (dt, a) in tensors.items():
        raw = np.ascontiguousarray(a).tobytes()
        meta[prefix + name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    text = (json.dumps(meta) if header is None else header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for b in blobs:
            f.write(b)


def _open(path, workers=2):
    import qmoe
    return qmoe.Checkpoint(str(path), workers)


def pattern(n, seed):
    return ((seed + np.arange(n) * 7) % 256).astype(np.uint8)


def test_basic_index(built, tmp_path):
    """c/tests/test_safetensors.c:63-110: names lose language_model., lookups
    of model.* fall back to it, and a whole tensor reads back exactly."""
    a = pattern(128, 1).view(np.uint16).reshape(4, 16)
    b = pattern(96, 9).reshape(3, 4, 8)
    write_st(tmp_path / "model.safetensors",
             {"language_model.model.layers.0.weight": ("BF16", a), "language_model.other": ("U8", b)})
    with _open(tmp_path) as ck:
        t = ck.find("model.layers.0.weight")
        assert t["dtype"] == "BF16" and t["shape"] == (4, 16) and t["nbytes"] == 128
        assert t["row_bytes"] == 32
        assert ck.find("other") is not None
        assert ck.find("model.missing") is None
        assert np.array_equal(ck.read_tensor("model.layers.0.weight"), a)
        assert np.array_equal(ck.read_tensor("other"), b)
        assert ck.names() == ["model.layers.0.weight", "other"]
        s = ck.stats()
        assert s["tensors_read"] == 2 and s["bytes_read"] == 128 + 96


F32x4 = np.zeros(4, np.float32)
MALFORMED = [
    # c/tests/test_safetensors.c:112-166
    ("bad dtype size", '{"t":{"dtype":"F16","shape":[4],"data_offsets":[0,16]}}', "invalid safetensors range"),
    ("overlap", '{"a":{"dtype":"F32","shape":[4],"data_offsets":[0,16]},'
                '"b":{"dtype":"F32","shape":[4],"data_offsets":[8,24]}}', "overlapping safetensors ranges"),
    ("beyond file", '{"t":{"dtype":"F32","shape":[4],"data_offsets":[0,100]}}', "invalid safetensors range"),
    ("size mismatch", '{"t":{"dtype":"F32","shape":[4],"data_offsets":[0,8]}}', "invalid safetensors range"),
    ("duplicate", '{"t":{"dtype":"F32","shape":[4],"data_offsets":[0,16]},'
                  '"language_model.t":{"dtype":"F32","shape":[4],"data_offsets":[16,32]}}', "duplicate tensor t"),
    ("not json", "{not json", "invalid safetensors JSON"),
    # storage.py:107-146 messages
    ("not an object", "[1, 2]", "must be an object"),
    ("entry not an object", '{"t": 3}', "invalid safetensors entry"),
    ("unknown dtype", '{"t":{"dtype":"Q4","shape":[4],"data_offsets":[0,16]}}', "unsupported safetensors dtype Q4"),
    ("no dtype", '{"t":{"shape":[4],"data_offsets":[0,16]}}', "unsupported safetensors dtype"),
    ("three offsets", '{"t":{"dtype":"F32","shape":[4],"data_offsets":[0,8,16]}}', "invalid safetensors metadata"),
    ("no shape", '{"t":{"dtype":"F32","data_offsets":[0,16]}}', "invalid safetensors metadata"),
    ("float offset", '{"t":{"dtype":"F32","shape":[4],"data_offsets":[0,16.0]}}', "invalid data offsets"),
    ("bool offset", '{"t":{"dtype":"F32","shape":[4],"data_offsets":[false,16]}}', "invalid data offsets"),
    ("negative dim", '{"t":{"dtype":"F32","shape":[-4],"data_offsets":[0,16]}}', "invalid tensor shape"),
    ("negative offset", '{"t":{"dtype":"F32","shape":[4],"data_offsets":[-16,0]}}', "invalid safetensors range"),
    ("huge offset", '{"t":{"dtype":"F32","shape":[4],"data_offsets":[0,99999999999999999999999]}}',
     "invalid safetensors range"),
    ("trailing text", '{"t":{"dtype":"F32","shape":[4],"data_offsets":[0,16]}} x', "invalid safetensors JSON"),
]


@pytest.mark.parametrize("case", MALFORMED, ids=[c[0] for c in MALFORMED])
def test_malformed_headers_are_rejected(built, tmp_path, case):
    import qmoe
    _, header, msg = case
    write_st(tmp_path / "bad.safetensors", {"t": ("F32", np.zeros(8, np.float32))}, header=header)
    with pytest.raises(qmoe.QmoeError, match=msg):
        _open(tmp_path)


def test_truncated_files_and_empty_directories(built, tmp_path):
    import qmoe
    with pytest.raises(qmoe.QmoeError, match="no safetensors"):
        _open(tmp_path)
    with open(tmp_path / "short.safetensors", "wb") as f:   # header length past the end
        f.write(struct.pack("<Q", 10000))
    with pytest.raises(qmoe.QmoeError, match="truncated safetensors JSON"):
        _open(tmp_path)
    with open(tmp_path / "short.safetensors", "wb") as f:
        f.write(b"\x01\x02")
    with pytest.raises(qmoe.QmoeError, match="truncated safetensors header"):
        _open(tmp_path)


def test_metadata_escapes_and_zero_length_tensors(built, tmp_path):
    """__metadata__ is skipped; names may use JSON escapes; an empty tensor
    sits at the start of another's range without overlapping it."""
    body = np.arange(4, dtype=np.float32)
    header = ('{"__metadata__":{"format":"pt","nested":{"a":[1,2,{"b":null}]}},'
              '"w\\u00e9ight\\/x":{"dtype":"F32","shape":[4],"data_offsets":[0,16]},'
              '"empty":{"dtype":"F32","shape":[0, 3],"data_offsets":[0,0]}}')
    write_st(tmp_path / "m.safetensors", {"t": ("F32", body)}, header=header)
    with _open(tmp_path) as ck:
        assert sorted(ck.names()) == ["empty", "wéight/x"]
        assert np.array_equal(ck.read_tensor("wéight/x"), body)
        assert ck.find("empty")["shape"] == (0, 3) and ck.find("empty")["row_bytes"] == 0


def test_deeply_nested_metadata(built, tmp_path):
    """json.loads takes a few hundred levels of nesting in __metadata__, and so
    does the index; far deeper nesting is refused, not a crash."""
    import qmoe
    t = '"t":{"dtype":"F32","shape":[4],"data_offsets":[0,16]}'
    for depth, ok in ((300, True), (100000, False)):
        write_st(tmp_path / "m.safetensors", {"t": ("F32", np.zeros(4, np.float32))},
                 header='{"__metadata__":' + "[" * depth + "]" * depth + "," + t + "}")
        if ok:
            with _open(tmp_path) as ck:
                assert ck.names() == ["t"]
        else:
            with pytest.raises(qmoe.QmoeError, match="invalid safetensors JSON"):
                _open(tmp_path)


def test_row_reads_restore_order_and_deduplicate(built, tmp_path):
    """tests/test_streaming.py:113-126 and :85-93: rows [3, 1, 3, 2] come
    back in request order from one pread of rows 1..3."""
    a = np.random.default_rng(1).integers(0, 2**32, size=(4, 32, 4), dtype=np.uint32)
    write_st(tmp_path / "m.safetensors", {"w": ("U32", a)}, prefix="language_model.")
    with _open(tmp_path) as ck:
        rows = ck.read_rows("w", [3, 1, 3, 2])
        assert np.array_equal(rows, a[[3, 1, 3, 2]])
        s = ck.stats()
        rb = ck.find("w")["row_bytes"]
        assert s["bytes_read"] == 3 * rb and s["pread_calls"] == 1 and s["rows_read"] == 4


def test_row_runs_and_empty_requests(built, tmp_path):
    """tests/test_streaming.py:43-57 (rows [1, 2, 5]: two reads) and :72-78
    (an empty request reads nothing); rows outside the tensor are refused."""
    import qmoe
    a = np.arange(16 * 8, dtype=np.uint16).reshape(16, 8)
    write_st(tmp_path / "m.safetensors", {"p": ("BF16", a), "s": ("F32", np.zeros((), np.float32))})
    with _open(tmp_path) as ck:
        assert np.array_equal(ck.read_rows("p", [1, 2, 5]), a[[1, 2, 5]])
        assert ck.stats()["pread_calls"] == 2 and ck.stats()["bytes_read"] == 3 * 16
        assert ck.read_rows("p", []).shape == (0, 8)
        assert ck.stats()["pread_calls"] == 2
        with pytest.raises(qmoe.QmoeError, match="row 16 outside"):
            ck.read_rows("p", [0, 16])
        with pytest.raises(qmoe.QmoeError, match="row -1 outside"):
            ck.read_rows("p", [-1])
        with pytest.raises(qmoe.QmoeError, match="no rows"):
            ck.read_rows("s", [0])
        # sorted unique rows go straight to the output, still one read per run
        assert np.array_equal(ck.read_rows("p", [0, 1, 2, 3, 9, 10]), a[[0, 1, 2, 3, 9, 10]])
        assert ck.stats()["pread_calls"] == 4
    ck.close()
    with pytest.raises(qmoe.QmoeError, match="closed"):
        ck.read_tensor("p")


def test_large_tensor_reads_in_pieces_on_several_threads(built, tmp_path):
    a = np.random.default_rng(2).integers(0, 255, size=(3, 25 << 20), dtype=np.uint8)  # 75 MiB
    write_st(tmp_path / "big.safetensors", {"big": ("U8", a)})
    with _open(tmp_path, workers=4) as ck:
        assert np.array_equal(ck.read_tensor("big"), a)
        assert ck.stats()["pread_calls"] >= 3   # 32 MiB pieces
        out = {}

        def reader(i):
            out[i] = ck.read_rows("big", [2 - (i % 3), i % 3])

        th = [threading.Thread(target=reader, args=(i,)) for i in range(6)]
        for t in th:
            t.start()
        for t in th:
            t.join()
        for i in range(6):
            assert np.array_equal(out[i], a[[2 - (i % 3), i % 3]])
        assert ck.stats()["rows_read"] == 12


def _layer_tensors(s, layer, drop=()):
    """SynthLayer arrays under the checkpoint's names (c/src/model.c:541-546,
    :1902-1923), in the disk shapes of model.c:555-557."""
    d, e, i, g = s.d, s.E, s.I, s.g
    base = f"model.layers.{layer}.mlp"
    out = {f"{base}.gate.weight": ("BF16", s.router.reshape(e, d)),
           f"{base}.shared_expert_gate.weight": ("BF16", s.shared_gate.reshape(1, d))}
    for key, name, rows, cols, stacked in (
            ("gate", "switch_mlp.gate_proj", i, d, True), ("up", "switch_mlp.up_proj", i, d, True),
            ("down", "switch_mlp.down_proj", d, i, True), ("sh_gate", "shared_expert.gate_proj", i, d, False),
            ("sh_up", "shared_expert.up_proj", i, d, False), ("sh_down", "shared_expert.down_proj", d, i, False)):
        q, sc, bi = s.t[key]
        lead = (e, rows) if stacked else (rows,)
        out[f"{base}.{name}.weight"] = ("U32", q.reshape(*lead, cols // 8))
        out[f"{base}.{name}.scales"] = ("BF16", sc.reshape(*lead, cols // g))
        out[f"{base}.{name}.biases"] = ("BF16", bi.reshape(*lead, cols // g))
    return {k: v for k, v in out.items() if not any(x in k for x in drop)}


def _bytes_at(w_ptr, n, dtype):
    import ctypes
    return np.frombuffer((ctypes.c_uint8 * (n * np.dtype(dtype).itemsize)).from_address(w_ptr),
                         dtype=dtype)


@pytest.fixture
def tiny_ckpt(built, tmp_path):
    """Two synthetic layers of configs[0] over two files, some names under
    language_model. (a multimodal checkpoint's text model)."""
    import qmoe
    cfg = qmoe.make_config(D, E, K, I, layers=2, max_tokens=32)
    layers = [qmoe.SynthLayer(cfg, 20261204, l) for l in range(2)]
    write_st(tmp_path / "model-00001-of-00002.safetensors", _layer_tensors(layers[0], 0),
             prefix="language_model.")
    write_st(tmp_path / "model-00002-of-00002.safetensors", _layer_tensors(layers[1], 1))
    return cfg, layers, tmp_path


def test_read_layer_equals_the_written_arrays(tiny_ckpt):
    cfg, layers, path = tiny_ckpt
    with _open(path, workers=3) as ck:
        assert ck.find("model.layers.0.mlp.gate.weight")["file"] == 0
        assert ck.find("model.layers.1.mlp.gate.weight")["file"] == 1
        for l, s in enumerate(layers):
            buf, w = ck.read_layer(cfg, l)
            assert w.logit_bias is None
            assert np.array_equal(_bytes_at(w.router, s.router.size, np.uint16), s.router)
            assert np.array_equal(_bytes_at(w.shared_gate, s.shared_gate.size, np.uint16), s.shared_gate)
            for key in ("gate", "up", "down", "sh_gate", "sh_up", "sh_down"):
                q, sc, bi = s.t[key]
                part = getattr(w, key)
                assert np.array_equal(_bytes_at(part.q, q.size, np.uint32), q), key
                assert np.array_equal(_bytes_at(part.scales, sc.size, np.uint16), sc), key
                assert np.array_equal(_bytes_at(part.biases, bi.size, np.uint16), bi), key
        assert ck.stats()["tensors_read"] == 40


def test_packed_slots_equal_an_independent_packing(tiny_ckpt):
    """qmoe_ckpt_pack_experts (rows read per tensor, packed in C) and
    qmoe_pack_expert against the numpy restatement of the slot layout."""
    import qmoe
    from test_zz_no_alloc import pack_slots
    cfg, layers, path = tiny_ckpt
    sb = qmoe.lib().qmoe_slot_bytes(cfg)
    with _open(path) as ck:
        for l, s in enumerate(layers):
            pool, sh = pack_slots(s, sb)
            ids = [5, 0, 15, 5, 7]
            got = ck.pack_experts(cfg, l, ids)
            assert np.array_equal(got, pool[ids])
            w = s.weights()
            assert np.array_equal(qmoe.pack_expert(cfg, w, 9), pool[9])
            assert np.array_equal(qmoe.pack_expert(cfg, w, -1), sh)


def test_contiguous_experts_share_one_read_per_tensor(tiny_ckpt):
    """tests/test_streaming.py:175-198: four contiguous experts, nine
    tensors, nine preads; scattered experts cost one per run."""
    cfg, _, path = tiny_ckpt
    with _open(path) as ck:
        ck.pack_experts(cfg, 0, [0, 1, 2, 3])
        assert ck.stats()["pread_calls"] == 9
        ck.pack_experts(cfg, 0, [9, 4, 11])
        assert ck.stats()["pread_calls"] == 9 + 27
        assert ck.stats()["rows_read"] == 9 * 7


def test_layer_reader_checks_names_types_and_shapes(built, tmp_path):
    import qmoe
    cfg = qmoe.make_config(D, E, K, I, layers=1, max_tokens=32)
    s = qmoe.SynthLayer(cfg, 20261205, 0)

    def attempt(tensors, sub):
        for f in tmp_path.glob("*.safetensors"):
            f.unlink()
        write_st(tmp_path / "m.safetensors", tensors)
        with _open(tmp_path) as ck:
            if sub is None:
                return ck.read_layer(cfg, 0)
            with pytest.raises(qmoe.QmoeError, match=sub):
                ck.read_layer(cfg, 0)

    full = _layer_tensors(s, 0)
    attempt({k: v for k, v in full.items() if "switch_mlp.up_proj.scales" not in k},
            "missing expert tensor model.layers.0.mlp.switch_mlp.up_proj.scales")
    attempt({k: v for k, v in full.items() if "mlp.gate.weight" not in k},
            "missing tensor model.layers.0.mlp.gate.weight")
    bad = dict(full)
    bad["model.layers.0.mlp.gate.weight"] = ("F32", np.zeros((E, D), np.float32))
    attempt(bad, "has dtype F32, expected BF16")
    bad = dict(full)
    bad["model.layers.0.mlp.switch_mlp.down_proj.weight"] = ("U32", np.zeros((E, D, I // 16), np.uint32))
    attempt(bad, r"configured shape \[16, 256, 16\]")
    # the shared expert's biases may be absent: they read as zeros
    buf, w = attempt({k: v for k, v in full.items() if "shared_expert.up_proj.biases" not in k}, None)
    assert not _bytes_at(w.sh_up.biases, s.t["sh_up"][2].size, np.uint16).any()
    assert np.array_equal(_bytes_at(w.sh_up.scales, s.t["sh_up"][1].size, np.uint16), s.t["sh_up"][1])
    with _open(tmp_path) as ck:
        with pytest.raises(qmoe.QmoeError, match="expert 16 out of range"):
            ck.pack_experts(cfg, 0, [16])
        with pytest.raises(qmoe.QmoeError, match="missing expert tensor"):
            ck.pack_experts(cfg, 3, [0])


@pytest.mark.gpu
def test_upload_from_checkpoint_equals_upload_from_memory(tiny_ckpt):
    """qmoe_upload_layer_ckpt (a layer read from the files, then uploaded)
    gives the same outputs, bit for bit, as qmoe_upload_layer of the arrays
    the files were written from; two layers, one per file."""
    import qmoe
    cfg, layers, path = tiny_ckpt
    a, b = qmoe.Context(cfg), qmoe.Context(cfg)
    with qmoe.Checkpoint(str(path), 2) as ck:
        for l, s in enumerate(layers):
            a.upload(l, s)
            b.upload_ckpt(l, ck, l)
    x = qmoe.synth_tokens(20261204, 3, 32, D)
    for l in range(2):
        for n in (1, 32):
            assert np.array_equal(a.forward(l, x[:n]), b.forward(l, x[:n])), (l, n)
    a.close()
    b.close()
