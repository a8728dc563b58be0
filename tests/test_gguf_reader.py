"""The library's GGUF reader (kq_gguf_*) on files written by gguf-py's
GGUFWriter: tensor directory, stored bytes and metadata as written, and
malformed files (bad magic or version, truncation anywhere, tensors outside
the file) rejected with KQ_ERR_FORMAT instead of crashing.  Host code only."""
import numpy as np
import pytest

from pesti_b200 import kq, synthetic

gguf = pytest.importorskip("gguf")


def _write(path, tensors, meta=(), alignment=None):
    w = gguf.GGUFWriter(str(path), "llama")
    if alignment:
        w.add_custom_alignment(alignment)
    for kind, key, val in meta:
        getattr(w, f"add_{kind}")(key, val)
    for name, arr, qt in tensors:
        if qt is None:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=qt)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.fixture
def model_file(tmp_path):
    q4 = synthetic.gguf_weight(kq.KQ_GGUF_Q4_K, 12, 512, seed=1)
    q6 = synthetic.gguf_weight(kq.KQ_GGUF_Q6_K, 5, 768, seed=2)
    norm = np.linspace(-1, 1, 512, dtype=np.float32)
    emb = np.arange(6 * 8, dtype=np.float16).reshape(6, 8)
    meta = [("uint32", "llama.block_count", 2), ("float32", "llama.rope.freq_base", 500000.0),
            ("string", "general.name", "tiny-é"), ("array", "tokenizer.ggml.scores", [0.5, -1.25, 3.0]),
            ("array", "tokenizer.ggml.tokens", ["<s>", "a", ""]), ("bool", "general.flag", True),
            ("uint64", "big.count", 1 << 40), ("int32", "neg", -7)]
    path = tmp_path / "m.gguf"
    _write(path, [("blk.0.ffn_up.weight", q4, gguf.GGMLQuantizationType.Q4_K),
                  ("blk.0.ffn_down.weight", q6, gguf.GGMLQuantizationType.Q6_K),
                  ("norm.weight", norm, None), ("tok_embd.weight", emb, None)], meta)
    return path, {"q4": q4, "q6": q6, "norm": norm, "emb": emb}


def test_directory_bytes_and_metadata_as_written(model_file):
    path, src = model_file
    with kq.GgufFile(str(path)) as f:
        t = f.tensors
        assert list(t) == ["blk.0.ffn_up.weight", "blk.0.ffn_down.weight", "norm.weight", "tok_embd.weight"]
        assert (t["blk.0.ffn_up.weight"].ggml_type, t["blk.0.ffn_up.weight"].shape) == (12, (12, 512))
        assert (t["blk.0.ffn_down.weight"].ggml_type, t["blk.0.ffn_down.weight"].shape) == (14, (5, 768))
        assert (t["norm.weight"].ggml_type, t["norm.weight"].shape) == (0, (512,))
        assert (t["tok_embd.weight"].ggml_type, t["tok_embd.weight"].shape) == (1, (6, 8))
        assert np.array_equal(f.read("blk.0.ffn_up.weight"), src["q4"].reshape(-1))
        assert np.array_equal(f.read("blk.0.ffn_down.weight"), src["q6"].reshape(-1))
        assert np.array_equal(f.read("norm.weight").view(np.float32), src["norm"])
        assert np.array_equal(f.read("tok_embd.weight").view(np.float16).reshape(6, 8), src["emb"])
        # offsets agree with gguf-py's own reader
        ref = {x.name: x for x in gguf.GGUFReader(str(path)).tensors}
        for name, x in t.items():
            assert x.offset == ref[name].data_offset and x.nbytes == ref[name].n_bytes
        m = f.metadata
        assert m["llama.block_count"] == 2 and m["llama.rope.freq_base"] == 500000.0
        assert m["general.name"] == "tiny-é"
        assert np.array_equal(m["tokenizer.ggml.scores"], np.array([0.5, -1.25, 3.0], np.float32))
        assert m["tokenizer.ggml.tokens"] == ["<s>", "a", ""]
        assert m["general.flag"] is True and m["big.count"] == 1 << 40 and m["neg"] == -7
        assert m["general.architecture"] == "llama"


def test_custom_alignment(tmp_path):
    q4 = synthetic.gguf_weight(kq.KQ_GGUF_Q4_K, 3, 256, seed=3)
    path = tmp_path / "a.gguf"
    _write(path, [("x", np.ones(5, np.float32), None), ("w", q4, gguf.GGMLQuantizationType.Q4_K)], alignment=64)
    with kq.GgufFile(str(path)) as f:
        assert f.metadata["general.alignment"] == 64
        assert f.tensors["w"].offset % 64 == 0
        assert np.array_equal(f.read("w"), q4.reshape(-1))


def _status(path):
    with pytest.raises(kq.KqError) as e:
        kq.GgufFile(str(path))
    return e.value.status


def test_malformed_files_are_rejected(model_file, tmp_path):
    path, _ = model_file
    data = path.read_bytes()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + data[4:])
    assert _status(bad) == kq.KQ_ERR_FORMAT
    bad.write_bytes(data[:4] + (1).to_bytes(4, "little") + data[8:])  # version 1 (32-bit counts)
    assert _status(bad) == kq.KQ_ERR_FORMAT
    bad.write_bytes(data[:8] + (1 << 40).to_bytes(8, "little") + data[16:])  # absurd tensor count
    assert _status(bad) == kq.KQ_ERR_FORMAT
    # every truncation point inside the header and directory, and inside the data
    first_data = min(x.offset for x in kq.GgufFile(str(path)).tensors.values())
    for cut in list(range(0, first_data, 7)) + [first_data + 1, len(data) - 1]:
        bad.write_bytes(data[:cut])
        assert _status(bad) == kq.KQ_ERR_FORMAT, cut
    assert _status(tmp_path / "missing.gguf") == kq.KQ_ERR_FORMAT


def test_read_rejects_a_short_buffer(model_file):
    path, _ = model_file
    with kq.GgufFile(str(path)) as f:
        t = f.tensors["norm.weight"]
        buf = np.empty(t.nbytes - 4, np.uint8)
        assert f.lib.kq_gguf_read_tensor(f.handle, t.index, buf.ctypes.data, buf.size) == kq.KQ_ERR_SHORT_BUFFER
        assert f.lib.kq_gguf_read_tensor(f.handle, 99, buf.ctypes.data, buf.size) == kq.KQ_ERR_INVALID_ARG
        assert f.lib.kq_gguf_find_tensor(f.handle, b"nope") == -1
        assert f.lib.kq_gguf_find_meta(f.handle, b"general.name") >= 0


def test_layer_from_a_tensor_that_is_not_a_k_quant_is_refused(model_file):
    path, _ = model_file
    with pytest.raises(kq.KqError) as e:
        kq.QuantizedLinear.from_gguf(str(path), "norm.weight")
    assert e.value.status == kq.KQ_ERR_UNSUPPORTED


def test_repeated_or_non_utf8_tensor_names_are_format_errors(tmp_path):
    # two tensors whose names differ in one byte; patching that byte makes the
    # directory repeat a name, or hold a name that is not UTF-8
    a = np.ones(4, np.float32)
    path = tmp_path / "n.gguf"
    _write(path, [("w.aa", a, None), ("w.ab", 2 * a, None)])
    data = path.read_bytes()
    at = data.index(b"w.ab")
    bad = tmp_path / "dup.gguf"
    bad.write_bytes(data[:at + 3] + b"a" + data[at + 4:])
    with pytest.raises(kq.KqError) as e:
        kq.GgufFile(str(bad))
    assert e.value.status == kq.KQ_ERR_FORMAT and "twice" in str(e.value)
    bad.write_bytes(data[:at + 3] + b"\xff" + data[at + 4:])
    with pytest.raises(kq.KqError) as e:
        kq.GgufFile(str(bad))
    assert e.value.status == kq.KQ_ERR_FORMAT and "UTF-8" in str(e.value)
    with kq.GgufFile(str(path)) as f:  # the unpatched file reads
        assert list(f.tensors) == ["w.aa", "w.ab"]


def test_layer_from_a_path_closes_the_file_it_opened(model_file, monkeypatch):
    path, _ = model_file
    closed = []
    orig = kq.GgufFile.close

    def spy(self):
        if self.handle:
            closed.append(self.path)
        orig(self)

    monkeypatch.setattr(kq.GgufFile, "close", spy)
    with pytest.raises(kq.KqError):
        kq.QuantizedLinear.from_gguf(str(path), "norm.weight")
    assert closed == [str(path)]
