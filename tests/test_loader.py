"""The reference's single-file model format: final_b200.modelfile.write and
the library's memory-mapped reader (include/b2loader.h, host code only, so
these run without a GPU).  Covers the index, shapes and data round trip,
configuration inference, an unaligned tensor offset, and every kind of
corrupt file the reader must refuse (bad magic, an index cut short, a tensor
running past the end of the file)."""
import ctypes as C
import struct

import numpy as np
import pytest

from final_b200 import _lib
from final_b200.modelfile import ModelFile, write

import lfm2_cases as lc


def _tensors():
    rng = np.random.default_rng(7)
    return {"embed_tokens.weight": rng.standard_normal((11, 64)).astype(np.float32),
            "layers.0.conv.conv.weight": rng.standard_normal((64, 1, 3)).astype(np.float32),
            "scalar": np.array(3.5, dtype=np.float32),
            "empty": np.zeros((0, 4), dtype=np.float32),
            "v": rng.standard_normal(5).astype(np.float32)}


def test_round_trip(tmp_path):
    t = _tensors()
    p = tmp_path / "m.bin"
    write(str(p), t)
    mf = ModelFile(str(p))
    assert list(mf.names()) == list(t)
    for n, a in t.items():
        assert mf.shape(n) == a.shape
        assert np.array_equal(mf.tensor(n), a)
    assert mf.has("v") and not mf.has("nope")
    lib = _lib.load()
    assert lib.b2_loader_weight(mf.handle, b"v", 5) is not None
    assert lib.b2_loader_weight(mf.handle, b"v", 6) is None
    assert lib.b2_loader_weight(mf.handle, b"nope", 5) is None
    mf.close()


def test_config_inferred_from_tensors(tmp_path):
    cfg = lc.TINY
    W = lc.Weights(cfg["seed"], cfg["vocab"], cfg)
    names = lc.model_names(cfg["layers"], cfg)
    p = tmp_path / "tiny.bin"
    write(str(p), {n: W(n) for n in names})
    mf = ModelFile(str(p))
    c = mf.config()
    assert c == dict(vocab=cfg["vocab"], hidden=cfg["H"], num_layers=cfg["layers"],
                     num_dense_layers=cfg["NUM_DENSE"], layer_types=list(cfg["TYPES"]),
                     num_heads=cfg["HQ"], num_kv_heads=cfg["HKV"], dense_inter=cfg["I_DENSE"],
                     num_experts=cfg["E"], moe_inter=cfg["I_MOE"], use_expert_bias=1)
    assert np.array_equal(mf.tensor("layers.3.feed_forward.experts.5.w2.weight"),
                          W("layers.3.feed_forward.experts.5.w2.weight"))
    mf.close()


def _raw(entries, data_blobs, version=1):
    """A file with hand-placed offsets: entries = [(name, shape, offset)]."""
    out = bytearray(b"LFM2" + struct.pack("<II", version, len(entries)))
    for n, shape, off in entries:
        nb = n.encode()
        out += struct.pack("<I", len(nb)) + nb + struct.pack("<I", len(shape))
        out += struct.pack(f"<{len(shape)}I", *shape) + struct.pack("<Q", off)
    for off, blob in data_blobs:
        if len(out) < off:
            out += b"\0" * (off - len(out))
        out[off:off + len(blob)] = blob
    return bytes(out)


def test_unaligned_offset_is_copied(tmp_path):
    a = np.arange(6, dtype=np.float32) * 1.25
    p = tmp_path / "u.bin"
    p.write_bytes(_raw([("a", (2, 3), 101)], [(101, a.tobytes())]))
    mf = ModelFile(str(p))
    assert np.array_equal(mf.tensor("a"), a.reshape(2, 3))
    mf.close()


@pytest.mark.parametrize("kind", ["magic", "short_index", "past_eof", "huge_dims", "missing"])
def test_corrupt_files_are_refused(tmp_path, kind):
    a = np.ones(4, dtype=np.float32)
    good = _raw([("a", (4,), 64)], [(64, a.tobytes())])
    p = tmp_path / "bad.bin"
    if kind == "magic":
        p.write_bytes(b"LFM3" + good[4:])
    elif kind == "short_index":
        p.write_bytes(good[:20])
    elif kind == "past_eof":
        p.write_bytes(_raw([("a", (4,), 64)], [(64, a.tobytes()[:8])]))
    elif kind == "huge_dims":
        p.write_bytes(_raw([("a", (1 << 20, 1 << 20), 64)], [(64, a.tobytes())]))
    lib = _lib.load()
    h = C.c_void_p()
    path = str(p if kind != "missing" else tmp_path / "does_not_exist.bin").encode()
    assert lib.b2_loader_open(path, C.byref(h)) == _lib.B2_ERR_INVALID
    assert not h.value
