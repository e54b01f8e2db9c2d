"""The reference engine's single-file model format (read by its ModelLoader,
src/model_loader.cpp:20-68): ``write`` produces it from named fp32 arrays,
``ModelFile`` reads it through the library's memory-mapped loader
(include/b2loader.h) and infers the model configuration from the tensor
names and shapes, for ``LFM2Model.from_file``.

Layout: b"LFM2", uint32 version, uint32 count, then per tensor uint32
name_len, name, uint32 ndim, uint32 dims[ndim], uint64 offset; fp32 data at
the offsets (64-byte aligned here).  Little-endian.
"""
from __future__ import annotations

import ctypes as C
import re
import struct
from typing import Dict, Iterable, Mapping, Tuple

import numpy as np

from . import _lib
from ._lib import check


def write(path: str, tensors: Mapping[str, np.ndarray], version: int = 1) -> None:
    """Write named arrays (converted to fp32) in the reference's format."""
    items = [(n, np.asarray(a, dtype=np.float32).copy(order="C")) for n, a in tensors.items()]
    index_size = 12 + sum(4 + len(n.encode()) + 4 + 4 * a.ndim + 8 for n, a in items)
    off = (index_size + 63) // 64 * 64
    offsets = []
    for _, a in items:
        offsets.append(off)
        off = (off + a.nbytes + 63) // 64 * 64
    with open(path, "wb") as f:
        f.write(b"LFM2" + struct.pack("<II", version, len(items)))
        for (n, a), o in zip(items, offsets):
            nb = n.encode()
            f.write(struct.pack("<I", len(nb)) + nb + struct.pack("<I", a.ndim))
            f.write(struct.pack(f"<{a.ndim}I", *a.shape) if a.ndim else b"")
            f.write(struct.pack("<Q", o))
        for (_, a), o in zip(items, offsets):
            f.seek(o)
            f.write(a.tobytes())


class ModelFile:
    """A model file opened through the library's loader (memory-mapped)."""

    def __init__(self, path: str):
        self.lib = _lib.load()
        h = C.c_void_p()
        check(self.lib.b2_loader_open(str(path).encode(), C.byref(h)), f"b2_loader_open({path})")
        self._h = h

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def names(self) -> Iterable[str]:
        return [self.lib.b2_loader_name(self._h, i).decode()
                for i in range(self.lib.b2_loader_num_tensors(self._h))]

    def shape(self, name: str) -> Tuple[int, ...]:
        shp = (C.c_int64 * 8)()
        nd = C.c_int(0)
        check(self.lib.b2_loader_tensor(self._h, name.encode(), None, None, shp, C.byref(nd)),
              f"tensor {name}")
        return tuple(shp[i] for i in range(nd.value))

    def has(self, name: str) -> bool:
        return self.lib.b2_loader_tensor(self._h, name.encode(), None, None, None, None) == 0

    def tensor(self, name: str) -> np.ndarray:
        """A read-only view of the tensor's fp32 data in the mapping."""
        p = C.c_void_p()
        n = C.c_int64(0)
        shp = (C.c_int64 * 8)()
        nd = C.c_int(0)
        check(self.lib.b2_loader_tensor(self._h, name.encode(), C.byref(p), C.byref(n), shp,
                                        C.byref(nd)), f"tensor {name}")
        if n.value == 0:
            return np.zeros(tuple(shp[i] for i in range(nd.value)), dtype=np.float32)
        a = np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), shape=(n.value,))
        a = a.reshape(tuple(shp[i] for i in range(nd.value)))
        a.flags.writeable = False
        return a

    def config(self) -> Dict[str, object]:
        """Model configuration implied by the tensors present."""
        names = set(self.names())
        layers = 1 + max(int(m.group(1)) for m in
                         (re.match(r"layers\.(\d+)\.", n) for n in names) if m)
        V, H = self.shape("embed_tokens.weight")
        types = [0 if f"layers.{i}.self_attn.q_proj.weight" in names else 1
                 for i in range(layers)]
        dense = 0
        while dense < layers and f"layers.{dense}.feed_forward.w1.weight" in names:
            dense += 1
        cfg = dict(vocab=V, hidden=H, num_layers=layers, num_dense_layers=dense,
                   layer_types=types)
        a = next((i for i in range(layers) if types[i] == 0), None)
        if a is not None:
            cfg["num_heads"] = self.shape(f"layers.{a}.self_attn.q_proj.weight")[0] // 64
            cfg["num_kv_heads"] = self.shape(f"layers.{a}.self_attn.k_proj.weight")[0] // 64
        else:
            cfg["num_heads"], cfg["num_kv_heads"] = H // 64, max(H // 256, 1)
        if dense:
            cfg["dense_inter"] = self.shape("layers.0.feed_forward.w1.weight")[0]
        if dense < layers:
            m = f"layers.{dense}.feed_forward."
            cfg["num_experts"] = self.shape(m + "gate.weight")[0]
            cfg["moe_inter"] = self.shape(m + "experts.0.w1.weight")[0]
            cfg["use_expert_bias"] = int(m + "expert_bias" in names)
        return cfg

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.b2_loader_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
