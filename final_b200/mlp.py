"""Python host mirror of the reference's dense MLP operator (include/layer.h:48-66).

``MLP(w1, w2, w3, max_tokens=...)`` hands the weights over once (the
reference's ``init_gpu``); ``forward_gpu(x, y, batch, seq_len, hidden_size,
stream)`` runs y = (silu(x.W1^T) * (x.W3^T)).W2^T on caller-owned fp32 device
buffers, stream-ordered, like MLP::forward_gpu (src/layer.cu:1230-1269).
Compute goes through ``b2_mlp_*`` of the C ABI (include/b2mlp.h).
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib
from ._lib import MlpDesc, check
from .moe import _DT, _stream_ptr


class MLP:
    """Dense SwiGLU MLP.  w1 (gate), w3 (up): [I, H] fp32; w2: [H, I] fp32, on
    one CUDA device.  ``dtype``: "bf16" (default) or "tf32" GEMM operands."""

    def __init__(self, w1: torch.Tensor, w2: torch.Tensor, w3: torch.Tensor, *, max_tokens: int,
                 dtype: str = "bf16", stream: Optional[torch.cuda.Stream] = None):
        self.lib = _lib.load()
        I, H = w1.shape
        assert w3.shape == (I, H) and w2.shape == (H, I)
        for w in (w1, w2, w3):
            assert w.is_cuda and w.dtype == torch.float32 and w.is_contiguous()
        self.H, self.I, self.max_tokens = H, I, max_tokens
        self.device = w1.device
        d = MlpDesc(hidden=H, inter=I, max_tokens=max_tokens, dtype=_DT[dtype])
        handle = C.c_void_p()
        with torch.cuda.device(self.device):
            check(self.lib.b2_mlp_create(C.byref(d), C.c_void_p(w1.data_ptr()),
                                         C.c_void_p(w2.data_ptr()), C.c_void_p(w3.data_ptr()), 0,
                                         C.c_void_p(_stream_ptr(stream)), C.byref(handle)),
                  "b2_mlp_create")
        self._h = handle

    def forward_gpu(self, x: torch.Tensor, y: torch.Tensor, batch: int, seq_len: int,
                    hidden_size: int, stream: Optional[torch.cuda.Stream] = None) -> None:
        assert hidden_size == self.H
        T = batch * seq_len
        assert x.is_contiguous() and y.is_contiguous() and x.numel() >= T * self.H
        check(self.lib.b2_mlp_forward(self._h, C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()),
                                      T, C.c_void_p(_stream_ptr(stream))), "b2_mlp_forward")

    def forward(self, x: torch.Tensor, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        T = x.shape[0]
        y = torch.empty(T, self.H, dtype=torch.float32, device=x.device)
        self.forward_gpu(x, y, 1, T, self.H, stream)
        return y

    def device_status(self) -> int:
        v = C.c_int(0)
        rc = self.lib.b2_mlp_get_status(self._h, C.c_void_p(_stream_ptr(None)), C.byref(v))
        if rc not in (_lib.B2_OK, _lib.B2_ERR_DEVICE):
            check(rc, "b2_mlp_get_status")
        return v.value

    def device_bytes(self) -> int:
        return int(self.lib.b2_mlp_device_bytes(self._h))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.b2_mlp_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
