"""Python host mirror of the reference's MoE / GEMM operator interface.

``SparseMoeBlock`` mirrors the reference class of the same name
(include/layer.h:72-123): weights are handed over once (``init_gpu``), then
``forward_gpu(x, y, batch, seq_len, hidden_size, stream)`` runs the layer on
caller-owned fp32 device buffers, stream-ordered, exactly like
SparseMoeBlock::forward_gpu (src/layer.cu:1428-1498).  All compute goes
through the C ABI of ``libb2moe.so``; PyTorch only provides device memory and
streams here.  Errors raise ``B2Error`` instead of exiting the process (the
reference's CHECK_CUDA calls exit(), include/tensor.h:9-17).
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import B2_BF16, B2_TF32, MoeDesc, MoeTrace, check

_DT = {"bf16": B2_BF16, "tf32": B2_TF32}


def _stream_ptr(stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _expert_ptrs(w) -> list:
    """Per-expert device pointers of a stacked [E, r, c] tensor or a list."""
    if isinstance(w, torch.Tensor):
        assert w.is_cuda and w.dtype == torch.float32 and w.is_contiguous()
        step = w[0].numel() * 4
        return [w.data_ptr() + e * step for e in range(w.shape[0])]
    out = []
    for t in w:
        assert t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()
        out.append(t.data_ptr())
    return out


class SparseMoeBlock:
    """MoE layer: router top-k, scatter, tcgen05 W1/W3-SwiGLU and W2, combine.

    gate: [E, H] fp32; w1, w3: [E, I, H] fp32 (or E tensors [I, H]);
    w2: [E, H, I] fp32; expert_bias: [E] fp32 or None.  All on one CUDA
    device.  ``dtype`` selects the expert-GEMM operand type: "bf16" (default,
    fp32 accumulate) or "tf32" (fp32 operands, fp32 accumulate).
    """

    def __init__(self, gate: torch.Tensor, w1, w2, w3, expert_bias: Optional[torch.Tensor] = None,
                 *, max_tokens: int, top_k: int = 4, routed_scale: float = 1.0,
                 dtype: str = "bf16", stream: Optional[torch.cuda.Stream] = None):
        self.lib = _lib.load()
        E, H = gate.shape
        I = (w1.shape[1] if isinstance(w1, torch.Tensor) else w1[0].shape[0])
        self.E, self.H, self.I, self.K = E, H, I, top_k
        self.max_tokens = max_tokens
        self.device = gate.device
        d = MoeDesc(hidden=H, inter=I, num_experts=E, top_k=top_k, max_tokens=max_tokens,
                    routed_scale=routed_scale, use_bias=1 if expert_bias is not None else 0,
                    dtype=_DT[dtype])
        p1, p2, p3 = (_expert_ptrs(w) for w in (w1, w2, w3))
        arr = C.c_void_p * E
        handle = C.c_void_p()
        with torch.cuda.device(self.device):
            gate = gate.contiguous()
            bias_ptr = expert_bias.contiguous().data_ptr() if expert_bias is not None else None
            check(self.lib.b2_moe_create(C.byref(d), arr(*p1), arr(*p2), arr(*p3),
                                         C.c_void_p(gate.data_ptr()), C.c_void_p(bias_ptr),
                                         0, C.c_void_p(_stream_ptr(stream)), C.byref(handle)),
                  "b2_moe_create")
        self._h = handle

    # -- reference-shaped entry point --------------------------------------
    def forward_gpu(self, x: torch.Tensor, y: torch.Tensor, batch: int, seq_len: int,
                    hidden_size: int, stream: Optional[torch.cuda.Stream] = None) -> None:
        assert hidden_size == self.H
        T = batch * seq_len
        assert x.is_contiguous() and y.is_contiguous() and x.numel() >= T * self.H
        check(self.lib.b2_moe_forward(self._h, C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()),
                                      T, C.c_void_p(_stream_ptr(stream))), "b2_moe_forward")

    def forward(self, x: torch.Tensor, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        T = x.shape[0]
        y = torch.empty(T, self.H, dtype=torch.float32, device=x.device)
        self.forward_gpu(x, y, 1, T, self.H, stream)
        return y

    def forward_traced(self, x: torch.Tensor) -> dict:
        """Forward that also returns every intermediate the parity tests check."""
        T, E, K = x.shape[0], self.E, self.K
        dev = x.device
        out = {
            "y": torch.empty(T, self.H, dtype=torch.float32, device=dev),
            "logits": torch.empty(T, E, dtype=torch.float32, device=dev),
            "topk_idx": torch.empty(T, K, dtype=torch.int32, device=dev),
            "topk_w": torch.empty(T, K, dtype=torch.float32, device=dev),
            "counts": torch.empty(E, dtype=torch.int32, device=dev),
            "offsets": torch.empty(E, dtype=torch.int32, device=dev),
            "mtile_offsets": torch.empty(E + 1, dtype=torch.int32, device=dev),
            "token_slot": torch.empty(T, K, dtype=torch.int32, device=dev),
            "sorted_token": torch.full((T * K,), -1, dtype=torch.int32, device=dev),
            "sorted_w": torch.zeros(T * K, dtype=torch.float32, device=dev),
        }
        tr = MoeTrace(**{k: C.c_void_p(v.data_ptr()) for k, v in out.items() if k != "y"})
        check(self.lib.b2_moe_forward_ex(self._h, C.c_void_p(x.data_ptr()),
                                         C.c_void_p(out["y"].data_ptr()), T, C.byref(tr),
                                         C.c_void_p(_stream_ptr(None))), "b2_moe_forward_ex")
        return out

    def device_status(self) -> int:
        v = C.c_int(0)
        rc = self.lib.b2_moe_get_status(self._h, C.c_void_p(_stream_ptr(None)), C.byref(v))
        if rc not in (_lib.B2_OK, _lib.B2_ERR_DEVICE):
            check(rc, "b2_moe_get_status")
        return v.value

    STAGES = ("route", "scan", "scatter", "gemm_w13", "gemm_w2", "combine")

    def profile(self, enable: bool) -> None:
        check(self.lib.b2_moe_profile_enable(self._h, 1 if enable else 0), "b2_moe_profile_enable")

    def profile_read(self) -> tuple:
        """(summed ms per stage as a dict, number of forwards recorded)."""
        ms = (C.c_float * 6)()
        n = C.c_int(0)
        check(self.lib.b2_moe_profile_read(self._h, ms, C.byref(n)), "b2_moe_profile_read")
        return dict(zip(self.STAGES, list(ms))), n.value

    def device_bytes(self) -> int:
        return int(self.lib.b2_moe_device_bytes(self._h))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.b2_moe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_KINDS = {"single": 0, "pair": 1, "splitk": 2, "pairsplit": 3}


def gemm_nt(A: torch.Tensor, B: torch.Tensor, out: Optional[torch.Tensor] = None,
            dtype: str = "bf16", status: Optional[torch.Tensor] = None,
            stream: Optional[torch.cuda.Stream] = None, config=None) -> torch.Tensor:
    """C[M,N] fp32 = A[M,K] . B[N,K]^T on the tcgen05 core.

    dtype "bf16": A, B bf16.  dtype "tf32": A, B fp32 (TF32 tensor-core math).
    config: None (the planner's choice) or (kind, bn, split) as gemm_plan
    returns it, to run one kernel configuration (b2_gemm_nt_config).
    Replaces attn_matmul_tiled_kernel (src/layer.cu:9-141) and the LM-head
    GEMM (src/model.cu:42-116).
    """
    lib = _lib.load()
    M, K = A.shape
    N = B.shape[0]
    want = torch.bfloat16 if dtype == "bf16" else torch.float32
    assert A.dtype == want and B.dtype == want and A.is_contiguous() and B.is_contiguous()
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32, device=A.device)
    st = C.c_void_p(status.data_ptr()) if status is not None else None
    args = (C.c_void_p(A.data_ptr()), C.c_void_p(B.data_ptr()), C.c_void_p(out.data_ptr()), M,
            N, K, out.stride(0), _DT[dtype])
    if config is None:
        check(lib.b2_gemm_nt(*args, st, C.c_void_p(_stream_ptr(stream))), "b2_gemm_nt")
    else:
        kind, bn, split = config
        check(lib.b2_gemm_nt_config(*args, _KINDS[kind], bn, split, st,
                                    C.c_void_p(_stream_ptr(stream))), "b2_gemm_nt_config")
    return out


def to_bf16(x: torch.Tensor, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """fp32 -> bf16 with the library's conversion kernel."""
    lib = _lib.load()
    assert x.dtype == torch.float32 and x.is_contiguous() and x.is_cuda
    out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    check(lib.b2_convert_f32_to_bf16(C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()),
                                     x.numel(), C.c_void_p(_stream_ptr(stream))),
          "b2_convert_f32_to_bf16")
    return out


def launch_count() -> int:
    return int(_lib.load().b2_kernel_launch_count())


def gemm_plan(M: int, N: int, K: int, dtype: str = "bf16", sms: int = 148):
    """The kernel b2_gemm_nt picks for an M x N x K product on `sms` SMs:
    ("single" | "pair" | "splitk" | "pairsplit", tile width, K splits).  Host
    only."""
    lib = _lib.load()
    kind, bn, split = C.c_int(), C.c_int(), C.c_int()
    check(lib.b2_gemm_plan(M, N, K, _DT[dtype], sms, C.byref(kind), C.byref(bn), C.byref(split)),
          "b2_gemm_plan")
    return ("single", "pair", "splitk", "pairsplit")[kind.value], bn.value, split.value
