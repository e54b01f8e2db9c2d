"""Expert-parallel MoE layer: one process per GPU, NCCL dispatch / combine.

``ExpertParallelMoE`` is the multi-GPU counterpart of ``SparseMoeBlock``: each
rank routes its own tokens, rows travel to the rank that computes them and
come back for the local combine.  All of it runs in the C ABI of
include/b2moe_ep.h; torch.distributed is only used here to hand the NCCL
unique id from rank 0 to the others.

Placement (``mode``): "owner" -- rank r holds experts [r*E/G, (r+1)*E/G);
"balanced" -- every rank holds all experts and computes a contiguous share of
the globally expert-sorted rows; the shares split the estimated GEMM cost
(rows + 128 per non-empty (expert, source) block + 320 per expert) evenly
(skew-proof).
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib
from ._lib import B2_EP_BALANCED, B2_EP_OWNER, EpPlan, MoeDesc, check
from .moe import _DT, _expert_ptrs, _stream_ptr

MODES = {"owner": B2_EP_OWNER, "balanced": B2_EP_BALANCED}


def plan(counts, rank: int, mode: str = "balanced") -> dict:
    """Exchange plan of `rank` for a [world][E] count matrix (pure host)."""
    lib = _lib.load()
    import numpy as np
    c = np.ascontiguousarray(np.asarray(counts, dtype=np.int32))
    world, E = c.shape
    p = EpPlan()
    check(lib.b2_ep_plan_compute(world, rank, E, MODES[mode], c.ctypes.data, C.byref(p)),
          "b2_ep_plan_compute")
    return p.to_dict(world)


def fused_schedule(counts, rank: int, mode: str = "balanced", w2: bool = False) -> dict:
    """The group list of one fused launch of `rank` (pure host): per group its
    row count, C row, A row, local expert, source whose flag it waits on (-1:
    none), the rank its rows came from and (W2) its return chunk; plus the
    256-row tile prefix."""
    lib = _lib.load()
    import numpy as np
    c = np.ascontiguousarray(np.asarray(counts, dtype=np.int32))
    world, E = c.shape
    n1 = _lib.EP_MAX_SEGMENTS + 1
    buf = np.zeros(8 * n1, dtype=np.int32)
    g, mt = C.c_int(0), C.c_int(0)
    check(lib.b2_ep_fused_schedule(world, rank, E, MODES[mode], c.ctypes.data, int(w2),
                                   buf.ctypes.data, C.byref(g), C.byref(mt)),
          "b2_ep_fused_schedule")
    n = g.value
    a = buf.reshape(8, n1)
    return {"count": a[0, :n].copy(), "c_row": a[1, :n].copy(), "mtile": a[2, :n + 1].copy(),
            "expert": a[3, :n].copy(), "a_row": a[4, :n].copy(), "source": a[5, :n].copy(),
            "dest": a[6, :n].copy(), "chunk": a[7, :n].copy(), "mtiles": mt.value}


def unique_id() -> bytes:
    lib = _lib.load()
    buf = (C.c_char * 128)()
    check(lib.b2_ep_unique_id(buf), "b2_ep_unique_id")
    return bytes(buf)


class ExpertParallelMoE:
    """gate [E,H], w1/w3 [E,I,H], w2 [E,H,I] fp32 on this rank's device: the
    full layer; the rank keeps the experts its mode needs.  ``uid`` is the
    NCCL unique id (bytes); when None it is created on rank 0 and broadcast
    over the default torch.distributed group."""

    def __init__(self, gate: torch.Tensor, w1, w2, w3, expert_bias: Optional[torch.Tensor] = None,
                 *, max_tokens: int, top_k: int = 4, routed_scale: float = 1.0,
                 dtype: str = "bf16", mode: str = "balanced", world: Optional[int] = None,
                 rank: Optional[int] = None, uid: Optional[bytes] = None,
                 timeout_s: float = 60.0, stream: Optional[torch.cuda.Stream] = None,
                 pipeline: str = "fused"):
        import torch.distributed as dist
        self.lib = _lib.load()
        if world is None:
            world = dist.get_world_size() if dist.is_initialized() else 1
        if rank is None:
            rank = dist.get_rank() if dist.is_initialized() else 0
        self.world, self.rank, self.mode = world, rank, mode
        E, H = gate.shape
        I = w1.shape[1]
        self.E, self.H, self.I, self.K = E, H, I, top_k
        if uid is None:
            if world == 1:
                uid = unique_id()
            else:
                obj = [unique_id() if rank == 0 else None]
                dist.broadcast_object_list(obj, src=0)
                uid = obj[0]
        if mode == "owner":
            el = E // world
            sel = slice(rank * el, (rank + 1) * el)
            w1, w2, w3 = w1[sel].contiguous(), w2[sel].contiguous(), w3[sel].contiguous()
        nw = w1.shape[0]
        arr = C.c_void_p * nw
        p1, p2, p3 = (_expert_ptrs(w) for w in (w1, w2, w3))
        d = MoeDesc(hidden=H, inter=I, num_experts=E, top_k=top_k, max_tokens=max_tokens,
                    routed_scale=routed_scale, use_bias=1 if expert_bias is not None else 0,
                    dtype=_DT[dtype])
        idbuf = (C.c_char * 128).from_buffer_copy(uid)
        handle = C.c_void_p()
        gate = gate.contiguous()
        bias_ptr = expert_bias.contiguous().data_ptr() if expert_bias is not None else None
        check(self.lib.b2_ep_create(C.byref(d), world, rank, idbuf, MODES[mode], arr(*p1),
                                    arr(*p2), arr(*p3), C.c_void_p(gate.data_ptr()),
                                    C.c_void_p(bias_ptr), 0, C.c_void_p(_stream_ptr(stream)),
                                    C.byref(handle)), "b2_ep_create")
        self._h = handle
        check(self.lib.b2_ep_set_timeout(self._h, C.c_double(timeout_s)), "b2_ep_set_timeout")
        self.set_pipeline(pipeline)

    def forward_gpu(self, x: torch.Tensor, y: torch.Tensor, num_tokens: int,
                    stream: Optional[torch.cuda.Stream] = None) -> None:
        check(self.lib.b2_ep_forward(self._h, C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()),
                                     num_tokens, C.c_void_p(_stream_ptr(stream))), "b2_ep_forward")

    def forward(self, x: torch.Tensor, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        y = torch.empty(x.shape[0], self.H, dtype=torch.float32, device=x.device)
        self.forward_gpu(x, y, x.shape[0], stream)
        return y

    def last_plan(self) -> dict:
        p = EpPlan()
        check(self.lib.b2_ep_last_plan(self._h, C.byref(p)), "b2_ep_last_plan")
        return p.to_dict(self.world)

    def _layer(self):
        return self.lib.b2_ep_layer(self._h)

    def profile(self, enable: bool) -> None:
        check(self.lib.b2_moe_profile_enable(self._layer(), 1 if enable else 0), "profile")

    def profile_read(self) -> tuple:
        ms = (C.c_float * 6)()
        n = C.c_int(0)
        check(self.lib.b2_moe_profile_read(self._layer(), ms, C.byref(n)), "profile_read")
        from .moe import SparseMoeBlock
        return dict(zip(SparseMoeBlock.STAGES, list(ms))), n.value

    TIMELINE = ("start", "scattered", "planned", "own_first", "arrived", "remote_done",
                "own_second", "returned", "done", "host_wait", "host_enqueue", "w13_done",
                "w2_done")
    PIPELINES = {"fused": 0, "staged": 1}

    def set_pipeline(self, pipeline: str) -> None:
        """"fused" (default): one W1||W3 and one W2 launch over every source's
        rows, results returned chunk by chunk by the copy engine as W2 counts
        them stored; "staged": a launch pair per source, results returned by
        the copy engine after each pair."""
        check(self.lib.b2_ep_set_pipeline(self._h, self.PIPELINES[pipeline]),
              "b2_ep_set_pipeline")

    def timeline(self) -> list:
        """[(mark, us since the forward started)] of the last forward run with
        profiling on (b2_ep_profile_timeline)."""
        tags, ms, n = (C.c_int * 64)(), (C.c_float * 64)(), C.c_int(0)
        check(self.lib.b2_ep_profile_timeline(self._h, 64, tags, ms, C.byref(n)),
              "b2_ep_profile_timeline")
        return [(self.TIMELINE[tags[i]], round(ms[i] * 1e3, 1)) for i in range(n.value)]

    def device_status(self) -> int:
        v = C.c_int(0)
        rc = self.lib.b2_moe_get_status(self._layer(), C.c_void_p(_stream_ptr(None)), C.byref(v))
        if rc not in (_lib.B2_OK, _lib.B2_ERR_DEVICE):
            check(rc, "b2_moe_get_status")
        return v.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.b2_ep_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
