"""Python host mirror of the reference's decoder operators around the MoE:
``RMSNorm``, ``rope_tables`` (RotaryEmbedding), ``Attention``, ``ShortConv``
and the whole-model ``LFM2Model`` (include/layer.h:10-176,
include/model.h:28-36 of the reference).

The weights are handed over once; ``forward_gpu`` runs on caller-owned fp32
device buffers, stream-ordered, with the reference's argument order.  All
compute goes through the C ABI of include/b2lfm2.h; errors raise B2Error.
"""
from __future__ import annotations

import ctypes as C
import zlib
from typing import Callable, Dict, Optional

import numpy as np
import torch

from . import _lib
from ._lib import AttnDesc, ConvDesc, Lfm2Desc, WEIGHT_FN, check
from .moe import _DT, _stream_ptr

# The reference model (include/config.h:3-31).
LAYER_TYPES = (1, 1, 0, 1, 1, 1, 0, 1, 1, 1, 0, 1, 1, 1, 0, 1, 1, 1, 0, 1, 1, 0, 1, 1)
CONFIG = dict(vocab=65536, hidden=2048, num_layers=24, num_heads=32, num_kv_heads=8,
              dense_inter=7168, moe_inter=1792, num_experts=32, top_k=4, num_dense_layers=2,
              eps=1e-5, rope_theta=1e6, routed_scale=1.0, use_expert_bias=1)


def _vp(t) -> C.c_void_p:
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p()


def _dev_f32(t: torch.Tensor) -> None:
    assert t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5,
            stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """RMSNorm over the last axis (RMSNorm::forward_gpu, src/layer.cu:1144-1148)."""
    _dev_f32(x)
    _dev_f32(w)
    dim = x.shape[-1]
    y = torch.empty_like(x)
    check(_lib.load().b2_rmsnorm(_vp(x), _vp(w), _vp(y), x.numel() // dim, dim, eps,
                                 C.c_void_p(_stream_ptr(stream))), "b2_rmsnorm")
    return y


def rope_tables(max_pos: int, head_dim: int = 64, base: float = 1e6):
    """Host cos / sin tables [max_pos][head_dim] (RotaryEmbedding::init_gpu)."""
    c = np.empty((max_pos, head_dim), dtype=np.float32)
    s = np.empty_like(c)
    check(_lib.load().b2_rope_tables(c.ctypes.data, s.ctypes.data, max_pos, head_dim, base),
          "b2_rope_tables")
    return c, s


def embed(ids: torch.Tensor, table: torch.Tensor,
          stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """hidden[t] = table[ids[t]] (embedding_lookup_kernel, src/model.cu:18-31)."""
    _dev_f32(table)
    ids = ids.to(torch.int32).contiguous()
    V, H = table.shape
    out = torch.empty(ids.numel(), H, dtype=torch.float32, device=table.device)
    status = torch.zeros(1, dtype=torch.int32, device=table.device)
    check(_lib.load().b2_embed(_vp(ids), _vp(table), _vp(out), ids.numel(), H, V, _vp(status),
                               C.c_void_p(_stream_ptr(stream))), "b2_embed")
    return out


class _Handle:
    _destroy = ""

    def close(self) -> None:
        if getattr(self, "_h", None):
            getattr(self.lib, self._destroy)(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Attention(_Handle):
    """GQA attention block (Attention, include/layer.h:126-159): wq [Hq*64, H],
    wk / wv [Hkv*64, H], wo [H, Hq*64], q_ln / k_ln [64], fp32 on one device."""
    _destroy = "b2_attn_destroy"

    def __init__(self, wq, wk, wv, wo, q_ln, k_ln, *, max_tokens: int, eps: float = 1e-5,
                 stream: Optional[torch.cuda.Stream] = None):
        self.lib = _lib.load()
        for t in (wq, wk, wv, wo, q_ln, k_ln):
            _dev_f32(t)
        self.H = wq.shape[1]
        d = AttnDesc(hidden=self.H, num_heads=wq.shape[0] // 64, num_kv_heads=wk.shape[0] // 64,
                     head_dim=64, max_tokens=max_tokens, eps=eps)
        h = C.c_void_p()
        with torch.cuda.device(wq.device):
            check(self.lib.b2_attn_create(C.byref(d), _vp(wq), _vp(wk), _vp(wv), _vp(wo),
                                          _vp(q_ln), _vp(k_ln), 0,
                                          C.c_void_p(_stream_ptr(stream)), C.byref(h)),
                  "b2_attn_create")
        self._h = h

    def forward_gpu(self, x, cos, sin, output, batch: int, seq_len: int, hidden_size: int,
                    stream: Optional[torch.cuda.Stream] = None) -> None:
        assert hidden_size == self.H
        check(self.lib.b2_attn_forward(self._h, _vp(x), _vp(cos), _vp(sin), _vp(output), batch,
                                       seq_len, C.c_void_p(_stream_ptr(stream))),
              "b2_attn_forward")

    def forward(self, x, cos, sin, batch: int, seq_len: int) -> torch.Tensor:
        y = torch.empty(batch * seq_len, self.H, dtype=torch.float32, device=x.device)
        self.forward_gpu(x, cos, sin, y, batch, seq_len, self.H)
        return y


class ShortConv(_Handle):
    """Gated short-convolution block (ShortConv, include/layer.h:161-194):
    conv_w [H, 1, 3], in_w [3H, H], out_w [H, H], fp32 on one device."""
    _destroy = "b2_conv_destroy"

    def __init__(self, conv_w, in_w, out_w, *, max_tokens: int,
                 stream: Optional[torch.cuda.Stream] = None):
        self.lib = _lib.load()
        for t in (conv_w, in_w, out_w):
            _dev_f32(t)
        self.H = out_w.shape[0]
        d = ConvDesc(hidden=self.H, kernel=conv_w.shape[-1], max_tokens=max_tokens)
        h = C.c_void_p()
        with torch.cuda.device(in_w.device):
            check(self.lib.b2_conv_create(C.byref(d), _vp(conv_w), _vp(in_w), _vp(out_w), 0,
                                          C.c_void_p(_stream_ptr(stream)), C.byref(h)),
                  "b2_conv_create")
        self._h = h

    def forward_gpu(self, x, y, batch: int, seq_len: int, hidden_size: int,
                    stream: Optional[torch.cuda.Stream] = None) -> None:
        assert hidden_size == self.H
        check(self.lib.b2_conv_forward(self._h, _vp(x), _vp(y), batch, seq_len,
                                       C.c_void_p(_stream_ptr(stream))), "b2_conv_forward")

    def forward(self, x, batch: int, seq_len: int) -> torch.Tensor:
        y = torch.empty(batch * seq_len, self.H, dtype=torch.float32, device=x.device)
        self.forward_gpu(x, y, batch, seq_len, self.H)
        return y


class LFM2Model(_Handle):
    """The whole model on one GPU (LFM2Model, include/model.h:28-36).

    ``weights(name, numel)`` returns the tensor of that reference name (an
    fp32 torch tensor on the device, or a numpy array with
    ``weights_on_host=True``) or None when the model has no such tensor; the
    returned objects are kept alive until construction ends.  Other
    keywords override the reference configuration (``CONFIG``).

    ``expert_parallel`` ("balanced" or "owner") builds the expert-parallel
    model instead (b2_lfm2_create_ep): one rank per GPU, every MoE layer an
    expert-parallel layer over ``world`` ranks, all of them sharing one NCCL
    communicator made from ``uid`` (created on rank 0 and broadcast over the
    default torch.distributed group when None).  Construction, forward and
    close are collective."""
    _destroy = "b2_lfm2_destroy"

    def __init__(self, weights: Callable[[str, int], object], *, max_batch: int, max_seq: int,
                 weights_on_host: bool = False, layer_types=LAYER_TYPES, dtype: str = "bf16",
                 device: Optional[torch.device] = None,
                 stream: Optional[torch.cuda.Stream] = None,
                 expert_parallel: Optional[str] = None, world: Optional[int] = None,
                 rank: Optional[int] = None, uid: Optional[bytes] = None, **cfg):
        self.lib = _lib.load()
        c = dict(CONFIG)
        c.update(cfg)
        self.cfg = c
        self.layers = c["num_layers"]
        d = Lfm2Desc(vocab=c["vocab"], hidden=c["hidden"], num_layers=c["num_layers"],
                     num_heads=c["num_heads"], num_kv_heads=c["num_kv_heads"],
                     dense_inter=c["dense_inter"], moe_inter=c["moe_inter"],
                     num_experts=c["num_experts"], top_k=c["top_k"],
                     num_dense_layers=c["num_dense_layers"], max_batch=max_batch,
                     max_seq=max_seq, eps=c["eps"], rope_theta=c["rope_theta"],
                     routed_scale=c["routed_scale"], use_expert_bias=c["use_expert_bias"],
                     dtype=_DT[dtype])
        for i in range(c["num_layers"]):
            d.layer_types[i] = int(layer_types[i])
        self.vocab, self.H = c["vocab"], c["hidden"]
        self.max_batch, self.max_seq = max_batch, max_seq
        keep: Dict[str, object] = {}

        def get(_ctx, name, numel):
            t = weights(name.decode(), int(numel))
            if t is None:
                return None
            if isinstance(t, np.ndarray):
                assert weights_on_host and t.dtype == np.float32 and t.flags.c_contiguous
                assert t.size == numel, (name, t.size, numel)
                keep[name] = t
                return t.ctypes.data
            assert not weights_on_host
            _dev_f32(t)
            assert t.numel() == numel, (name, t.numel(), numel)
            keep[name] = t
            return t.data_ptr()

        from .modelfile import ModelFile
        if isinstance(weights, ModelFile):
            # straight from the memory-mapped file: the C loader is the source
            cb, ctx, weights_on_host = C.cast(self.lib.b2_loader_weight, WEIGHT_FN), \
                weights.handle, True
        else:
            cb, ctx = WEIGHT_FN(get), None
        h = C.c_void_p()
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.expert_parallel = expert_parallel
        with torch.cuda.device(self.device):
            if expert_parallel is None:
                check(self.lib.b2_lfm2_create(C.byref(d), cb, ctx, int(weights_on_host),
                                              C.c_void_p(_stream_ptr(stream)), C.byref(h)),
                      "b2_lfm2_create")
            else:
                from .ep import MODES, unique_id
                import torch.distributed as dist
                if world is None:
                    world = dist.get_world_size() if dist.is_initialized() else 1
                if rank is None:
                    rank = dist.get_rank() if dist.is_initialized() else 0
                if uid is None:
                    if world == 1:
                        uid = unique_id()
                    else:
                        obj = [unique_id() if rank == 0 else None]
                        dist.broadcast_object_list(obj, src=0)
                        uid = obj[0]
                self.world, self.rank = world, rank
                idbuf = C.create_string_buffer(bytes(uid), len(uid))
                check(self.lib.b2_lfm2_create_ep(C.byref(d), cb, ctx, int(weights_on_host),
                                                 world, rank, idbuf, MODES[expert_parallel],
                                                 C.c_void_p(_stream_ptr(stream)), C.byref(h)),
                      "b2_lfm2_create_ep")
        keep.clear()
        self._h = h

    @classmethod
    def from_file(cls, path: str, *, max_batch: int, max_seq: int, dtype: str = "bf16",
                  device: Optional[torch.device] = None, **overrides) -> "LFM2Model":
        """Load a model file in the reference's format (final_b200.modelfile);
        the configuration is inferred from its tensors."""
        from .modelfile import ModelFile
        mf = ModelFile(path)
        try:
            cfg = mf.config()
            cfg.update(overrides)
            types = cfg.pop("layer_types")
            return cls(mf, max_batch=max_batch, max_seq=max_seq, layer_types=types,
                       dtype=dtype, device=device, **cfg)
        finally:
            mf.close()

    def forward_gpu(self, ids: torch.Tensor, logits: torch.Tensor, batch: int, seq_len: int,
                    stream: Optional[torch.cuda.Stream] = None, hidden_out=None) -> None:
        assert ids.dtype == torch.int32 and ids.is_contiguous() and ids.is_cuda
        fn = self.lib.b2_lfm2_forward_ex
        check(fn(self._h, _vp(ids), batch, seq_len, _vp(logits), _vp(hidden_out),
                 C.c_void_p(_stream_ptr(stream))), "b2_lfm2_forward")

    def forward(self, ids: torch.Tensor, want_hidden: bool = False):
        """ids [B, S] int -> logits [B, vocab] of each sequence's last position."""
        B, S = ids.shape
        ids = ids.to(device=self.device, dtype=torch.int32).contiguous()
        logits = torch.empty(B, self.vocab, dtype=torch.float32, device=self.device)
        hidden = (torch.empty(self.layers, B * S, self.H, dtype=torch.float32, device=self.device)
                  if want_hidden else None)
        self.forward_gpu(ids, logits, B, S, hidden_out=hidden)
        return (logits, hidden) if want_hidden else logits

    def device_status(self) -> int:
        v = C.c_int(0)
        rc = self.lib.b2_lfm2_get_status(self._h, C.c_void_p(_stream_ptr(None)), C.byref(v))
        if rc not in (_lib.B2_OK, _lib.B2_ERR_DEVICE):
            check(rc, "b2_lfm2_get_status")
        return v.value

    def device_bytes(self) -> int:
        return int(self.lib.b2_lfm2_device_bytes(self._h))


def synthetic_weights(device, seed: int = 0):
    """Random-init weights of the reference architecture, by tensor name, as
    fp32 tensors on `device`: embedding N(0,1); RMSNorm weights N(1,0.1);
    conv taps N(0,0.3); projections, experts, router and expert bias
    N(0,0.02); no separate lm_head.weight (tied, as the reference model).
    Each tensor's values depend only on (seed, name), so a rank that fetches
    a subset (an expert-parallel owner) gets the same tensors as a full model.
    For benchmarks: no checkpoint is needed."""
    g = torch.Generator(device=device)

    def get(name: str, numel: int):
        if name == "lm_head.weight":
            return None
        g.manual_seed((seed << 32) ^ zlib.crc32(name.encode()))
        last = name.split(".")[-2] if name.count(".") else name
        if name == "embed_tokens.weight":
            mean, std = 0.0, 1.0
        elif "norm" in last:
            mean, std = 1.0, 0.1
        elif name.endswith("conv.conv.weight"):
            mean, std = 0.0, 0.3
        else:
            mean, std = 0.0, 0.02
        return torch.empty(numel, dtype=torch.float32, device=device).normal_(mean, std,
                                                                              generator=g)
    return get


def model_flop(batch: int, seq: int, cfg=None, layer_types=LAYER_TYPES) -> float:
    """Algorithmic FLOP of one forward (2 per multiply-add): projections,
    causal attention core, dense MLP / MoE experts and router, last-token LM
    head; elementwise work not counted."""
    c = dict(CONFIG)
    c.update(cfg or {})
    H, Hq, Hkv = c["hidden"], c["num_heads"], c["num_kv_heads"]
    T = batch * seq
    f = 0.0
    for i in range(c["num_layers"]):
        if layer_types[i] == 0:
            f += T * 2.0 * H * (Hq + 2 * Hkv) * 64 + T * 2.0 * Hq * 64 * H
            f += batch * 4.0 * Hq * 64 * seq * (seq + 1) / 2
        else:
            f += T * 2.0 * H * 3 * H + T * 2.0 * H * H
        if i < c["num_dense_layers"]:
            f += T * 6.0 * H * c["dense_inter"]
        else:
            f += T * (2.0 * H * c["num_experts"] + c["top_k"] * 6.0 * H * c["moe_inter"])
    return f + batch * 2.0 * H * c["vocab"]
