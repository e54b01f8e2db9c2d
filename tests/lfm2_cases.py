"""Seeded LFM2 decoder cases shared by the golden-fixture generator, the CPU
oracle tests and the GPU parity tests.

Weights are named as the reference engine names them in its model file
(src/layer.cu:1274-1297, 1508-1522, 1680-1690, 1797-1812; src/model.cu:
158-180) and drawn from the oracle's splitmix64/Box-Muller generator with one
stream per tensor name (crc32 of the name), so every tensor is bit-identical
wherever it is regenerated.  The oracle-side compositions below follow
DecoderLayer::forward_gpu (src/layer.cu:1895-1919) and the last pipeline
stage (src/model.cu:485-548).
"""
from __future__ import annotations

import zlib

import numpy as np

import oracle as o

# The reference model's shape (include/config.h:3-31).
H, HQ, HKV, HD = 2048, 32, 8, 64
E, K, I_MOE, I_DENSE = 32, 4, 1792, 7168
LAYER_TYPES = (1, 1, 0, 1, 1, 1, 0, 1, 1, 1, 0, 1, 1, 1, 0, 1, 1, 1, 0, 1, 1, 0, 1, 1)
NUM_DENSE = 2
THETA = 1000000.0

# A model with the reference's layer shapes but 4 layers (conv+MLP, conv+MLP,
# attention+MoE, conv+MoE: the first four of LAYER_TYPES) and a 1024-entry
# vocabulary, small enough for the CPU oracle.
MINI = dict(layers=4, vocab=1024, batch=2, seq=16, seed=21)

# Shapes of a model: the reference's, and a tiny one (model-file and C++
# class tests, where the whole model is written to disk).
REF = dict(H=H, HQ=HQ, HKV=HKV, E=E, K=K, I_MOE=I_MOE, I_DENSE=I_DENSE, NUM_DENSE=NUM_DENSE,
           TYPES=LAYER_TYPES)
TINY = dict(H=256, HQ=4, HKV=2, E=8, K=4, I_MOE=128, I_DENSE=384, NUM_DENSE=2,
            TYPES=(1, 1, 0, 1, 0), layers=5, vocab=300, batch=3, seq=23, seed=22)


def stream_of(name: str) -> int:
    return zlib.crc32(name.encode()) & 0xFFFFFFFF


def weight_spec(name: str, vocab: int, cfg=REF):
    """(shape, mean, std) of a tensor by its reference name."""
    H, HQ, HKV, E = cfg["H"], cfg["HQ"], cfg["HKV"], cfg["E"]
    I_MOE, I_DENSE = cfg["I_MOE"], cfg["I_DENSE"]
    p = name.split(".")
    if name == "embed_tokens.weight":
        return (vocab, H), 0.0, 1.0
    if name == "lm_head.weight":
        return (vocab, H), 0.0, 0.02
    if name == "embedding_norm.weight" or p[-2].endswith("norm") or p[-2].endswith("layernorm"):
        n = HD if "layernorm" in p[-2] else H
        return (n,), 1.0, 0.1
    if "self_attn" in p:
        return {"q_proj": (HQ * HD, H), "k_proj": (HKV * HD, H), "v_proj": (HKV * HD, H),
                "out_proj": (H, HQ * HD)}[p[-2]], 0.0, 0.02
    if "conv" in p:
        return {"conv": (H, 1, 3), "in_proj": (3 * H, H), "out_proj": (H, H)}[p[-2]], 0.0, \
            (0.3 if p[-2] == "conv" else 0.02)
    if "experts" in p:
        return {"w1": (I_MOE, H), "w3": (I_MOE, H), "w2": (H, I_MOE)}[p[-2]], 0.0, 0.02
    if p[-2] == "gate":
        return (E, H), 0.0, 0.02
    if p[-1] == "expert_bias":
        return (E,), 0.0, 0.02
    if "feed_forward" in p:
        return {"w1": (I_DENSE, H), "w3": (I_DENSE, H), "w2": (H, I_DENSE)}[p[-2]], 0.0, 0.02
    raise KeyError(name)


class Weights:
    """Lazily generated, cached tensors by reference name."""

    def __init__(self, seed: int, vocab: int, cfg=REF):
        self.seed, self.vocab, self.cache, self.cfg = seed, vocab, {}, cfg

    def __call__(self, name: str) -> np.ndarray:
        if name not in self.cache:
            shape, mean, std = weight_spec(name, self.vocab, self.cfg)
            a = o.randn(shape, self.seed, stream_of(name), std)
            if mean:
                a = (a + np.float32(mean)).astype(np.float32)
            self.cache[name] = a
        return self.cache[name]

    def drop(self, prefix: str) -> None:
        for k in [k for k in self.cache if k.startswith(prefix)]:
            del self.cache[k]


def layer_names(i: int, is_attention: bool, cfg=REF):
    E, NUM_DENSE = cfg["E"], cfg["NUM_DENSE"]
    pre = f"layers.{i}."
    names = [pre + "operator_norm.weight", pre + "ffn_norm.weight"]
    if is_attention:
        names += [pre + f"self_attn.{n}.weight" for n in ("q_proj", "k_proj", "v_proj", "out_proj",
                                                          "q_layernorm", "k_layernorm")]
    else:
        names += [pre + f"conv.{n}.weight" for n in ("conv", "in_proj", "out_proj")]
    if i >= NUM_DENSE:
        names += [pre + "feed_forward.gate.weight", pre + "feed_forward.expert_bias"]
        for e in range(E):
            names += [pre + f"feed_forward.experts.{e}.{w}.weight" for w in ("w1", "w2", "w3")]
    else:
        names += [pre + f"feed_forward.{w}.weight" for w in ("w1", "w2", "w3")]
    return names


def model_names(layers: int, cfg=REF):
    """Every tensor name of a model with `layers` layers (tied LM head)."""
    names = ["embed_tokens.weight", "embedding_norm.weight"]
    for i in range(layers):
        names += layer_names(i, cfg["TYPES"][i] == 0, cfg)
    return names


def experts(W: Weights, i: int):
    E = W.cfg["E"]
    pre = f"layers.{i}.feed_forward."
    w1 = np.stack([W(pre + f"experts.{e}.w1.weight") for e in range(E)])
    w2 = np.stack([W(pre + f"experts.{e}.w2.weight") for e in range(E)])
    w3 = np.stack([W(pre + f"experts.{e}.w3.weight") for e in range(E)])
    return w1, w2, w3


def mixer_oracle(W: Weights, i: int, xn: np.ndarray, B: int, S: int, cos, sin):
    """The layer's attention or short-conv block on its normed input."""
    pre = f"layers.{i}."
    if W.cfg["TYPES"][i] == 0:
        return o.attention_block(xn, W(pre + "self_attn.q_proj.weight"),
                                 W(pre + "self_attn.k_proj.weight"),
                                 W(pre + "self_attn.v_proj.weight"),
                                 W(pre + "self_attn.out_proj.weight"),
                                 W(pre + "self_attn.q_layernorm.weight"),
                                 W(pre + "self_attn.k_layernorm.weight"), cos, sin, B, S)
    return o.shortconv_block(xn, W(pre + "conv.in_proj.weight"), W(pre + "conv.conv.weight"),
                             W(pre + "conv.out_proj.weight"), B, S)


def ffn_oracle(W: Weights, i: int, hn: np.ndarray):
    pre = f"layers.{i}.feed_forward."
    if i < W.cfg["NUM_DENSE"]:
        return o.dense_mlp(hn, W(pre + "w1.weight"), W(pre + "w3.weight"), W(pre + "w2.weight"))
    w1, w2, w3 = experts(W, i)
    return o.moe_forward(hn, W(pre + "gate.weight"), W(pre + "expert_bias"), w1, w2, w3,
                         K=W.cfg["K"])["y"]


def decoder_layer_oracle(W: Weights, i: int, x: np.ndarray, B: int, S: int, cos, sin):
    """DecoderLayer::forward_gpu (src/layer.cu:1895-1919)."""
    pre = f"layers.{i}."
    xn = o.rmsnorm(x, W(pre + "operator_norm.weight"))
    h = x + mixer_oracle(W, i, xn, B, S, cos, sin)
    hn = o.rmsnorm(h, W(pre + "ffn_norm.weight"))
    return h + ffn_oracle(W, i, hn)


def token_ids(B: int, S: int, vocab: int, seed: int) -> np.ndarray:
    u = o.randu(B * S, seed, 9)
    return np.minimum((u * vocab).astype(np.int32), vocab - 1).reshape(B, S)


def model_oracle(W: Weights, ids: np.ndarray, layers: int, want_hidden=False):
    """Embedding, `layers` decoder layers, final norm of each sequence's last
    token and the LM head (src/model.cu:404-548, tied weights when the model
    has no lm_head.weight, src/model.cu:172-179)."""
    B, S = ids.shape
    H = W.cfg["H"]
    cos, sin = o.rope_tables(S)
    x = W("embed_tokens.weight")[ids.reshape(-1)].astype(np.float32)
    hidden = []
    for i in range(layers):
        x = decoder_layer_oracle(W, i, x, B, S, cos, sin)
        hidden.append(x)
    last = x.reshape(B, S, H)[:, -1, :]
    hn = o.rmsnorm(last, W("embedding_norm.weight"))
    logits = o.gemm_nt(hn, W("embed_tokens.weight"))
    return (logits, hidden) if want_hidden else logits
