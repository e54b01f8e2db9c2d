"""ctypes wrapper of the CPU oracle (oracle/moe_oracle.c) and of the
reference-kernel harness (oracle/_ref/libref_moe.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference leg of bench.py.  The product path
(final_b200/) never imports this module.

Also defines the seeded synthetic inputs every test, fixture and bench
configuration uses, so that they can be regenerated bit-identically on any
machine from (seed, stream) pairs.
"""
from __future__ import annotations

import ctypes as C
import math
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libref_moe.so"

_o = None
_r = None

f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")


def lib():
    """Load (building with make if needed) the oracle library."""
    global _o
    if _o is not None:
        return _o
    if not LIB.exists():
        subprocess.run(["make", "-C", str(HERE), "liboracle.so"], check=True,
                       stdout=subprocess.DEVNULL)
    o = C.CDLL(str(LIB))
    vp = C.c_void_p
    o.b2o_gemm_nt.argtypes = [f32p, f32p, f32p, C.c_int, C.c_int, C.c_int]
    o.b2o_router_logits.argtypes = [f32p, f32p, f32p, C.c_int, C.c_int, C.c_int]
    o.b2o_route_topk.argtypes = [f32p, vp, C.c_int, C.c_int, C.c_int, C.c_float, i32p, f32p, vp]
    o.b2o_scan.argtypes = [i32p, C.c_int, C.c_int, i32p, i32p]
    o.b2o_scatter_canonical.argtypes = [i32p, f32p, C.c_int, C.c_int, C.c_int, i32p, vp, vp, i32p]
    o.b2o_expert_ffn.argtypes = [f32p, i32p, i32p, i32p, C.c_int, C.c_int, C.c_int,
                                 vp, vp, vp, vp, f32p]
    o.b2o_combine.argtypes = [f32p, i32p, f32p, C.c_int, C.c_int, C.c_int, f32p]
    o.b2o_randn.argtypes = [f32p, C.c_size_t, C.c_uint64, C.c_uint64, C.c_float]
    o.b2o_randu.argtypes = [f64p, C.c_size_t, C.c_uint64, C.c_uint64]
    o.b2o_set_num_threads.argtypes = [C.c_int]
    o.b2o_rmsnorm.argtypes = [f32p, f32p, f32p, C.c_int, C.c_int]
    o.b2o_rope_tables.argtypes = [f32p, f32p, C.c_int, C.c_int, C.c_float]
    o.b2o_attention_core.argtypes = [f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                     f32p, f32p, f32p, f32p, f32p]
    o.b2o_shortconv_core.argtypes = [f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int, f32p]
    _o = o
    return o


def set_threads(n: int) -> None:
    lib().b2o_set_num_threads(n)


def num_threads() -> int:
    return lib().b2o_num_threads()


# ------------------------------------------------------------------ inputs
def randn(shape, seed: int, stream: int, std: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    a = np.empty(n, dtype=np.float32)
    lib().b2o_randn(a, n, seed, stream, std)
    return a.reshape(shape)


def randu(n: int, seed: int, stream: int) -> np.ndarray:
    a = np.empty(n, dtype=np.float64)
    lib().b2o_randu(a, n, seed, stream)
    return a


# streams used for each tensor of an MoE layer
S_X, S_GATE, S_BIAS, S_W1, S_W3, S_W2, S_GUMBEL = 0, 1, 2, 100, 200, 300, 7


def moe_inputs(T, H, E, I, seed, *, x_std=1.0, w_std=0.02, bias_std=0.02, bias=True):
    """x ~ N(0,x_std), gate / w1 / w3 / w2 ~ N(0,w_std), bias ~ N(0,bias_std)."""
    x = randn((T, H), seed, S_X, x_std)
    gate = randn((E, H), seed, S_GATE, w_std)
    b = randn((E,), seed, S_BIAS, bias_std) if bias else None
    w1 = np.stack([randn((I, H), seed, S_W1 + e, w_std) for e in range(E)])
    w3 = np.stack([randn((I, H), seed, S_W3 + e, w_std) for e in range(E)])
    w2 = np.stack([randn((H, I), seed, S_W2 + e, w_std) for e in range(E)])
    return dict(x=x, gate=gate, bias=b, w1=w1, w2=w2, w3=w3)


def zipf_logits(T, E, seed, s=1.1):
    """L[t,e] = ln p_e + Gumbel(0,1), p_e ~ e^-s: the top-k of each row is a
    draw without replacement with probabilities p (Gumbel-top-k)."""
    p = np.arange(1, E + 1, dtype=np.float64) ** (-s)
    p /= p.sum()
    u = randu(T * E, seed, S_GUMBEL).reshape(T, E)
    return (np.log(p)[None, :] - np.log(-np.log(u))).astype(np.float32)


def inject_logits(x: np.ndarray, gate: np.ndarray, L: np.ndarray) -> None:
    """Make x . gate^T == L exactly: gate = [I_E | 0], x[:, :E] = L (in place).
    The router GEMM still runs over all H columns; every other product is an
    exact zero, so the sequential-k FMA chain returns L bit-for-bit."""
    E = gate.shape[0]
    gate[:] = 0.0
    gate[np.arange(E), np.arange(E)] = 1.0
    x[:, :E] = L


# ------------------------------------------------------------------ oracle
def gemm_nt(A, B):
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M, K = A.shape
    N = B.shape[0]
    Cm = np.empty((M, N), dtype=np.float32)
    lib().b2o_gemm_nt(A, B, Cm, M, N, K)
    return Cm


def route(logits, bias, K, routed_scale=1.0):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    idx = np.empty((T, K), dtype=np.int32)
    w = np.empty((T, K), dtype=np.float32)
    counts = np.zeros(E, dtype=np.int32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().b2o_route_topk(logits, b.ctypes.data if b is not None else None, T, E, K,
                         routed_scale, idx, w, counts.ctypes.data)
    return idx, w, counts


def scan(counts, tile):
    counts = np.ascontiguousarray(counts, dtype=np.int32)
    E = counts.shape[0]
    off = np.empty(E, dtype=np.int32)
    toff = np.empty(E + 1, dtype=np.int32)
    lib().b2o_scan(counts, E, tile, off, toff)
    return off, toff


def scatter(idx, w, E, offsets):
    T, K = idx.shape
    st = np.full(T * K, -1, dtype=np.int32)
    sw = np.zeros(T * K, dtype=np.float32)
    slot = np.empty((T, K), dtype=np.int32)
    lib().b2o_scatter_canonical(np.ascontiguousarray(idx, dtype=np.int32),
                                np.ascontiguousarray(w, dtype=np.float32), T, K, E,
                                np.ascontiguousarray(offsets, dtype=np.int32),
                                st.ctypes.data, sw.ctypes.data, slot)
    return st, sw, slot


def expert_ffn(x, sorted_token, offsets, counts, w1, w3, w2, want_inter=False):
    E, I, H = w1.shape
    R = int(counts.sum())
    out = np.zeros((max(R, 1), H), dtype=np.float32)
    inter = np.zeros((max(R, 1), I), dtype=np.float32) if want_inter else None
    arr = C.c_void_p * E
    w1 = np.ascontiguousarray(w1, dtype=np.float32)
    w3 = np.ascontiguousarray(w3, dtype=np.float32)
    w2 = np.ascontiguousarray(w2, dtype=np.float32)
    p1 = arr(*[w1[e].ctypes.data for e in range(E)])
    p3 = arr(*[w3[e].ctypes.data for e in range(E)])
    p2 = arr(*[w2[e].ctypes.data for e in range(E)])
    lib().b2o_expert_ffn(np.ascontiguousarray(x, dtype=np.float32),
                         np.ascontiguousarray(sorted_token, dtype=np.int32),
                         np.ascontiguousarray(offsets, dtype=np.int32),
                         np.ascontiguousarray(counts, dtype=np.int32), E, H, I,
                         C.cast(p1, C.c_void_p), C.cast(p3, C.c_void_p), C.cast(p2, C.c_void_p),
                         inter.ctypes.data if inter is not None else None, out)
    return (out, inter) if want_inter else out


def dense_mlp(x, w1, w3, w2):
    """Dense SwiGLU MLP of the layers without experts, MLP::forward_gpu
    (src/layer.cu:1230-1269): gate = x.W1^T, up = x.W3^T (attn_matmul_tiled_kernel,
    src/layer.cu:9-141), silu(gate) * up (moe_swiglu_kernel, :670-692), then
    .W2^T.  Every row goes through the expert FFN restatement as one expert
    holding all rows (the same arithmetic, row by row)."""
    T = x.shape[0]
    counts = np.array([T], dtype=np.int32)
    offsets = np.zeros(1, dtype=np.int32)
    order = np.arange(T, dtype=np.int32)
    return expert_ffn(x, order, offsets, counts, w1[None], w3[None], w2[None])[:T]


def combine(out, token_slot, w, H):
    T, K = token_slot.shape
    y = np.empty((T, H), dtype=np.float32)
    lib().b2o_combine(np.ascontiguousarray(out, dtype=np.float32),
                      np.ascontiguousarray(token_slot, dtype=np.int32),
                      np.ascontiguousarray(w, dtype=np.float32), T, K, H, y)
    return y


def moe_forward(x, gate, bias, w1, w2, w3, K=4, routed_scale=1.0, tile=128):
    """Whole layer in SparseMoeBlock::forward_gpu order; returns every
    intermediate the parity tests compare."""
    T, H = x.shape
    E = gate.shape[0]
    logits = gemm_nt(x, gate)
    idx, w, counts = route(logits, bias, K, routed_scale)
    off, toff = scan(counts, tile)
    st, sw, slot = scatter(idx, w, E, off)
    out = expert_ffn(x, st, off, counts, w1, w3, w2)
    y = combine(out, slot, w, H)
    return dict(y=y, logits=logits, topk_idx=idx, topk_w=w, counts=counts, offsets=off,
                mtile_offsets=toff, sorted_token=st, sorted_w=sw, token_slot=slot)


# ------------------------------------------------------ LFM2 decoder glue
def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def rmsnorm(x, w):
    """rms_norm_kernel (src/layer.cu:144-191) over the last axis."""
    x = _f32(x)
    dim = x.shape[-1]
    y = np.empty_like(x)
    lib().b2o_rmsnorm(x, _f32(w), y, x.size // dim, dim)
    return y


def rope_tables(npos, head_dim=64, theta=1000000.0):
    """RotaryEmbedding::init_gpu tables (src/layer.cu:1167-1190), [npos][head_dim]."""
    c = np.empty((npos, head_dim), dtype=np.float32)
    s = np.empty((npos, head_dim), dtype=np.float32)
    lib().b2o_rope_tables(c, s, npos, head_dim, theta)
    return c, s


def attention_core(qkv, B, S, Hq, Hkv, q_ln, k_ln, cos, sin, hd=64):
    out = np.zeros((B * S, Hq * hd), dtype=np.float32)
    lib().b2o_attention_core(_f32(qkv), B, S, Hq, Hkv, hd, _f32(q_ln), _f32(k_ln), _f32(cos),
                             _f32(sin), out)
    return out


def attention_block(x, wq, wk, wv, wo, q_ln, k_ln, cos, sin, B, S, want_core=False):
    """Attention::forward_gpu (src/layer.cu:1584-1659): projections by the
    sequential-k GEMM, q/k norm + RoPE + causal GQA core, out projection."""
    hd = q_ln.shape[0]
    Hq, Hkv = wq.shape[0] // hd, wk.shape[0] // hd
    qkv = np.concatenate([gemm_nt(x, wq), gemm_nt(x, wk), gemm_nt(x, wv)], axis=1)
    core = attention_core(qkv, B, S, Hq, Hkv, q_ln, k_ln, cos, sin, hd)
    y = gemm_nt(core, wo)
    return (y, core) if want_core else y


def shortconv_core(in_proj_out, conv_w, B, S):
    H, L = conv_w.shape[0], conv_w.shape[-1]
    y = np.empty((B * S, H), dtype=np.float32)
    lib().b2o_shortconv_core(_f32(in_proj_out), _f32(conv_w.reshape(H, L)), B, S, H, L, y)
    return y


def shortconv_block(x, in_w, conv_w, out_w, B, S, want_core=False):
    """ShortConv::forward_gpu (src/layer.cu:1735-1777)."""
    core = shortconv_core(gemm_nt(x, in_w), conv_w, B, S)
    y = gemm_nt(core, out_w)
    return (y, core) if want_core else y


# ------------------------------------------------------ reference kernels
def ref_lib():
    """The reference's own CUDA kernels compiled from its sources (oracle/_ref).
    Returns None when that library was not built here."""
    global _r
    if _r is not None:
        return _r
    if not REF_LIB.exists():
        return None
    r = C.CDLL(str(REF_LIB))
    vp, i = C.c_void_p, C.c_int
    r.ref_gemm_nt.argtypes = [vp, vp, vp, i, i, i, vp]
    r.ref_lm_head.argtypes = [vp, vp, vp, i, i, i, vp]
    r.ref_moe_create.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, i, i, C.POINTER(vp)]
    r.ref_moe_destroy.argtypes = [vp]
    r.ref_moe_forward.argtypes = [vp, vp, vp, i, vp, vp, vp, vp, vp, vp, vp, vp]
    r.ref_rmsnorm.argtypes = [vp, vp, vp, i, i, vp]
    r.ref_add.argtypes = [vp, vp, vp, i, vp]
    r.ref_embed.argtypes = [vp, vp, vp, i, i, vp]
    r.ref_rope_tables.argtypes = [vp, vp, i]
    r.ref_attention.argtypes = [vp] * 11 + [i] * 5 + [vp]
    r.ref_shortconv.argtypes = [vp] * 6 + [i] * 3 + [vp]
    r.ref_mlp.argtypes = [vp] * 5 + [i] * 3 + [vp]
    _r = r
    return r


def gflop_moe(T, H, E, K, I):
    """Algorithmic FLOP of one MoE layer: router 2HE + experts K*(2*2HI + 2IH) per token."""
    return T * (2 * H * E + K * (4 * H * I + 2 * I * H)) / 1e9


__all__ = [n for n in dir() if not n.startswith("_")] + ["math"]
