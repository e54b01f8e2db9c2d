"""Generate tests/golden/ref_lfm2.npz by running the REFERENCE engine's own
CUDA kernels (compiled unmodified from its src/layer.cu and src/model.cu into
oracle/_ref/libref_moe.so by oracle/Makefile) on a GPU, on the seeded inputs
of tests/lfm2_cases.py:

  rope      the reference RotaryEmbedding's cos/sin tables (first rows + a
            SHA-256 of the first 4096 positions)
  rms       rms_norm_kernel over hidden 2048 and head_dim 64 rows
  attn      Attention::forward_gpu, layer 2 weights, batch 2 x seq 16
  conv      ShortConv::forward_gpu, layer 0 weights, 2 x 16 and 1 x 37
  mlp       MLP::forward_gpu, layer 0 weights, 32 tokens
  model     embedding, 4 decoder layers (conv+MLP, conv+MLP, attention+MoE,
            conv+MoE), final norm, last-token LM head (vocab 1024, tied),
            launched piece by piece in DecoderLayer::forward_gpu order

Run on a CUDA machine from the repository root:
    python tests/golden/make_golden_lfm2.py [outdir]
Large outputs keep a subset of rows plus float64 row sums; inputs are not
stored (they are regenerated from the seeds).
"""
import ctypes as C
import hashlib
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))
import oracle as o  # noqa: E402
import lfm2_cases as lc  # noqa: E402

ROWS = [0, 3, 7, 15, 16, 20, 27, 31]
ROPE_HASH_POS = 4096


def vp(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def keep(prefix, a, out, rows=ROWS):
    a = np.asarray(a, dtype=np.float32)
    out[prefix + "_rows"] = a[[r for r in rows if r < a.shape[0]]]
    out[prefix + "_rowsum"] = a.astype(np.float64).sum(axis=1)
    out[prefix + "_absmax"] = np.array(np.abs(a).max())


def main():
    outdir = sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__))
    r = o.ref_lib()
    if r is None:
        raise SystemExit("oracle/_ref/libref_moe.so missing: run `make -C oracle` where the "
                         "reference tree is present")
    dev = torch.device("cuda:0")
    alive = []  # device copies must outlive the (asynchronous) launches that read them

    def t(a):
        d = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        alive.append(d)
        return d

    res = {}

    # rotary tables
    c = np.empty((ROPE_HASH_POS, lc.HD), dtype=np.float32)
    s = np.empty_like(c)
    assert r.ref_rope_tables(c.ctypes.data, s.ctypes.data, ROPE_HASH_POS) == 0
    res["rope_cos_rows"], res["rope_sin_rows"] = c[:32], s[:32]
    res["rope_cos_sha256"] = np.array(hashlib.sha256(c.tobytes()).hexdigest())
    res["rope_sin_sha256"] = np.array(hashlib.sha256(s.tobytes()).hexdigest())
    cos_d, sin_d = t(c), t(s)

    # rmsnorm
    for tag, (rows, dim) in (("rms2048", (8, 2048)), ("rms64", (96, 64))):
        x = o.randn((rows, dim), 31, dim, 3.0)
        w = (o.randn((dim,), 31, dim + 1, 0.1) + np.float32(1.0)).astype(np.float32)
        y = torch.empty(rows, dim, device=dev)
        assert r.ref_rmsnorm(vp(y), vp(t(x)), vp(t(w)), rows, dim, None) == 0
        torch.cuda.synchronize()
        res[tag] = y.cpu().numpy()

    W = lc.Weights(lc.MINI["seed"], lc.MINI["vocab"])

    # attention block (layer 2), batch 2 x seq 16
    B, S = 2, 16
    x = o.randn((B * S, lc.H), 41, 0, 1.0)
    pre = "layers.2.self_attn."
    y = torch.empty(B * S, lc.H, device=dev)
    core = torch.empty(B * S, lc.HQ * lc.HD, device=dev)
    assert r.ref_attention(vp(t(x)), *[vp(t(W(pre + n + ".weight"))) for n in (
        "q_proj", "k_proj", "v_proj", "out_proj", "q_layernorm", "k_layernorm")],
        vp(cos_d), vp(sin_d), vp(y), vp(core), B, S, lc.H, lc.HQ, lc.HKV, None) == 0
    torch.cuda.synchronize()
    keep("attn_y", y.cpu().numpy(), res)
    keep("attn_core", core.cpu().numpy(), res)

    # short conv (layer 0)
    for tag, (B, S) in (("conv", (2, 16)), ("conv37", (1, 37))):
        x = o.randn((B * S, lc.H), 42, S, 1.0)
        pre = "layers.0.conv."
        y = torch.empty(B * S, lc.H, device=dev)
        core = torch.empty(B * S, lc.H, device=dev)
        assert r.ref_shortconv(vp(t(x)), vp(t(W(pre + "in_proj.weight"))),
                               vp(t(W(pre + "conv.weight"))), vp(t(W(pre + "out_proj.weight"))),
                               vp(y), vp(core), B, S, lc.H, None) == 0
        torch.cuda.synchronize()
        rows = ROWS if B * S == 32 else [0, 1, 2, 3, 17, 35, 36]
        keep(tag + "_y", y.cpu().numpy(), res, rows)
        keep(tag + "_core", core.cpu().numpy(), res, rows)

    # dense MLP (layer 0)
    x = o.randn((32, lc.H), 43, 0, 1.0)
    pre = "layers.0.feed_forward."
    y = torch.empty(32, lc.H, device=dev)
    assert r.ref_mlp(vp(t(x)), vp(t(W(pre + "w1.weight"))), vp(t(W(pre + "w2.weight"))),
                     vp(t(W(pre + "w3.weight"))), vp(y), 32, lc.H, lc.I_DENSE, None) == 0
    torch.cuda.synchronize()
    keep("mlp_y", y.cpu().numpy(), res)

    # mini model
    B, S, L, V = lc.MINI["batch"], lc.MINI["seq"], lc.MINI["layers"], lc.MINI["vocab"]
    T = B * S
    ids = lc.token_ids(B, S, V, lc.MINI["seed"])
    emb = t(W("embed_tokens.weight"))
    hid = torch.empty(T, lc.H, device=dev)
    assert r.ref_embed(vp(hid), vp(t(ids.reshape(-1))), vp(emb), T, lc.H, None) == 0
    xn = torch.empty_like(hid)
    mix = torch.empty_like(hid)
    for i in range(L):
        pre = f"layers.{i}."
        assert r.ref_rmsnorm(vp(xn), vp(hid), vp(t(W(pre + "operator_norm.weight"))), T, lc.H,
                             None) == 0
        if lc.LAYER_TYPES[i] == 0:
            a = pre + "self_attn."
            assert r.ref_attention(vp(xn), *[vp(t(W(a + n + ".weight"))) for n in (
                "q_proj", "k_proj", "v_proj", "out_proj", "q_layernorm", "k_layernorm")],
                vp(cos_d), vp(sin_d), vp(mix), None, B, S, lc.H, lc.HQ, lc.HKV, None) == 0
        else:
            cv = pre + "conv."
            assert r.ref_shortconv(vp(xn), vp(t(W(cv + "in_proj.weight"))),
                                   vp(t(W(cv + "conv.weight"))),
                                   vp(t(W(cv + "out_proj.weight"))), vp(mix), None, B, S, lc.H,
                                   None) == 0
        assert r.ref_add(vp(hid), vp(hid), vp(mix), T * lc.H, None) == 0
        assert r.ref_rmsnorm(vp(xn), vp(hid), vp(t(W(pre + "ffn_norm.weight"))), T, lc.H,
                             None) == 0
        ff = pre + "feed_forward."
        if i < lc.NUM_DENSE:
            assert r.ref_mlp(vp(xn), vp(t(W(ff + "w1.weight"))), vp(t(W(ff + "w2.weight"))),
                             vp(t(W(ff + "w3.weight"))), vp(mix), T, lc.H, lc.I_DENSE,
                             None) == 0
        else:
            w1, w2, w3 = (t(a) for a in lc.experts(W, i))
            arr = C.c_void_p * lc.E
            p1 = arr(*[w1[e].data_ptr() for e in range(lc.E)])
            p2 = arr(*[w2[e].data_ptr() for e in range(lc.E)])
            p3 = arr(*[w3[e].data_ptr() for e in range(lc.E)])
            h = C.c_void_p()
            gate, bias = t(W(ff + "gate.weight")), t(W(ff + "expert_bias"))
            assert r.ref_moe_create(C.cast(p1, C.c_void_p), C.cast(p2, C.c_void_p),
                                    C.cast(p3, C.c_void_p), vp(gate), vp(bias), lc.E, lc.K,
                                    lc.H, lc.I_MOE, T, 288, C.byref(h)) == 0
            assert r.ref_moe_forward(h, vp(xn), vp(mix), T, None, None, None, None, None, None,
                                     None, None) == 0
            torch.cuda.synchronize()
            r.ref_moe_destroy(h)
            del w1, w2, w3
            W.drop(ff + "experts")
        assert r.ref_add(vp(hid), vp(hid), vp(mix), T * lc.H, None) == 0
        torch.cuda.synchronize()
        keep(f"model_h{i}", hid.cpu().numpy(), res)
        alive.clear()
    normed = torch.empty_like(hid)
    assert r.ref_rmsnorm(vp(normed), vp(hid), vp(t(W("embedding_norm.weight"))), T, lc.H,
                         None) == 0
    last = normed.view(B, S, lc.H)[:, -1, :].contiguous()
    logits = torch.empty(B, V, device=dev)
    assert r.ref_lm_head(vp(logits), vp(last), vp(emb), B, V, lc.H, None) == 0
    torch.cuda.synchronize()
    res["model_logits"] = logits.cpu().numpy()
    res["model_ids"] = ids
    np.savez_compressed(os.path.join(outdir, "ref_lfm2.npz"), **res)
    print("wrote ref_lfm2.npz", {k: v.shape for k, v in res.items()}, flush=True)


if __name__ == "__main__":
    main()
