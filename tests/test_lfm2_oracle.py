"""The CPU oracle of the decoder glue (oracle/lfm2_oracle.c + oracle.py)
against the reference engine's own kernels: tests/golden/ref_lfm2.npz was
written by tests/golden/make_golden_lfm2.py running the reference's
rms_norm / RoPE / attention / short-conv / MLP / MoE / embedding / LM-head
kernels (built unmodified from its sources) on a B200.

Bars: RoPE tables, RMSNorm, the attention block and the short-conv block are
bit-exact (same operation order, same FFMA contractions).  The dense MLP and
the model differ only through SiLU's expf (glibc here, CUDA's there): a few
1e-7 relative.  No GPU is needed."""
import hashlib
from pathlib import Path

import numpy as np
import pytest

import oracle as o
import lfm2_cases as lc

G = np.load(Path(__file__).parent / "golden" / "ref_lfm2.npz")
ROWS = [0, 3, 7, 15, 16, 20, 27, 31]


def _rows_equal(name, a, rows=ROWS):
    want = G[name + "_rows"]
    assert np.array_equal(a[rows], want), name
    assert np.array_equal(a.astype(np.float64).sum(axis=1), G[name + "_rowsum"]), name


def _rel(a, want):
    return float(np.abs(a - want).max() / np.abs(want).max())


@pytest.fixture(scope="module")
def W():
    return lc.Weights(lc.MINI["seed"], lc.MINI["vocab"])


@pytest.fixture(scope="module")
def rope():
    return o.rope_tables(4096)


def test_rope_tables_bit_exact(rope):
    c, s = rope
    assert np.array_equal(c[:32], G["rope_cos_rows"])
    assert np.array_equal(s[:32], G["rope_sin_rows"])
    assert hashlib.sha256(c.tobytes()).hexdigest() == str(G["rope_cos_sha256"])
    assert hashlib.sha256(s.tobytes()).hexdigest() == str(G["rope_sin_sha256"])


@pytest.mark.parametrize("tag,rows,dim", [("rms2048", 8, 2048), ("rms64", 96, 64)])
def test_rmsnorm_bit_exact(tag, rows, dim):
    x = o.randn((rows, dim), 31, dim, 3.0)
    w = (o.randn((dim,), 31, dim + 1, 0.1) + np.float32(1.0)).astype(np.float32)
    assert np.array_equal(o.rmsnorm(x, w), G[tag])


def test_attention_block_bit_exact(W, rope):
    c, s = rope
    B, S = 2, 16
    x = o.randn((B * S, lc.H), 41, 0, 1.0)
    pre = "layers.2.self_attn."
    y, core = o.attention_block(x, *[W(pre + n + ".weight") for n in (
        "q_proj", "k_proj", "v_proj", "out_proj", "q_layernorm", "k_layernorm")], c, s, B, S,
        want_core=True)
    _rows_equal("attn_core", core)
    _rows_equal("attn_y", y)


@pytest.mark.parametrize("tag,B,S", [("conv", 2, 16), ("conv37", 1, 37)])
def test_shortconv_block_bit_exact(W, tag, B, S):
    x = o.randn((B * S, lc.H), 42, S, 1.0)
    pre = "layers.0.conv."
    y, core = o.shortconv_block(x, W(pre + "in_proj.weight"), W(pre + "conv.weight"),
                                W(pre + "out_proj.weight"), B, S, want_core=True)
    rows = ROWS if B * S == 32 else [0, 1, 2, 3, 17, 35, 36]
    _rows_equal(tag + "_core", core, rows)
    _rows_equal(tag + "_y", y, rows)


def test_dense_mlp_matches(W):
    x = o.randn((32, lc.H), 43, 0, 1.0)
    pre = "layers.0.feed_forward."
    y = o.dense_mlp(x, W(pre + "w1.weight"), W(pre + "w3.weight"), W(pre + "w2.weight"))
    assert _rel(y[ROWS], G["mlp_y_rows"]) < 5e-7


def test_mini_model_matches(W):
    ids = lc.token_ids(lc.MINI["batch"], lc.MINI["seq"], lc.MINI["vocab"], lc.MINI["seed"])
    assert np.array_equal(ids, G["model_ids"])
    logits, hidden = lc.model_oracle(W, ids, lc.MINI["layers"], want_hidden=True)
    for i, h in enumerate(hidden):
        assert _rel(h[ROWS], G[f"model_h{i}_rows"]) < 5e-6, i
    assert _rel(logits, G["model_logits"]) < 5e-6
