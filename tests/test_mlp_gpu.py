"""Dense SwiGLU MLP (b2_mlp_*, include/b2mlp.h) on the GPU against the CPU
oracle's restatement of MLP::forward_gpu (src/layer.cu:1230-1269).

Tolerance (max |y - y_ref| / max |y_ref|, y_ref = fp32 oracle): 1e-2 for bf16
operands, 5e-3 for TF32 -- the same bar as the MoE experts.  Rows are
independent, so large cases are checked on a row sample.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {"bf16": 1e-2, "tf32": 5e-3}


def _rel(a, b):
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(np.asarray(a, dtype=np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


def _weights(oracle, H, I, seed):
    w1 = oracle.randn((I, H), seed, oracle.S_W1, 0.02)
    w3 = oracle.randn((I, H), seed, oracle.S_W3, 0.02)
    w2 = oracle.randn((H, I), seed, oracle.S_W2, 0.02)
    return w1, w3, w2


# (tokens, hidden, inter): the model's shape (H 2048, I 7168) at decode, mid
# and prefill sizes -- single-CTA kernels with 64/128/256-column tiles and the
# CTA-pair kernels -- plus a ragged shape with I padded to 128.
CASES = [(1, 2048, 7168), (257, 2048, 7168), (2048, 2048, 7168), (300, 512, 1000)]


@pytest.mark.parametrize("dtype", ["bf16", "tf32"])
@pytest.mark.parametrize("T,H,I", CASES)
def test_mlp_vs_oracle(cuda_dev, oracle, T, H, I, dtype):
    from final_b200 import MLP
    seed = 11 + T
    x = oracle.randn((T, H), seed, oracle.S_X)
    w1, w3, w2 = _weights(oracle, H, I, seed)
    t = lambda a: torch.from_numpy(a).to(cuda_dev)
    mlp = MLP(t(w1), t(w2), t(w3), max_tokens=T, dtype=dtype)
    y = mlp.forward(t(x))
    torch.cuda.synchronize()
    assert mlp.device_status() == 0
    rows = np.arange(T) if T <= 300 else np.sort(np.random.default_rng(0).choice(T, 48, replace=False))
    y_ref = oracle.dense_mlp(x[rows], w1, w3, w2)
    err = _rel(y.cpu().numpy()[rows], y_ref)
    assert err < TOL[dtype], f"T={T} H={H} I={I} {dtype}: rel err {err:.3e}"


def test_mlp_deterministic_capacity_and_empty(cuda_dev, oracle):
    from final_b200 import MLP, B2Error
    T, H, I = 96, 512, 640
    x = oracle.randn((T, H), 5, oracle.S_X)
    w1, w3, w2 = _weights(oracle, H, I, 5)
    t = lambda a: torch.from_numpy(a).to(cuda_dev)
    mlp = MLP(t(w1), t(w2), t(w3), max_tokens=T)
    xd = t(x)
    y1, y2 = mlp.forward(xd), mlp.forward(xd)
    y3 = mlp.forward(xd[:7].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert torch.equal(y3, y1[:7])
    with pytest.raises(B2Error):
        mlp.forward(torch.zeros(T + 1, H, device=cuda_dev))
    assert mlp.forward(xd[:0]).shape == (0, H)
    assert mlp.device_status() == 0
