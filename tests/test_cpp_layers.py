"""The C++ drop-in layer classes (final_b200/cpp/b2_layers.h): reference
class names and entry points over the C ABI.

CPU: the adapter library and its driver are built and load without a GPU.
GPU: b2_layers_run constructs SparseMoeBlock(layer_idx) / MLP(w1, w2, w3) from
weights stored under the reference's tensor names (src/layer.cu:1274-1297),
runs init_gpu() + forward_gpu(x, y, 1, T, H, stream) as
DecoderLayer::forward_gpu does, and y is compared with the CPU oracle
(tolerance 1e-2 bf16 / 5e-3 TF32, as for the C ABI tests).
"""
import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
LIBDIR = ROOT / "final_b200" / "lib"
RUN = LIBDIR / "b2_layers_run"
TOL = {"bf16": 1e-2, "tf32": 5e-3}


def _built():
    from final_b200 import build as b
    b.build()
    b.build_cpp()


def test_adapter_builds_and_loads():
    _built()
    ctypes.CDLL(str(LIBDIR / "libb2layers.so"))
    r = subprocess.run([str(RUN), "--help"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "usage" in r.stderr


def _store(d: Path, name: str, a: np.ndarray) -> None:
    a = np.ascontiguousarray(a, dtype=np.float32)
    (d / f"{name}.f32").write_bytes(a.tobytes())
    (d / f"{name}.shape").write_text(" ".join(str(s) for s in a.shape))


def _run(kind, d, layer, x, dtype):
    xf, yf = d / "x.f32", d / "y.f32"
    xf.write_bytes(np.ascontiguousarray(x, dtype=np.float32).tobytes())
    r = subprocess.run([str(RUN), kind, str(d), str(layer), str(x.shape[0]), str(xf), str(yf),
                        dtype], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    return np.frombuffer(yf.read_bytes(), dtype=np.float32).reshape(x.shape)


def _rel(a, b):
    return float(np.abs(a.astype(np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["bf16", "tf32"])
def test_cpp_sparse_moe_block(cuda_dev, oracle, tmp_path, dtype):
    _built()
    T, H, E, I, layer = 77, 512, 8, 256, 3
    inp = oracle.moe_inputs(T, H, E, I, seed=21)
    pre = f"layers.{layer}.feed_forward."
    _store(tmp_path, pre + "gate.weight", inp["gate"])
    _store(tmp_path, pre + "expert_bias", inp["bias"])
    for e in range(E):
        for w in ("w1", "w2", "w3"):
            _store(tmp_path, f"{pre}experts.{e}.{w}.weight", inp[w][e])
    y = _run("moe", tmp_path, layer, inp["x"], dtype)
    ref = oracle.moe_forward(inp["x"], inp["gate"], inp["bias"], inp["w1"], inp["w2"], inp["w3"])
    assert _rel(y, ref["y"]) < TOL[dtype]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["bf16", "tf32"])
def test_cpp_mlp(cuda_dev, oracle, tmp_path, dtype):
    _built()
    T, H, I, layer = 130, 1024, 1536, 0
    x = oracle.randn((T, H), 8, oracle.S_X)
    w1 = oracle.randn((I, H), 8, oracle.S_W1, 0.02)
    w3 = oracle.randn((I, H), 8, oracle.S_W3, 0.02)
    w2 = oracle.randn((H, I), 8, oracle.S_W2, 0.02)
    pre = f"layers.{layer}.feed_forward."
    for n, a in (("w1", w1), ("w2", w2), ("w3", w3)):
        _store(tmp_path, f"{pre}{n}.weight", a)
    y = _run("mlp", tmp_path, layer, x, dtype)
    assert _rel(y, oracle.dense_mlp(x, w1, w3, w2)) < TOL[dtype]


# ---------------------------------------------------------------- decoder
# The rest of the reference's classes (Attention, ShortConv, DecoderLayer,
# LFM2Model with its ModelLoader) over a tiny model written in the
# reference's file format: weights under the reference's names, read by the
# C++ ModelLoader, results against the CPU oracle.
import lfm2_cases as lc  # noqa: E402


@pytest.fixture(scope="module")
def tiny_file(tmp_path_factory):
    from final_b200.modelfile import write
    cfg = lc.TINY
    W = lc.Weights(cfg["seed"], cfg["vocab"], cfg)
    p = tmp_path_factory.mktemp("tiny") / "tiny.bin"
    write(str(p), {n: W(n) for n in lc.model_names(cfg["layers"], cfg)})
    return p, W


def _run_seq(kind, src, layer, B, S, x, extra=()):
    d = Path(str(src)).parent
    xf, yf = d / f"x_{kind}_{layer}.f32", d / f"y_{kind}_{layer}.f32"
    xf.write_bytes(np.ascontiguousarray(x, dtype=np.float32).tobytes())
    r = subprocess.run([str(RUN), kind, str(src), str(layer), *[str(e) for e in extra], str(B),
                        str(S), str(xf), str(yf)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    return np.frombuffer(yf.read_bytes(), dtype=np.float32).reshape(x.shape)


@pytest.mark.gpu
@pytest.mark.parametrize("kind,layer", [("attn", 2), ("conv", 0)])
def test_cpp_attention_and_shortconv(cuda_dev, oracle, tiny_file, kind, layer):
    _built()
    p, W = tiny_file
    B, S, H = 2, 37, lc.TINY["H"]
    x = oracle.randn((B * S, H), 50, layer, 1.0)
    y = _run_seq(kind, p, layer, B, S, x)
    c, s = oracle.rope_tables(S)
    want = lc.mixer_oracle(W, layer, x, B, S, c, s)
    assert _rel(y, want) < 1e-2


@pytest.mark.gpu
@pytest.mark.parametrize("layer", [0, 2, 3])
def test_cpp_decoder_layer(cuda_dev, oracle, tiny_file, layer):
    _built()
    p, W = tiny_file
    B, S, H = 3, 23, lc.TINY["H"]
    x = oracle.randn((B * S, H), 51, layer, 1.0)
    is_attn = int(lc.TINY["TYPES"][layer] == 0)
    y = _run_seq("decoder", p, layer, B, S, x, extra=(is_attn,))
    c, s = oracle.rope_tables(S)
    want = lc.decoder_layer_oracle(W, layer, x, B, S, c, s)
    # the layer's update (output - input), per token
    err = np.abs((y - x) - (want - x)).max(axis=1) / np.abs(want - x).max(axis=1)
    assert np.sort(err)[-2] < 1e-2, err.max()   # at most one token may flip a near-tie expert


@pytest.mark.gpu
def test_cpp_model_from_file(cuda_dev, tiny_file, tmp_path):
    """LFM2Model(model_file) + forward + sync as the reference's main drives it."""
    _built()
    p, W = tiny_file
    cfg = lc.TINY
    B, S = cfg["batch"], cfg["seq"]
    ids = lc.token_ids(B, S, cfg["vocab"], cfg["seed"])
    idf, lf = tmp_path / "ids.i32", tmp_path / "logits.f32"
    idf.write_bytes(ids.astype(np.int32).tobytes())
    r = subprocess.run([str(RUN), "model", str(p), str(B), str(S), str(idf), str(lf)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    logits = np.frombuffer(lf.read_bytes(), dtype=np.float32).reshape(B, cfg["vocab"])
    want = lc.model_oracle(W, ids, cfg["layers"])
    print(f"C++ LFM2Model logits vs oracle: {_rel(logits, want):.2e}")
    assert _rel(logits, want) < 5e-3  # measured 5.5e-4 on a B200


def _cpp_model_logits(p, ids, B, S, V, out):
    idf = out.with_suffix(".i32")
    idf.write_bytes(ids.astype(np.int32).tobytes())
    r = subprocess.run([str(RUN), "model", str(p), str(B), str(S), str(idf), str(out)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    return np.frombuffer(out.read_bytes(), dtype=np.float32).reshape(B, V)


def _cpp_model_ep(p, ids_list, B, S, V, tmp_path, placement):
    """Start one model_ep rank per entry of ids_list; returns their logits."""
    world = len(ids_list)
    idfile = tmp_path / f"uid_{placement}_{world}"
    procs, outs = [], []
    for rank, ids in enumerate(ids_list):
        idf, lf = tmp_path / f"ep_ids{rank}.i32", tmp_path / f"ep_logits{rank}.f32"
        idf.write_bytes(ids.astype(np.int32).tobytes())
        outs.append(lf)
        procs.append(subprocess.Popen(
            [str(RUN), "model_ep", str(p), str(B), str(S), str(idf), str(lf), str(world),
             str(rank), str(idfile), placement],
            stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    for pr in procs:
        out, _ = pr.communicate(timeout=300)
        assert pr.returncode == 0, out
    return [np.frombuffer(lf.read_bytes(), dtype=np.float32).reshape(B, V) for lf in outs]


@pytest.mark.gpu
@pytest.mark.parametrize("placement", ["balanced", "owner"])
def test_cpp_model_ep_one_rank(cuda_dev, tiny_file, tmp_path, placement):
    """LFM2Model(file, world=1, rank=0, id): the expert-parallel constructor
    gives the replica model's logits bit for bit."""
    _built()
    p, _ = tiny_file
    cfg = lc.TINY
    B, S, V = cfg["batch"], cfg["seq"], cfg["vocab"]
    ids = lc.token_ids(B, S, V, cfg["seed"])
    want = _cpp_model_logits(p, ids, B, S, V, tmp_path / "single.f32")
    (got,) = _cpp_model_ep(p, [ids], B, S, V, tmp_path, placement)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("placement", ["balanced", "owner"])
def test_cpp_model_ep_two_ranks(cuda_dev, tiny_file, tmp_path, placement):
    """Two processes, one per GPU, each with its own batch: each rank's
    logits equal the single-GPU model's on the same ids, bit for bit."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _built()
    p, _ = tiny_file
    cfg = lc.TINY
    B, S, V = cfg["batch"], cfg["seq"], cfg["vocab"]
    ids = [lc.token_ids(B, S, V, cfg["seed"] + 7 * r) for r in range(2)]
    want = [_cpp_model_logits(p, ids[r], B, S, V, tmp_path / f"single{r}.f32") for r in range(2)]
    got = _cpp_model_ep(p, ids, B, S, V, tmp_path, placement)
    for r in range(2):
        assert np.array_equal(got[r].view(np.uint32), want[r].view(np.uint32)), r
