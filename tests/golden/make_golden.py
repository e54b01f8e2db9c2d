"""Generate the golden fixtures in tests/golden/ by running the REFERENCE
engine's own CUDA kernels (compiled unmodified from its src/layer.cu and
src/model.cu into oracle/_ref/libref_moe.so by oracle/Makefile) on a GPU, on
the seeded inputs of tests/moe_cases.py.

Run on a CUDA machine from the repository root:
    python tests/golden/make_golden.py [outdir]
It writes one ref_<case>.npz per MoE case plus ref_gemm.npz.  The inputs are
not stored: they are regenerated from the case's seeds by the oracle's
splitmix64/Box-Muller generator.  tests/test_oracle.py checks the CPU oracle
against these files.
"""
import ctypes as C
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))
import oracle as o  # noqa: E402
from moe_cases import CASES, build_case  # noqa: E402

# outputs of config1 are large: keep the first rows plus whole-output checksums
Y_ROWS_KEPT = {"config1": 8, "zipf": 32, "hot_expert": 32}


def vp(t):
    return C.c_void_p(t.data_ptr())


def run_case(r, name, dev):
    inp = build_case(name)
    T, H = inp["x"].shape
    E, I = inp["w1"].shape[:2]
    K = inp["K"]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    w1, w2, w3 = t(inp["w1"]), t(inp["w2"]), t(inp["w3"])
    gate = t(inp["gate"])
    bias = t(inp["bias"]) if inp["bias"] is not None else None
    arr = C.c_void_p * E
    p1 = arr(*[w1[e].data_ptr() for e in range(E)])
    p2 = arr(*[w2[e].data_ptr() for e in range(E)])
    p3 = arr(*[w3[e].data_ptr() for e in range(E)])
    h = C.c_void_p()
    rc = r.ref_moe_create(C.cast(p1, C.c_void_p), C.cast(p2, C.c_void_p), C.cast(p3, C.c_void_p),
                          vp(gate), vp(bias) if bias is not None else None, E, K, H, I, T, 288,
                          C.byref(h))
    assert rc == 0, rc
    x = t(inp["x"])
    y = torch.empty(T, H, device=dev)
    logits = torch.empty(T, E, device=dev)
    idx = torch.empty(T, K, dtype=torch.int32, device=dev)
    w = torch.empty(T, K, device=dev)
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    offsets = torch.empty(E, dtype=torch.int32, device=dev)
    tok_pos = torch.empty(T, K, dtype=torch.int32, device=dev)
    sorted_idx = torch.empty(T * K, dtype=torch.int32, device=dev)
    rc = r.ref_moe_forward(h, vp(x), vp(y), T, vp(logits), vp(idx), vp(w), vp(counts), vp(offsets),
                           vp(tok_pos), vp(sorted_idx), None)
    assert rc == 0, rc
    torch.cuda.synchronize()
    r.ref_moe_destroy(h)
    yn = y.cpu().numpy()
    keep = Y_ROWS_KEPT.get(name, T)
    return dict(
        case=np.array(name), shape=np.array([T, H, E, I, K], dtype=np.int32),
        logits=logits.cpu().numpy(), topk_idx=idx.cpu().numpy(), topk_w=w.cpu().numpy(),
        counts=counts.cpu().numpy(), offsets=offsets.cpu().numpy(),
        token_expert_pos=tok_pos.cpu().numpy(), sorted_idx=sorted_idx.cpu().numpy(),
        y=yn[:keep], y_rowsum=yn.astype(np.float64).sum(axis=1),
        y_absmax=np.array(np.abs(yn).max()),
    )


def run_gemm(r, dev):
    out = {}
    for tag, (M, N, K), fn in (("attn", (100, 96, 256), r.ref_gemm_nt),
                               ("lmhead", (5, 320, 256), r.ref_lm_head)):
        A = o.randn((M, K), 3, 0, 1.0)
        B = o.randn((N, K), 3, 1, 0.02)
        Ct = torch.empty(M, N, device=dev)
        At, Bt = torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev)
        assert fn(vp(Ct), vp(At), vp(Bt), M, N, K, None) == 0
        torch.cuda.synchronize()
        out[f"{tag}_shape"] = np.array([M, N, K], dtype=np.int32)
        out[f"{tag}_C"] = Ct.cpu().numpy()
    return out


def main():
    outdir = sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__))
    os.makedirs(outdir, exist_ok=True)
    r = o.ref_lib()
    if r is None:
        raise SystemExit("oracle/_ref/libref_moe.so missing: run `make -C oracle` where the "
                         "reference tree is present")
    dev = torch.device("cuda:0")
    for name in CASES:
        np.savez_compressed(os.path.join(outdir, f"ref_{name}.npz"), **run_case(r, name, dev))
        print("wrote", name, flush=True)
    np.savez_compressed(os.path.join(outdir, "ref_gemm.npz"), **run_gemm(r, dev))
    print("wrote gemm", flush=True)


if __name__ == "__main__":
    main()
