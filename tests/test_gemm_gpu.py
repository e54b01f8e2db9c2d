"""Dense NT GEMM on the tcgen05 core against an fp64 PyTorch reference of the
same op (C = A . B^T), and against the reference engine's own tiled kernel
(attn_matmul_tiled_kernel, src/layer.cu:9-141) when oracle/_ref is built.

Tolerances (max |C - C_ref| / max |C_ref|):
  bf16 operands, fp32 accumulate vs fp64 of the same bf16 values: 1e-4
      (only the accumulation order differs)
  bf16 / tf32 vs the reference's fp32 result on fp32 inputs: 1e-2
      (the north-star tolerance for bf16/TF32 tensor-core math)
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

# Shapes across the planner's choices on 148 SMs (final_b200.moe.gemm_plan):
# CTA pairs (256x256 tiles), single CTAs with 128-column tiles, split-K
# clusters of 2..6 CTAs; test_every_configuration below runs every kernel
# configuration, chosen or not, on the same operands.
SHAPES = [
    (128, 256, 64),       # one k-block
    (200, 300, 128),      # ragged M and N, partial k-blocks
    (512, 2048, 2048),    # out projection, M=512: split-K 2 x 128
    (1280, 2048, 2048),   # single CTA, 128-column tiles, two waves
    (300, 1000, 512),     # ragged split-K 2 x 128
    (384, 3072, 2048),    # fused QKV width
    (64, 65536, 2048),    # LM head, batch rows only (CTA pairs)
    (1, 512, 2048),       # single row: split-K 6
    (1000, 520, 1032),    # K not a multiple of the 64-wide k-block: split-K 3
    (4096, 3072, 2048),   # enough 256x256 tiles for the CTA-pair kernel
    (2000, 4096, 1024),   # CTA-pair kernel with a ragged last row tile
    (512, 3072, 2048),    # single CTA, 128-column tiles, one wave
    (64, 2048, 7168),     # decode-size down projection: split-K 6
    (1, 4096, 2048),      # one token: split-K 4
    (333, 1000, 1000),    # ragged split-K 4
]

CONFIGS = ([("single", bn, 1) for bn in (64, 128, 256)] + [("pair", 256, 1)] +
           [("splitk", bn, sp) for bn in (128, 256) for sp in (2, 3, 4, 6, 8)] +
           [("pairsplit", 256, sp) for sp in (2, 3, 4)])


def _rel(a, b):
    return ((a.double() - b.double()).abs().max() / b.double().abs().max().clamp_min(1e-30)).item()


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_bf16_vs_fp64(cuda_dev, M, N, K):
    from final_b200 import gemm_nt
    g = torch.Generator(device=cuda_dev).manual_seed(M * 7 + N * 3 + K)
    A = torch.randn(M, K, device=cuda_dev, generator=g).to(torch.bfloat16)
    B = (torch.randn(N, K, device=cuda_dev, generator=g) * 0.02).to(torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    Cm = gemm_nt(A, B, dtype="bf16", status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    ref = A.double() @ B.double().T
    assert _rel(Cm, ref) < 1e-4


@pytest.mark.parametrize("M,N,K", SHAPES[:5] + [(1000, 520, 1032), (64, 2048, 7168)])
def test_gemm_tf32_vs_fp64(cuda_dev, M, N, K):
    from final_b200 import gemm_nt
    g = torch.Generator(device=cuda_dev).manual_seed(M + N + K)
    A = torch.randn(M, K, device=cuda_dev, generator=g)
    B = torch.randn(N, K, device=cuda_dev, generator=g) * 0.02
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    Cm = gemm_nt(A, B, dtype="tf32", status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    ref = A.double() @ B.double().T
    assert _rel(Cm, ref) < 1e-2


def test_gemm_ldc_and_stream(cuda_dev):
    """Output written with a row stride > N on a side stream leaves the gap untouched."""
    from final_b200 import gemm_nt
    M, N, K = 256, 512, 256
    A = torch.randn(M, K, device=cuda_dev).to(torch.bfloat16)
    B = torch.randn(N, K, device=cuda_dev).to(torch.bfloat16)
    big = torch.full((M, N + 64), 7.0, device=cuda_dev)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        gemm_nt(A, B, out=big[:, :N], dtype="bf16", stream=s)
    s.synchronize()
    assert _rel(big[:, :N], A.double() @ B.double().T) < 1e-4
    assert torch.all(big[:, N:] == 7.0)


def test_gemm_vs_reference_kernel(cuda_dev, oracle):
    """Our bf16/tf32 GEMM against the reference's own fp32 tiled kernel."""
    r = oracle.ref_lib()
    if r is None:
        pytest.skip("oracle/_ref not built (reference tree absent when building)")
    from final_b200 import gemm_nt
    M, N, K = 300, 3072, 2048
    A = torch.randn(M, K, device=cuda_dev)
    B = torch.randn(N, K, device=cuda_dev) * 0.02
    Cref = torch.empty(M, N, device=cuda_dev)
    assert r.ref_gemm_nt(C.c_void_p(Cref.data_ptr()), C.c_void_p(A.data_ptr()),
                         C.c_void_p(B.data_ptr()), M, N, K, None) == 0
    torch.cuda.synchronize()
    exact = A.double() @ B.double().T
    assert _rel(Cref, exact) < 1e-5  # the reference kernel itself is fp32-exact-ish
    Cb = gemm_nt(A.to(torch.bfloat16), B.to(torch.bfloat16), dtype="bf16")
    Ct = gemm_nt(A, B, dtype="tf32")
    torch.cuda.synchronize()
    assert _rel(Cb, Cref) < 1e-2
    assert _rel(Ct, Cref) < 1e-2


def test_gemm_invalid_args(cuda_dev):
    from final_b200 import B2Error, gemm_nt
    A = torch.zeros(4, 12, device=cuda_dev, dtype=torch.bfloat16)  # K=12: not a multiple of 8
    B = torch.zeros(8, 12, device=cuda_dev, dtype=torch.bfloat16)
    with pytest.raises(B2Error):
        gemm_nt(A, B, dtype="bf16")


@pytest.mark.parametrize("M,N,K", [(333, 1000, 1000), (512, 2048, 2048), (64, 520, 7168)])
@pytest.mark.parametrize("dtype", ["bf16", "tf32"])
def test_every_configuration(cuda_dev, M, N, K, dtype):
    """Every kernel configuration (b2_gemm_nt_config) on the same operands:
    single-CTA 64/128/256-column tiles, CTA pairs, split-K with 128/256-column
    tiles and 2..8 CTAs per cluster, split-K over 2..4 CTA pairs."""
    from final_b200 import gemm_nt
    g = torch.Generator(device=cuda_dev).manual_seed(M + 3 * N + 7 * K)
    A = torch.randn(M, K, device=cuda_dev, generator=g)
    B = torch.randn(N, K, device=cuda_dev, generator=g) * 0.02
    if dtype == "bf16":
        A, B = A.to(torch.bfloat16), B.to(torch.bfloat16)
    ref = A.double() @ B.double().T
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    for cfg in CONFIGS:
        Cm = gemm_nt(A, B, dtype=dtype, status=status, config=cfg)
        torch.cuda.synchronize()
        assert status.item() == 0, cfg
        assert _rel(Cm, ref) < (1e-4 if dtype == "bf16" else 1e-2), cfg


def test_splitk_is_deterministic(cuda_dev):
    """The split-K reduction runs in a fixed CTA order: repeated calls give
    identical bits."""
    from final_b200 import gemm_nt
    A = torch.randn(512, 2048, device=cuda_dev).to(torch.bfloat16)
    B = (torch.randn(3072, 2048, device=cuda_dev) * 0.02).to(torch.bfloat16)
    c0 = gemm_nt(A, B, dtype="bf16")
    for _ in range(3):
        assert torch.equal(gemm_nt(A, B, dtype="bf16"), c0)


@pytest.mark.parametrize("split", [2, 3, 4])
def test_pair_splitk_is_deterministic(cuda_dev, split):
    """Split-K over CTA pairs reduces its slices in a fixed order: repeated
    calls give identical bits, on a shape whose last row and column tiles and
    last k-block are partial."""
    from final_b200 import gemm_nt
    g = torch.Generator(device=cuda_dev).manual_seed(split)
    A = torch.randn(300, 1000, device=cuda_dev, generator=g).to(torch.bfloat16)
    B = (torch.randn(700, 1000, device=cuda_dev, generator=g) * 0.02).to(torch.bfloat16)
    ref = A.double() @ B.double().T
    cfg = ("pairsplit", 256, split)
    c0 = gemm_nt(A, B, dtype="bf16", config=cfg)
    assert _rel(c0, ref) < 1e-4
    for _ in range(3):
        assert torch.equal(gemm_nt(A, B, dtype="bf16", config=cfg), c0)
