"""The dense GEMM planner (b2_gemm_plan, host only: no GPU needed): which
kernel configuration each shape gets on a 148-SM B200."""
import pytest

from final_b200.moe import gemm_plan


@pytest.mark.parametrize("M,N,K,want", [
    (16384, 2048, 2048, ("pair", 256, 1)),      # prefill projections
    (16384, 6144, 2048, ("pair", 256, 1)),      # conv in-projection
    (32, 65536, 2048, ("pair", 256, 1)),        # LM head over the last tokens
    (512, 2048, 2048, ("splitk", 128, 2)),      # config 2, M = 512
    (512, 3072, 2048, ("single", 128, 1)),      # 96 tiles: one wave, no split
    (64, 2048, 7168, ("splitk", 128, 6)),       # decode MLP down projection
    (1, 4096, 2048, ("splitk", 128, 4)),
    (1280, 2048, 2048, ("single", 256, 1)),     # 80 wide tiles in one wave, not 160 in two
    (2048, 2048, 2048, ("single", 256, 1)),     # one wave: 15.9 us against 24.4 in two
    (128, 256, 64, ("single", 128, 1)),         # too little K to split
])
def test_plan(M, N, K, want):
    assert gemm_plan(M, N, K, "bf16", 148) == want


def test_split_fits_one_wave_and_keeps_four_k_blocks():
    for M in (1, 64, 200, 512, 777):
        for N in (512, 2048, 3072, 5000):
            for K in (512, 1024, 2048, 7168):
                kind, bn, sp = gemm_plan(M, N, K, "bf16", 148)
                if kind != "splitk":
                    continue
                tiles = -(-M // 128) * -(-N // bn)
                assert bn == 128 and 2 <= sp <= 6 and tiles * sp <= 148
                assert (K * 2 // 128) // sp >= 4
                assert tiles <= (148 // 18) * (18 // sp)  # clusters co-resident


def test_plan_rejects_bad_arguments():
    from final_b200 import B2Error
    with pytest.raises(B2Error):
        gemm_plan(0, 16, 16)
