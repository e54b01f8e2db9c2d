// gemm_sm100_pair_splitk.cuh -- split-K over CTA pairs: the tcgen05 GEMM for
// dense products with too few 256 x 256 tiles to fill the GPU (M of a few
// hundred rows: config 2's M = 512 projections, short prompts).
//
//   C[M, n] = A[M, K] . B[n, K]^T
//
// One thread-block cluster of 2*S CTAs (S = 2..4 K-slices) per 256 x 256
// output tile.  CTAs 2p and 2p+1 form pair p (cta_group::2): as in
// gemm_sm100_pair.cuh, CTA c of the pair loads A rows [m0 + 128c, +128) and B
// rows [n0 + 128c, +128) of each k-block, and the pair's even CTA issues
// M=256 x N=256 UMMAs over both CTAs' shared memory into both CTAs' TMEM
// (128 rows x 256 columns each); pair p accumulates k-blocks
// [p*KB/S, (p+1)*KB/S).  Per CTA and k-block that is 32 KB of operands for
// 4.2 MFLOP -- half the bytes per FLOP of the single-CTA split-K kernel, whose
// products are bound by how fast the SMs pull operands from L2 -- and the S
// slices put S times as many SMs on the tile.
//
// The S partials of each 128-row half are then reduced through distributed
// shared memory, 128 columns at a time, exactly as gemm_sm100_splitk.cuh does
// for its S CTAs, over the CTAs of that half (cluster ranks c, 2+c, 4+c, ...)
// in fixed slice order, so results are deterministic.  Each cluster runs one
// tile; every thread reaches the same cluster barriers because every loop
// before them is bounded.
#pragma once
#include "gemm_sm100_pair.cuh"
#include "gemm_sm100_splitk.cuh"

namespace b2 {

constexpr int kPairSplitMax = 4;   // K-slices: clusters of up to 8 CTAs
constexpr int kPairSplitStages = 4;

constexpr size_t pair_splitk_smem_bytes() {
  return 1024 + (size_t)kPairSplitStages * (kPairABytes + kPairBBytes) + kSplitPartBytes + 256;
}

template <int EPI, bool TF32, typename TOut>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_pair_splitk_kernel(const __grid_constant__ CUtensorMap tmA,
                            const __grid_constant__ CUtensorMap tmB, const SplitArgs g) {
  constexpr int S_ = kPairSplitStages;
  constexpr int BN = kBN;  // 256 output (SwiGLU: 128 gate + 128 up) columns per tile
  constexpr int NSLICE = BN / kSplitSlice;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + S_ * kPairABytes;
  uint8_t *sPart = sB + S_ * kPairBBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sPart + kSplitPartBytes);
  // bars[0..S) full, [S..2S) empty, 2S tmem_full, 2S+1 drain; then the TMEM
  // base and the abort flag
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * S_ + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = g.splits;                 // K-slices = pairs per cluster
  const uint32_t rank = cluster_ctarank();
  const uint32_t half = rank & 1u;        // which 128 rows of the tile
  const uint32_t lead = rank & ~1u;       // the pair's MMA-issuing CTA
  const int slice = (int)(rank >> 1);
  const bool leader = half == 0;
  const int tile = blockIdx.x / (2 * S);
  const int m_tile = tile % g.m_tiles, n_tile = tile / g.m_tiles;
  const int kb0 = (int)((long long)g.num_k_blocks * slice / S);
  const int kb1 = (int)((long long)g.num_k_blocks * (slice + 1) / S);
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[S_ + s]); };
  const uint32_t tfull_bar = smem_u32(&bars[2 * S_]);
  const uint32_t drain_bar = smem_u32(&bars[2 * S_ + 1]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S_; ++s) {
      mbar_init(full_bar(s), 2);  // both producers of the pair arrive (the lead's copy is used)
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  cluster_sync();  // every CTA's barriers exist before any remote arrive
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_holder), BN);
    tmem_relinquish_pair();
  }
  pdl_wait();
  pdl_trigger();
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer (both CTAs)
      const uint64_t pol = policy_evict_last();
      uint32_t issued = 0, last_par = 0;
      const int a_row = m_tile * kPairBM + 128 * (int)half;
      const int b_row = n_tile * BN + 128 * (int)half;
      for (int kb = kb0; kb < kb1; ++kb) {
        const int i = kb - kb0, stage = i % S_;
        const uint32_t phase = (uint32_t)(i / S_) & 1;
        if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, g.status, kDevTimeoutProducer))
          break;
        const uint32_t lead_full = mapa_shared(full_bar(stage), lead);
        if (leader)
          mbar_arrive_expect_tx(full_bar(stage), 2 * (kPairABytes + kPairBBytes));
        else
          mbar_arrive_cluster(lead_full);
        const int kc = kb * (TF32 ? 32 : 64);
        tma_load_2d_pair(smem_u32(sA + stage * kPairABytes), &tmA, lead_full, kc, a_row, pol);
        tma_load_2d_pair(smem_u32(sB + stage * kPairBBytes), &tmB, lead_full, kc, b_row, pol);
        issued |= 1u << stage;
        last_par = (last_par & ~(1u << stage)) | (phase << stage);
      }
      // both CTAs' copies complete on the lead's full barriers: the lead
      // waits (bounded) for the last phase of every stage it filled
      if (leader)
        for (int s = 0; s < S_; ++s)
          if (issued >> s & 1) mbar_drain(full_bar(s), (last_par >> s) & 1, g.status);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------ UMMA issuer (pair lead)
      constexpr uint32_t idesc = make_idesc(TF32 ? 2u : 1u, 2 * 128, BN);
      bool issued_any = false, ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        const int i = kb - kb0, stage = i % S_;
        const uint32_t phase = (uint32_t)(i / S_) & 1;
        if (!mbar_wait(full_bar(stage), phase, abort_flag, g.status, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t a0 = make_sw128_desc(smem_u32(sA + stage * kPairABytes));
        const uint64_t b0 = make_sw128_desc(smem_u32(sB + stage * kPairBBytes));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (TF32)
            umma_tf32_pair(tmem_base, a0 + 2 * k, b0 + 2 * k, idesc, (i | k) != 0);
          else
            umma_f16_pair(tmem_base, a0 + 2 * k, b0 + 2 * k, idesc, (i | k) != 0);
        }
        issued_any = true;
        umma_commit_pair(empty_bar(stage));
        umma_commit_pair(mapa_shared(empty_bar(stage), rank | 1u));
      }
      if (ok && issued_any) {
        umma_commit_pair(tfull_bar);
        umma_commit_pair(mapa_shared(tfull_bar, rank | 1u));
      }
      if (issued_any) {
        umma_commit_pair(drain_bar);
        mbar_drain(drain_bar, 0, g.status);
      }
    }
  }
  __syncwarp();

  // ------------------------------------ reduction (epilogue warps 2..5)
  const bool epi = warp >= 2;
  const int q = warp & 3;           // TMEM lane quarter of an epilogue warp
  const int et = threadIdx.x - 64;  // 0..127 in the epilogue warps
  const int row = q * 32 + lane;    // accumulator row (of this CTA's 128) this thread drains
  const uint32_t part_base = smem_u32(sPart);
  const int R = (128 + S - 1) / S;  // rows of this half this CTA reduces
  const int r0 = min(128, slice * R), r1 = min(128, r0 + R);
  // empty slices (more slices than k-blocks) contribute zeros
  bool have_acc = false, ok = true;
  if (epi && kb1 > kb0) {
    have_acc = mbar_wait(tfull_bar, 0, abort_flag, g.status, kDevTimeoutEpilogue);
    have_acc = __all_sync(0xffffffffu, have_acc);  // tcgen05.ld is warp-collective
    ok = have_acc;
    tc_fence_after();
  }
  const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16);
  TOut *out = reinterpret_cast<TOut *>(g.out);
  const bool vec_ok = (g.ldo % 4) == 0;
  const int row_base = m_tile * kPairBM + 128 * (int)half;
#pragma unroll 1
  for (int h = 0; h < NSLICE; ++h) {
    // 1. our slice h of the partial into shared memory
    if (epi && ok) {
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        const int col = EPI == kEpiSwiGLU ? (c < 2 ? 64 * h + 32 * c : 128 + 64 * h + 32 * (c - 2))
                                          : kSplitSlice * h + 32 * c;
        uint32_t r[32];
        if (have_acc) {
          tmem_ld32(trow + (uint32_t)col, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        }
#pragma unroll
        for (int v = 0; v < 8; ++v)
          *reinterpret_cast<float4 *>(sPart + part_off(row, c * 8 + v)) =
              make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                          __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
      }
    }
    // 2. every CTA's slice is visible to every CTA
    __syncwarp();
    cluster_sync();
    // 3. reduce our rows of this half over the S slices in order (cluster
    //    ranks half, 2 + half, ...), write C
    if (epi && ok) {
      if constexpr (EPI == kEpiStore) {
        const int nu = (r1 - r0) * 32;
        for (int u0 = et; u0 < nu; u0 += 2 * kEpiThreads) {
          float4 v[2][kPairSplitMax];
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            const int u = min(u0 + w * kEpiThreads, nu - 1);
            const uint32_t a = part_base + part_off(r0 + u / 32, u % 32);
#pragma unroll
            for (int j = 0; j < kPairSplitMax; ++j)
              if (j < S) v[w][j] = ld_cluster_f4(mapa_shared(a, (uint32_t)(2 * j) + half));
          }
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            const int u = u0 + w * kEpiThreads;
            if (u >= nu) break;
            const int lr = r0 + u / 32, cu = u % 32;
            const int grow = row_base + lr;
            const int gcol = n_tile * BN + kSplitSlice * h + cu * 4;
            if (grow >= g.M || gcol >= g.N) continue;
            float4 acc = v[w][0];
#pragma unroll
            for (int j = 1; j < kPairSplitMax; ++j)
              if (j < S) {
                acc.x += v[w][j].x;
                acc.y += v[w][j].y;
                acc.z += v[w][j].z;
                acc.w += v[w][j].w;
              }
            store4(out + (long long)grow * g.ldo + gcol, acc.x, acc.y, acc.z, acc.w, vec_ok,
                   g.N - gcol, g.accumulate != 0);
          }
        }
      } else {
        const int nu = (r1 - r0) * 16;
        for (int u = et; u < nu; u += kEpiThreads) {
          const int lr = r0 + u / 16, cu = u % 16;
          float4 gv[kPairSplitMax], uv[kPairSplitMax];
          const uint32_t ag = part_base + part_off(lr, cu), au = part_base + part_off(lr, cu + 16);
#pragma unroll
          for (int j = 0; j < kPairSplitMax; ++j)
            if (j < S) {
              gv[j] = ld_cluster_f4(mapa_shared(ag, (uint32_t)(2 * j) + half));
              uv[j] = ld_cluster_f4(mapa_shared(au, (uint32_t)(2 * j) + half));
            }
          const int grow = row_base + lr;
          const int gcol = n_tile * (BN / 2) + 64 * h + cu * 4;
          if (grow >= g.M || gcol >= g.N) continue;
          float4 ga = gv[0], ua = uv[0];
#pragma unroll
          for (int j = 1; j < kPairSplitMax; ++j)
            if (j < S) {
              ga.x += gv[j].x; ga.y += gv[j].y; ga.z += gv[j].z; ga.w += gv[j].w;
              ua.x += uv[j].x; ua.y += uv[j].y; ua.z += uv[j].z; ua.w += uv[j].w;
            }
          store4(out + (long long)grow * g.ldo + gcol, swiglu(ga.x, ua.x), swiglu(ga.y, ua.y),
                 swiglu(ga.z, ua.z), swiglu(ga.w, ua.w), vec_ok, g.N - gcol);
        }
      }
    }
    // 4. the slice has been read everywhere (the last one: nobody leaves early)
    __syncwarp();
    cluster_sync();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, BN);
  }
}

}  // namespace b2
