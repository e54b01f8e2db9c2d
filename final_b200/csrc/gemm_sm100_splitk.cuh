// gemm_sm100_splitk.cuh -- split-K tcgen05 GEMM for dense products too small
// to give every SM an output tile (M of a few hundred rows or fewer: decode
// batches, short prompts, config 2's M = 512 projections).
//
//   C[M, n] = A[M, K] . B[n, K]^T
//
// One thread-block cluster of S CTAs (2 <= S <= 8) per 128 x BN output tile;
// cluster rank r accumulates k-blocks [r*KB/S, (r+1)*KB/S) into its own TMEM
// accumulator with the single-CTA pipeline of gemm_sm100.cuh (warp 0 TMA
// producer, warp 1 UMMA issuer, warps 2..5 epilogue).  The S partial tiles
// are then reduced through distributed shared memory, 128 columns at a time:
//   1. each CTA writes its partial slice [128 rows][128 cols] fp32 into its
//      own shared memory (16-byte units XOR-swizzled by row);
//   2. cluster barrier (release / acquire at cluster scope): every slice is
//      visible to every CTA;
//   3. CTA r sums rows [r*R, r*R+R) of the slice over the S partials in rank
//      order 0..S-1 (ld.shared::cluster), applies the epilogue (plain store
//      or SwiGLU, fp32 or bf16 out) and writes C with whole-row coalesced
//      stores;
//   4. cluster barrier: every CTA is done reading the slice, which may now be
//      overwritten by the next one (after the last slice: nobody exits while a
//      peer may still read its shared memory).
// Each cluster runs exactly one tile, so all warps are idle by step 1 and the
// hardware cluster barrier replaces any hand-built signalling: every thread of
// every CTA executes the same 2 x (slices) barriers, whatever its role did.
// The reduction order is fixed, so results are deterministic.  Every wait of
// the main loop is bounded (status codes as in gemm_sm100.cuh); the barriers
// are reached by all threads because every loop before them is bounded.
//
// SwiGLU: the 256-column accumulator holds gate columns [0,128) and up
// columns [128,256); slice h carries gate [64h, 64h+64) and up
// [128+64h, 128+64h+64), so each reducing CTA sees the matching halves.
#pragma once
#include "gemm_sm100.cuh"

namespace b2 {

constexpr int kSplitMax = 8;        // portable cluster size
constexpr int kSplitSlice = 128;    // columns of one reduction slice
constexpr int kSplitPartBytes = kBM * kSplitSlice * 4;  // 64 KB
constexpr int kEpiThreads = 128;

struct SplitArgs {
  int M, N;              // rows of A / C, output columns (SwiGLU: gated outputs)
  int num_k_blocks;      // 128-byte k-blocks of K
  int splits;            // S = cluster size
  int m_tiles;           // ceil(M / 128)
  void *out;
  long long ldo;         // output row stride (elements)
  int *status;
  int accumulate;        // fp32 plain epilogue only: C += result
};

constexpr int splitk_stages(int bn) { return bn == 256 ? 3 : 4; }

constexpr size_t splitk_smem_bytes(int bn) {
  return 1024 + (size_t)splitk_stages(bn) * (kABytes + bn * kBKBytes) + kSplitPartBytes + 256;
}

// A 16-byte load from another CTA's shared memory.  volatile keeps it after
// the (volatile) mbarrier wait that acquires the data; no memory clobber, so
// several loads can be in flight at once.
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}

// byte offset of 16-byte unit u (0..31) of partial row `row`
__device__ __forceinline__ uint32_t part_off(int row, int u) {
  return (uint32_t)(row * (kSplitSlice * 4) + ((u ^ (row & 7)) << 4));
}

// Four consecutive outputs of one row as TOut (16-byte fp32 / 8-byte bf16
// store when aligned and whole, else element by element up to n_valid).
template <typename TOut>
__device__ __forceinline__ void store4(TOut *dst, float a, float b, float c, float d, bool vec,
                                       int n_valid, bool add = false) {
  const float v[4] = {a, b, c, d};
  if constexpr (sizeof(TOut) == 4) {
    if (add) {  // C = C + result
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (i < n_valid) dst[i] = __fadd_rn(dst[i], v[i]);
      return;
    }
  }
  if (vec && n_valid >= 4) {
    if constexpr (sizeof(TOut) == 4)
      *reinterpret_cast<float4 *>(dst) = make_float4(a, b, c, d);
    else
      *reinterpret_cast<uint2 *>(dst) = make_uint2(pack_bf16(a, b), pack_bf16(c, d));
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // constant indices keep v in registers
    if (i >= n_valid) break;
    if constexpr (sizeof(TOut) == 4) dst[i] = v[i];
    else dst[i] = __float2bfloat16_rn(v[i]);
  }
}

template <int EPI, bool TF32, typename TOut, int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_splitk_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB, const SplitArgs g) {
  static_assert(BN == 128 || BN == 256, "split-K tile width");
  static_assert(EPI == kEpiStore || BN == 256, "SwiGLU pairs 128 gate and 128 up columns");
  constexpr int S_ = splitk_stages(BN);
  constexpr int BB_ = BN * kBKBytes;
  constexpr int NSLICE = BN / kSplitSlice;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + S_ * kABytes;
  uint8_t *sPart = sB + S_ * BB_;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sPart + kSplitPartBytes);
  // bars[0..S) full, [S..2S) empty, 2S tmem_full, 2S+1 drain; then the TMEM
  // base and the abort flag
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * S_ + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = g.splits;
  const uint32_t rank = cluster_ctarank();
  const int tile = blockIdx.x / S;
  const int m_tile = tile % g.m_tiles, n_tile = tile / g.m_tiles;
  const int kb0 = (int)((long long)g.num_k_blocks * rank / S);
  const int kb1 = (int)((long long)g.num_k_blocks * (rank + 1) / S);
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[S_ + s]); };
  const uint32_t tfull_bar = smem_u32(&bars[2 * S_]);
  const uint32_t drain_bar = smem_u32(&bars[2 * S_ + 1]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S_; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), BN);
    tmem_relinquish();
  }
  pdl_wait();
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      const uint64_t pol = policy_evict_last();
      uint32_t issued = 0, last_par = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        const int i = kb - kb0, stage = i % S_;
        const uint32_t phase = (uint32_t)(i / S_) & 1;
        if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, g.status, kDevTimeoutProducer))
          break;
        mbar_arrive_expect_tx(full_bar(stage), kABytes + BB_);
        const int kc = kb * (TF32 ? 32 : 64);
        tma_load_2d(smem_u32(sA + stage * kABytes), &tmA, full_bar(stage), kc, m_tile * kBM, pol);
        tma_load_2d(smem_u32(sB + stage * BB_), &tmB, full_bar(stage), kc, n_tile * BN, pol);
        issued |= 1u << stage;
        last_par = (last_par & ~(1u << stage)) | (phase << stage);
      }
      for (int s = 0; s < S_; ++s)
        if (issued >> s & 1) mbar_drain(full_bar(s), (last_par >> s) & 1, g.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ UMMA issuer
      constexpr uint32_t idesc = make_idesc(TF32 ? 2u : 1u, kBM, BN);
      bool issued_any = false, ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        const int i = kb - kb0, stage = i % S_;
        const uint32_t phase = (uint32_t)(i / S_) & 1;
        if (!mbar_wait(full_bar(stage), phase, abort_flag, g.status, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t a0 = make_sw128_desc(smem_u32(sA + stage * kABytes));
        const uint64_t b0 = make_sw128_desc(smem_u32(sB + stage * BB_));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (TF32)
            umma_tf32(tmem_base, a0 + 2 * k, b0 + 2 * k, idesc, (i | k) != 0);
          else
            umma_f16(tmem_base, a0 + 2 * k, b0 + 2 * k, idesc, (i | k) != 0);
        }
        issued_any = true;
        umma_commit(empty_bar(stage));
      }
      if (ok && issued_any) umma_commit(tfull_bar);
      if (issued_any) {
        umma_commit(drain_bar);
        mbar_drain(drain_bar, 0, g.status);
      }
    }
  }
  __syncwarp();

  // -------------------------------------------- reduction (epilogue warps 2..5)
  const bool epi = warp >= 2;
  const int q = warp & 3;           // TMEM lane quarter of an epilogue warp
  const int et = threadIdx.x - 64;  // 0..127 in the epilogue warps
  const int row = q * 32 + lane;    // accumulator row this thread drains
  const uint32_t part_base = smem_u32(sPart);
  const int R = (kBM + S - 1) / S;  // rows this CTA reduces
  const int r0 = min(kBM, (int)rank * R), r1 = min(kBM, r0 + R);
  // empty splits (more CTAs than k-blocks) contribute zeros
  bool have_acc = false, ok = true;
  if (epi && kb1 > kb0) {
    have_acc = mbar_wait(tfull_bar, 0, abort_flag, g.status, kDevTimeoutEpilogue);
    // tcgen05.ld is warp-collective: the whole warp takes the same branch
    have_acc = __all_sync(0xffffffffu, have_acc);
    ok = have_acc;
    tc_fence_after();
  }
  const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16);
  TOut *out = reinterpret_cast<TOut *>(g.out);
  const bool vec_ok = (g.ldo % 4) == 0;
#pragma unroll 1
  for (int h = 0; h < NSLICE; ++h) {
    // 1. our slice h of the partial into shared memory
    if (epi && ok) {
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        // TMEM columns of 32-wide chunk c of slice h
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
    // 3. reduce our rows over the S partials in rank order, write C; all S
    //    remote loads of a unit are issued before any is used
    if (epi && ok) {
      if constexpr (EPI == kEpiStore) {
        const int nu = (r1 - r0) * 32;
        for (int u0 = et; u0 < nu; u0 += 2 * kEpiThreads) {
          float4 v[2][kSplitMax];
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            const int u = min(u0 + w * kEpiThreads, nu - 1);
            const uint32_t a = part_base + part_off(r0 + u / 32, u % 32);
#pragma unroll
            for (int j = 0; j < kSplitMax; ++j)
              if (j < S) v[w][j] = ld_cluster_f4(mapa_shared(a, (uint32_t)j));
          }
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            const int u = u0 + w * kEpiThreads;
            if (u >= nu) break;
            const int lr = r0 + u / 32, cu = u % 32;
            const int grow = m_tile * kBM + lr;
            const int gcol = n_tile * BN + kSplitSlice * h + cu * 4;
            if (grow >= g.M || gcol >= g.N) continue;
            float4 acc = v[w][0];
#pragma unroll
            for (int j = 1; j < kSplitMax; ++j)
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
          float4 gv[kSplitMax], uv[kSplitMax];
          const uint32_t ag = part_base + part_off(lr, cu), au = part_base + part_off(lr, cu + 16);
#pragma unroll
          for (int j = 0; j < kSplitMax; ++j)
            if (j < S) {
              gv[j] = ld_cluster_f4(mapa_shared(ag, (uint32_t)j));
              uv[j] = ld_cluster_f4(mapa_shared(au, (uint32_t)j));
            }
          const int grow = m_tile * kBM + lr;
          const int gcol = n_tile * (BN / 2) + 64 * h + cu * 4;
          if (grow >= g.M || gcol >= g.N) continue;
          float4 ga = gv[0], ua = uv[0];
#pragma unroll
          for (int j = 1; j < kSplitMax; ++j)
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
    tmem_dealloc(tmem_base, BN);
  }
}

}  // namespace b2
