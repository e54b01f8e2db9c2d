// gemm_sm100.cuh -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[rows, n] = A[rows, K] . B[n, K]^T        (both operands K-major)
//
// One CTA per SM walks a static round-robin list of 128 x BN output tiles
// (BN = 256, or 128 / 64 for dense problems with too few wide tiles):
//   warp 0      TMA producer (one elected lane): A/B k-blocks of 128 bytes
//               (64 bf16 or 32 fp32) into a SW128 smem ring of 192 KB
//               (4 stages at BN 256, 6 at 128, 8 at 64);
//   warp 1      TMEM allocator + UMMA issuer (one lane): 4 x (128xBNxK16/K8)
//               MMAs per k-block into a double-buffered fp32 TMEM accumulator
//               (2 x BN columns), tcgen05.commit frees smem stages;
//   warps 2..5  epilogue: tcgen05.ld 32x32b of the warp's TMEM lane quarter,
//               fused SwiGLU / bf16 / fp32 conversion, stores staged through
//               a per-warp smem block so each instruction writes whole row
//               segments.
//
// Two schedules share the kernel:
//   grouped  (MoE experts): rows of A are expert segments [offsets[e],
//            offsets[e]+counts[e]) of the scattered activations, cut into
//            128-row tiles by the prefix mtile_offsets[]; tile order is
//            (expert, m-tile, n-tile) with n fastest, so the tiles in flight
//            share one expert's weights in L2.  B rows of expert e start at
//            e * b_rows_per_group.
//   dense    one group of M rows, rastered in bands of group_m m-tiles so a
//            band's A tiles and the B tiles in flight stay L2-resident.
// This replaces the reference's FFMA kernels attn_matmul_tiled_kernel
// (src/layer.cu:9-141), moe_persistent_fused_w1w3_kernel (:773-972) and
// moe_persistent_w2_kernel (:974-1126).
#pragma once
#include "sm100_ptx.cuh"

namespace b2 {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBKBytes = 128;
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBKBytes;  // 16 KB
constexpr int kBBytes = kBN * kBKBytes;  // 32 KB
constexpr int kMaxGroups = 256;
constexpr int kGemmThreads = 192;
constexpr int kTmemCols = 512;
// Per-warp staging block of the coalesced epilogue store: 32 rows x 32 fp32.
constexpr int kEpiWarpBytes = 32 * 32 * 4;
constexpr int kEpiStageBytes = 4 * kEpiWarpBytes;  // 4 epilogue warps

enum EpiKind { kEpiStore = 0, kEpiSwiGLU = 1 };

// SwiGLU of one accumulator pair, silu(g) * u, with the sigmoid written as
// 0.5 + 0.5 tanh(g / 2) on the hardware tanh: one MUFU operation and no
// branch, so a chunk's 32 outputs pipeline (an IEEE division's slow-path
// branch serialised them).  The approximate tanh's error (about 2^-11) is
// below the bf16 rounding of the stored intermediate.  Every GEMM kernel's
// SwiGLU epilogue uses this function, so they all give the same bits.
__device__ __forceinline__ float swiglu(float g, float u) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * g));
  return g * fmaf(0.5f, t, 0.5f) * u;
}

struct GemmArgs {
  const int *counts;         // grouped: rows per group
  const int *offsets;        // grouped: first row of each group in A / C
  const int *mtile_offsets;  // grouped: exclusive prefix of ceil(count/128), [G+1]
  const int *group_b;        // grouped, optional: B block of each group (default: the group index)
  int num_groups;            // grouped: G (<= kMaxGroups); dense: 0
  const int *num_groups_dev; // CTA-pair grouped schedule built on the GPU: G read here
  int b_rows_per_group;      // grouped: rows of B per group
  int M;                     // dense rows
  int N;                     // output columns (SwiGLU: gated output columns)
  int num_n_tiles;
  int num_k_blocks;
  int group_m;               // dense raster band height (m-tiles)
  void *out;
  long long ldo;             // output row stride in elements
  int *status;
  int accumulate;            // fp32 output only: C += A . B^T (the residual add, fused)
  // ---- expert-parallel extensions of the grouped CTA-pair schedule (all
  // optional; zero / null keeps the plain grouped GEMM):
  const int *a_offsets;      // first A row of each group when it differs from its C row
  const int *group_src;      // -1: A rows in tmA now; s >= 0: A rows in tmA2, published
                             // when flags[s] >= flag_target (a peer's copy engine)
  const uint64_t *flags;
  uint64_t flag_target;
  void *const *out_ptrs;     // output base of each destination (this GPU's buffers)
  const int *group_dst;      // destination of each group (index into out_ptrs)
  long long c_rows;          // rows of every output buffer (> 0: rows beyond are refused)
  const int *group_chunk;    // return chunk of each group (-1: none) ...
  unsigned long long *chunk_done;  // ... whose counter every epilogue warp bumps (after
                             // a fence) once its rows of a tile are stored
  uint64_t wait_ns;          // bound of every wait of the kernel (0: kWaitTimeoutNs)
};

// Ring depth for an N-tile width: 192 KB of A+B stages (4 at 256, 6 at 128,
// 8 at 64 columns).
constexpr int gemm_stages(int bn) { return (4 * (kABytes + kBBytes)) / (kABytes + bn * kBKBytes); }

constexpr size_t gemm_smem_bytes(int bn = kBN) {
  return 1024 + (size_t)gemm_stages(bn) * (kABytes + bn * kBKBytes) + kEpiStageBytes + 256 +
         4 * (kMaxGroups + 1) * 4;
}

struct TileInfo {
  int a_row, b_row, rows_valid, n_tile, cols_valid;
  int c_row;  // first output row (= a_row unless the group has its own A offset)
  int src;    // -1, or the peer whose flag publishes the A rows
  int dst;    // output destination (index into GemmArgs::out_ptrs)
  int chunk;  // return chunk of the group (-1: none)
};

__device__ __forceinline__ TileInfo decode_tile(int tile, const GemmArgs &g,
                                                const int *s_mt, const int *s_off,
                                                const int *s_cnt, const int *s_grp,
                                                int out_tile_cols, int bn = kBN) {
  TileInfo t;
  const int NT = g.num_n_tiles;
  if (g.num_groups > 0) {
    const int gm = tile / NT;
    const int n = tile - gm * NT;
    int lo = 0, hi = g.num_groups;  // s_mt[lo] <= gm < s_mt[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_mt[mid] <= gm) lo = mid; else hi = mid;
    }
    const int m = gm - s_mt[lo];
    t.a_row = s_off[lo] + m * kBM;
    t.rows_valid = min(kBM, s_cnt[lo] - m * kBM);
    t.b_row = s_grp[lo] * g.b_rows_per_group + n * bn;
    t.n_tile = n;
  } else {
    const int MT = (g.M + kBM - 1) / kBM;
    const int band = g.group_m * NT;
    const int b = tile / band;
    const int m0 = b * g.group_m;
    const int gh = min(g.group_m, MT - m0);
    const int idx = tile - b * band;
    const int n = idx / gh;
    const int m = m0 + (idx - n * gh);
    t.a_row = m * kBM;
    t.rows_valid = min(kBM, g.M - t.a_row);
    t.b_row = n * bn;
    t.n_tile = n;
  }
  t.cols_valid = min(out_tile_cols, g.N - t.n_tile * out_tile_cols);
  t.c_row = t.a_row;
  t.src = -1;
  t.dst = 0;
  t.chunk = -1;
  return t;
}

// Waits that must complete even while the CTA is aborting (draining our own
// asynchronous copies / MMAs before the CTA's smem and TMEM are released).
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity, int *status) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      if (status) atomicCAS(status, 0, (int)kDevTimeoutDrain);
      return;
    }
  }
}

// Store up to 32 consecutive fp32 values of one output row as TOut.
template <typename TOut>
__device__ __forceinline__ void store_cols(TOut *dst, const float (&h)[32], int valid,
                                           bool vec_ok, bool add = false) {
  if (valid <= 0) return;
  if (add) {  // fp32 accumulate into C: C = C + result, element by element
    if constexpr (sizeof(TOut) == 4) {
#pragma unroll
      for (int i = 0; i < 32; ++i)  // constant indices keep h in registers
        if (i < valid) dst[i] = __fadd_rn(dst[i], h[i]);
    }
    return;
  }
  if (valid >= 32 && vec_ok) {
    if constexpr (sizeof(TOut) == 2) {
      uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
      for (int v = 0; v < 4; ++v)
        d[v] = make_uint4(pack_bf16(h[8 * v], h[8 * v + 1]), pack_bf16(h[8 * v + 2], h[8 * v + 3]),
                          pack_bf16(h[8 * v + 4], h[8 * v + 5]), pack_bf16(h[8 * v + 6], h[8 * v + 7]));
    } else {
      float4 *d = reinterpret_cast<float4 *>(dst);
#pragma unroll
      for (int v = 0; v < 8; ++v) d[v] = make_float4(h[4 * v], h[4 * v + 1], h[4 * v + 2], h[4 * v + 3]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < valid) {
        if constexpr (sizeof(TOut) == 2) dst[i] = __float2bfloat16_rn(h[i]);
        else dst[i] = h[i];
      }
  }
}

// Writes a warp's 32 rows x 32 columns (lane i holds row i in h) through a
// per-warp shared-memory block so that each global store instruction covers
// whole row segments: 128 B of each of 4 rows (fp32) or 64 B of each of 8
// rows (bf16), instead of 16 B of each of 32 rows.  The 16-byte units of a row
// are XOR-swizzled by the row index, so the row-wise writes and the
// column-wise reads of the block are both free of bank conflicts.
// out0 = the warp's first row at the chunk's first column; rows >= rows_valid
// are skipped.  Needs 16-byte aligned rows and 32 valid columns; the whole
// warp calls it.
template <typename TOut>
__device__ __forceinline__ void store_block_coalesced(uint8_t *stage, const float (&h)[32],
                                                      TOut *out0, long long ldo, int rows_valid,
                                                      int lane, bool add = false) {
  if constexpr (sizeof(TOut) == 4) {
    float4 *srow = reinterpret_cast<float4 *>(stage + lane * 128);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      srow[u ^ (lane & 7)] = make_float4(h[4 * u], h[4 * u + 1], h[4 * u + 2], h[4 * u + 3]);
    __syncwarp();
    const int u = lane & 7;
    if (add) {
      // C = C + result: all eight loads of C are in flight before any store
      float4 o[8];
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int r = it * 4 + (lane >> 3);
        o[it] = r < rows_valid ? reinterpret_cast<const float4 *>(out0 + r * ldo)[u]
                               : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int r = it * 4 + (lane >> 3);
        const float4 v = reinterpret_cast<const float4 *>(stage + r * 128)[u ^ (r & 7)];
        if (r < rows_valid)
          reinterpret_cast<float4 *>(out0 + r * ldo)[u] =
              make_float4(__fadd_rn(o[it].x, v.x), __fadd_rn(o[it].y, v.y),
                          __fadd_rn(o[it].z, v.z), __fadd_rn(o[it].w, v.w));
      }
    } else {
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int r = it * 4 + (lane >> 3);
        const float4 v = reinterpret_cast<const float4 *>(stage + r * 128)[u ^ (r & 7)];
        if (r < rows_valid) reinterpret_cast<float4 *>(out0 + r * ldo)[u] = v;
      }
    }
  } else {
    uint4 *srow = reinterpret_cast<uint4 *>(stage + lane * 64);
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int u = 0; u < 4; ++u)
      srow[u ^ sw] = make_uint4(pack_bf16(h[8 * u], h[8 * u + 1]), pack_bf16(h[8 * u + 2], h[8 * u + 3]),
                                pack_bf16(h[8 * u + 4], h[8 * u + 5]),
                                pack_bf16(h[8 * u + 6], h[8 * u + 7]));
    __syncwarp();
    const int u = lane & 3;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int r = it * 8 + (lane >> 2);
      const uint4 v = reinterpret_cast<const uint4 *>(stage + r * 64)[u ^ ((r >> 1) & 3)];
      if (r < rows_valid) reinterpret_cast<uint4 *>(out0 + r * ldo)[u] = v;
    }
  }
  __syncwarp();
}

// One 32-column chunk of a warp's 32 output rows: coalesced through shared
// memory when the chunk is whole and rows are 16-byte aligned, else row-wise.
template <typename TOut>
__device__ __forceinline__ void store_chunk(uint8_t *stage, const float (&h)[32], TOut *out0,
                                           long long ldo, int rows_valid, int cols_valid,
                                           bool vec_ok, int lane, bool add = false) {
  if (rows_valid <= 0 || cols_valid <= 0) return;
  if (vec_ok && cols_valid >= 32) {
    store_block_coalesced(stage, h, out0, ldo, rows_valid, lane, add);
  } else if (lane < rows_valid) {
    store_cols(out0 + lane * ldo, h, cols_valid, vec_ok, add);
  }
}

template <int EPI, bool TF32, typename TOut, int BN = kBN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB, const GemmArgs g) {
  static_assert(BN == 64 || BN == 128 || BN == 256, "N tile");
  static_assert(EPI == kEpiStore || BN == kBN, "SwiGLU pairs 128 gate and 128 up columns");
  constexpr int S_ = gemm_stages(BN);  // ring stages
  constexpr int BB_ = BN * kBKBytes;  // B bytes per stage
  constexpr uint32_t TC_ = 2 * BN;  // two accumulators
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + S_ * kABytes;
  uint8_t *sEpi = sB + S_ * BB_;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sEpi + kEpiStageBytes);
  // bars[0..S) full, [S..2S) empty, 2S..2S+1 tmem_full, 2S+2..2S+3 tmem_empty, 2S+4 drain
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * S_ + 5);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  int *s_mt = reinterpret_cast<int *>(bars) + 64;  // 256 B past the barrier block
  int *s_off = s_mt + (kMaxGroups + 1);
  int *s_cnt = s_off + (kMaxGroups + 1);
  int *s_grp = s_cnt + (kMaxGroups + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[S_ + s]); };
  auto tfull_bar = [&](int a) { return smem_u32(&bars[2 * S_ + a]); };
  auto tempty_bar = [&](int a) { return smem_u32(&bars[2 * S_ + 2 + a]); };
  const uint32_t drain_bar = smem_u32(&bars[2 * S_ + 4]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S_; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 128);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), TC_);
    tmem_relinquish();
  }
  // everything above overlaps the previous kernel's tail; the schedule and
  // the A operand are that kernel's output
  pdl_wait();
  pdl_trigger();
  if (g.num_groups > 0) {
    for (int i = threadIdx.x; i <= g.num_groups; i += blockDim.x) {
      s_mt[i] = g.mtile_offsets[i];
      if (i < g.num_groups) {
        s_off[i] = g.offsets[i];
        s_cnt[i] = g.counts[i];
        s_grp[i] = g.group_b ? g.group_b[i] : i;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  const int NT = g.num_n_tiles;
  const int total_tiles = g.num_groups > 0
                              ? s_mt[g.num_groups] * NT
                              : ((g.M + kBM - 1) / kBM) * NT;
  constexpr int out_tile_cols = (EPI == kEpiSwiGLU) ? BN / 2 : BN;
  const int KB = g.num_k_blocks;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      const uint64_t pol = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      uint32_t last_par = 0;
      for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
        const TileInfo t = decode_tile(tile, g, s_mt, s_off, s_cnt, s_grp, out_tile_cols, BN);
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, g.status,
                         kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(stage), kABytes + BB_);
          const int kc = kb * (TF32 ? 32 : 64);
          tma_load_2d(smem_u32(sA + stage * kABytes), &tmA, full_bar(stage), kc, t.a_row, pol);
          tma_load_2d(smem_u32(sB + stage * BB_), &tmB, full_bar(stage), kc, t.b_row, pol);
          issued |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == S_) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
      // our own copies must have landed before the CTA may exit
      for (int s = 0; s < S_; ++s)
        if (issued >> s & 1) mbar_drain(full_bar(s), (last_par >> s) & 1, g.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ UMMA issuer
      constexpr uint32_t idesc = make_idesc(TF32 ? 2u : 1u, kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_par = 0;
      bool issued_any = false;
      for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
        if (!mbar_wait(tempty_bar(acc), acc_par ^ 1, abort_flag, g.status, kDevTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, g.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a0 = make_sw128_desc(smem_u32(sA + stage * kABytes));
          const uint64_t b0 = make_sw128_desc(smem_u32(sB + stage * BB_));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // +32 bytes per K step inside the 128-byte swizzle atom (>>4 = 2)
            if (TF32)
              umma_tf32(d, a0 + 2 * k, b0 + 2 * k, idesc, (kb | k) != 0);
            else
              umma_f16(d, a0 + 2 * k, b0 + 2 * k, idesc, (kb | k) != 0);
          }
          issued_any = true;
          umma_commit(empty_bar(stage));
          if (++stage == S_) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));
        acc ^= 1;
        if (acc == 0) acc_par ^= 1;
      }
      if (issued_any) {
        umma_commit(drain_bar);
        mbar_drain(drain_bar, 0, g.status);
      }
    }
  } else {
    // -------------------------------------------------- epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint8_t *stage = sEpi + q * kEpiWarpBytes;
    // 16-byte vector stores need 16-byte aligned rows
    const bool vec_ok = (g.ldo * (long long)sizeof(TOut)) % 16 == 0;
    int acc = 0;
    uint32_t acc_par = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      const TileInfo t = decode_tile(tile, g, s_mt, s_off, s_cnt, s_grp, out_tile_cols, BN);
      if (!mbar_wait(tfull_bar(acc), acc_par, abort_flag, g.status, kDevTimeoutEpilogue))
        break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const int rows_valid = t.rows_valid - q * 32;  // of this warp's 32 rows
      TOut *out = reinterpret_cast<TOut *>(g.out) + (long long)(t.a_row + q * 32) * g.ldo +
                  (long long)t.n_tile * out_tile_cols;
      if constexpr (EPI == kEpiSwiGLU) {
        // columns [0,128) of the accumulator are gate (W1), [128,256) up (W3)
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t gr[32], ur[32];
          tmem_ld32(tbase + c * 32, gr);
          tmem_ld32(tbase + 128 + c * 32, ur);
          tmem_ld_wait();
          float h[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) h[i] = swiglu(__uint_as_float(gr[i]), __uint_as_float(ur[i]));
          store_chunk(stage, h, out + c * 32, g.ldo, rows_valid, t.cols_valid - c * 32, vec_ok,
                      lane);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          tmem_ld_wait();
          float h[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) h[i] = __uint_as_float(r[i]);
          store_chunk(stage, h, out + c * 32, g.ldo, rows_valid, t.cols_valid - c * 32, vec_ok,
                      lane, g.accumulate != 0);
        }
      }
      tc_fence_before();
      mbar_arrive(tempty_bar(acc));
      acc ^= 1;
      if (acc == 0) acc_par ^= 1;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TC_);
  }
}

}  // namespace b2
