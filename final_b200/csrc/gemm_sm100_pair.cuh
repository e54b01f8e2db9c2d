// gemm_sm100_pair.cuh -- the tcgen05 GEMM of gemm_sm100.cuh run by CTA pairs
// (cta_group::2): each pair of CTAs of a 2-CTA cluster computes a 256 x 256
// output tile.
//
//   CTA c of the pair loads A rows [m0 + 128c, +128) and B rows [n0 + 128c,
//   +128) of each 128-byte k-block into its own shared memory (a 6-stage ring
//   of 32 KB stages); the pair leader (c = 0) issues M=256 x N=256 UMMAs that
//   read both CTAs' shared memory and accumulate into both CTAs' TMEM (each CTA
//   holds its 128 rows x 256 columns); every CTA runs the epilogue of its own
//   rows.  Per CTA and k-block that is 32 KB of operand traffic instead of the
//   48 KB of a single-CTA 128 x 256 tile.
//
// Synchronisation (all waits bounded as in sm100_ptx.cuh):
//   full[s]    leader's barrier; both producers arrive, both CTAs' TMA bytes
//              complete on it (cta_group::2 loads, no multicast);
//   empty[s]   one per CTA; the leader commits its MMAs to both;
//   tfull[a]   one per CTA; the leader commits the last k-block's MMAs to both;
//   tempty[a]  leader's barrier; one arrival per epilogue warp of both CTAs.
// The grouped schedule's m-tiles are 256 rows (mtile_offsets in 256-row units).
//
// Expert-parallel form (GemmArgs' optional fields; ep.cu): one launch covers a
// rank's own rows and every source rank's rows.  A group may read its A rows
// from a second tensor map (the receive buffer) once that source's arrival
// flag reaches the forward's sequence number -- the producer waits on it,
// bounded, before its first load of the group's rows -- may store its output
// rows into another of this GPU's buffers, and may belong to a return chunk
// whose completion counter each epilogue warp bumps once its rows of a tile
// are stored, so the copy engine returns the chunk to its source while the
// launch continues: the exchange overlaps the GEMM instead of splitting it
// into one launch per source.
#pragma once
#include "gemm_sm100.cuh"

namespace b2 {

constexpr int kPairBM = 256;  // rows per CTA-pair tile (128 per CTA)
constexpr int kPairStages = 6;
constexpr int kPairABytes = 128 * kBKBytes;  // 16 KB
constexpr int kPairBBytes = 128 * kBKBytes;  // 16 KB: half of the 256-wide B tile
// per-group schedule arrays in shared memory: m-tile prefix, C offset, count,
// B block, A offset, source, destination, return chunk
constexpr int kPairSchedArrays = 8;

constexpr size_t gemm_pair_smem_bytes() {
  return 1024 + (size_t)kPairStages * (kPairABytes + kPairBBytes) + kEpiStageBytes + 512 +
         kPairSchedArrays * (kMaxGroups + 1) * 4;
}

__device__ __forceinline__ TileInfo decode_pair_tile(int tile, const GemmArgs &g, const int *s_mt,
                                                     const int *s_off, const int *s_cnt,
                                                     const int *s_grp, const int *s_aoff,
                                                     const int *s_src, const int *s_dst,
                                                     const int *s_chunk, int out_tile_cols,
                                                     int crank, int ngroups) {
  TileInfo t;
  const int NT = g.num_n_tiles;
  t.src = -1;
  t.dst = 0;
  t.chunk = -1;
  if (ngroups > 0) {
    const int gm = tile / NT;
    const int n = tile - gm * NT;
    int lo = 0, hi = ngroups;  // s_mt[lo] <= gm < s_mt[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_mt[mid] <= gm) lo = mid; else hi = mid;
    }
    const int m = gm - s_mt[lo];
    const int within = m * kPairBM + 128 * crank;
    t.c_row = s_off[lo] + within;
    t.a_row = (g.a_offsets ? s_aoff[lo] : s_off[lo]) + within;
    t.rows_valid = min(128, s_cnt[lo] - within);
    t.b_row = s_grp[lo] * g.b_rows_per_group + n * kBN + 128 * crank;
    t.n_tile = n;
    if (g.group_src) t.src = s_src[lo];
    if (g.group_dst) t.dst = s_dst[lo];
    if (g.group_chunk) t.chunk = s_chunk[lo];
  } else {
    const int MT = (g.M + kPairBM - 1) / kPairBM;
    const int band = g.group_m * NT;
    const int b = tile / band;
    const int m0 = b * g.group_m;
    const int gh = min(g.group_m, MT - m0);
    const int idx = tile - b * band;
    const int n = idx / gh;
    const int m = m0 + (idx - n * gh);
    t.a_row = m * kPairBM + 128 * crank;
    t.c_row = t.a_row;
    t.rows_valid = min(128, g.M - t.a_row);
    t.b_row = n * kBN + 128 * crank;
    t.n_tile = n;
  }
  t.cols_valid = min(out_tile_cols, g.N - t.n_tile * out_tile_cols);
  return t;
}

template <int EPI, bool TF32, typename TOut>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmA2, const GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + kPairStages * kPairABytes;
  uint8_t *sEpi = sB + kPairStages * kPairBBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sEpi + kEpiStageBytes);
  // bars[0..S) full, [S..2S) empty, 2S..2S+1 tmem_full, 2S+2..2S+3 tmem_empty, 2S+4 drain
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * kPairStages + 5);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  int *s_mt = reinterpret_cast<int *>(bars) + 128;  // 512 B past the barrier block
  int *s_off = s_mt + (kMaxGroups + 1);
  int *s_cnt = s_off + (kMaxGroups + 1);
  int *s_grp = s_cnt + (kMaxGroups + 1);
  int *s_aoff = s_grp + (kMaxGroups + 1);
  int *s_src = s_aoff + (kMaxGroups + 1);
  int *s_dst = s_src + (kMaxGroups + 1);
  int *s_chunk = s_dst + (kMaxGroups + 1);
  const uint64_t wait_ns = g.wait_ns ? g.wait_ns : kWaitTimeoutNs;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[kPairStages + s]); };
  auto tfull_bar = [&](int a) { return smem_u32(&bars[2 * kPairStages + a]); };
  auto tempty_bar = [&](int a) { return smem_u32(&bars[2 * kPairStages + 2 + a]); };
  const uint32_t drain_bar = smem_u32(&bars[2 * kPairStages + 4]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(full_bar(s), 2);   // both producers of the pair arrive (leader's copy is used)
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 8);  // 4 epilogue warps x 2 CTAs (leader's copy is used)
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (g.group_src) tma_prefetch_desc(&tmA2);
  }
  cluster_sync();  // both CTAs' barriers exist before any remote arrive
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_holder), kTmemCols);
    tmem_relinquish_pair();
  }
  pdl_wait();
  pdl_trigger();
  // grouped schedule: the group count is a launch parameter, or (when the
  // schedule itself was built on the GPU) read from device memory; a count
  // outside [0, kMaxGroups] runs no tile
  int ngroups = g.num_groups;
  if (g.num_groups_dev) {
    ngroups = *g.num_groups_dev;
    if (ngroups < 0 || ngroups > kMaxGroups) ngroups = 0;
  }
  const bool grouped = g.num_groups > 0 || g.num_groups_dev != nullptr;
  if (grouped) {
    for (int i = threadIdx.x; i <= ngroups; i += blockDim.x) {
      s_mt[i] = g.mtile_offsets[i];
      if (i < ngroups) {
        s_off[i] = g.offsets[i];
        s_cnt[i] = g.counts[i];
        s_grp[i] = g.group_b ? g.group_b[i] : i;
        if (g.a_offsets) s_aoff[i] = g.a_offsets[i];
        if (g.group_src) s_src[i] = g.group_src[i];
        if (g.group_dst) s_dst[i] = g.group_dst[i];
        if (g.group_chunk) s_chunk[i] = g.group_chunk[i];
      }
    }
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  const int NT = g.num_n_tiles;
  const int total_tiles = grouped
                              ? s_mt[ngroups] * NT
                              : ((g.M + kPairBM - 1) / kPairBM) * NT;
  constexpr int out_tile_cols = (EPI == kEpiSwiGLU) ? kBN / 2 : kBN;
  const int KB = g.num_k_blocks;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer (both CTAs)
      const uint64_t pol = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, last_par = 0;
      uint64_t arrived = 0;  // sources whose rows this producer has seen published
      for (int tile = pair; tile < total_tiles; tile += npairs) {
        const TileInfo t = decode_pair_tile(tile, g, s_mt, s_off, s_cnt, s_grp, s_aoff, s_src,
                                            s_dst, s_chunk, out_tile_cols, (int)crank,
                                            grouped ? ngroups : 0);
        const CUtensorMap *ta = &tmA;
        if (t.src >= 0) {
          ta = &tmA2;
          if (!((arrived >> (t.src & 63)) & 1)) {
            if (!flag_wait_ge(g.flags + t.src, g.flag_target, abort_flag, g.status, wait_ns))
              break;
            fence_proxy_async_global();  // the rows the flag published, for the TMA loads
            arrived |= 1ull << (t.src & 63);
          }
        }
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, g.status,
                         kDevTimeoutProducer, wait_ns)) {
            ok = false;
            break;
          }
          const uint32_t lead_full = mapa_shared(full_bar(stage), 0);
          if (leader)
            mbar_arrive_expect_tx(full_bar(stage), 2 * (kPairABytes + kPairBBytes));
          else
            mbar_arrive_cluster(lead_full);
          const int kc = kb * (TF32 ? 32 : 64);
          tma_load_2d_pair(smem_u32(sA + stage * kPairABytes), ta, lead_full, kc, t.a_row, pol);
          tma_load_2d_pair(smem_u32(sB + stage * kPairBBytes), &tmB, lead_full, kc, t.b_row, pol);
          issued |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
      // Both CTAs' copies complete on the leader's full barriers: the leader
      // waits (bounded) for the last phase of every stage it filled before
      // the pair leaves; the peer stays resident meanwhile in the final
      // cluster barrier.  Without an abort this returns at once (the MMA
      // warp has consumed every stage).
      if (leader)
        for (int s = 0; s < kPairStages; ++s)
          if (issued >> s & 1) mbar_drain(full_bar(s), (last_par >> s) & 1, g.status);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------ UMMA issuer (pair leader)
      constexpr uint32_t idesc = make_idesc(TF32 ? 2u : 1u, 2 * 128, kBN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_par = 0;
      bool issued_any = false;
      for (int tile = pair; tile < total_tiles; tile += npairs) {
        if (!mbar_wait(tempty_bar(acc), acc_par ^ 1, abort_flag, g.status, kDevTimeoutMma,
                       wait_ns))
          break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * kBN);
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, g.status, kDevTimeoutMma, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a0 = make_sw128_desc(smem_u32(sA + stage * kPairABytes));
          const uint64_t b0 = make_sw128_desc(smem_u32(sB + stage * kPairBBytes));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (TF32)
              umma_tf32_pair(d, a0 + 2 * k, b0 + 2 * k, idesc, (kb | k) != 0);
            else
              umma_f16_pair(d, a0 + 2 * k, b0 + 2 * k, idesc, (kb | k) != 0);
          }
          issued_any = true;
          umma_commit_pair(empty_bar(stage));
          umma_commit_pair(mapa_shared(empty_bar(stage), 1));
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(tfull_bar(acc));
        umma_commit_pair(mapa_shared(tfull_bar(acc), 1));
        acc ^= 1;
        if (acc == 0) acc_par ^= 1;
      }
      if (issued_any) {
        umma_commit_pair(drain_bar);
        mbar_drain(drain_bar, 0, g.status);
      }
    }
  } else {
    // -------------------------------------------------- epilogue (both CTAs)
    const int q = warp & 3;
    uint8_t *stage = sEpi + q * kEpiWarpBytes;
    const bool vec_ok = (g.ldo * (long long)sizeof(TOut)) % 16 == 0;
    int acc = 0;
    uint32_t acc_par = 0;
    for (int tile = pair; tile < total_tiles; tile += npairs) {
      const TileInfo t = decode_pair_tile(tile, g, s_mt, s_off, s_cnt, s_grp, s_aoff, s_src,
                                          s_dst, s_chunk, out_tile_cols, (int)crank,
                                            grouped ? ngroups : 0);
      if (!mbar_wait(tfull_bar(acc), acc_par, abort_flag, g.status, kDevTimeoutEpilogue,
                     wait_ns))
        break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * kBN);
      int rows_valid = t.rows_valid - q * 32;  // of this warp's 32 rows
      // an output row outside the destination buffer (a corrupt schedule) is
      // refused and recorded instead of written
      if (g.c_rows > 0 && rows_valid > 0 &&
          (t.c_row < 0 || (long long)t.c_row + t.rows_valid > g.c_rows)) {
        if (lane == 0 && g.status) atomicCAS(g.status, 0, (int)kDevBadSlot);
        rows_valid = 0;
      }
      TOut *obase = reinterpret_cast<TOut *>(g.out_ptrs ? g.out_ptrs[t.dst] : g.out);
      TOut *out = obase + (long long)(t.c_row + q * 32) * g.ldo +
                  (long long)t.n_tile * out_tile_cols;
      if constexpr (EPI == kEpiSwiGLU) {
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
        for (int c = 0; c < kBN / 32; ++c) {
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
      if (t.chunk >= 0) {
        // this warp's rows of the tile are stored: count it for the chunk's
        // return copy (fence first, so the copy engine that waits on the
        // counter reads the stored rows)
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(g.chunk_done + t.chunk, 1ull);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty_bar(acc), 0));
      acc ^= 1;
      if (acc == 0) acc_par ^= 1;
    }
  }

  __syncthreads();
  cluster_sync();  // the leader's MMAs into this CTA's TMEM are drained
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace b2
