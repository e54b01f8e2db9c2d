// moe_kernels.cuh -- routing, scan, scatter and combine kernels of the MoE
// layer (everything around the two grouped GEMMs), plus weight packing.
//
// Pipeline per forward (all stream-ordered, no host sync):
//   route_kernel    x . gate^T in fp32 with the reference's sequential-k FFMA
//                   order, sigmoid / bias / insertion top-k / renormalise,
//                   per-block expert histogram          (src/layer.cu:439-499)
//   scan_kernel     expert counts, offsets, 128-row tile prefix, per-block
//                   slot bases                          (src/layer.cu:730-768)
//   scatter_kernel  canonical (token, rank) slot order, fp32 -> bf16 row copy
//                                                       (src/layer.cu:501-542)
//   [grouped GEMMs: gemm_sm100.cuh]
//   combine_kernel  y[t] = sum_k w[t,k] * out[slot(t,k)] in k order
//                                                       (src/layer.cu:695-721)
#pragma once
#include "sm100_ptx.cuh"

// Non-template kernels are `static`: each .cu that includes this header owns
// its copy, so several translation units of the library can launch them.
namespace b2 {

constexpr int kRouteTB = 32;   // tokens per route / scatter block
constexpr int kRouteKC = 32;   // k-chunk of the router dot products
constexpr int kMaxExperts = 32;
constexpr int kMaxTopK = 8;

// ---------------------------------------------------------------------------
// route_kernel: one block of two warps per 32 tokens, 16 tokens per warp.
// logits[t,e] = fold_k fma(x[t,k], gate[e,k], acc) from 0.0f -- the order of
// attn_matmul_tiled_kernel (src/layer.cu:70-130), so logits are bit-exact.
// Every dot product is one sequential chain, so the only parallelism is
// (token, expert) pairs: at 16k tokens that is 16k lanes of 32 accumulators or
// 32k lanes of 16.  The narrower split gives every SM sub-partition two warps
// to interleave (one warp alone waits on its own shared-memory and cp.async
// latencies) and 2x the blocks to even out the last wave.
//
// x and gateT (= gate^T, [H][32]) stream through a kRouteStages-deep cp.async
// ring of 32-wide k-chunks shared by the block: xs[t][k] holds 32 tokens x
// 32 k fp32 in rows padded to 36 floats (the 4 rows one 128-bit load touches
// fall in distinct bank groups, and every load offset is a compile-time
// constant); gs[k][e] is the gate chunk, read by both warps.  One 64-thread
// barrier per chunk.  Lane (tg = lane%4, eg = lane/4) of warp w owns tokens
// 16w+tg+4i (i<4) x experts 4eg..4eg+3 (16 accumulators): per 4 k-steps,
// 8 128-bit shared loads (broadcasts: one wavefront each) feed 64 FFMAs, each
// accumulator updated in strict k order.
// ---------------------------------------------------------------------------
constexpr int kRouteStages = 4;
constexpr int kRouteThreads = 64;
constexpr int kRouteXRow = kRouteKC + 4;  // padded row (floats)

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

static __global__ void __launch_bounds__(kRouteThreads)
    route_kernel(const float *__restrict__ x, const float *__restrict__ gateT,
                 const float *__restrict__ bias, int T, int H, int E, int K,
                 float routed_scale, int *__restrict__ topk_idx,
                 float *__restrict__ topk_w, int *__restrict__ block_counts,
                 float *__restrict__ logits_out) {
  __shared__ __align__(16) float xs[kRouteStages][kRouteTB * kRouteXRow];
  __shared__ __align__(16) float gs[kRouteStages][kRouteKC * kMaxExperts];
  __shared__ float lg[kRouteTB][kMaxExperts + 1];
  __shared__ int hist[kMaxExperts];

  const int tid = threadIdx.x;
  const int lane = tid & 31, w = tid >> 5;
  const int t0 = blockIdx.x * kRouteTB;
  const int NC = H / kRouteKC;
  if (tid < kMaxExperts) hist[tid] = 0;
  pdl_wait();
  pdl_trigger();

  // chunk kc -> stage st: per thread 4 x 16 B of x (rows of its own warp) and
  // 4 x 16 B of the gate; rows past T are zero-filled (src-size 0)
  auto issue = [&](int kc, int st) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int idx = lane + 32 * m;  // 0..127 within the warp's 16 rows
      const int row = 16 * w + (idx >> 3), c = idx & 7;
      const int t = t0 + row;
      const bool ok = t < T;
      const float *src = x + (size_t)(ok ? t : 0) * H + kc * kRouteKC + c * 4;
      cp_async16(smem_u32(&xs[st][row * kRouteXRow + c * 4]), src, ok ? 16u : 0u);
    }
    const float *gsrc = gateT + (size_t)kc * kRouteKC * kMaxExperts;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int idx = tid + kRouteThreads * m;  // 0..255
      cp_async16(smem_u32(&gs[st][idx * 4]), gsrc + idx * 4, 16u);
    }
  };

  const int tg = lane & 3, eg = lane >> 2;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[i][e] = 0.0f;

#pragma unroll
  for (int st = 0; st < kRouteStages - 1; ++st) {
    if (st < NC) issue(st, st);
    cp_async_commit();
  }
  for (int kc = 0; kc < NC; ++kc) {
    cp_async_wait<kRouteStages - 2>();
    // chunk kc has landed for every thread, and every thread is done with
    // chunk kc-1, whose stage the next issue refills
    __syncthreads();
    const int nk = kc + kRouteStages - 1;
    if (nk < NC) issue(nk, nk % kRouteStages);
    cp_async_commit();
    const float *xb = xs[kc % kRouteStages] + (16 * w + tg) * kRouteXRow;
    const float *gb = gs[kc % kRouteStages] + eg * 4;
#pragma unroll 4
    for (int q = 0; q < kRouteKC / 4; ++q) {  // k-quad q: k = 4q .. 4q+3
      float4 xv[4], gv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        xv[i] = *reinterpret_cast<const float4 *>(xb + 4 * i * kRouteXRow + 4 * q);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        gv[j] = *reinterpret_cast<const float4 *>(gb + (4 * q + j) * kMaxExperts);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float ge[4] = {gv[j].x, gv[j].y, gv[j].z, gv[j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float xk = j == 0 ? xv[i].x : j == 1 ? xv[i].y : j == 2 ? xv[i].z : xv[i].w;
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[i][e] = __fmaf_rn(xk, ge[e], acc[i][e]);
        }
      }
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) lg[16 * w + tg + 4 * i][eg * 4 + e] = acc[i][e];
  __syncthreads();

  if (threadIdx.x < kRouteTB) {
    const int tl = threadIdx.x;
    const int t = t0 + tl;
    if (t < T) {
      if (logits_out)
        for (int e = 0; e < E; ++e) logits_out[(size_t)t * E + e] = lg[tl][e];
      float mp[kMaxTopK];
      int mi[kMaxTopK];
      if (K == 4) {
        // the reference's 4-slot insertion (src/layer.cu:468-487) unrolled into
        // registers: same strict '>' comparisons in the same order
        float s0 = -1e30f, s1 = -1e30f, s2 = -1e30f, s3 = -1e30f;
        float p0 = 0.0f, p1 = 0.0f, p2 = 0.0f, p3 = 0.0f;
        int i0 = -1, i1 = -1, i2 = -1, i3 = -1;
        for (int e = 0; e < E; ++e) {
          const float prob = 1.0f / (1.0f + (float)exp(-(double)lg[tl][e]));
          const float sc = prob + (bias ? bias[e] : 0.0f);
          if (sc > s3) {
            if (sc > s2) {
              s3 = s2; p3 = p2; i3 = i2;
              if (sc > s1) {
                s2 = s1; p2 = p1; i2 = i1;
                if (sc > s0) {
                  s1 = s0; p1 = p0; i1 = i0;
                  s0 = sc; p0 = prob; i0 = e;
                } else {
                  s1 = sc; p1 = prob; i1 = e;
                }
              } else {
                s2 = sc; p2 = prob; i2 = e;
              }
            } else {
              s3 = sc; p3 = prob; i3 = e;
            }
          }
        }
        mp[0] = p0; mp[1] = p1; mp[2] = p2; mp[3] = p3;
        mi[0] = i0; mi[1] = i1; mi[2] = i2; mi[3] = i3;
      } else {
        float ms[kMaxTopK];
#pragma unroll
        for (int i = 0; i < kMaxTopK; ++i) {
          ms[i] = -1e30f;
          mp[i] = 0.0f;
          mi[i] = -1;
        }
        for (int e = 0; e < E; ++e) {
          const float prob = 1.0f / (1.0f + (float)exp(-(double)lg[tl][e]));
          const float score = prob + (bias ? bias[e] : 0.0f);
          if (score > ms[K - 1]) {
            int pos = K - 1;
            while (pos > 0 && score > ms[pos - 1]) {
              ms[pos] = ms[pos - 1];
              mp[pos] = mp[pos - 1];
              mi[pos] = mi[pos - 1];
              pos--;
            }
            ms[pos] = score;
            mp[pos] = prob;
            mi[pos] = e;
          }
        }
      }
      float sum = 0.0f;
      for (int i = 0; i < K; ++i) sum = __fadd_rn(sum, mp[i]);
      const float scale = (sum > 1e-6f) ? __fdiv_rn(1.0f, sum) : 1.0f;
      for (int i = 0; i < K; ++i) {
        topk_idx[(size_t)t * K + i] = mi[i];
        topk_w[(size_t)t * K + i] = __fmul_rn(__fmul_rn(mp[i], scale), routed_scale);
        if (mi[i] >= 0 && mi[i] < E) atomicAdd(&hist[mi[i]], 1);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < kMaxExperts) block_counts[(size_t)blockIdx.x * kMaxExperts + threadIdx.x] = hist[threadIdx.x];
}

// ---------------------------------------------------------------------------
// scan_kernel: one block of 1024 threads (32 warps x 32 expert lanes).
// counts[e] = sum_b block_counts[b][e]; offsets = exclusive prefix of counts;
// mtile_offsets = exclusive prefix of ceil(count/128) (+ sentinel);
// block_base[b][e] = offsets[e] + sum_{b'<b} block_counts[b'][e].
// ---------------------------------------------------------------------------
static __global__ void __launch_bounds__(1024)
    scan_kernel(const int *__restrict__ block_counts, int nb, int E, int tile_rows,
                int *__restrict__ counts, int *__restrict__ offsets,
                int *__restrict__ mtile_offsets, int *__restrict__ block_base) {
  __shared__ int part[32][33];
  __shared__ int ebase[32];
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  pdl_wait();
  pdl_trigger();
  const int per = (nb + 31) / 32;
  const int b0 = w * per, b1 = min(nb, b0 + per);
  int s = 0;
  for (int b = b0; b < b1; ++b) s += block_counts[(size_t)b * kMaxExperts + lane];
  part[w][lane] = s;
  __syncthreads();
  if (w == 0) {
    int run = 0;
    for (int i = 0; i < 32; ++i) {
      const int v = part[i][lane];
      part[i][lane] = run;
      run += v;
    }
    const int cnt = lane < E ? run : 0;
    const int tiles = (cnt + tile_rows - 1) / tile_rows;
    int ic = cnt, it = tiles;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int nc = __shfl_up_sync(0xffffffffu, ic, d);
      const int nt = __shfl_up_sync(0xffffffffu, it, d);
      if (lane >= d) {
        ic += nc;
        it += nt;
      }
    }
    ebase[lane] = ic - cnt;
    if (lane < E) {
      counts[lane] = cnt;
      offsets[lane] = ic - cnt;
      mtile_offsets[lane] = it - tiles;
    }
    if (lane == E - 1) mtile_offsets[E] = it;
  }
  __syncthreads();
  int run = ebase[lane] + part[w][lane];
  for (int b = b0; b < b1; ++b) {
    block_base[(size_t)b * kMaxExperts + lane] = run;
    run += block_counts[(size_t)b * kMaxExperts + lane];
  }
}

// ---------------------------------------------------------------------------
// scatter_kernel: block b handles tokens [32b, 32b+32) (kRouteTB) with 32*K
// threads (rounded up to whole warps); thread p owns pair (token 32b + p/K,
// rank p%K).  Its slot is
//   block_base[b][e] + #{pairs p' < p in this block with the same expert}
// which is the canonical token-major order of the CPU oracle.  Then the block
// copies each token row once from fp32 x into its K slots as bf16 (or fp32).
// An expert id of -1 (no expert selected) is dropped (slot -1); an id outside
// [-1, E) is dropped the same way and recorded as kDevBadExpert in *status.
// ---------------------------------------------------------------------------
__host__ __device__ constexpr int scatter_threads(int K) { return (kRouteTB * K + 31) / 32 * 32; }

template <typename TOut>
__global__ void __launch_bounds__(256)
    scatter_kernel(const float *__restrict__ x, const int *__restrict__ topk_idx,
                   const float *__restrict__ topk_w, const int *__restrict__ block_base,
                   int T, int H, int E, int K, TOut *__restrict__ sorted_x,
                   int *__restrict__ token_slot, int *__restrict__ sorted_token,
                   float *__restrict__ sorted_w, int *__restrict__ status) {
  __shared__ int wcnt[8][kMaxExperts];
  __shared__ int slot_s[kRouteTB * kMaxTopK];
  const int p = threadIdx.x;
  const int npairs = kRouteTB * K;
  const int lane = p & 31, w = p >> 5;
  const int t = blockIdx.x * kRouteTB + p / K;
  for (int i = p; i < 8 * kMaxExperts; i += blockDim.x) (&wcnt[0][0])[i] = 0;
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  int e = -1;
  if (p < npairs && t < T) {
    e = topk_idx[(size_t)t * K + (p % K)];
    if (e >= E || e < -1) {
      if (status) atomicCAS(status, 0, (int)kDevBadExpert);
      e = -1;
    } else if (e < 0) {
      e = -1;
    }
  }
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank_w = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && rank_w == 0) wcnt[w][e] = __popc(peers);
  __syncthreads();
  int slot = -1;
  if (e >= 0) {
    int r = rank_w;
    for (int i = 0; i < w; ++i) r += wcnt[i][e];
    slot = block_base[(size_t)blockIdx.x * kMaxExperts + e] + r;
  }
  if (p < npairs) {
    slot_s[p] = slot;
    if (t < T) {
      token_slot[(size_t)t * K + (p % K)] = slot;
      if (slot >= 0) {
        if (sorted_token) sorted_token[slot] = t;
        if (sorted_w) sorted_w[slot] = topk_w[(size_t)t * K + (p % K)];
      }
    }
  }
  __syncthreads();
  // row copy: 4 tokens per pass so each thread keeps 8 x 16 B loads in flight
  const int ntok = min(kRouteTB, T - blockIdx.x * kRouteTB);
  const float *xblk = x + (size_t)blockIdx.x * kRouteTB * H;
  for (int tl0 = 0; tl0 < ntok; tl0 += 4) {
    for (int c = p * 8; c < H; c += blockDim.x * 8) {
      float4 a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (tl0 + u < ntok) {
          const float *src = xblk + (size_t)(tl0 + u) * H + c;
          a[u] = *reinterpret_cast<const float4 *>(src);
          b[u] = *reinterpret_cast<const float4 *>(src + 4);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (tl0 + u >= ntok) break;
        const int tl = tl0 + u;
        if constexpr (sizeof(TOut) == 2) {
          const uint4 v = make_uint4(pack_bf16(a[u].x, a[u].y), pack_bf16(a[u].z, a[u].w),
                                     pack_bf16(b[u].x, b[u].y), pack_bf16(b[u].z, b[u].w));
          for (int k = 0; k < K; ++k) {
            const int s = slot_s[tl * K + k];
            if (s >= 0) *reinterpret_cast<uint4 *>(sorted_x + (size_t)s * H + c) = v;
          }
        } else {
          for (int k = 0; k < K; ++k) {
            const int s = slot_s[tl * K + k];
            if (s >= 0) {
              float4 *d = reinterpret_cast<float4 *>(sorted_x + (size_t)s * H + c);
              d[0] = a[u];
              d[1] = b[u];
            }
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// hist_kernel: the per-block expert histogram route_kernel produces, for
// expert ids the caller computed (b2_moe_dispatch_slots).  One block of 128
// threads per kRouteTB tokens; ids outside [0, E) are not counted (the
// scatter drops and records them).
// ---------------------------------------------------------------------------
static __global__ void __launch_bounds__(128)
    hist_kernel(const int *__restrict__ topk_idx, int T, int E, int K,
                int *__restrict__ block_counts) {
  __shared__ int hist[kMaxExperts];
  if (threadIdx.x < kMaxExperts) hist[threadIdx.x] = 0;
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  const int t0 = blockIdx.x * kRouteTB;
  const int n = min(kRouteTB, T - t0) * K;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = topk_idx[(size_t)t0 * K + i];
    if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  if (threadIdx.x < kMaxExperts)
    block_counts[(size_t)blockIdx.x * kMaxExperts + threadIdx.x] = hist[threadIdx.x];
}

// ---------------------------------------------------------------------------
// combine_kernel: one block (256 threads) per token; thread handles 8 columns.
// y[t,h] = fold over k of fma(out[slot_k,h], w[t,k], sum) from 0 -- the
// reference's `sum += val * weight` in fixed k order (src/layer.cu:709-718).
// Dropped pairs (slot -1) contribute nothing.  With `accumulate` the sum is
// added to y (y = y + sum, the decoder layer's residual add fused).
// ---------------------------------------------------------------------------
template <typename TIn>
__global__ void __launch_bounds__(256)
    combine_kernel(const TIn *__restrict__ sorted_out, const int *__restrict__ token_slot,
                   const float *__restrict__ topk_w, int T, int H, int K,
                   float *__restrict__ y, int accumulate = 0) {
  const int t = blockIdx.x;
  __shared__ int ss[kMaxTopK];
  __shared__ float sw[kMaxTopK];
  pdl_wait();
  if (threadIdx.x < K) {
    ss[threadIdx.x] = token_slot[(size_t)t * K + threadIdx.x];
    sw[threadIdx.x] = topk_w[(size_t)t * K + threadIdx.x];
  }
  __syncthreads();
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    for (int k = 0; k < K; ++k) {
      const int s = ss[k];
      if (s < 0) continue;
      const float wk = sw[k];
      float v[8];
      if constexpr (sizeof(TIn) == 2) {
        const uint4 r = *reinterpret_cast<const uint4 *>(sorted_out + (size_t)s * H + c);
        v[0] = bf16lo(r.x); v[1] = bf16hi(r.x); v[2] = bf16lo(r.y); v[3] = bf16hi(r.y);
        v[4] = bf16lo(r.z); v[5] = bf16hi(r.z); v[6] = bf16lo(r.w); v[7] = bf16hi(r.w);
      } else {
        const float4 a = *reinterpret_cast<const float4 *>(sorted_out + (size_t)s * H + c);
        const float4 b = *reinterpret_cast<const float4 *>(sorted_out + (size_t)s * H + c + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __fmaf_rn(v[i], wk, acc[i]);
    }
    float4 *dst = reinterpret_cast<float4 *>(y + (size_t)t * H + c);
    if (accumulate) {
      const float4 o0 = dst[0], o1 = dst[1];
      acc[0] = __fadd_rn(o0.x, acc[0]); acc[1] = __fadd_rn(o0.y, acc[1]);
      acc[2] = __fadd_rn(o0.z, acc[2]); acc[3] = __fadd_rn(o0.w, acc[3]);
      acc[4] = __fadd_rn(o1.x, acc[4]); acc[5] = __fadd_rn(o1.y, acc[5]);
      acc[6] = __fadd_rn(o1.z, acc[6]); acc[7] = __fadd_rn(o1.w, acc[7]);
    }
    dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// ---------------------------------------------------------------------------
// Weight packing (create time).
// W1||W3 interleaved per 128-row block: packed row blk*256 + r holds
//   r <  128: w1[e][blk*128 + r]      r >= 128: w3[e][blk*128 + r - 128]
// (zero rows past I), so one 256-wide tile yields 128 gate and the matching
// 128 up columns and the SwiGLU happens in the GEMM epilogue.
// W2 is copied to [E][H][Ip] with zero columns past I.
// ---------------------------------------------------------------------------
template <typename TW>
__global__ void pack_w13_single(const float *__restrict__ w1, const float *__restrict__ w3,
                                int H, int I, int Ip, TW *__restrict__ out) {
  const int prow = blockIdx.x;  // 0 .. 2*Ip-1
  const int blk = prow / 256, r = prow % 256;
  const int src_row = blk * 128 + (r & 127);
  const float *src = (src_row < I) ? ((r < 128 ? w1 : w3) + (size_t)src_row * H) : nullptr;
  TW *dst = out + (size_t)prow * H;
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    const float v = src ? src[h] : 0.0f;
    if constexpr (sizeof(TW) == 2) dst[h] = __float2bfloat16_rn(v);
    else dst[h] = v;
  }
}

template <typename TW>
__global__ void pack_w2_single(const float *__restrict__ w2, int H, int I, int Ip,
                               TW *__restrict__ out) {
  const int h = blockIdx.x;
  const float *src = w2 + (size_t)h * I;
  TW *dst = out + (size_t)h * Ip;
  for (int i = threadIdx.x; i < Ip; i += blockDim.x) {
    const float v = i < I ? src[i] : 0.0f;
    if constexpr (sizeof(TW) == 2) dst[i] = __float2bfloat16_rn(v);
    else dst[i] = v;
  }
}

// gateT[h][e] = gate[e][h] for e < E, 0 otherwise (32 columns).
static __global__ void pack_gate_kernel(const float *__restrict__ gate, int E, int H,
                                 float *__restrict__ gateT) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)H * kMaxExperts) return;
  const int h = (int)(i / kMaxExperts), e = (int)(i % kMaxExperts);
  gateT[i] = e < E ? gate[(size_t)e * H + h] : 0.0f;
}

// fp32 -> bf16 (round to nearest even), 8 elements per thread and step.  May
// be launched with programmatic stream serialization: reads `in` only after
// the predecessor kernel has completed.
static __global__ void f32_to_bf16_kernel(const float *__restrict__ in, __nv_bfloat16 *__restrict__ out,
                                   size_t n) {
  pdl_wait();
  pdl_trigger();
  size_t i = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const size_t stride = (size_t)gridDim.x * blockDim.x * 8;
  for (; i + 8 <= n; i += stride) {
    const float4 a = *reinterpret_cast<const float4 *>(in + i);
    const float4 b = *reinterpret_cast<const float4 *>(in + i + 4);
    *reinterpret_cast<uint4 *>(out + i) =
        make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(b.x, b.y), pack_bf16(b.z, b.w));
  }
  if (i < n)
    for (; i < n; ++i) out[i] = __float2bfloat16_rn(in[i]);
}

}  // namespace b2
