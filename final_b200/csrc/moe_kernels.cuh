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
// route_kernel: one block of 64 threads per 32 tokens.
// logits[t,e] = fold_k fma(x[t,k], gate[e,k], acc) from 0.0f -- the order of
// attn_matmul_tiled_kernel (src/layer.cu:70-130), so logits are bit-exact.
// Thread (tg = tid%8, eg = tid/8) owns tokens 4tg..4tg+3 x experts 4eg..4eg+3.
// gateT is the gate transposed to [H][32] (zero columns for e >= E).
// ---------------------------------------------------------------------------
static __global__ void __launch_bounds__(64)
    route_kernel(const float *__restrict__ x, const float *__restrict__ gateT,
                 const float *__restrict__ bias, int T, int H, int E, int K,
                 float routed_scale, int *__restrict__ topk_idx,
                 float *__restrict__ topk_w, int *__restrict__ block_counts,
                 float *__restrict__ logits_out) {
  __shared__ __align__(16) float xs[2][kRouteKC][kRouteTB + 4];
  __shared__ __align__(16) float gs[2][kRouteKC][kMaxExperts];
  __shared__ float lg[kRouteTB][kMaxExperts + 1];
  __shared__ int hist[kMaxExperts];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int wid = tid >> 5;
  const int t0 = blockIdx.x * kRouteTB;
  const int tg = tid & 7, eg = tid >> 3;
  const int NC = H / kRouteKC;
  const bool tok_ok = (t0 + lane) < T;
  const float *xrow = x + (size_t)(t0 + lane) * H;

  if (tid < kMaxExperts) hist[tid] = 0;

  // x chunk: lane = token, warp w loads k-quads 4w..4w+3 (float4 each)
  float4 xr[4];
  auto load_x = [&](int kc) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k0 = (wid * 4 + i) * 4;
      xr[i] = tok_ok ? *reinterpret_cast<const float4 *>(xrow + kc * kRouteKC + k0)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto store_x = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k0 = (wid * 4 + i) * 4;
      xs[buf][k0 + 0][lane] = xr[i].x;
      xs[buf][k0 + 1][lane] = xr[i].y;
      xs[buf][k0 + 2][lane] = xr[i].z;
      xs[buf][k0 + 3][lane] = xr[i].w;
    }
  };
  // gate chunk [KC][32] fp32 = 4 KB: 256 x 16 B, 4 per thread
  auto load_g = [&](int kc, int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int v = tid + i * 64;  // 16-byte vector index within the chunk
      const float4 *src = reinterpret_cast<const float4 *>(gateT + (size_t)kc * kRouteKC * kMaxExperts) + v;
      reinterpret_cast<float4 *>(&gs[buf][0][0])[v] = *src;
    }
  };

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  load_x(0);
  store_x(0);
  load_g(0, 0);
  __syncthreads();
  for (int kc = 0; kc < NC; ++kc) {
    const int buf = kc & 1;
    const bool more = kc + 1 < NC;
    if (more) load_x(kc + 1);
#pragma unroll 8
    for (int k = 0; k < kRouteKC; ++k) {
      const float4 xv = *reinterpret_cast<const float4 *>(&xs[buf][k][tg * 4]);
      const float4 gv = *reinterpret_cast<const float4 *>(&gs[buf][k][eg * 4]);
      const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
      const float ga[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(xa[i], ga[j], acc[i][j]);
    }
    if (more) {
      store_x(buf ^ 1);
      load_g(kc + 1, buf ^ 1);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) lg[tg * 4 + i][eg * 4 + j] = acc[i][j];
  __syncthreads();

  if (tid < kRouteTB) {
    const int t = t0 + tid;
    if (t < T) {
      if (logits_out)
        for (int e = 0; e < E; ++e) logits_out[(size_t)t * E + e] = lg[tid][e];
      float ms[kMaxTopK], mp[kMaxTopK];
      int mi[kMaxTopK];
#pragma unroll
      for (int i = 0; i < kMaxTopK; ++i) {
        ms[i] = -1e30f;
        mp[i] = 0.0f;
        mi[i] = -1;
      }
      for (int e = 0; e < E; ++e) {
        const float prob = 1.0f / (1.0f + (float)exp(-(double)lg[tid][e]));
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
  if (tid < kMaxExperts) block_counts[(size_t)blockIdx.x * kMaxExperts + tid] = hist[tid];
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
// scatter_kernel: block b handles tokens [32b, 32b+32) with 32*K threads,
// thread p owns pair (token 32b + p/K, rank p%K).  Its slot is
//   block_base[b][e] + #{pairs p' < p in this block with the same expert}
// which is the canonical token-major order of the CPU oracle.  Then the block
// copies each token row once from fp32 x into its K slots as bf16 (or fp32).
// ---------------------------------------------------------------------------
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
  __syncthreads();
  int e = -1;
  if (p < npairs && t < T) {
    e = topk_idx[(size_t)t * K + (p % K)];
    if (e < 0 || e >= E) e = -1;
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
  const int ntok = min(kRouteTB, T - blockIdx.x * kRouteTB);
  for (int tl = 0; tl < ntok; ++tl) {
    const float *src = x + (size_t)(blockIdx.x * kRouteTB + tl) * H;
    for (int c = p * 8; c < H; c += blockDim.x * 8) {
      const float4 a = *reinterpret_cast<const float4 *>(src + c);
      const float4 b = *reinterpret_cast<const float4 *>(src + c + 4);
      if constexpr (sizeof(TOut) == 2) {
        const uint4 v = make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w),
                                   pack_bf16(b.x, b.y), pack_bf16(b.z, b.w));
        for (int k = 0; k < K; ++k) {
          const int s = slot_s[tl * K + k];
          if (s >= 0) *reinterpret_cast<uint4 *>(sorted_x + (size_t)s * H + c) = v;
        }
      } else {
        for (int k = 0; k < K; ++k) {
          const int s = slot_s[tl * K + k];
          if (s >= 0) {
            float4 *d = reinterpret_cast<float4 *>(sorted_x + (size_t)s * H + c);
            d[0] = a;
            d[1] = b;
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// combine_kernel: one block (256 threads) per token; thread handles 8 columns.
// y[t,h] = fold over k of fma(out[slot_k,h], w[t,k], sum) from 0 -- the
// reference's `sum += val * weight` in fixed k order (src/layer.cu:709-718).
// Dropped pairs (slot -1) contribute nothing.
// ---------------------------------------------------------------------------
template <typename TIn>
__global__ void __launch_bounds__(256)
    combine_kernel(const TIn *__restrict__ sorted_out, const int *__restrict__ token_slot,
                   const float *__restrict__ topk_w, int T, int H, int K,
                   float *__restrict__ y) {
  const int t = blockIdx.x;
  __shared__ int ss[kMaxTopK];
  __shared__ float sw[kMaxTopK];
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

static __global__ void f32_to_bf16_kernel(const float *__restrict__ in, __nv_bfloat16 *__restrict__ out,
                                   size_t n) {
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
