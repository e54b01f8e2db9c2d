// lfm2_kernels.cuh -- the decoder-layer glue of the LFM2 model around the
// tcgen05 GEMMs: embedding gather, fused residual-add + RMSNorm, per-head q/k
// RMSNorm + RoPE, causal GQA flash attention and the short-convolution
// gating.  All of them are HBM- or latency-bound; none is a matrix product
// big enough for the tensor-core GEMM (the attention's two 64-wide products
// per key block run on mma.sync inside the kernel, see flash_attn_kernel).
//
// Replaces embedding_lookup_kernel (src/model.cu:18-31), rms_norm_kernel
// (src/layer.cu:144-191) with add_kernel (:1872-1893), rope_transpose_kernel
// / transpose_v_kernel (:193-245), fused_attn_gqa_kernel (:296-393) and the
// three conv kernels (:397-465) of the reference.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include "sm100_ptx.cuh"

namespace b2 {

constexpr int kDevBadToken = 0x203;  // token id outside [0, vocab)

// ------------------------------------------------------------ embedding
// out[t][:] = table[ids[t]][:], one block per token, 16-byte vectors
// (H % 4 == 0).  An id outside [0, V) records kDevBadToken and writes zeros.
static __global__ void __launch_bounds__(256)
    embed_kernel(const int *__restrict__ ids, const float *__restrict__ table, int H, int V,
                 float *__restrict__ out, int *status) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0 && status) atomicCAS(status, 0, kDevBadToken);
    id = -1;
  }
  const int h4 = H >> 2;
  const float4 *src = reinterpret_cast<const float4 *>(table) + (size_t)(id < 0 ? 0 : id) * h4;
  float4 *dst = reinterpret_cast<float4 *>(out) + (size_t)t * h4;
  for (int i = threadIdx.x; i < h4; i += blockDim.x)
    dst[i] = id < 0 ? make_float4(0.f, 0.f, 0.f, 0.f) : __ldg(src + i);
}

// ------------------------------------------------------------ add + RMSNorm
// One block of 256 threads per RPB output rows.  Input row of output row o =
// o * step + off (step 1 / off 0 for every row; step S / off S-1 for the last
// token of each sequence).  With ADD, v = resid + delta (written back to
// resid when write_resid), else v = resid.  y = v * r * w with
// r = 1 / sqrtf(sum(v^2) / dim + eps), written as fp32 and/or bf16.
//
// The sum is formed in exactly the order of the reference's rms_norm_kernel
// launched with 256 threads: thread t accumulates elements t, t+256, ... by
// FFMA, warps reduce by __shfl_down 16..1, warp 0 reduces the eight warp sums
// by __shfl_down 4, 2, 1.  The division and square root are the IEEE ones
// (no fast-math), so y equals the reference's bit for bit.
// NPT > 0: dim == 256 * NPT, the rows stay in registers: the RPB rows and the
// weights are all loaded before the first reduction, so a block keeps
// RPB * dim * 4 bytes in flight and its reduction latency is paid once for
// RPB rows; each row is reduced in its own tree, in the order above.
// NPT == 0 (RPB 1): any dim, two passes, the same order.
template <int NPT, int RPB>
__global__ void __launch_bounds__(256)
    add_rmsnorm_kernel(float *__restrict__ resid, const float *__restrict__ delta,
                       const float *__restrict__ w, int rows, int dim, int step, int off,
                       int write_resid, float eps, float *__restrict__ y32,
                       __nv_bfloat16 *__restrict__ y16) {
  static_assert(NPT > 0 || RPB == 1, "the two-pass path handles one row per block");
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float ws[RPB][8];
  __shared__ float total[RPB];
  float s[RPB];
  float v[RPB][NPT > 0 ? NPT : 1];
  float wv[NPT > 0 ? NPT : 1];
  bool ok[RPB];
  float *r[RPB];
  const float *dl[RPB];
#pragma unroll
  for (int q = 0; q < RPB; ++q) {
    const int o = blockIdx.x * RPB + q;
    ok[q] = o < rows;
    const size_t row_in = (size_t)(ok[q] ? o : 0) * step + off;
    r[q] = resid + row_in * dim;
    dl[q] = delta ? delta + row_in * dim : nullptr;
    s[q] = 0.0f;
  }
  if constexpr (NPT > 0) {
#pragma unroll
    for (int q = 0; q < RPB; ++q)
#pragma unroll
      for (int j = 0; j < NPT; ++j) v[q][j] = ok[q] ? r[q][tid + 256 * j] : 0.0f;
#pragma unroll
    for (int j = 0; j < NPT; ++j) wv[j] = w[tid + 256 * j];
    if (delta) {
#pragma unroll
      for (int q = 0; q < RPB; ++q) {
        if (!ok[q]) continue;
#pragma unroll
        for (int j = 0; j < NPT; ++j) v[q][j] = __fadd_rn(v[q][j], dl[q][tid + 256 * j]);
        if (write_resid)
#pragma unroll
          for (int j = 0; j < NPT; ++j) r[q][tid + 256 * j] = v[q][j];
      }
    }
#pragma unroll
    for (int q = 0; q < RPB; ++q)
#pragma unroll
      for (int j = 0; j < NPT; ++j) s[q] = __fmaf_rn(v[q][j], v[q][j], s[q]);
  } else {
    for (int i = tid; i < dim; i += 256) {
      float x = r[0][i];
      if (dl[0]) {
        x = __fadd_rn(x, dl[0][i]);
        if (write_resid) r[0][i] = x;
      }
      s[0] = __fmaf_rn(x, x, s[0]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int q = 0; q < RPB; ++q) s[q] += __shfl_down_sync(0xffffffffu, s[q], o);
  if (lane == 0)
#pragma unroll
    for (int q = 0; q < RPB; ++q) ws[q][warp] = s[q];
  __syncthreads();
  if (warp == 0) {
    float t[RPB];
#pragma unroll
    for (int q = 0; q < RPB; ++q) t[q] = lane < 8 ? ws[q][lane] : 0.0f;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1)
#pragma unroll
      for (int q = 0; q < RPB; ++q) t[q] += __shfl_down_sync(0xffffffffu, t[q], o);
    if (lane == 0)
#pragma unroll
      for (int q = 0; q < RPB; ++q) total[q] = t[q];
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < RPB; ++q) {
    if (!ok[q]) continue;
    const float rms =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total[q], (float)dim), eps)));
    const size_t row_out = (size_t)blockIdx.x * RPB + q;
    if constexpr (NPT > 0) {
#pragma unroll
      for (int j = 0; j < NPT; ++j) {
        const int i = tid + 256 * j;
        const float o = __fmul_rn(__fmul_rn(v[q][j], rms), wv[j]);
        if (y32) y32[row_out * dim + i] = o;
        if (y16) y16[row_out * dim + i] = __float2bfloat16_rn(o);
      }
    } else {
      for (int i = tid; i < dim; i += 256) {
        float x = r[q][i];
        if (dl[q] && !write_resid) x = __fadd_rn(x, dl[q][i]);
        const float o = __fmul_rn(__fmul_rn(x, rms), w[i]);
        if (y32) y32[row_out * dim + i] = o;
        if (y16) y16[row_out * dim + i] = __float2bfloat16_rn(o);
      }
    }
  }
}

// ------------------------------------------------------------ q/k norm + RoPE
// qkv: [T][(Hq + 2 Hkv) * 64] bf16 projections (q heads, k heads, v heads;
// the projection GEMM writes bf16, half the bytes of fp32 both ways).
// One block per token, one warp per head (lane l holds elements l and l+32,
// which are exactly the pair RoPE rotates).  q / k heads: RMSNorm over the
// 64 values in the reference's order for a 64-wide row (rms_norm_kernel,
// src/layer.cu:144-191: two 32-lane shuffle trees, then their sum; the mean
// x/64 is taken as x * 2^-6, the same correctly rounded value), then RoPE at
// position s = t % S with the caller's [pos][64] cos / sin tables
// (rope_transpose_kernel, :193-227):
//   o1 = n1*c1 - n2*s1,  o2 = n2*c2 + n1*s2   (one FFMA each).
// Written as bf16 in [B][heads][S][64] (one contiguous 128-byte row per
// head and position), v heads converted only.  A warp loads all of its heads
// (up to kQkHeadsInFlight) before computing any, so their HBM latencies
// overlap instead of adding up head after head; the position's tables and
// the two norm weights are loaded once per warp, and the heads' 1/rms are
// computed together (head j's sum in lane j).
constexpr int kQkHeadsInFlight = 8;  // per warp (48 heads over 8 warps: 6)

static __global__ void __launch_bounds__(256)
    qk_norm_rope_kernel(const __nv_bfloat16 *__restrict__ qkv, const float *__restrict__ q_ln,
                        const float *__restrict__ k_ln, const float *__restrict__ cosv,
                        const float *__restrict__ sinv, int S, int Hq, int Hkv, float eps,
                        __nv_bfloat16 *__restrict__ q, __nv_bfloat16 *__restrict__ k,
                        __nv_bfloat16 *__restrict__ v) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x, b = t / S, s = t - b * S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nh = Hq + 2 * Hkv;
  const __nv_bfloat16 *row = qkv + (size_t)t * nh * 64;
  const float *cs = cosv + (size_t)s * 64, *sn = sinv + (size_t)s * 64;
  const float c1 = cs[lane], c2 = cs[lane + 32], s1 = sn[lane], s2 = sn[lane + 32];
  const float wq1 = q_ln[lane], wq2 = q_ln[lane + 32];
  const float wk1 = k_ln[lane], wk2 = k_ln[lane + 32];
  for (int h0 = warp; h0 < nh; h0 += 8 * kQkHeadsInFlight) {
    __nv_bfloat16 r1[kQkHeadsInFlight], r2[kQkHeadsInFlight];
#pragma unroll
    for (int j = 0; j < kQkHeadsInFlight; ++j) {
      const int h = h0 + 8 * j;
      if (h < nh) {
        r1[j] = row[h * 64 + lane];
        r2[j] = row[h * 64 + lane + 32];
      }
    }
    // sums of squares of the q / k heads, head j's in lane j, so one IEEE
    // divide and square root serve all of them
    float mine = 0.0f;
#pragma unroll
    for (int j = 0; j < kQkHeadsInFlight; ++j) {
      const int h = h0 + 8 * j;  // warp-uniform
      if (h >= nh || h >= Hq + Hkv) break;
      const float x1 = __bfloat162float(r1[j]);
      const float x2 = __bfloat162float(r2[j]);
      float a = __fmul_rn(x1, x1), c = __fmul_rn(x2, x2);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_down_sync(0xffffffffu, a, o);
        c += __shfl_down_sync(0xffffffffu, c, o);
      }
      const float tot = __shfl_sync(0xffffffffu, __fadd_rn(a, c), 0);
      if (lane == j) mine = tot;
    }
    const float rms_mine =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(mine, 0.015625f), eps)));
#pragma unroll
    for (int j = 0; j < kQkHeadsInFlight; ++j) {
      const int h = h0 + 8 * j;  // warp-uniform
      if (h >= nh) break;
      if (h >= Hq + Hkv) {
        __nv_bfloat16 *dst = v + (((size_t)b * Hkv + (h - Hq - Hkv)) * S + s) * 64;
        dst[lane] = r1[j];
        dst[lane + 32] = r2[j];
        continue;
      }
      const float x1 = __bfloat162float(r1[j]);
      const float x2 = __bfloat162float(r2[j]);
      const float rms = __shfl_sync(0xffffffffu, rms_mine, j);
      const bool isq = h < Hq;
      const float n1 = __fmul_rn(__fmul_rn(x1, rms), isq ? wq1 : wk1);
      const float n2 = __fmul_rn(__fmul_rn(x2, rms), isq ? wq2 : wk2);
      const float o1 = __fmaf_rn(n1, c1, -__fmul_rn(n2, s1));
      const float o2 = __fmaf_rn(n2, c2, __fmul_rn(n1, s2));
      __nv_bfloat16 *dst = isq ? q + (((size_t)b * Hq + h) * S + s) * 64
                               : k + (((size_t)b * Hkv + (h - Hq)) * S + s) * 64;
      dst[lane] = __float2bfloat16_rn(o1);
      dst[lane + 32] = __float2bfloat16_rn(o2);
    }
  }
}

// ------------------------------------------------------------ flash attention
// Causal GQA attention, head_dim 64, bf16 operands, fp32 softmax state.
// Grid (ceil(S/64) query blocks, Hq, B), 128 threads: warp w owns query rows
// [16w, 16w+16) of the block.  Key / value blocks of 64 rows stream through a
// two-stage cp.async ring; S = Q K^T and O += P V are m16n8k16 bf16 MMAs with
// fp32 accumulators in registers (the P fragments are the S accumulators
// re-packed, never touching shared memory); the softmax is online in the
// log2 domain (ex2.approx).  Causal: query block i reads key blocks 0..i
// only, the diagonal one masked per element; query blocks are issued
// heaviest first.  Output O[t][h*64 + d] bf16, token-major (the A operand of
// the out projection).  Attention is ~1% of the model's FLOPs at seq 512, so
// the per-warp MMA path is enough here; the GEMMs that dominate run on
// tcgen05.
constexpr int kAttnB = 64;   // query / key rows per block
constexpr int kAttnLd = 72;  // padded smem row (bf16): 144 B, ldmatrix conflict-free

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                          uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void attn_cp16(uint32_t dst, const void *src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes)
               : "memory");
}

static __global__ void __launch_bounds__(128)
    flash_attn_kernel(const __nv_bfloat16 *__restrict__ Q, const __nv_bfloat16 *__restrict__ K,
                      const __nv_bfloat16 *__restrict__ V, int S, int Hq, int Hkv,
                      float scale_log2, __nv_bfloat16 *__restrict__ O) {
  __shared__ __align__(128) __nv_bfloat16 sQ[kAttnB * kAttnLd];
  __shared__ __align__(128) __nv_bfloat16 sK[2][kAttnB * kAttnLd];
  __shared__ __align__(128) __nv_bfloat16 sV[2][kAttnB * kAttnLd];
  const int qb = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (Hq / Hkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __nv_bfloat16 *Qb = Q + ((size_t)b * Hq + h) * S * 64;
  const __nv_bfloat16 *Kb = K + ((size_t)b * Hkv + hk) * S * 64;
  const __nv_bfloat16 *Vb = V + ((size_t)b * Hkv + hk) * S * 64;
  const int q0 = qb * kAttnB;

  // 64 rows x 8 chunks of 16 bytes; rows past S are zero-filled
  auto load_tile = [&](__nv_bfloat16 *dst, const __nv_bfloat16 *src, int row0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = tid + i * 128, r = c >> 3, u = c & 7;
      const int gr = row0 + r;
      const __nv_bfloat16 *g = src + (size_t)(gr < S ? gr : 0) * 64 + u * 8;
      attn_cp16(smem_u32(dst + r * kAttnLd + u * 8), g, gr < S ? 16u : 0u);
    }
  };

  pdl_wait();
  pdl_trigger();
  load_tile(sQ, Qb, q0);
  load_tile(sK[0], Kb, 0);
  load_tile(sV[0], Vb, 0);
  asm volatile("cp.async.commit_group;" ::: "memory");

  const int nkb = qb + 1;
  const int g = lane >> 2, qd = lane & 3;
  const int row0 = q0 + warp * 16 + g, row1 = row0 + 8;
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F, l0 = 0.0f, l1 = 0.0f;
  uint32_t qf[4][4];
  const int lm = lane >> 3, lr = lane & 7;

  for (int j = 0; j < nkb; ++j) {
    if (j + 1 < nkb) {
      load_tile(sK[(j + 1) & 1], Kb, (j + 1) * kAttnB);
      load_tile(sV[(j + 1) & 1], Vb, (j + 1) * kAttnB);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kc = 0; kc < 4; ++kc)
        ldsm_x4(smem_u32(sQ + (warp * 16 + (lane & 15)) * kAttnLd + kc * 16 + (lane >> 4) * 8),
                qf[kc][0], qf[kc][1], qf[kc][2], qf[kc][3]);
    }
    const __nv_bfloat16 *ks = sK[j & 1], *vs = sV[j & 1];
    float sc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.0f;
#pragma unroll
    for (int kc = 0; kc < 4; ++kc)
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(ks + (np * 16 + (lm >> 1) * 8 + lr) * kAttnLd + kc * 16 + (lm & 1) * 8),
                b0, b1, b2, b3);
        mma_bf16_16816(sc[2 * np], qf[kc], b0, b1);
        mma_bf16_16816(sc[2 * np + 1], qf[kc], b2, b3);
      }
    // scale to the log2 domain, mask the future and the padding
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = j * kAttnB + nt * 8 + qd * 2 + (e & 1);
        const int row = e < 2 ? row0 : row1;
        float v = sc[nt][e] * scale_log2;
        if (key > row || key >= S) v = -CUDART_INF_F;
        sc[nt][e] = v;
        if (e < 2) mx0 = fmaxf(mx0, v); else mx1 = fmaxf(mx1, v);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float r0 = mx0 == -CUDART_INF_F ? 0.0f : mx0;
    const float r1 = mx1 == -CUDART_INF_F ? 0.0f : mx1;
    const float a0 = ex2_approx(m0 - r0), a1 = ex2_approx(m1 - r1);
    m0 = mx0;
    m1 = mx1;
    l0 *= a0;
    l1 *= a1;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      o[nt][0] *= a0;
      o[nt][1] *= a0;
      o[nt][2] *= a1;
      o[nt][3] *= a1;
      sc[nt][0] = ex2_approx(sc[nt][0] - r0);
      sc[nt][1] = ex2_approx(sc[nt][1] - r0);
      sc[nt][2] = ex2_approx(sc[nt][2] - r1);
      sc[nt][3] = ex2_approx(sc[nt][3] - r1);
      l0 += sc[nt][0] + sc[nt][1];
      l1 += sc[nt][2] + sc[nt][3];
    }
    // O += P V over the block's 64 keys (4 chunks of 16)
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      const uint32_t pa[4] = {pack_bf16(sc[2 * kc][0], sc[2 * kc][1]),
                              pack_bf16(sc[2 * kc][2], sc[2 * kc][3]),
                              pack_bf16(sc[2 * kc + 1][0], sc[2 * kc + 1][1]),
                              pack_bf16(sc[2 * kc + 1][2], sc[2 * kc + 1][3])};
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(vs + (kc * 16 + (lm & 1) * 8 + lr) * kAttnLd + dp * 16 + (lm >> 1) * 8),
                  b0, b1, b2, b3);
        mma_bf16_16816(o[2 * dp], pa, b0, b1);
        mma_bf16_16816(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncthreads();  // every warp is done with this stage before it is refilled
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
  const size_t ld = (size_t)Hq * 64;
  __nv_bfloat16 *ob = O + (size_t)b * S * ld + (size_t)h * 64;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int d = nt * 8 + qd * 2;
    if (row0 < S)
      *reinterpret_cast<uint32_t *>(ob + (size_t)row0 * ld + d) =
          pack_bf16(o[nt][0] * inv0, o[nt][1] * inv0);
    if (row1 < S)
      *reinterpret_cast<uint32_t *>(ob + (size_t)row1 * ld + d) =
          pack_bf16(o[nt][2] * inv1, o[nt][3] * inv1);
  }
}

// ------------------------------------------------------------ short conv
// in_proj output ip: [T][3H] bf16 = (B | C | gate) per token (the projection
// GEMM writes bf16: half the bytes of fp32 both ways); conv_w [H][3].
// y[t][h] = C[t][h] * sum_k w[h][k] * Bx[t-2+k][h] over positions of the
// same sequence (Bx = B * gate), the reference's FFMA chain from 0 in k order
// (conv_transpose_split_kernel, causal_conv1d_kernel and
// conv_gating_transpose_kernel fused, src/layer.cu:397-465), written bf16.
// A thread owns 4 adjacent channels over kConvRun consecutive positions and
// keeps the two previous Bx in registers.
constexpr int kConvRun = 16;
constexpr int kConvL = 3;
static __global__ void __launch_bounds__(128)
    conv_glue_kernel(const __nv_bfloat16 *__restrict__ ip, const float *__restrict__ cw, int S,
                     int H, __nv_bfloat16 *__restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const int h4 = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (h4 >= H) return;
  const int b = blockIdx.z, s0 = blockIdx.y * kConvRun;
  float w[4][kConvL];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int k = 0; k < kConvL; ++k) w[c][k] = cw[(size_t)(h4 + c) * kConvL + k];
  const size_t ld = (size_t)3 * H;
  const __nv_bfloat16 *base = ip + (size_t)b * S * ld + h4;
  auto ld4 = [&](const __nv_bfloat16 *p) {  // 4 bf16 (8 bytes) as fp32
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    return make_float4(bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y));
  };
  auto bx_at = [&](int s) {
    const float4 bv = ld4(base + (size_t)s * ld);
    const float4 gv = ld4(base + (size_t)s * ld + 2 * H);
    return make_float4(__fmul_rn(bv.x, gv.x), __fmul_rn(bv.y, gv.y), __fmul_rn(bv.z, gv.z),
                       __fmul_rn(bv.w, gv.w));
  };
  float4 hist[kConvL - 1];  // Bx at s-2, s-1
#pragma unroll
  for (int k = 0; k < kConvL - 1; ++k) {
    const int p = s0 - (kConvL - 1) + k;
    hist[k] = p >= 0 ? bx_at(p) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const int s_end = min(S, s0 + kConvRun);
  for (int s = s0; s < s_end; ++s) {
    const float4 cur = bx_at(s);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < kConvL; ++k) {
      if (s - (kConvL - 1) + k < 0) continue;
      const float4 v = k == kConvL - 1 ? cur : hist[k];
      acc[0] = __fmaf_rn(v.x, w[0][k], acc[0]);
      acc[1] = __fmaf_rn(v.y, w[1][k], acc[1]);
      acc[2] = __fmaf_rn(v.z, w[2][k], acc[2]);
      acc[3] = __fmaf_rn(v.w, w[3][k], acc[3]);
    }
#pragma unroll
    for (int k = 0; k < kConvL - 2; ++k) hist[k] = hist[k + 1];
    hist[kConvL - 2] = cur;
    const float4 cv = ld4(base + (size_t)s * ld + H);
    const uint2 out = make_uint2(pack_bf16(__fmul_rn(cv.x, acc[0]), __fmul_rn(cv.y, acc[1])),
                                 pack_bf16(__fmul_rn(cv.z, acc[2]), __fmul_rn(cv.w, acc[3])));
    *reinterpret_cast<uint2 *>(y + ((size_t)b * S + s) * H + h4) = out;
  }
}

}  // namespace b2
