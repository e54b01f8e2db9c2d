/*
 * moe_oracle.c -- CPU restatement of the reference engine's MoE / tiled-GEMM
 * semantics.  TEST INFRASTRUCTURE ONLY: the parity tests, smoke() and the
 * cpu_baseline leg of bench.py use this library as the checker (and as the
 * timed CPU stand-in for the reference, which ships no CPU implementation of
 * this path -- every CPU forward() in src/layer.cu is an empty stub,
 * src/layer.cu:1499-1503).  The product path never links or calls it.
 *
 * Parity pin: the routing results (logits, expert ids, weights, counts) are
 * bit-exact with the reference's own CUDA kernels compiled from source
 * (oracle/ref_harness.cu), and the expert-FFN output agrees with them to a few
 * fp32 ulps (the only difference is expf: glibc here, CUDA's libdevice there).
 * The committed fixtures under tests/golden/ were produced by those reference
 * kernels on a B200 and are checked against this file by tests/test_oracle.py.
 *
 * Every function names the reference lines it restates.  Floating-point
 * operation order is the reference's: every dot product is a sequential-k
 * chain of fused multiply-adds starting from 0.0f (nvcc contracts
 * `acc += a*b` to FFMA), which fmaf() reproduces bit-for-bit.  This file must
 * be compiled with -ffp-contract=off so the compiler adds no other fusions.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define B2O_MAXK 8

int b2o_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void b2o_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ------------------------------------------------------------------------ */
/* Dense NT GEMM: C[M,N] = A[M,K] . B[N,K]^T, fp32.                          */
/* Restates attn_matmul_tiled_kernel (src/layer.cu:9-141): each output is a  */
/* single accumulator updated in k order by `acc += a*b` (FFMA), starting at */
/* 0.0f.  The loop below keeps that per-output order exactly and vectorises  */
/* across rows of A instead (transposed into a small panel).                 */
/* ------------------------------------------------------------------------ */
#define B2O_MT 64
void b2o_gemm_nt(const float *A, const float *B, float *C, int M, int N,
                 int K) {
  int mtiles = (M + B2O_MT - 1) / B2O_MT;
#pragma omp parallel
  {
    float *panel = (float *)malloc(sizeof(float) * (size_t)K * B2O_MT);
    float acc[B2O_MT];
#pragma omp for schedule(dynamic, 1)
    for (int mt = 0; mt < mtiles; ++mt) {
      int m0 = mt * B2O_MT;
      int mr = M - m0 < B2O_MT ? M - m0 : B2O_MT;
      for (int k = 0; k < K; ++k)
        for (int r = 0; r < B2O_MT; ++r)
          panel[(size_t)k * B2O_MT + r] =
              r < mr ? A[(size_t)(m0 + r) * K + k] : 0.0f;
      for (int n = 0; n < N; ++n) {
        const float *b = B + (size_t)n * K;
        for (int r = 0; r < B2O_MT; ++r) acc[r] = 0.0f;
        for (int k = 0; k < K; ++k) {
          const float bk = b[k];
          const float *p = panel + (size_t)k * B2O_MT;
          for (int r = 0; r < B2O_MT; ++r) acc[r] = fmaf(p[r], bk, acc[r]);
        }
        for (int r = 0; r < mr; ++r) C[(size_t)(m0 + r) * N + n] = acc[r];
      }
    }
    free(panel);
  }
}

/* Router logits = x . gate^T (src/layer.cu:1440-1450 launches the tiled GEMM
 * above with N = num_experts). */
void b2o_router_logits(const float *x, const float *gate, float *logits, int T,
                       int E, int H) {
  b2o_gemm_nt(x, gate, logits, T, E, H);
}

/* d_sigmoid (src/layer.cu:435): float result of a double-precision exp. */
static float sigmoid_ref(float v) {
  return 1.0f / (1.0f + (float)exp(-(double)v));
}

/* d_silu_opt (src/layer.cu:728). */
static float silu_ref(float v) { return v / (1.0f + expf(-v)); }

/* ------------------------------------------------------------------------ */
/* moe_router_topk_kernel (src/layer.cu:439-499).                            */
/*  prob  = sigmoid(logit); score = prob + bias[e] (selection only)          */
/*  top-K by insertion with strict '>' (ties keep the lower expert id)       */
/*  initial slot score -1e30f, id -1, prob 0                                 */
/*  sum   = sequential fp32 sum of the K selected probs                      */
/*  scale = sum > 1e-6f ? 1/sum : 1;  w_i = prob_i * scale * routed_scale    */
/*  counts[e] += 1 for each selected id in [0,E)                             */
/* counts may be NULL; it is accumulated into (not cleared).                 */
/* ------------------------------------------------------------------------ */
void b2o_route_topk(const float *logits, const float *bias, int T, int E,
                    int K, float routed_scale, int32_t *idx, float *w,
                    int32_t *counts) {
  if (K > B2O_MAXK) K = B2O_MAXK;
  for (int t = 0; t < T; ++t) {
    float ms[B2O_MAXK], mp[B2O_MAXK];
    int mi[B2O_MAXK];
    for (int i = 0; i < K; ++i) {
      ms[i] = -1e30f;
      mp[i] = 0.0f;
      mi[i] = -1;
    }
    for (int e = 0; e < E; ++e) {
      float prob = sigmoid_ref(logits[(size_t)t * E + e]);
      float score = prob + (bias ? bias[e] : 0.0f);
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
    for (int i = 0; i < K; ++i) sum += mp[i];
    float scale = (sum > 1e-6f) ? (1.0f / sum) : 1.0f;
    for (int i = 0; i < K; ++i) {
      idx[(size_t)t * K + i] = mi[i];
      w[(size_t)t * K + i] = mp[i] * scale * routed_scale;
      if (counts && mi[i] >= 0 && mi[i] < E) counts[mi[i]]++;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* moe_scan_kernel (src/layer.cu:730-768): exclusive prefix of counts and of */
/* ceil(count/tile) -> offsets[E], tile_offsets[E+1] (sentinel = total).     */
/* ------------------------------------------------------------------------ */
void b2o_scan(const int32_t *counts, int E, int tile, int32_t *offsets,
              int32_t *tile_offsets) {
  int32_t off = 0, toff = 0;
  for (int e = 0; e < E; ++e) {
    offsets[e] = off;
    tile_offsets[e] = toff;
    off += counts[e];
    toff += (counts[e] + tile - 1) / tile;
  }
  tile_offsets[E] = toff;
}

/* ------------------------------------------------------------------------ */
/* Scatter bookkeeping (moe_scatter_kernel, src/layer.cu:501-542) in the    */
/* canonical deterministic order: within each expert segment, slots follow  */
/* (token, rank) order.  The reference assigns slots with atomicAdd in block */
/* scheduling order, so only the per-expert SET of (token, rank) pairs is    */
/* comparable with it; this order is the one the B200 kernels must produce.  */
/* Out-of-range ids (the reference's -1 when fewer than K experts scored)    */
/* get token_slot = -1 and no slot.                                          */
/* ------------------------------------------------------------------------ */
void b2o_scatter_canonical(const int32_t *idx, const float *w, int T, int K,
                           int E, const int32_t *offsets,
                           int32_t *sorted_token, float *sorted_w,
                           int32_t *token_slot) {
  int32_t *fill = (int32_t *)calloc((size_t)E, sizeof(int32_t));
  for (int t = 0; t < T; ++t)
    for (int k = 0; k < K; ++k) {
      int e = idx[(size_t)t * K + k];
      if (e < 0 || e >= E) {
        token_slot[(size_t)t * K + k] = -1;
        continue;
      }
      int s = offsets[e] + fill[e]++;
      if (sorted_token) sorted_token[s] = t;
      if (sorted_w) sorted_w[s] = w[(size_t)t * K + k];
      token_slot[(size_t)t * K + k] = s;
    }
  free(fill);
}

/* ------------------------------------------------------------------------ */
/* Expert FFN over the sorted rows.                                          */
/*  inter[s,n] = silu(x_s . w1[e][n]) * (x_s . w3[e][n])                     */
/*      (moe_persistent_fused_w1w3_kernel, src/layer.cu:773-972; the        */
/*       epilogue at :964 is d_silu_opt(s1) * s3)                            */
/*  out[s,h]   = inter_s . w2[e][h]                                          */
/*      (moe_persistent_w2_kernel, src/layer.cu:974-1126)                    */
/* w1/w3 are per-expert [I,H] row-major, w2 per-expert [H,I] (the reference's*/
/* float** tables, src/layer.cu:1377-1396).  Row s of expert e reads          */
/* x[sorted_token[s]].  inter may be NULL (then a private buffer is used).   */
/* ------------------------------------------------------------------------ */
#define B2O_RT 32
void b2o_expert_ffn(const float *x, const int32_t *sorted_token,
                    const int32_t *offsets, const int32_t *counts, int E,
                    int H, int I, const float *const *w1,
                    const float *const *w3, const float *const *w2,
                    float *inter, float *out) {
  /* work items: (expert, row-tile) */
  int total = 0;
  for (int e = 0; e < E; ++e) total += (counts[e] + B2O_RT - 1) / B2O_RT;
  int *item_e = (int *)malloc(sizeof(int) * (total + 1));
  int *item_r = (int *)malloc(sizeof(int) * (total + 1));
  int n_items = 0;
  for (int e = 0; e < E; ++e)
    for (int r = 0; r < counts[e]; r += B2O_RT) {
      item_e[n_items] = e;
      item_r[n_items] = r;
      n_items++;
    }
#pragma omp parallel
  {
    float *xT = (float *)malloc(sizeof(float) * (size_t)H * B2O_RT);
    float *iT = (float *)malloc(sizeof(float) * (size_t)I * B2O_RT);
    float a1[B2O_RT], a3[B2O_RT];
#pragma omp for schedule(dynamic, 1)
    for (int it = 0; it < n_items; ++it) {
      int e = item_e[it];
      int r0 = item_r[it];
      int rows = counts[e] - r0 < B2O_RT ? counts[e] - r0 : B2O_RT;
      int s0 = offsets[e] + r0;
      for (int k = 0; k < H; ++k)
        for (int r = 0; r < B2O_RT; ++r)
          xT[(size_t)k * B2O_RT + r] =
              r < rows ? x[(size_t)sorted_token[s0 + r] * H + k] : 0.0f;
      const float *W1 = w1[e], *W3 = w3[e], *W2 = w2[e];
      for (int n = 0; n < I; ++n) {
        const float *b1 = W1 + (size_t)n * H, *b3 = W3 + (size_t)n * H;
        for (int r = 0; r < B2O_RT; ++r) a1[r] = a3[r] = 0.0f;
        for (int k = 0; k < H; ++k) {
          const float *p = xT + (size_t)k * B2O_RT;
          const float c1 = b1[k], c3 = b3[k];
          for (int r = 0; r < B2O_RT; ++r) {
            a1[r] = fmaf(p[r], c1, a1[r]);
            a3[r] = fmaf(p[r], c3, a3[r]);
          }
        }
        for (int r = 0; r < B2O_RT; ++r) {
          float v = silu_ref(a1[r]) * a3[r];
          iT[(size_t)n * B2O_RT + r] = v;
          if (inter && r < rows) inter[(size_t)(s0 + r) * I + n] = v;
        }
      }
      for (int h = 0; h < H; ++h) {
        const float *b2 = W2 + (size_t)h * I;
        for (int r = 0; r < B2O_RT; ++r) a1[r] = 0.0f;
        for (int n = 0; n < I; ++n) {
          const float *p = iT + (size_t)n * B2O_RT;
          const float c = b2[n];
          for (int r = 0; r < B2O_RT; ++r) a1[r] = fmaf(p[r], c, a1[r]);
        }
        for (int r = 0; r < rows; ++r) out[(size_t)(s0 + r) * H + h] = a1[r];
      }
    }
    free(xT);
    free(iT);
  }
  free(item_e);
  free(item_r);
}

/* ------------------------------------------------------------------------ */
/* moe_gather_deterministic_kernel (src/layer.cu:695-721):                   */
/*  y[t,h] = sum over k in order of (out[slot(t,k),h] * w[t,k]) via FFMA.    */
/* Slots of -1 (dropped) contribute nothing (the reference would read an     */
/* unwritten position there).                                                */
/* ------------------------------------------------------------------------ */
void b2o_combine(const float *out, const int32_t *token_slot, const float *w,
                 int T, int K, int H, float *y) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t)
    for (int h = 0; h < H; ++h) {
      float sum = 0.0f;
      for (int k = 0; k < K; ++k) {
        int s = token_slot[(size_t)t * K + k];
        if (s < 0) continue;
        sum = fmaf(out[(size_t)s * H + h], w[(size_t)t * K + k], sum);
      }
      y[(size_t)t * H + h] = sum;
    }
}

/* ------------------------------------------------------------------------ */
/* Whole layer, SparseMoeBlock::forward_gpu order (src/layer.cu:1428-1498).  */
/* Caller-provided outputs (any may be NULL except y): logits[T,E],           */
/* idx[T,K], w[T,K], counts[E], offsets[E], token_slot[T,K].                 */
/* ------------------------------------------------------------------------ */
int b2o_moe_forward(const float *x, const float *gate, const float *bias,
                    const float *const *w1, const float *const *w3,
                    const float *const *w2, int T, int H, int E, int K, int I,
                    float routed_scale, float *y, float *logits_out,
                    int32_t *idx_out, float *w_out, int32_t *counts_out,
                    int32_t *offsets_out, int32_t *token_slot_out) {
  if (K > B2O_MAXK || K <= 0 || E <= 0 || T < 0) return -1;
  size_t TK = (size_t)T * K;
  float *logits = logits_out ? logits_out
                             : (float *)malloc(sizeof(float) * (size_t)T * E + 4);
  int32_t *idx = idx_out ? idx_out : (int32_t *)malloc(sizeof(int32_t) * TK + 4);
  float *w = w_out ? w_out : (float *)malloc(sizeof(float) * TK + 4);
  int32_t *counts = counts_out ? counts_out
                               : (int32_t *)malloc(sizeof(int32_t) * E);
  int32_t *offsets = offsets_out ? offsets_out
                                 : (int32_t *)malloc(sizeof(int32_t) * E);
  int32_t *tiles = (int32_t *)malloc(sizeof(int32_t) * (E + 1));
  int32_t *slot = token_slot_out ? token_slot_out
                                 : (int32_t *)malloc(sizeof(int32_t) * TK + 4);
  int32_t *stok = (int32_t *)malloc(sizeof(int32_t) * TK + 4);
  float *sout = (float *)malloc(sizeof(float) * TK * (size_t)H + 4);

  b2o_router_logits(x, gate, logits, T, E, H);
  memset(counts, 0, sizeof(int32_t) * E);
  b2o_route_topk(logits, bias, T, E, K, routed_scale, idx, w, counts);
  b2o_scan(counts, E, 64, offsets, tiles);
  b2o_scatter_canonical(idx, w, T, K, E, offsets, stok, NULL, slot);
  b2o_expert_ffn(x, stok, offsets, counts, E, H, I, w1, w3, w2, NULL, sout);
  b2o_combine(sout, slot, w, T, K, H, y);

  if (!logits_out) free(logits);
  if (!idx_out) free(idx);
  if (!w_out) free(w);
  if (!counts_out) free(counts);
  if (!offsets_out) free(offsets);
  if (!token_slot_out) free(slot);
  free(tiles);
  free(stok);
  free(sout);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Seeded synthetic inputs shared by tests and fixtures: splitmix64 + Box-   */
/* Muller, so C, Python and the GPU box agree without depending on a library */
/* RNG.  Element i of stream `stream` depends only on (seed, stream, i).     */
/* ------------------------------------------------------------------------ */
static uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

void b2o_randn(float *out, size_t n, uint64_t seed, uint64_t stream,
               float stddev) {
  uint64_t base = splitmix64(seed ^ splitmix64(stream + 0x632BE59BD9B4E019ull));
#pragma omp parallel for schedule(static)
  for (long long p = 0; p < (long long)((n + 1) / 2); ++p) {
    uint64_t a = splitmix64(base + 2 * (uint64_t)p);
    uint64_t b = splitmix64(base + 2 * (uint64_t)p + 1);
    /* 53-bit uniforms in (0,1] and [0,1) */
    double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
    double r = sqrt(-2.0 * log(u1));
    double th = 6.283185307179586476925286766559 * u2;
    size_t i0 = 2 * (size_t)p;
    out[i0] = (float)(r * cos(th)) * stddev;
    if (i0 + 1 < n) out[i0 + 1] = (float)(r * sin(th)) * stddev;
  }
}

/* uniform integers in [0, bound) (for token ids / injected routing draws) */
void b2o_randu(double *out, size_t n, uint64_t seed, uint64_t stream) {
  uint64_t base = splitmix64(seed ^ splitmix64(stream + 0x2545F4914F6CDD1Dull));
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)n; ++i)
    out[i] = ((double)(splitmix64(base + (uint64_t)i) >> 11) + 0.5) *
             (1.0 / 9007199254740992.0);
}
