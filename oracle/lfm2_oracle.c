/*
 * lfm2_oracle.c -- CPU restatement of the reference engine's decoder-layer
 * glue around the matrix multiplications: RMSNorm, the rotary tables, the
 * attention core (per-head q/k norm, RoPE, causal GQA softmax-attention) and
 * the short-convolution gating.  TEST INFRASTRUCTURE ONLY: parity tests and
 * the golden-fixture generator use it as the checker; the product path never
 * links it.  Built into liboracle.so together with moe_oracle.c and compiled
 * with -ffp-contract=off, so every fused multiply-add below is an explicit
 * fmaf() standing for an FFMA that nvcc forms from the reference's
 * `acc += a * b` (its default -fmad=true), and nothing else is fused.
 *
 * Parity pin: tests/golden/ref_lfm2_*.npz hold the reference's own kernels'
 * outputs (built from its sources by oracle/Makefile, launched by
 * oracle/ref_harness.cu on a B200); tests/test_lfm2_oracle.py checks these
 * functions against them.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Sum of one warp's 32 values as __shfl_down_sync(…, 16..1) leaves it in
 * lane 0 (warpReduceSum, src/layer.cu:289-293; the loop in rms_norm_kernel,
 * src/layer.cu:163-164): v[i] += v[i + off] for off = 16, 8, 4, 2, 1.  Lanes
 * past the end read their own value back on hardware, but only lane 0's
 * result is used and it never reads past lane 31. */
static float warp_tree(const float *v_in) {
  float v[32];
  memcpy(v, v_in, sizeof(v));
  for (int off = 16; off > 0; off >>= 1)
    for (int i = 0; i + off < 32; ++i) v[i] = v[i] + v[i + off];
  return v[0];
}

/* rms_norm_kernel (src/layer.cu:144-191) with blockDim.x = 256, the launch of
 * RMSNorm::forward_gpu (:1144-1148): thread t accumulates x[i]^2 for
 * i = t, t+256, ... in order (FFMA); each warp reduces by the shuffle tree;
 * warp 0 then reduces the 8 warp sums with offsets 4, 2, 1;
 * r = 1 / sqrtf(sum / dim + 1e-5f); y = x * r * w. */
void b2o_rmsnorm(const float *x, const float *w, float *y, int rows, int dim) {
  for (int r = 0; r < rows; ++r) {
    const float *src = x + (size_t)r * dim;
    float *dst = y + (size_t)r * dim;
    float part[256];
    for (int t = 0; t < 256; ++t) {
      float s = 0.0f;
      for (int i = t; i < dim; i += 256) s = fmaf(src[i], src[i], s);
      part[t] = s;
    }
    float ws[8];
    for (int wi = 0; wi < 8; ++wi) ws[wi] = warp_tree(part + 32 * wi);
    for (int off = 4; off > 0; off >>= 1)
      for (int i = 0; i + off < 8; ++i) ws[i] = ws[i] + ws[i + off];
    const float rms = 1.0f / sqrtf(ws[0] / (float)dim + 1e-5f);
    for (int i = 0; i < dim; ++i) dst[i] = src[i] * rms * w[i];
  }
}

/* RotaryEmbedding::init_gpu (src/layer.cu:1167-1190): for position i and
 * j < head_dim/2, theta = powf(base, -2j/head_dim), angle = i * theta (fp32),
 * cos(angle) / sin(angle) of the float angle (the float overloads, cosf /
 * sinf, that C++ picks for a float argument), duplicated at j and
 * j + head_dim/2.  Tables are [npos][head_dim]. */
void b2o_rope_tables(float *cosv, float *sinv, int npos, int head_dim, float base) {
  const int half = head_dim / 2;
  for (int i = 0; i < npos; ++i)
    for (int j = 0; j < half; ++j) {
      const float theta = powf(base, -2.0f * (float)j / (float)head_dim);
      const float angle = (float)i * theta;
      const float c = cosf(angle), s = sinf(angle);
      cosv[(size_t)i * head_dim + j] = c;
      cosv[(size_t)i * head_dim + j + half] = c;
      sinv[(size_t)i * head_dim + j] = s;
      sinv[(size_t)i * head_dim + j + half] = s;
    }
}

/* rope_transpose_kernel (src/layer.cu:193-227) for one head vector:
 * out[d] = q1*c1 - q2*s1, out[d+half] = q2*c2 + q1*s2.  nvcc fuses each of
 * these into one FFMA with the other product rounded first. */
static void rope_one(const float *in, const float *c, const float *s, float *out, int hd) {
  const int half = hd / 2;
  for (int d = 0; d < half; ++d) {
    const float q1 = in[d], q2 = in[d + half];
    out[d] = fmaf(q1, c[d], -(q2 * s[d]));
    out[d + half] = fmaf(q2, c[d + half], q1 * s[d + half]);
  }
}

/* Attention::forward_gpu between the projections (src/layer.cu:1615-1655):
 *   q/k RMSNorm per head over head_dim (q_layernorm / k_layernorm),
 *   RoPE at the token's position s (rope_transpose_kernel),
 *   fused_attn_gqa_kernel (:296-393): score_j = (q . k_j) * scale with the
 *   dot product as lane partials q[l]*k[l] + q[l+32]*k[l+32] summed by the
 *   warp shuffle tree; j > i masked to -1e30; p_j = (float)exp((double)(
 *   score_j - max)) summed in double; out = sum_j (p_j * inv_sum) * v_j in j
 *   order (FFMA), inv_sum = (float)(1 / sum).
 * qkv: [B*S][(Hq + 2*Hkv)*hd] projections (q | k | v per token);
 * out: [B*S][Hq*hd].  The reference kernel is written for head_dim 64 (two
 * values per lane); so is this restatement (other sizes leave out untouched). */
void b2o_attention_core(const float *qkv, int B, int S, int Hq, int Hkv, int hd,
                        const float *q_ln, const float *k_ln, const float *cosv,
                        const float *sinv, float *out) {
  if (hd != 64) return; /* the reference kernel is written for head_dim 64 */
  const int W = (Hq + 2 * Hkv) * hd;
  const int G = Hq / Hkv;
  const float scale = 1.0f / sqrtf((float)hd);
  float *q = (float *)malloc(sizeof(float) * (size_t)B * S * Hq * hd);
  float *k = (float *)malloc(sizeof(float) * (size_t)B * S * Hkv * hd);
  float *tmp = (float *)malloc(sizeof(float) * hd);
  float *logit = (float *)malloc(sizeof(float) * S);
  /* norms + rope: q[b][h][s][:], k[b][h][s][:] */
  for (int b = 0; b < B; ++b)
    for (int s = 0; s < S; ++s) {
      const float *row = qkv + (size_t)(b * S + s) * W;
      for (int h = 0; h < Hq + Hkv; ++h) {
        const int isq = h < Hq;
        const float *src = row + (size_t)h * hd;
        b2o_rmsnorm(src, isq ? q_ln : k_ln, tmp, 1, hd);
        float *dst = isq ? q + (((size_t)b * Hq + h) * S + s) * hd
                         : k + (((size_t)b * Hkv + (h - Hq)) * S + s) * hd;
        rope_one(tmp, cosv + (size_t)s * hd, sinv + (size_t)s * hd, dst, hd);
      }
    }
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < Hq; ++h) {
      const int hk = h / G;
      const float *kh = k + ((size_t)b * Hkv + hk) * S * hd;
      for (int i = 0; i < S; ++i) {
        const float *qi = q + (((size_t)b * Hq + h) * S + i) * hd;
        float mx = -1e30f;
        for (int j = 0; j < S; ++j) {
          /* lane l holds q[l], q[l+32]: q0*k0 + q1*k1 -> fmaf(q0, k0, q1*k1) */
          const float *kj = kh + (size_t)j * hd;
          float part[32];
          for (int l = 0; l < 32; ++l) part[l] = fmaf(qi[l], kj[l], qi[l + 32] * kj[l + 32]);
          float sc = warp_tree(part) * scale;
          if (j > i) sc = -1e30f;
          logit[j] = sc;
          if (sc > mx) mx = sc;
        }
        double sum = 0.0;
        for (int j = 0; j < S; ++j) {
          const float v = (float)exp((double)(logit[j] - mx));
          logit[j] = v;
          sum += (double)v;
        }
        const float inv = (float)(1.0 / sum);
        const float *vbase = qkv + (size_t)(Hq + Hkv) * hd;
        float *o = out + (size_t)(b * S + i) * Hq * hd + (size_t)h * hd;
        for (int d = 0; d < hd; ++d) {
          float acc = 0.0f;
          for (int j = 0; j < S; ++j) {
            const float v = vbase[(size_t)(b * S + j) * W + (size_t)hk * hd + d];
            acc = fmaf(logit[j] * inv, v, acc);
          }
          o[d] = acc;
        }
      }
    }
  free(q);
  free(k);
  free(tmp);
  free(logit);
}

/* ShortConv::forward_gpu between the projections (src/layer.cu:1755-1771):
 * conv_transpose_split_kernel (:397-420) Bx = B * gate, causal_conv1d_kernel
 * (:422-445) sum over k of Bx[s - (L-1) + k] * w[h][k] for in-range positions
 * (FFMA chain from 0), conv_gating_transpose_kernel (:447-465) y = C * conv.
 * in_proj_out: [B*S][3H] = (B | C | gate) per token; conv_w: [H][L];
 * y: [B*S][H]. */
void b2o_shortconv_core(const float *in_proj_out, const float *conv_w, int B, int S,
                        int H, int L, float *y) {
  for (int b = 0; b < B; ++b)
    for (int s = 0; s < S; ++s)
      for (int h = 0; h < H; ++h) {
        float acc = 0.0f;
        for (int kk = 0; kk < L; ++kk) {
          const int pos = s - (L - 1) + kk;
          if (pos < 0) continue;
          const float *r = in_proj_out + (size_t)(b * S + pos) * 3 * H;
          const float bx = r[h] * r[2 * H + h];
          acc = fmaf(bx, conv_w[(size_t)h * L + kk], acc);
        }
        y[(size_t)(b * S + s) * H + h] = in_proj_out[(size_t)(b * S + s) * 3 * H + H + h] * acc;
      }
}
