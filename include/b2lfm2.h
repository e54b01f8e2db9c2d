/*
 * b2lfm2.h -- C ABI of the LFM2 decoder around the MoE / GEMM hot path:
 * the attention and short-convolution blocks, RMSNorm, the rotary tables,
 * the embedding, and the whole model forward (embedding, decoder layers,
 * final norm, last-token LM head) on one GPU.
 *
 * Conventions as in b2moe.h: plain pointers and sizes, stream-ordered calls,
 * b2_status returns, no process exit.  Activations are fp32 row-major
 * [tokens][hidden] with tokens = batch * seq_len, sequence-major (token
 * b * seq_len + s).  Projections run on the tcgen05 GEMM in bf16 with fp32
 * accumulation; norms, RoPE tables and the softmax state are fp32.
 */
#ifndef B2LFM2_H
#define B2LFM2_H

#include <stddef.h>
#include <stdint.h>

#include "b2moe.h"
#include "b2moe_ep.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- norms */

/* Replaces RMSNorm::forward_gpu (include/layer.h:16-17, src/layer.cu:1144-1148):
 * y[r] = x[r] * w / sqrt(mean(x[r]^2) + eps) for `rows` rows of `dim`,
 * summed in the reference kernel's order (bit-identical results for the
 * reference's eps 1e-5).  x, w, y: fp32 device pointers. */
b2_status b2_rmsnorm(const float *x, const float *w, float *y, int rows, int dim,
                     float eps, b2_stream stream);

/* Replaces DecoderLayer's residual add_kernel followed by the next RMSNorm
 * (src/layer.cu:1872-1893, 1905-1911): resid += delta (in place), then
 * y = RMSNorm(resid) as b2_rmsnorm.  Either output may be NULL: y_f32 fp32,
 * y_bf16 bf16 (the A operand of the next projection). */
b2_status b2_add_rmsnorm(float *resid, const float *delta, const float *w, float *y_f32,
                         void *y_bf16, int rows, int dim, float eps, b2_stream stream);

/* Replaces RotaryEmbedding::init_gpu (include/layer.h:22-38,
 * src/layer.cu:1167-1190): host fp32 tables cos/sin [max_pos][head_dim],
 * theta_j = base^(-2j/head_dim), angle = pos * theta_j in fp32, cos/sin of
 * that float, duplicated in both halves.  Host pointers; no device work. */
b2_status b2_rope_tables(float *cos_out, float *sin_out, int max_pos, int head_dim,
                         float base);

/* Replaces embedding_lookup_kernel (src/model.cu:18-31):
 * hidden[t] = table[ids[t]] for t < tokens (table [vocab][hidden] fp32,
 * hidden % 4 == 0).  An id outside [0, vocab) writes a zero row and records
 * 0x203 in the device int *status (may be NULL). */
b2_status b2_embed(const int32_t *ids, const float *table, float *hidden, int tokens,
                   int hidden_size, int vocab, int *status, b2_stream stream);

/* ------------------------------------------------------------ attention */

typedef struct b2_attn_desc {
  int hidden;       /* H (multiple of 64) */
  int num_heads;    /* Hq (32 in the reference model) */
  int num_kv_heads; /* Hkv, divides Hq (8) */
  int head_dim;     /* 64 (the only size supported, as in the reference) */
  int max_tokens;   /* capacity of batch * seq_len per forward */
  float eps;        /* q/k RMSNorm epsilon (1e-5) */
} b2_attn_desc;

typedef struct b2_attn b2_attn;

/* Replaces Attention::Attention + init_gpu (include/layer.h:126-137,
 * src/layer.cu:1508-1582): wq [Hq*64][H], wk/wv [Hkv*64][H], wo [H][Hq*64],
 * q_ln/k_ln [64], fp32, host (weights_on_host != 0) or device pointers.
 * Packs q|k|v into one bf16 [(Hq+2Hkv)*64][H] weight.  Synchronises stream. */
b2_status b2_attn_create(const b2_attn_desc *desc, const float *wq, const float *wk,
                         const float *wv, const float *wo, const float *q_ln,
                         const float *k_ln, int weights_on_host, b2_stream stream,
                         b2_attn **out);

/* Replaces Attention::forward_gpu(x, cos, sin, output, batch, seq_len,
 * hidden, stream) (include/layer.h:135-136, src/layer.cu:1584-1659): y[T,H] =
 * out_proj(causal GQA attention of RoPE(norm(q)), RoPE(norm(k)), v) for T =
 * batch * seq_len tokens, any seq_len (the reference kernel is limited to
 * 16).  cos/sin: device tables [>= seq_len][64] (b2_rope_tables layout). */
b2_status b2_attn_forward(b2_attn *attn, const float *x, const float *cos, const float *sin,
                          float *y, int batch, int seq_len, b2_stream stream);

b2_status b2_attn_destroy(b2_attn *attn);

/* ----------------------------------------------------------- short conv */

typedef struct b2_conv_desc {
  int hidden;      /* H (multiple of 64) */
  int kernel;      /* causal conv width L (3, CONV_L_CACHE; the only one supported) */
  int max_tokens;
} b2_conv_desc;

typedef struct b2_conv b2_conv;

/* Replaces ShortConv::ShortConv + init_gpu (include/layer.h:161-176,
 * src/layer.cu:1680-1733): conv_w [H][1][L], in_w [3H][H] (rows B | C | gate),
 * out_w [H][H], fp32 host or device pointers.  Synchronises stream. */
b2_status b2_conv_create(const b2_conv_desc *desc, const float *conv_w, const float *in_w,
                         const float *out_w, int weights_on_host, b2_stream stream,
                         b2_conv **out);

/* Replaces ShortConv::forward_gpu(x, y, batch, seq_len, hidden, stream)
 * (include/layer.h:174-175, src/layer.cu:1735-1777): in projection,
 * y = C * causal_conv(B * gate) per channel and sequence, out projection. */
b2_status b2_conv_forward(b2_conv *conv, const float *x, float *y, int batch, int seq_len,
                          b2_stream stream);

b2_status b2_conv_destroy(b2_conv *conv);

/* ---------------------------------------------------------------- model */

/* Weight source for b2_lfm2_create: returns a pointer to the fp32 tensor
 * `name` (the reference's tensor names, e.g. "layers.3.conv.in_proj.weight",
 * "layers.2.feed_forward.experts.7.w1.weight", "embed_tokens.weight") holding
 * `numel` elements, or NULL if the model has no such tensor.  Pointers must
 * stay valid until b2_lfm2_create returns. */
typedef const float *(*b2_weight_fn)(void *ctx, const char *name, int64_t numel);

typedef struct b2_lfm2_desc {
  int vocab;            /* 65536 */
  int hidden;           /* 2048 */
  int num_layers;       /* 24 (at most 64) */
  int num_heads;        /* 32 */
  int num_kv_heads;     /* 8 */
  int dense_inter;      /* 7168 (layers below num_dense_layers) */
  int moe_inter;        /* 1792 */
  int num_experts;      /* 32 */
  int top_k;            /* 4 */
  int num_dense_layers; /* 2 */
  int max_batch;        /* sequences per forward */
  int max_seq;          /* positions per sequence */
  float eps;            /* RMSNorm epsilon, 1e-5 */
  float rope_theta;     /* 1e6 */
  float routed_scale;   /* 1.0 */
  int use_expert_bias;  /* 1 */
  int layer_types[64];  /* 0 = attention, 1 = short conv (include/config.h:31) */
  int dtype;            /* expert / MLP GEMM operands: B2_BF16 or B2_TF32 */
} b2_lfm2_desc;

typedef struct b2_lfm2 b2_lfm2;

/* Replaces LFM2Model::LFM2Model + init_gpu_pipeline (include/model.h:28-36,
 * src/model.cu:142-331) on ONE GPU (the current device): every layer's
 * weights fetched through `get` by the reference's names, the LM head tied to
 * the embedding when the model has no "lm_head.weight" (src/model.cu:
 * 172-179), rotary tables for max_seq positions.  Synchronises stream. */
b2_status b2_lfm2_create(const b2_lfm2_desc *desc, b2_weight_fn get, void *ctx,
                         int weights_on_host, b2_stream stream, b2_lfm2 **out);

/* The expert-parallel model over `world` GPUs, one process (rank) per GPU;
 * replaces the 24-stage pipeline of init_gpu_pipeline / worker_stage
 * (src/model.cu:235-562), which moves the whole residual stream between
 * GPUs at stage boundaries.  Here every rank runs the embedding, attention /
 * conv blocks, dense MLPs and LM head on its own batch, and each MoE layer is
 * a b2_ep layer (include/b2moe_ep.h) in `mode`: only expert rows cross NVLink.
 * In B2_EP_OWNER mode `get` is asked only for this rank's experts
 * [rank*E/world, (rank+1)*E/world).  All MoE layers share one NCCL
 * communicator made from unique_id (b2_ep_unique_id on rank 0, shared by the
 * caller).  Collective: create, every forward and destroy are called by all
 * ranks in the same order; a rank with no tokens calls b2_lfm2_forward with
 * batch 0 and still takes part in every layer's exchange.  Each forward
 * waits on the host once per MoE layer (the count all-gather of
 * b2_ep_forward); logits are bit-identical to b2_lfm2_create's model on the
 * same tokens. */
b2_status b2_lfm2_create_ep(const b2_lfm2_desc *desc, b2_weight_fn get, void *ctx,
                            int weights_on_host, int world, int rank, const void *unique_id,
                            int mode, b2_stream stream, b2_lfm2 **out);

/* Host-side bound (seconds) on every wait for peers of an expert-parallel
 * model (default 60); B2_OK and no effect on a single-GPU model. */
b2_status b2_lfm2_set_timeout(b2_lfm2 *model, double seconds);

/* Replaces LFM2Model::forward(sample_idx, batch, ids, seq_len, out) as the
 * pipeline computes it (src/model.cu:385-548): logits[batch][vocab] (fp32,
 * device) of the last position of each sequence, ids [batch][seq_len] int32
 * device.  Stream-ordered; no host synchronisation. */
b2_status b2_lfm2_forward(b2_lfm2 *model, const int32_t *ids, int batch, int seq_len,
                          float *logits, b2_stream stream);

/* Same as b2_lfm2_forward, also copying the residual stream after every
 * layer into hidden_out [num_layers][batch*seq_len][hidden] (device). */
b2_status b2_lfm2_forward_ex(b2_lfm2 *model, const int32_t *ids, int batch, int seq_len,
                             float *logits, float *hidden_out, b2_stream stream);

/* Synchronises stream; returns and clears the first device-side error any
 * kernel of the model recorded (0 = none). */
b2_status b2_lfm2_get_status(b2_lfm2 *model, b2_stream stream, int *device_status);

/* Bytes of device memory the model holds. */
size_t b2_lfm2_device_bytes(const b2_lfm2 *model);

b2_status b2_lfm2_destroy(b2_lfm2 *model);

#ifdef __cplusplus
}
#endif

#endif /* B2LFM2_H */
