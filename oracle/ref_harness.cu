// ref_harness.cu -- TEST INFRASTRUCTURE ONLY.
//
// Launches the reference engine's own CUDA kernels, compiled unmodified from
// the reference's src/layer.cu and src/model.cu (see oracle/Makefile), in
// exactly the sequence SparseMoeBlock::forward_gpu uses (src/layer.cu:1428-1498),
// so that the CPU oracle (oracle/moe_oracle.c) and the golden fixtures under
// tests/golden/ are pinned to what the reference itself computes on a B200.
//
// The reference's SparseMoeBlock class cannot be constructed here: its
// constructor loads weights through ModelLoader (src/model_loader.cpp does not
// compile), so this harness owns the buffers that init_gpu() would allocate
// (src/layer.cu:1357-1426) and launches the kernels with the same grids.
// The output of the library built from this file lives only in oracle/_ref/.
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <vector>

#include "layer.h"  // RotaryEmbedding (reference header)

// Kernels defined in the reference's src/layer.cu (signatures as declared there).
__global__ void attn_matmul_tiled_kernel(float *out, const float *A,
                                         const float *B, int M, int N, int K);
__global__ void moe_router_topk_kernel(int *__restrict__ expert_counts,
                                       int *__restrict__ topk_indices_out,
                                       float *__restrict__ topk_weights_out,
                                       const float *__restrict__ logits,
                                       const float *__restrict__ bias,
                                       int num_experts, int k_experts,
                                       int num_tokens, float routed_scale,
                                       bool use_bias);
__global__ void moe_scan_kernel(int *offsets, int *write_pos, int *tile_offsets,
                                int *task_counters, const int *counts,
                                int num_experts, int tile_size);
__global__ void moe_scatter_kernel(
    float *__restrict__ sorted_x, int *__restrict__ sorted_idx_map,
    float *__restrict__ sorted_weights, int *__restrict__ expert_offsets,
    int *__restrict__ token_expert_pos, const float *__restrict__ x,
    const int *__restrict__ topk_indices, const float *__restrict__ topk_weights,
    int hidden_size, int k_experts, int num_tokens);
__global__ void moe_persistent_fused_w1w3_kernel(
    float *__restrict__ inter_out, const float *__restrict__ x,
    float **__restrict__ w1_ptrs, float **__restrict__ w3_ptrs,
    const int *__restrict__ tile_offsets, const int *__restrict__ offsets,
    const int *__restrict__ counts, int *__restrict__ task_counter,
    int hidden_size, int inter_size, int num_experts);
__global__ void moe_persistent_w2_kernel(
    float *__restrict__ final_out, const float *__restrict__ inter_in,
    float **__restrict__ w2_ptrs, const int *__restrict__ tile_offsets,
    const int *__restrict__ offsets, const int *__restrict__ counts,
    int *__restrict__ task_counter, int hidden_size, int inter_size,
    int num_experts);
__global__ void moe_gather_deterministic_kernel(
    float *__restrict__ output, const float *__restrict__ sorted_out,
    const int *__restrict__ token_expert_pos,
    const float *__restrict__ topk_weights, int num_tokens, int hidden_size,
    int k_experts);
__global__ void rms_norm_kernel(float *out, const float *in, const float *weight,
                                int total_rows, int hidden_dim);
__global__ void rope_transpose_kernel(float *out, const float *in, const float *cos,
                                      const float *sin, int batch, int seq_len,
                                      int num_heads, int head_dim);
__global__ void transpose_v_kernel(float *out, const float *in, int batch,
                                   int seq_len, int num_heads, int head_dim);
__global__ void fused_attn_gqa_kernel(float *__restrict__ output,
                                      const float *__restrict__ Q,
                                      const float *__restrict__ K,
                                      const float *__restrict__ V, int seq_len,
                                      int head_dim, int num_heads,
                                      int num_kv_heads, float scale);
__global__ void conv_transpose_split_kernel(float *Bx, float *C, const float *in_proj,
                                            int batch, int seq_len, int hidden_size);
__global__ void causal_conv1d_kernel(float *out, const float *input, const float *weight,
                                     int batch, int hidden_size, int seq_len,
                                     int kernel_size);
__global__ void conv_gating_transpose_kernel(float *out, const float *C,
                                             const float *conv_out, int batch,
                                             int hidden_size, int seq_len);
__global__ void add_kernel(float *out, const float *a, const float *b, int n);
__global__ void moe_swiglu_kernel(float *interm, const float *w1_out,
                                  const float *w3_out, int size);
// Defined in the reference's src/model.cu.
__global__ void lm_head_gemm_kernel(float *__restrict__ C,
                                    const float *__restrict__ A,
                                    const float *__restrict__ B, int M, int N,
                                    int K);
__global__ void embedding_lookup_kernel(float *hidden_states, const int *input_ids,
                                        const float *embed_table, int seq_len,
                                        int hidden_size);

#define RH_CHECK(call)                                                        \
  do {                                                                        \
    cudaError_t e_ = (call);                                                  \
    if (e_ != cudaSuccess) {                                                  \
      fprintf(stderr, "ref_harness %s:%d %s\n", __FILE__, __LINE__,           \
              cudaGetErrorString(e_));                                        \
      return (int)e_;                                                         \
    }                                                                         \
  } while (0)

extern "C" {

// C = A[M,K] . B[N,K]^T with the reference's 128x128 tiled kernel, launched as
// its call sites do (e.g. src/layer.cu:1250-1256).
int ref_gemm_nt(float *C, const float *A, const float *B, int M, int N, int K,
                cudaStream_t stream) {
  dim3 block(16, 16);
  dim3 grid((N + 127) / 128, (M + 127) / 128);
  attn_matmul_tiled_kernel<<<grid, block, 0, stream>>>(C, A, B, M, N, K);
  RH_CHECK(cudaGetLastError());
  return 0;
}

// LM-head GEMM as launched at src/model.cu:540-547.
int ref_lm_head(float *C, const float *A, const float *B, int M, int N, int K,
                cudaStream_t stream) {
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  dim3 block(32, 8);
  lm_head_gemm_kernel<<<grid, block, 0, stream>>>(C, A, B, M, N, K);
  RH_CHECK(cudaGetLastError());
  return 0;
}

struct RefMoe {
  int E, K, H, I, max_tokens, persistent_blocks;
  float **w1_tab, **w2_tab, **w3_tab;
  const float *gate, *bias;
  int *counts, *offsets, *sorted_idx, *topk_idx, *tok_pos, *tile_off, *task,
      *write_pos;
  float *sorted_w, *sorted_x, *sorted_inter, *sorted_out, *topk_w;
};

// Mirrors SparseMoeBlock::init_gpu (src/layer.cu:1357-1426): device weight
// pointer tables and scratch sized for max_tokens.  w1/w2/w3 are host arrays
// of E device pointers (w1,w3: [I,H]; w2: [H,I]).  persistent_blocks is the
// persistent-kernel grid (the reference ships 72*4 = 288, src/layer.cu:1474-1475).
int ref_moe_create(const float *const *w1, const float *const *w2,
                   const float *const *w3, const float *gate,
                   const float *bias, int E, int K, int H, int I,
                   int max_tokens, int persistent_blocks, void **out) {
  if (E != 32 || K != 4) return -1;  // kernels hard-wire 32 experts / 4 slots
  RefMoe *m = new RefMoe();
  m->E = E; m->K = K; m->H = H; m->I = I; m->max_tokens = max_tokens;
  m->persistent_blocks = persistent_blocks > 0 ? persistent_blocks : 288;
  m->gate = gate; m->bias = bias;
  RH_CHECK(cudaMalloc(&m->w1_tab, E * sizeof(float *)));
  RH_CHECK(cudaMalloc(&m->w2_tab, E * sizeof(float *)));
  RH_CHECK(cudaMalloc(&m->w3_tab, E * sizeof(float *)));
  RH_CHECK(cudaMemcpy(m->w1_tab, w1, E * sizeof(float *), cudaMemcpyHostToDevice));
  RH_CHECK(cudaMemcpy(m->w2_tab, w2, E * sizeof(float *), cudaMemcpyHostToDevice));
  RH_CHECK(cudaMemcpy(m->w3_tab, w3, E * sizeof(float *), cudaMemcpyHostToDevice));
  size_t ex = (size_t)max_tokens * K;
  size_t xs = ex * H;
  if ((size_t)max_tokens * E > xs) xs = (size_t)max_tokens * E;
  RH_CHECK(cudaMalloc(&m->counts, E * sizeof(int)));
  RH_CHECK(cudaMalloc(&m->offsets, E * sizeof(int)));
  RH_CHECK(cudaMalloc(&m->sorted_idx, ex * sizeof(int)));
  RH_CHECK(cudaMalloc(&m->sorted_w, ex * sizeof(float)));
  RH_CHECK(cudaMalloc(&m->sorted_x, xs * sizeof(float)));
  RH_CHECK(cudaMalloc(&m->sorted_inter, ex * I * 2 * sizeof(float)));
  RH_CHECK(cudaMalloc(&m->sorted_out, ex * H * sizeof(float)));
  RH_CHECK(cudaMalloc(&m->topk_idx, ex * sizeof(int)));
  RH_CHECK(cudaMalloc(&m->topk_w, ex * sizeof(float)));
  RH_CHECK(cudaMalloc(&m->tok_pos, ex * sizeof(int)));
  RH_CHECK(cudaMalloc(&m->tile_off, (E + 1) * sizeof(int)));
  RH_CHECK(cudaMalloc(&m->task, 2 * sizeof(int)));
  RH_CHECK(cudaMemset(m->task, 0, 2 * sizeof(int)));
  RH_CHECK(cudaMalloc(&m->write_pos, E * sizeof(int)));
  *out = m;
  return 0;
}

int ref_moe_destroy(void *h) {
  RefMoe *m = (RefMoe *)h;
  if (!m) return 0;
  void *ptrs[] = {m->w1_tab, m->w2_tab, m->w3_tab, m->counts, m->offsets,
                  m->sorted_idx, m->sorted_w, m->sorted_x, m->sorted_inter,
                  m->sorted_out, m->topk_idx, m->topk_w, m->tok_pos,
                  m->tile_off, m->task, m->write_pos};
  for (void *p : ptrs) cudaFree(p);
  delete m;
  return 0;
}

// SparseMoeBlock::forward_gpu (src/layer.cu:1428-1498), launch for launch.
// Optional outputs (device pointers, may be null) are copied out of the
// reference's scratch after the step that produced them: logits [T,E] right
// after the top-k kernel (they alias sorted_x, which scatter then overwrites),
// then idx/w [T,K], counts/offsets [E], token_expert_pos [T,K] and the
// slot->token map [T*K].
int ref_moe_forward(void *h, const float *x, float *y, int num_tokens,
                    float *logits_out, int *idx_out, float *w_out,
                    int *counts_out, int *offsets_out, int *tok_pos_out,
                    int *sorted_idx_out, cudaStream_t stream) {
  RefMoe *m = (RefMoe *)h;
  if (num_tokens > m->max_tokens) return -2;
  const int E = m->E, K = m->K, H = m->H, I = m->I;
  RH_CHECK(cudaMemsetAsync(y, 0, (size_t)num_tokens * H * sizeof(float), stream));
  RH_CHECK(cudaMemsetAsync(m->counts, 0, E * sizeof(int), stream));
  float *router_logits = m->sorted_x;
  {
    dim3 grid((E + 127) / 128, (num_tokens + 127) / 128);
    dim3 block(16, 16);
    attn_matmul_tiled_kernel<<<grid, block, 0, stream>>>(router_logits, x,
                                                         m->gate, num_tokens,
                                                         E, H);
  }
  int threads = 256;
  int blocks = (num_tokens + threads - 1) / threads;
  moe_router_topk_kernel<<<blocks, threads, 0, stream>>>(
      m->counts, m->topk_idx, m->topk_w, router_logits, m->bias, E, K,
      num_tokens, 1.0f, m->bias != nullptr);
  if (logits_out)
    RH_CHECK(cudaMemcpyAsync(logits_out, router_logits,
                             (size_t)num_tokens * E * sizeof(float),
                             cudaMemcpyDeviceToDevice, stream));
  moe_scan_kernel<<<1, 32, 0, stream>>>(m->offsets, m->write_pos, m->tile_off,
                                        m->task, m->counts, E, 64);
  moe_scatter_kernel<<<num_tokens, 256, 0, stream>>>(
      m->sorted_x, m->sorted_idx, m->sorted_w, m->write_pos, m->tok_pos, x,
      m->topk_idx, m->topk_w, H, K, num_tokens);
  dim3 dimBlock(32, 8);
  moe_persistent_fused_w1w3_kernel<<<m->persistent_blocks, dimBlock, 0, stream>>>(
      m->sorted_inter, m->sorted_x, m->w1_tab, m->w3_tab, m->tile_off,
      m->offsets, m->counts, &m->task[0], H, I, E);
  moe_persistent_w2_kernel<<<m->persistent_blocks, dimBlock, 0, stream>>>(
      m->sorted_out, m->sorted_inter, m->w2_tab, m->tile_off, m->offsets,
      m->counts, &m->task[1], H, I, E);
  int out_size = num_tokens * H;
  moe_gather_deterministic_kernel<<<(out_size + 255) / 256, 256, 0, stream>>>(
      y, m->sorted_out, m->tok_pos, m->topk_w, num_tokens, H, K);
  RH_CHECK(cudaGetLastError());
  size_t tk = (size_t)num_tokens * K;
  if (idx_out) RH_CHECK(cudaMemcpyAsync(idx_out, m->topk_idx, tk * sizeof(int), cudaMemcpyDeviceToDevice, stream));
  if (w_out) RH_CHECK(cudaMemcpyAsync(w_out, m->topk_w, tk * sizeof(float), cudaMemcpyDeviceToDevice, stream));
  if (counts_out) RH_CHECK(cudaMemcpyAsync(counts_out, m->counts, E * sizeof(int), cudaMemcpyDeviceToDevice, stream));
  if (offsets_out) RH_CHECK(cudaMemcpyAsync(offsets_out, m->offsets, E * sizeof(int), cudaMemcpyDeviceToDevice, stream));
  if (tok_pos_out) RH_CHECK(cudaMemcpyAsync(tok_pos_out, m->tok_pos, tk * sizeof(int), cudaMemcpyDeviceToDevice, stream));
  if (sorted_idx_out) RH_CHECK(cudaMemcpyAsync(sorted_idx_out, m->sorted_idx, tk * sizeof(int), cudaMemcpyDeviceToDevice, stream));
  return 0;
}

// ------------------------------------------------------------------ glue
// RMSNorm::forward_gpu (src/layer.cu:1144-1148).
int ref_rmsnorm(float *y, const float *x, const float *w, int rows, int dim,
                cudaStream_t stream) {
  rms_norm_kernel<<<rows, 256, 0, stream>>>(y, x, w, rows, dim);
  RH_CHECK(cudaGetLastError());
  return 0;
}

// add_kernel as DecoderLayer::forward_gpu launches it (src/layer.cu:1905-1918).
int ref_add(float *out, const float *a, const float *b, int n, cudaStream_t stream) {
  add_kernel<<<(n + 255) / 256, 256, 0, stream>>>(out, a, b, n);
  RH_CHECK(cudaGetLastError());
  return 0;
}

// embedding_lookup_kernel as worker_stage launches it (src/model.cu:409-412).
int ref_embed(float *hidden, const int *ids, const float *table, int tokens,
              int hidden_size, cudaStream_t stream) {
  int n = tokens * hidden_size;
  embedding_lookup_kernel<<<(n + 255) / 256, 256, 0, stream>>>(hidden, ids, table,
                                                               tokens, hidden_size);
  RH_CHECK(cudaGetLastError());
  return 0;
}

// The reference's own RotaryEmbedding (constructed and initialised exactly as
// a pipeline stage does, src/model.cu:298-300); copies its first npos rows of
// the cos / sin tables ([npos][HEAD_DIM] fp32) to host buffers.
int ref_rope_tables(float *cos_out, float *sin_out, int npos) {
  RotaryEmbedding r;
  r.init_gpu();
  RH_CHECK(cudaMemcpy(cos_out, r.cos_gpu_, (size_t)npos * HEAD_DIM * sizeof(float),
                      cudaMemcpyDeviceToHost));
  RH_CHECK(cudaMemcpy(sin_out, r.sin_gpu_, (size_t)npos * HEAD_DIM * sizeof(float),
                      cudaMemcpyDeviceToHost));
  return 0;
}

// Attention::forward_gpu (src/layer.cu:1584-1659), launch for launch, on
// caller buffers: x [T,H]; wq [Hq*64,H], wk/wv [Hkv*64,H], wo [H,Hq*64];
// q_ln/k_ln [64]; cos/sin [>=S][64]; y [T,H].  The reference kernel serves
// exactly seq_len 16 (block (32,16), 16 logits per thread): other lengths are
// refused.  `core_out` (may be null) receives the attention output before the
// out projection, [T, Hq*64].
int ref_attention(const float *x, const float *wq, const float *wk, const float *wv,
                  const float *wo, const float *q_ln, const float *k_ln,
                  const float *cos, const float *sin, float *y, float *core_out,
                  int batch, int seq_len, int hidden, int num_heads, int num_kv_heads,
                  cudaStream_t stream) {
  if (seq_len != 16) return -3;
  const int hd = 64, T = batch * seq_len;
  const size_t qn = (size_t)T * num_heads * hd, kn = (size_t)T * num_kv_heads * hd;
  float *q, *k, *v, *qn_, *kn_, *qt, *kt, *vt, *ot;
  RH_CHECK(cudaMalloc(&q, qn * 4));
  RH_CHECK(cudaMalloc(&k, kn * 4));
  RH_CHECK(cudaMalloc(&v, kn * 4));
  RH_CHECK(cudaMalloc(&qn_, qn * 4));
  RH_CHECK(cudaMalloc(&kn_, kn * 4));
  RH_CHECK(cudaMalloc(&qt, qn * 4));
  RH_CHECK(cudaMalloc(&kt, kn * 4));
  RH_CHECK(cudaMalloc(&vt, kn * 4));
  RH_CHECK(cudaMalloc(&ot, qn * 4));
  dim3 block(16, 16);
  dim3 grid_q((num_heads * hd + 127) / 128, (T + 127) / 128);
  attn_matmul_tiled_kernel<<<grid_q, block, 0, stream>>>(q, x, wq, T, num_heads * hd, hidden);
  dim3 grid_k((num_kv_heads * hd + 127) / 128, (T + 127) / 128);
  attn_matmul_tiled_kernel<<<grid_k, block, 0, stream>>>(k, x, wk, T, num_kv_heads * hd, hidden);
  attn_matmul_tiled_kernel<<<grid_k, block, 0, stream>>>(v, x, wv, T, num_kv_heads * hd, hidden);
  rms_norm_kernel<<<T * num_heads, 256, 0, stream>>>(qn_, q, q_ln, T * num_heads, hd);
  rms_norm_kernel<<<T * num_kv_heads, 256, 0, stream>>>(kn_, k, k_ln, T * num_kv_heads, hd);
  int rq = batch * num_heads * seq_len * (hd / 2);
  rope_transpose_kernel<<<(rq + 255) / 256, 256, 0, stream>>>(qt, qn_, cos, sin, batch,
                                                              seq_len, num_heads, hd);
  int rk = batch * num_kv_heads * seq_len * (hd / 2);
  rope_transpose_kernel<<<(rk + 255) / 256, 256, 0, stream>>>(kt, kn_, cos, sin, batch,
                                                              seq_len, num_kv_heads, hd);
  int vtot = batch * num_kv_heads * seq_len * hd;
  transpose_v_kernel<<<(vtot + 255) / 256, 256, 0, stream>>>(vt, v, batch, seq_len,
                                                             num_kv_heads, hd);
  dim3 grid_attn(batch, num_heads);
  dim3 block_attn(32, 16);
  size_t smem = 2 * seq_len * hd * sizeof(float);
  fused_attn_gqa_kernel<<<grid_attn, block_attn, smem, stream>>>(
      ot, qt, kt, vt, seq_len, hd, num_heads, num_kv_heads, 1.0f / sqrtf((float)hd));
  dim3 grid_o((hidden + 127) / 128, (T + 127) / 128);
  attn_matmul_tiled_kernel<<<grid_o, block, 0, stream>>>(y, ot, wo, T, hidden, num_heads * hd);
  RH_CHECK(cudaGetLastError());
  if (core_out)
    RH_CHECK(cudaMemcpyAsync(core_out, ot, qn * 4, cudaMemcpyDeviceToDevice, stream));
  RH_CHECK(cudaStreamSynchronize(stream));
  float *bufs[] = {q, k, v, qn_, kn_, qt, kt, vt, ot};
  for (float *b : bufs) cudaFree(b);
  return 0;
}

// ShortConv::forward_gpu (src/layer.cu:1735-1777), launch for launch:
// x [T,H]; in_w [3H,H]; conv_w [H][3]; out_w [H,H]; y [T,H].  `core_out`
// (may be null) receives the gated conv output before the out projection.
int ref_shortconv(const float *x, const float *in_w, const float *conv_w,
                  const float *out_w, float *y, float *core_out, int batch,
                  int seq_len, int hidden, cudaStream_t stream) {
  const int T = batch * seq_len;
  float *ip, *bx, *c, *co, *yt;
  RH_CHECK(cudaMalloc(&ip, (size_t)T * 3 * hidden * 4));
  RH_CHECK(cudaMalloc(&bx, (size_t)T * hidden * 4));
  RH_CHECK(cudaMalloc(&c, (size_t)T * hidden * 4));
  RH_CHECK(cudaMalloc(&co, (size_t)T * hidden * 4));
  RH_CHECK(cudaMalloc(&yt, (size_t)T * hidden * 4));
  dim3 block(16, 16);
  dim3 grid_in((3 * hidden + 127) / 128, (T + 127) / 128);
  attn_matmul_tiled_kernel<<<grid_in, block, 0, stream>>>(ip, x, in_w, T, 3 * hidden, hidden);
  int tot = T * hidden;
  conv_transpose_split_kernel<<<(tot + 255) / 256, 256, 0, stream>>>(bx, c, ip, batch,
                                                                     seq_len, hidden);
  causal_conv1d_kernel<<<(tot + 255) / 256, 256, 0, stream>>>(co, bx, conv_w, batch, hidden,
                                                              seq_len, CONV_KERNEL);
  conv_gating_transpose_kernel<<<(tot + 255) / 256, 256, 0, stream>>>(yt, c, co, batch,
                                                                      hidden, seq_len);
  dim3 grid_out((hidden + 127) / 128, (T + 127) / 128);
  attn_matmul_tiled_kernel<<<grid_out, block, 0, stream>>>(y, yt, out_w, T, hidden, hidden);
  RH_CHECK(cudaGetLastError());
  if (core_out)
    RH_CHECK(cudaMemcpyAsync(core_out, yt, (size_t)tot * 4, cudaMemcpyDeviceToDevice, stream));
  RH_CHECK(cudaStreamSynchronize(stream));
  float *bufs[] = {ip, bx, c, co, yt};
  for (float *b : bufs) cudaFree(b);
  return 0;
}

// MLP::forward_gpu (src/layer.cu:1233-1269) with the scratch
// DecoderLayer::init_gpu gives it (:1860-1866): gate/up [T, inter] each.
int ref_mlp(const float *x, const float *w1, const float *w2, const float *w3, float *y,
            int tokens, int hidden, int inter, cudaStream_t stream) {
  float *tmp;
  RH_CHECK(cudaMalloc(&tmp, (size_t)tokens * inter * 2 * sizeof(float)));
  float *gate = tmp, *up = tmp + (size_t)tokens * inter;
  dim3 block(16, 16);
  dim3 grid_gate((inter + 127) / 128, (tokens + 127) / 128);
  attn_matmul_tiled_kernel<<<grid_gate, block, 0, stream>>>(gate, x, w1, tokens, inter, hidden);
  attn_matmul_tiled_kernel<<<grid_gate, block, 0, stream>>>(up, x, w3, tokens, inter, hidden);
  int tot = tokens * inter;
  moe_swiglu_kernel<<<(tot + 255) / 256, 256, 0, stream>>>(gate, gate, up, tot);
  dim3 grid_down((hidden + 127) / 128, (tokens + 127) / 128);
  attn_matmul_tiled_kernel<<<grid_down, block, 0, stream>>>(y, gate, w2, tokens, hidden, inter);
  RH_CHECK(cudaGetLastError());
  RH_CHECK(cudaStreamSynchronize(stream));
  cudaFree(tmp);
  return 0;
}

}  // extern "C"
