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
// Defined in the reference's src/model.cu.
__global__ void lm_head_gemm_kernel(float *__restrict__ C,
                                    const float *__restrict__ A,
                                    const float *__restrict__ B, int M, int N,
                                    int K);

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

}  // extern "C"
