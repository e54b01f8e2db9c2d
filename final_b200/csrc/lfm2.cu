// lfm2.cu -- the LFM2 decoder around the MoE / GEMM hot path: attention and
// short-conv blocks, norms, embedding, and the one-GPU model runtime
// (include/b2lfm2.h).
//
// Every projection is one call of the dense tcgen05 GEMM (gemm_sm100*.cuh)
// with bf16 operands and fp32 output; the glue between them is the
// kernels of lfm2_kernels.cuh.  A decoder layer is
//   rmsnorm(resid) -> xb bf16
//   attention:  xb.Wqkv^T -> qk_norm_rope -> flash_attn -> resid += core.Wo^T
//   short conv: xb.Win^T  -> conv_glue                  -> resid += core.Wout^T
//   rmsnorm(resid) -> hn fp32 -> MoE (b2_moe) or MLP (b2_mlp), adding into resid
// with every launch programmatic-dependent on its predecessor.  The layers
// of a model share one workspace (the activations between the projections);
// each layer owns only its packed weights.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/b2lfm2.h"
#include "../../include/b2mlp.h"
#include "lfm2_kernels.cuh"
#include "moe_internal.h"

using namespace b2;

namespace b2 {

// Device allocations owned by one object.
struct Arena {
  std::vector<void *> ptrs;
  size_t bytes = 0;
  template <typename T>
  b2_status get(T **p, size_t count) {
    void *v = nullptr;
    const size_t n = std::max<size_t>(count * sizeof(T), 16);
    B2_CUDA(cudaMalloc(&v, n));
    ptrs.push_back(v);
    bytes += n;
    *p = reinterpret_cast<T *>(v);
    return B2_OK;
  }
  void release() {
    for (void *p : ptrs) cudaFree(p);
    ptrs.clear();
    bytes = 0;
  }
};

// A bf16 weight [N][K] (row-major, K contiguous) with TMA maps for every B
// box height the dense planner uses (128 for the CTA-pair kernel; 64 / 128 /
// 256 for the single-CTA kernel's tile widths).
struct DenseW {
  __nv_bfloat16 *w = nullptr;
  int N = 0, K = 0;
  CUtensorMap tm64, tm128, tm256;
};

// Staging of fp32 weights into bf16: host sources go through a device
// buffer chunk by chunk, device sources are converted in place.
struct Stager {
  float *buf = nullptr;
  size_t elems = 0;
  bool on_host = false;
  cudaStream_t s = nullptr;
  b2_status convert(const float *src, __nv_bfloat16 *dst, size_t n) {
    if (!src) return B2_ERR_INVALID;
    if (!on_host) {
      f32_to_bf16_kernel<<<(unsigned)std::min<size_t>((n / 8 + 255) / 256 + 1, 4096), 256, 0, s>>>(
          src, dst, n);
      B2_LAUNCHED();
      return B2_OK;
    }
    for (size_t o = 0; o < n; o += elems) {
      const size_t c = std::min(elems, n - o);
      B2_CUDA(cudaMemcpyAsync(buf, src + o, c * 4, cudaMemcpyHostToDevice, s));
      f32_to_bf16_kernel<<<(unsigned)std::min<size_t>((c / 8 + 255) / 256 + 1, 4096), 256, 0, s>>>(
          buf, dst + o, c);
      B2_LAUNCHED();
      B2_CUDA(cudaStreamSynchronize(s));  // the staging buffer is reused
    }
    return B2_OK;
  }
  // fp32 copy (small vectors, the embedding table)
  b2_status copy(const float *src, float *dst, size_t n) {
    if (!src) return B2_ERR_INVALID;
    B2_CUDA(cudaMemcpyAsync(dst, src, n * 4, on_host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice,
                            s));
    return B2_OK;
  }
};

static bool dense_maps(DenseW *d) {
  const uint64_t st = (uint64_t)d->K * 2;
  return make_tmap(&d->tm64, d->w, false, d->K, d->N, st, 64) &&
         make_tmap(&d->tm128, d->w, false, d->K, d->N, st, 128) &&
         make_tmap(&d->tm256, d->w, false, d->K, d->N, st, 256);
}

// W = rows of parts[0] | parts[1] | ... (each rows[i] x K fp32) as bf16.
static b2_status dense_make(Arena &a, Stager &sg, DenseW *d, int K, const float *const *parts,
                            const int *rows, int nparts) {
  d->K = K;
  d->N = 0;
  for (int i = 0; i < nparts; ++i) d->N += rows[i];
  B2_RETURN_IF(a.get(&d->w, (size_t)d->N * K));
  size_t r0 = 0;
  for (int i = 0; i < nparts; ++i) {
    B2_RETURN_IF(sg.convert(parts[i], d->w + r0 * K, (size_t)rows[i] * K));
    r0 += rows[i];
  }
  return dense_maps(d) ? B2_OK : B2_ERR_CUDA;
}

// C[M][N] (fp32 or bf16, row stride ldc) = A . W^T; ta is a bf16 map over
// A's rows with 128-row boxes and K inner elements.
template <typename TOut>
static b2_status dense_gemm(const CUtensorMap &ta, int M, const DenseW &W, TOut *C, long long ldc,
                            int *status, int sms, cudaStream_t s, bool accumulate = false) {
  if (M <= 0) return B2_OK;
  const int kblocks = (W.K * 2 + kBKBytes - 1) / kBKBytes;
  const DensePlan p = plan_dense(M, W.N, sms, false, kblocks, splitk_cluster_caps(false));
  const CUtensorMap &tb = p.b_box_rows == 64 ? W.tm64 : p.b_box_rows == 128 ? W.tm128 : W.tm256;
  GemmArgs g{};
  g.M = M;
  g.N = W.N;
  g.num_k_blocks = kblocks;
  g.out = C;
  g.ldo = ldc;
  g.status = status;
  g.accumulate = accumulate ? 1 : 0;
  return launch_dense<kEpiStore, false, TOut>(p, ta, tb, g, sms, s);
}

// Activations between the projections, shared by every layer of a model.
struct Work {
  int maxT = 0, H = 0, Hq = 0, Hkv = 0;
  __nv_bfloat16 *wide = nullptr;     // [maxT][max((Hq+2Hkv)*64, 3H)] bf16 projection output
  __nv_bfloat16 *q = nullptr;        // [maxT * Hq * 64]  ([B][Hq][S][64])
  __nv_bfloat16 *k = nullptr, *v = nullptr;  // [maxT * Hkv * 64]
  __nv_bfloat16 *xb = nullptr;       // [maxT][H] normed input (A of the first projection)
  __nv_bfloat16 *core = nullptr;     // [maxT][max(Hq*64, H)] A of the out projection
  CUtensorMap tm_xb, tm_core_attn, tm_core_conv;
};

static b2_status work_make(Arena &a, Work *w, int maxT, int H, int Hq, int Hkv) {
  w->maxT = maxT;
  w->H = H;
  w->Hq = Hq;
  w->Hkv = Hkv;
  const size_t T = (size_t)maxT;
  const size_t wide = std::max<size_t>((size_t)(Hq + 2 * Hkv) * 64, (size_t)3 * H);
  const size_t ccol = std::max<size_t>((size_t)Hq * 64, (size_t)H);
  B2_RETURN_IF(a.get(&w->wide, T * wide));
  B2_RETURN_IF(a.get(&w->q, T * std::max(Hq, 1) * 64));
  B2_RETURN_IF(a.get(&w->k, T * std::max(Hkv, 1) * 64));
  B2_RETURN_IF(a.get(&w->v, T * std::max(Hkv, 1) * 64));
  B2_RETURN_IF(a.get(&w->xb, T * H));
  B2_RETURN_IF(a.get(&w->core, T * ccol));
  B2_CUDA(cudaMemset(w->xb, 0, T * H * 2));
  B2_CUDA(cudaMemset(w->core, 0, T * ccol * 2));
  bool ok = make_tmap(&w->tm_xb, w->xb, false, H, T, (uint64_t)H * 2, kBM) &&
            make_tmap(&w->tm_core_conv, w->core, false, H, T, (uint64_t)H * 2, kBM);
  if (Hq > 0)
    ok = ok && make_tmap(&w->tm_core_attn, w->core, false, (uint64_t)Hq * 64, T,
                         (uint64_t)Hq * 128, kBM);
  return ok ? B2_OK : B2_ERR_CUDA;
}

struct AttnW {
  int H = 0, Hq = 0, Hkv = 0;
  float eps = 1e-5f;
  DenseW qkv, o;
  float *q_ln = nullptr, *k_ln = nullptr;
};

struct ConvW {
  int H = 0;
  DenseW in, out;
  float *cw = nullptr;  // [H][3]
};

static b2_status attn_make(Arena &a, Stager &sg, AttnW *w, int H, int Hq, int Hkv, float eps,
                           const float *wq, const float *wk, const float *wv, const float *wo,
                           const float *q_ln, const float *k_ln) {
  w->H = H;
  w->Hq = Hq;
  w->Hkv = Hkv;
  w->eps = eps;
  const float *parts[3] = {wq, wk, wv};
  const int rows[3] = {Hq * 64, Hkv * 64, Hkv * 64};
  B2_RETURN_IF(dense_make(a, sg, &w->qkv, H, parts, rows, 3));
  const int orow[1] = {H};
  B2_RETURN_IF(dense_make(a, sg, &w->o, Hq * 64, &wo, orow, 1));
  B2_RETURN_IF(a.get(&w->q_ln, 64));
  B2_RETURN_IF(a.get(&w->k_ln, 64));
  B2_RETURN_IF(sg.copy(q_ln, w->q_ln, 64));
  return sg.copy(k_ln, w->k_ln, 64);
}

static b2_status conv_make(Arena &a, Stager &sg, ConvW *w, int H, const float *conv_w,
                           const float *in_w, const float *out_w) {
  w->H = H;
  const int irow[1] = {3 * H}, orow[1] = {H};
  B2_RETURN_IF(dense_make(a, sg, &w->in, H, &in_w, irow, 1));
  B2_RETURN_IF(dense_make(a, sg, &w->out, H, &out_w, orow, 1));
  B2_RETURN_IF(a.get(&w->cw, (size_t)H * kConvL));
  return sg.copy(conv_w, w->cw, (size_t)H * kConvL);
}

// y[T][H] = attention block of w.xb (already normed, bf16); accumulate: y +=.
static b2_status attn_run(const AttnW &a, const Work &w, int B, int S, const float *cos,
                          const float *sin, float *y, int *status, int sms, cudaStream_t s,
                          bool accumulate = false) {
  const int T = B * S;
  const int W3 = a.qkv.N;
  B2_RETURN_IF(dense_gemm(w.tm_xb, T, a.qkv, w.wide, W3, status, sms, s));
  B2_RETURN_IF(launch_pdl(qk_norm_rope_kernel, dim3(T), dim3(256), 0, s,
                          (const __nv_bfloat16 *)w.wide,
                          (const float *)a.q_ln, (const float *)a.k_ln, cos, sin, S, a.Hq, a.Hkv,
                          a.eps, w.q, w.k, w.v));
  const float scale_log2 = (1.0f / sqrtf(64.0f)) * 1.4426950408889634f;
  B2_RETURN_IF(launch_pdl(flash_attn_kernel, dim3((S + kAttnB - 1) / kAttnB, a.Hq, B), dim3(128),
                          0, s, (const __nv_bfloat16 *)w.q, (const __nv_bfloat16 *)w.k,
                          (const __nv_bfloat16 *)w.v, S, a.Hq, a.Hkv, scale_log2, w.core));
  return dense_gemm(w.tm_core_attn, T, a.o, y, a.H, status, sms, s, accumulate);
}

// y[T][H] = short-conv block of w.xb; accumulate: y +=.
static b2_status conv_run(const ConvW &c, const Work &w, int B, int S, float *y, int *status,
                          int sms, cudaStream_t s, bool accumulate = false) {
  const int T = B * S, H = c.H;
  B2_RETURN_IF(dense_gemm(w.tm_xb, T, c.in, w.wide, 3LL * H, status, sms, s));
  B2_RETURN_IF(launch_pdl(conv_glue_kernel, dim3((H + 511) / 512, (S + kConvRun - 1) / kConvRun, B),
                          dim3(128), 0, s, (const __nv_bfloat16 *)w.wide, (const float *)c.cw, S,
                          H, w.core));
  return dense_gemm(w.tm_core_conv, T, c.out, y, H, status, sms, s, accumulate);
}

static b2_status to_bf16_async(const float *x, __nv_bfloat16 *out, size_t n, int sms,
                               cudaStream_t s) {
  const size_t blocks = std::min<size_t>((n / 8 + 255) / 256 + 1, (size_t)sms * 16);
  return launch_pdl(f32_to_bf16_kernel, dim3((unsigned)blocks), dim3(256), 0, s, x, out, n);
}

static b2_status norm_launch(float *resid, const float *delta, const float *w, int rows, int dim,
                             int step, int off, int write_resid, float eps, float *y32,
                             __nv_bfloat16 *y16, cudaStream_t s) {
  if (rows <= 0) return B2_OK;
  const dim3 b(256), g1(rows), g2((rows + 1) / 2);
  switch (dim % 256 == 0 ? dim / 256 : 0) {
    case 8:
      return launch_pdl(add_rmsnorm_kernel<8, 2>, g2, b, 0, s, resid, delta, w, rows, dim, step,
                        off, write_resid, eps, y32, y16);
    case 16:
      return launch_pdl(add_rmsnorm_kernel<16, 1>, g1, b, 0, s, resid, delta, w, rows, dim,
                        step, off, write_resid, eps, y32, y16);
    case 4:
      return launch_pdl(add_rmsnorm_kernel<4, 2>, g2, b, 0, s, resid, delta, w, rows, dim, step,
                        off, write_resid, eps, y32, y16);
    default:
      return launch_pdl(add_rmsnorm_kernel<0, 1>, g1, b, 0, s, resid, delta, w, rows, dim, step,
                        off, write_resid, eps, y32, y16);
  }
}

static b2_status device_ok(DevInfo *di) {
  if (!dev_info(di)) return B2_ERR_NO_DEVICE;
  if (di->cc_major != 10) return B2_ERR_NO_DEVICE;
  return B2_OK;
}

}  // namespace b2

// ================================================================ norms, rope, embed
extern "C" b2_status b2_rmsnorm(const float *x, const float *w, float *y, int rows, int dim,
                                float eps, b2_stream stream) {
  if (rows < 0 || dim <= 0 || (rows > 0 && (!x || !w || !y))) return B2_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return norm_launch(const_cast<float *>(x), nullptr, w, rows, dim, 1, 0, 0, eps, y, nullptr, s);
}

extern "C" b2_status b2_add_rmsnorm(float *resid, const float *delta, const float *w, float *y_f32,
                                    void *y_bf16, int rows, int dim, float eps, b2_stream stream) {
  if (rows < 0 || dim <= 0 || (rows > 0 && (!resid || !w))) return B2_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return norm_launch(resid, delta, w, rows, dim, 1, 0, delta ? 1 : 0, eps, y_f32,
                     reinterpret_cast<__nv_bfloat16 *>(y_bf16), s);
}

extern "C" b2_status b2_rope_tables(float *cos_out, float *sin_out, int max_pos, int head_dim,
                                    float base) {
  if (!cos_out || !sin_out || max_pos < 0 || head_dim <= 0 || head_dim % 2) return B2_ERR_INVALID;
  const int half = head_dim / 2;
  for (int i = 0; i < max_pos; ++i)
    for (int j = 0; j < half; ++j) {
      const float theta = powf(base, -2.0f * (float)j / (float)head_dim);
      const float angle = (float)i * theta;
      const float c = cosf(angle), sn = sinf(angle);
      cos_out[(size_t)i * head_dim + j] = cos_out[(size_t)i * head_dim + j + half] = c;
      sin_out[(size_t)i * head_dim + j] = sin_out[(size_t)i * head_dim + j + half] = sn;
    }
  return B2_OK;
}

extern "C" b2_status b2_embed(const int32_t *ids, const float *table, float *hidden, int tokens,
                              int hidden_size, int vocab, int *status, b2_stream stream) {
  if (tokens < 0 || hidden_size <= 0 || hidden_size % 4 || vocab <= 0 ||
      (tokens > 0 && (!ids || !table || !hidden)))
    return B2_ERR_INVALID;
  if (tokens == 0) return B2_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return launch_pdl(embed_kernel, dim3(tokens), dim3(256), 0, s, (const int *)ids, table,
                    hidden_size, vocab, hidden, status);
}

// ================================================================ attention object
struct b2_attn {
  int device = 0, sms = 0;
  b2_attn_desc d{};
  Arena mem;
  AttnW w;
  Work work;
  int *status = nullptr;
};

extern "C" b2_status b2_attn_destroy(b2_attn *a) {
  if (!a) return B2_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(a->device);
  a->mem.release();
  cudaSetDevice(prev);
  delete a;
  return B2_OK;
}

extern "C" b2_status b2_attn_create(const b2_attn_desc *desc, const float *wq, const float *wk,
                                    const float *wv, const float *wo, const float *q_ln,
                                    const float *k_ln, int weights_on_host, b2_stream stream,
                                    b2_attn **out) {
  if (!desc || !out || !wq || !wk || !wv || !wo || !q_ln || !k_ln) return B2_ERR_INVALID;
  *out = nullptr;
  const b2_attn_desc &d = *desc;
  if (d.hidden <= 0 || d.hidden % 64 || d.head_dim != 64 || d.num_heads <= 0 ||
      d.num_kv_heads <= 0 || d.num_heads % d.num_kv_heads || d.max_tokens < 1)
    return B2_ERR_INVALID;
  DevInfo di;
  B2_RETURN_IF(device_ok(&di));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  b2_attn *a = new b2_attn();
  a->d = d;
  a->sms = di.sms;
  cudaGetDevice(&a->device);
  Stager sg;
  sg.on_host = weights_on_host != 0;
  sg.s = s;
  sg.elems = (size_t)8 << 20;
  b2_status st = B2_OK;
  if (sg.on_host) st = a->mem.get(&sg.buf, sg.elems);
  if (st == B2_OK) st = a->mem.get(&a->status, 1);
  if (st == B2_OK && cudaMemsetAsync(a->status, 0, sizeof(int), s) != cudaSuccess) st = B2_ERR_CUDA;
  if (st == B2_OK)
    st = attn_make(a->mem, sg, &a->w, d.hidden, d.num_heads, d.num_kv_heads,
                   d.eps > 0 ? d.eps : 1e-5f, wq, wk, wv, wo, q_ln, k_ln);
  if (st == B2_OK) st = work_make(a->mem, &a->work, d.max_tokens, d.hidden, d.num_heads, d.num_kv_heads);
  if (st == B2_OK && cudaStreamSynchronize(s) != cudaSuccess) st = B2_ERR_CUDA;
  if (st != B2_OK) {
    b2_attn_destroy(a);
    return st;
  }
  *out = a;
  return B2_OK;
}

extern "C" b2_status b2_attn_forward(b2_attn *a, const float *x, const float *cos,
                                     const float *sin, float *y, int batch, int seq_len,
                                     b2_stream stream) {
  if (!a || batch < 0 || seq_len < 0) return B2_ERR_INVALID;
  const long long T = (long long)batch * seq_len;
  if (T == 0) return B2_OK;
  if (!x || !cos || !sin || !y) return B2_ERR_INVALID;
  if (T > a->d.max_tokens) return B2_ERR_CAPACITY;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  B2_RETURN_IF(to_bf16_async(x, a->work.xb, (size_t)T * a->d.hidden, a->sms, s));
  return attn_run(a->w, a->work, batch, seq_len, cos, sin, y, a->status, a->sms, s);
}

// ================================================================ short-conv object
struct b2_conv {
  int device = 0, sms = 0;
  b2_conv_desc d{};
  Arena mem;
  ConvW w;
  Work work;
  int *status = nullptr;
};

extern "C" b2_status b2_conv_destroy(b2_conv *c) {
  if (!c) return B2_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  c->mem.release();
  cudaSetDevice(prev);
  delete c;
  return B2_OK;
}

extern "C" b2_status b2_conv_create(const b2_conv_desc *desc, const float *conv_w,
                                    const float *in_w, const float *out_w, int weights_on_host,
                                    b2_stream stream, b2_conv **out) {
  if (!desc || !out || !conv_w || !in_w || !out_w) return B2_ERR_INVALID;
  *out = nullptr;
  const b2_conv_desc &d = *desc;
  if (d.hidden <= 0 || d.hidden % 64 || d.kernel != kConvL || d.max_tokens < 1)
    return B2_ERR_INVALID;
  DevInfo di;
  B2_RETURN_IF(device_ok(&di));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  b2_conv *c = new b2_conv();
  c->d = d;
  c->sms = di.sms;
  cudaGetDevice(&c->device);
  Stager sg;
  sg.on_host = weights_on_host != 0;
  sg.s = s;
  sg.elems = (size_t)8 << 20;
  b2_status st = B2_OK;
  if (sg.on_host) st = c->mem.get(&sg.buf, sg.elems);
  if (st == B2_OK) st = c->mem.get(&c->status, 1);
  if (st == B2_OK && cudaMemsetAsync(c->status, 0, sizeof(int), s) != cudaSuccess) st = B2_ERR_CUDA;
  if (st == B2_OK) st = conv_make(c->mem, sg, &c->w, d.hidden, conv_w, in_w, out_w);
  if (st == B2_OK) st = work_make(c->mem, &c->work, d.max_tokens, d.hidden, 0, 0);
  if (st == B2_OK && cudaStreamSynchronize(s) != cudaSuccess) st = B2_ERR_CUDA;
  if (st != B2_OK) {
    b2_conv_destroy(c);
    return st;
  }
  *out = c;
  return B2_OK;
}

extern "C" b2_status b2_conv_forward(b2_conv *c, const float *x, float *y, int batch, int seq_len,
                                     b2_stream stream) {
  if (!c || batch < 0 || seq_len < 0) return B2_ERR_INVALID;
  const long long T = (long long)batch * seq_len;
  if (T == 0) return B2_OK;
  if (!x || !y) return B2_ERR_INVALID;
  if (T > c->d.max_tokens) return B2_ERR_CAPACITY;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  B2_RETURN_IF(to_bf16_async(x, c->work.xb, (size_t)T * c->d.hidden, c->sms, s));
  return conv_run(c->w, c->work, batch, seq_len, y, c->status, c->sms, s);
}

// ================================================================ model
namespace {
struct Layer {
  bool attention = false;
  AttnW a;
  ConvW c;
  float *op_norm = nullptr, *ffn_norm = nullptr;
  b2_moe *moe = nullptr;
  b2_mlp *mlp = nullptr;
  b2_ep *ep = nullptr;  // expert-parallel MoE (models made by b2_lfm2_create_ep)
};

struct EpCfg {
  int world = 1, rank = 0, mode = 0;
  const void *unique_id = nullptr;
};
}  // namespace

struct b2_lfm2 {
  int device = 0, sms = 0;
  b2_lfm2_desc d{};
  Arena mem;
  Work work;
  std::vector<Layer> layers;
  float *embed = nullptr;       // [V][H] fp32
  DenseW lm_head;               // [V][H] bf16
  float *final_norm = nullptr;  // [H]
  float *cos = nullptr, *sin = nullptr;  // [max_seq][64]
  float *resid = nullptr, *hn = nullptr;  // [maxT][H] fp32: residual stream, FFN input
  __nv_bfloat16 *lastb = nullptr;  // [max_batch][H]
  CUtensorMap tm_lastb;
  int *status = nullptr;
  int world = 1, rank = 0;  // expert-parallel group (world 1: a single-GPU model)
  bool ep = false;
};

extern "C" b2_status b2_lfm2_destroy(b2_lfm2 *m) {
  if (!m) return B2_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(m->device);
  // expert-parallel layers are destroyed collectively, in the same order on every rank
  for (Layer &l : m->layers) {
    if (l.moe) b2_moe_destroy(l.moe);
    if (l.mlp) b2_mlp_destroy(l.mlp);
    if (l.ep) b2_ep_destroy(l.ep);
  }
  m->mem.release();
  cudaSetDevice(prev);
  delete m;
  return B2_OK;
}

namespace {
struct Fetch {
  b2_weight_fn get;
  void *ctx;
  std::string missing;
  const float *operator()(const std::string &name, int64_t numel) {
    const float *p = get(ctx, name.c_str(), numel);
    if (!p && missing.empty()) missing = name;
    return p;
  }
};
}  // namespace

static b2_status lfm2_create_impl(const b2_lfm2_desc *desc, b2_weight_fn get, void *ctx,
                                  int weights_on_host, b2_stream stream, const EpCfg *ep,
                                  b2_lfm2 **out) {
  if (!desc || !get || !out) return B2_ERR_INVALID;
  *out = nullptr;
  const b2_lfm2_desc &d = *desc;
  if (d.vocab <= 0 || d.hidden <= 0 || d.hidden % 64 || d.num_layers < 1 || d.num_layers > 64 ||
      d.num_heads <= 0 || d.num_kv_heads <= 0 || d.num_heads % d.num_kv_heads ||
      d.hidden % d.num_heads || d.hidden / d.num_heads != 64 || d.max_batch < 1 || d.max_seq < 1 ||
      d.num_dense_layers < 0 || (d.dtype != B2_BF16 && d.dtype != B2_TF32))
    return B2_ERR_INVALID;
  for (int i = 0; i < d.num_layers; ++i)
    if (d.layer_types[i] != 0 && d.layer_types[i] != 1) return B2_ERR_INVALID;
  DevInfo di;
  B2_RETURN_IF(device_ok(&di));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int H = d.hidden, V = d.vocab, Hq = d.num_heads, Hkv = d.num_kv_heads;
  const long long maxT = (long long)d.max_batch * d.max_seq;
  if (maxT > (1LL << 30)) return B2_ERR_INVALID;
  const float eps = d.eps > 0 ? d.eps : 1e-5f;

  b2_lfm2 *m = new b2_lfm2();
  m->d = d;
  m->sms = di.sms;
  if (ep) {
    m->ep = true;
    m->world = ep->world;
    m->rank = ep->rank;
  }
  cudaGetDevice(&m->device);
  Fetch f{get, ctx, {}};
  Stager sg;
  sg.on_host = weights_on_host != 0;
  sg.s = s;
  sg.elems = (size_t)16 << 20;
  b2_status st = B2_OK;
  auto fail = [&](b2_status e) {
    if (!f.missing.empty())
      fprintf(stderr, "[b2lfm2] weight source has no tensor \"%s\"\n", f.missing.c_str());
    cudaStreamSynchronize(s);
    b2_lfm2_destroy(m);
    return e;
  };
#define B2_TRY(x)                          \
  do {                                     \
    st = (x);                              \
    if (st != B2_OK) return fail(st);      \
  } while (0)
  if (sg.on_host) B2_TRY(m->mem.get(&sg.buf, sg.elems));
  B2_TRY(m->mem.get(&m->status, 1));
  B2_TRY(cudaMemsetAsync(m->status, 0, sizeof(int), s) == cudaSuccess ? B2_OK : B2_ERR_CUDA);
  B2_TRY(work_make(m->mem, &m->work, (int)maxT, H, Hq, Hkv));
  B2_TRY(m->mem.get(&m->resid, maxT * H));
  B2_TRY(m->mem.get(&m->hn, maxT * H));
  B2_TRY(m->mem.get(&m->lastb, (size_t)d.max_batch * H));
  B2_TRY(cudaMemsetAsync(m->lastb, 0, (size_t)d.max_batch * H * 2, s) == cudaSuccess ? B2_OK
                                                                                   : B2_ERR_CUDA);
  if (!make_tmap(&m->tm_lastb, m->lastb, false, H, d.max_batch, (uint64_t)H * 2, kBM))
    return fail(B2_ERR_CUDA);

  // rotary tables (host math of the reference, uploaded once)
  {
    std::vector<float> c((size_t)d.max_seq * 64), sn((size_t)d.max_seq * 64);
    b2_rope_tables(c.data(), sn.data(), d.max_seq, 64, d.rope_theta > 0 ? d.rope_theta : 1e6f);
    B2_TRY(m->mem.get(&m->cos, c.size()));
    B2_TRY(m->mem.get(&m->sin, sn.size()));
    B2_TRY(cudaMemcpy(m->cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess
               ? B2_OK : B2_ERR_CUDA);
    B2_TRY(cudaMemcpy(m->sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess
               ? B2_OK : B2_ERR_CUDA);
  }
  // embedding, final norm, LM head (tied when the model has no lm_head.weight)
  const float *emb = f("embed_tokens.weight", (int64_t)V * H);
  if (!emb) return fail(B2_ERR_INVALID);
  B2_TRY(m->mem.get(&m->embed, (size_t)V * H));
  B2_TRY(sg.copy(emb, m->embed, (size_t)V * H));
  const float *lm = get(ctx, "lm_head.weight", (int64_t)V * H);
  const int vrow[1] = {V};
  const float *lmsrc = lm ? lm : emb;
  B2_TRY(dense_make(m->mem, sg, &m->lm_head, H, &lmsrc, vrow, 1));
  const float *fn = f("embedding_norm.weight", H);
  if (!fn) return fail(B2_ERR_INVALID);
  B2_TRY(m->mem.get(&m->final_norm, H));
  B2_TRY(sg.copy(fn, m->final_norm, H));

  m->layers.resize(d.num_layers);
  for (int i = 0; i < d.num_layers; ++i) {
    Layer &L = m->layers[i];
    const std::string pre = "layers." + std::to_string(i) + ".";
    L.attention = d.layer_types[i] == 0;
    const float *opn = f(pre + "operator_norm.weight", H);
    const float *ffn = f(pre + "ffn_norm.weight", H);
    if (!opn || !ffn) return fail(B2_ERR_INVALID);
    B2_TRY(m->mem.get(&L.op_norm, H));
    B2_TRY(m->mem.get(&L.ffn_norm, H));
    B2_TRY(sg.copy(opn, L.op_norm, H));
    B2_TRY(sg.copy(ffn, L.ffn_norm, H));
    if (L.attention) {
      const std::string a = pre + "self_attn.";
      const float *wq = f(a + "q_proj.weight", (int64_t)Hq * 64 * H);
      const float *wk = f(a + "k_proj.weight", (int64_t)Hkv * 64 * H);
      const float *wv = f(a + "v_proj.weight", (int64_t)Hkv * 64 * H);
      const float *wo = f(a + "out_proj.weight", (int64_t)H * Hq * 64);
      const float *ql = f(a + "q_layernorm.weight", 64);
      const float *kl = f(a + "k_layernorm.weight", 64);
      if (!wq || !wk || !wv || !wo || !ql || !kl) return fail(B2_ERR_INVALID);
      B2_TRY(attn_make(m->mem, sg, &L.a, H, Hq, Hkv, eps, wq, wk, wv, wo, ql, kl));
    } else {
      const std::string c = pre + "conv.";
      const float *cw = f(c + "conv.weight", (int64_t)H * kConvL);
      const float *iw = f(c + "in_proj.weight", 3LL * H * H);
      const float *ow = f(c + "out_proj.weight", (int64_t)H * H);
      if (!cw || !iw || !ow) return fail(B2_ERR_INVALID);
      B2_TRY(conv_make(m->mem, sg, &L.c, H, cw, iw, ow));
    }
    const std::string ff = pre + "feed_forward.";
    if (i < d.num_dense_layers) {
      const int I = d.dense_inter;
      const float *w1 = f(ff + "w1.weight", (int64_t)I * H);
      const float *w2 = f(ff + "w2.weight", (int64_t)H * I);
      const float *w3 = f(ff + "w3.weight", (int64_t)I * H);
      if (!w1 || !w2 || !w3) return fail(B2_ERR_INVALID);
      b2_mlp_desc md{H, I, (int)maxT, d.dtype};
      B2_TRY(b2_mlp_create(&md, w1, w2, w3, weights_on_host, stream, &L.mlp));
    } else {
      const int E = d.num_experts, I = d.moe_inter;
      // an expert-parallel owner fetches only its experts [rank*E/world, ...)
      const bool owner = ep && ep->mode == B2_EP_OWNER;
      const int e0 = owner ? ep->rank * (E / ep->world) : 0;
      const int ne = owner ? E / ep->world : E;
      std::vector<const float *> w1(ne), w2(ne), w3(ne);
      for (int j = 0; j < ne; ++j) {
        const std::string x = ff + "experts." + std::to_string(e0 + j) + ".";
        w1[j] = f(x + "w1.weight", (int64_t)I * H);
        w2[j] = f(x + "w2.weight", (int64_t)H * I);
        w3[j] = f(x + "w3.weight", (int64_t)I * H);
        if (!w1[j] || !w2[j] || !w3[j]) return fail(B2_ERR_INVALID);
      }
      const float *gate = f(ff + "gate.weight", (int64_t)E * H);
      const float *bias = d.use_expert_bias ? f(ff + "expert_bias", E) : nullptr;
      if (!gate || (d.use_expert_bias && !bias)) return fail(B2_ERR_INVALID);
      b2_moe_desc md{H, I, E, d.top_k, (int)maxT, d.routed_scale, d.use_expert_bias ? 1 : 0,
                     d.dtype};
      if (ep) {
        // the first MoE layer creates the communicator, the others share it
        b2_ep *first = nullptr;
        for (int j = 0; j < i && !first; ++j) first = m->layers[j].ep;
        B2_TRY(ep_create_impl(&md, ep->world, ep->rank, ep->unique_id, first, ep->mode,
                              w1.data(), w2.data(), w3.data(), gate, bias, weights_on_host,
                              stream, &L.ep));
      } else {
        B2_TRY(b2_moe_create(&md, w1.data(), w2.data(), w3.data(), gate, bias, weights_on_host,
                             stream, &L.moe));
      }
    }
  }
  B2_TRY(cudaStreamSynchronize(s) == cudaSuccess ? B2_OK : B2_ERR_CUDA);
#undef B2_TRY
  *out = m;
  return B2_OK;
}

extern "C" b2_status b2_lfm2_create(const b2_lfm2_desc *desc, b2_weight_fn get, void *ctx,
                                    int weights_on_host, b2_stream stream, b2_lfm2 **out) {
  return lfm2_create_impl(desc, get, ctx, weights_on_host, stream, nullptr, out);
}

extern "C" b2_status b2_lfm2_create_ep(const b2_lfm2_desc *desc, b2_weight_fn get, void *ctx,
                                       int weights_on_host, int world, int rank,
                                       const void *unique_id, int mode, b2_stream stream,
                                       b2_lfm2 **out) {
  if (!unique_id || world < 1 || world > B2_EP_MAX_WORLD || rank < 0 || rank >= world ||
      (mode != B2_EP_OWNER && mode != B2_EP_BALANCED))
    return B2_ERR_INVALID;
  if (!desc || desc->num_dense_layers >= desc->num_layers) return B2_ERR_INVALID;
  if (mode == B2_EP_OWNER && desc->num_experts % world) return B2_ERR_INVALID;
  EpCfg ep;
  ep.world = world;
  ep.rank = rank;
  ep.mode = mode;
  ep.unique_id = unique_id;
  return lfm2_create_impl(desc, get, ctx, weights_on_host, stream, &ep, out);
}

extern "C" b2_status b2_lfm2_set_timeout(b2_lfm2 *m, double seconds) {
  if (!m || !(seconds > 0)) return B2_ERR_INVALID;
  for (Layer &L : m->layers)
    if (L.ep) B2_RETURN_IF(b2_ep_set_timeout(L.ep, seconds));
  return B2_OK;
}

static b2_status lfm2_forward_impl(b2_lfm2 *m, const int32_t *ids, int B, int S, float *logits,
                                   float *hidden_out, cudaStream_t s) {
  const b2_lfm2_desc &d = m->d;
  const int H = d.hidden, T = B * S;
  const float eps = d.eps > 0 ? d.eps : 1e-5f;
  B2_RETURN_IF(launch_pdl(embed_kernel, dim3(T), dim3(256), 0, s, (const int *)ids,
                          (const float *)m->embed, H, d.vocab, m->resid, m->status));
  // Every block adds its output into the residual stream inside its last
  // kernel (the out projection's epilogue, the MoE combine, the MLP's down
  // projection): DecoderLayer's two add_kernel passes (src/layer.cu:1905-1918)
  // cost no separate read / write of the stream.
  for (int i = 0; i < d.num_layers; ++i) {
    Layer &L = m->layers[i];
    // xb = operator_norm(resid)
    B2_RETURN_IF(norm_launch(m->resid, nullptr, L.op_norm, T, H, 1, 0, 0, eps, nullptr,
                             m->work.xb, s));
    // resid += attention / short conv
    if (L.attention)
      B2_RETURN_IF(attn_run(L.a, m->work, B, S, m->cos, m->sin, m->resid, m->status, m->sms, s,
                            true));
    else
      B2_RETURN_IF(conv_run(L.c, m->work, B, S, m->resid, m->status, m->sms, s, true));
    // hn = ffn_norm(resid); resid += MoE / MLP
    B2_RETURN_IF(norm_launch(m->resid, nullptr, L.ffn_norm, T, H, 1, 0, 0, eps, m->hn, nullptr, s));
    if (L.moe)
      B2_RETURN_IF(moe_forward_impl(L.moe, m->hn, m->resid, T, nullptr, s, true));
    else if (L.ep)
      B2_RETURN_IF(ep_forward_impl(L.ep, m->hn, m->resid, T, s, true));
    else
      B2_RETURN_IF(mlp_forward_impl(L.mlp, m->hn, m->resid, T, s, true));
    if (hidden_out)
      B2_CUDA(cudaMemcpyAsync(hidden_out + (size_t)i * T * H, m->resid, (size_t)T * H * 4,
                              cudaMemcpyDeviceToDevice, s));
  }
  // final norm of each sequence's last token only
  B2_RETURN_IF(norm_launch(m->resid, nullptr, m->final_norm, B, H, S, S - 1, 0, eps, nullptr,
                           m->lastb, s));
  return dense_gemm(m->tm_lastb, B, m->lm_head, logits, d.vocab, m->status, m->sms, s);
}

extern "C" b2_status b2_lfm2_forward_ex(b2_lfm2 *m, const int32_t *ids, int batch, int seq_len,
                                        float *logits, float *hidden_out, b2_stream stream) {
  if (!m || batch < 0 || seq_len < 0) return B2_ERR_INVALID;
  if (batch > m->d.max_batch || seq_len > m->d.max_seq) return B2_ERR_CAPACITY;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (batch == 0 || seq_len == 0) {
    // an expert-parallel rank without tokens still takes part in every
    // layer's exchange, in layer order
    if (m->ep)
      for (Layer &L : m->layers)
        if (L.ep) B2_RETURN_IF(ep_forward_impl(L.ep, nullptr, nullptr, 0, s, true));
    return B2_OK;
  }
  if (!ids || !logits) return B2_ERR_INVALID;
  return lfm2_forward_impl(m, ids, batch, seq_len, logits, hidden_out, s);
}

extern "C" b2_status b2_lfm2_forward(b2_lfm2 *m, const int32_t *ids, int batch, int seq_len,
                                     float *logits, b2_stream stream) {
  return b2_lfm2_forward_ex(m, ids, batch, seq_len, logits, nullptr, stream);
}

extern "C" b2_status b2_lfm2_get_status(b2_lfm2 *m, b2_stream stream, int *device_status) {
  if (!m || !device_status) return B2_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  B2_CUDA(cudaStreamSynchronize(s));
  int v = 0;
  B2_CUDA(cudaMemcpy(&v, m->status, sizeof(int), cudaMemcpyDeviceToHost));
  B2_CUDA(cudaMemset(m->status, 0, sizeof(int)));
  for (Layer &L : m->layers) {
    int lv = 0;
    if (L.moe) b2_moe_get_status(L.moe, stream, &lv);
    if (L.mlp) b2_mlp_get_status(L.mlp, stream, &lv);
    if (L.ep) b2_moe_get_status(b2_ep_layer(L.ep), stream, &lv);
    if (!v) v = lv;
  }
  *device_status = v;
  return v ? B2_ERR_DEVICE : B2_OK;
}

extern "C" size_t b2_lfm2_device_bytes(const b2_lfm2 *m) {
  if (!m) return 0;
  size_t b = m->mem.bytes;
  for (const Layer &L : m->layers) {
    if (L.moe) b += b2_moe_device_bytes(L.moe);
    if (L.mlp) b += b2_mlp_device_bytes(L.mlp);
    if (L.ep) b += b2_moe_device_bytes(b2_ep_layer(L.ep));
  }
  return b;
}
