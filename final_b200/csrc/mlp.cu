// mlp.cu -- dense SwiGLU MLP (layers without experts) on the tcgen05 GEMM core.
//
//   forward:  x fp32 --f32_to_bf16_kernel--> xc bf16 [T][H]       (bf16 mode)
//             xc . [W1||W3]^T, SwiGLU in the epilogue --> inter [T][Ip]
//             inter . W2^T --> y fp32 [T][H]
//
// Weights are packed once at create exactly as one MoE expert's: W1||W3
// interleaved per 128-row block (gate rows then up rows) into [2*Ip][H], W2
// into [H][Ip], with I padded to Ip = ceil(I/128)*128 by zero rows/columns
// (silu(0) * 0 = 0, so the padding adds nothing).  The GEMM kernel and tile
// width are chosen per forward from T (plan_dense); all three launches use
// programmatic dependent launch.  Replaces MLP::init_gpu / MLP::forward_gpu
// (include/layer.h:48-66, src/layer.cu:1217-1269).
#include "../../include/b2mlp.h"
#include "moe_internal.h"

using namespace b2;

struct b2_mlp {
  b2_mlp_desc d;
  int device = 0;
  int sms = 0;
  int Ip = 0;
  bool tf32 = false;
  size_t bytes = 0;
  void *w13 = nullptr;    // [2*Ip][H]
  void *w2 = nullptr;     // [H][Ip]
  void *xc = nullptr;     // [max_tokens][H] bf16 copy of x (bf16 mode)
  void *inter = nullptr;  // [max_tokens][Ip]
  int *status = nullptr;
  CUtensorMap tm_xc, tm_inter;
  CUtensorMap tm_w13_128, tm_w13_256;          // W1||W3 boxes of 128 (pair) / 256 rows
  CUtensorMap tm_w2_64, tm_w2_128, tm_w2_256;  // W2 boxes of 64 / 128 / 256 rows
  std::vector<void *> allocs;
};

static b2_status mlp_alloc(b2_mlp *m, void **p, size_t bytes) {
  B2_CUDA(cudaMalloc(p, bytes ? bytes : 16));
  m->allocs.push_back(*p);
  m->bytes += bytes;
  return B2_OK;
}

extern "C" b2_status b2_mlp_destroy(b2_mlp *m) {
  if (!m) return B2_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(m->device);
  for (void *p : m->allocs) cudaFree(p);
  cudaSetDevice(prev);
  delete m;
  return B2_OK;
}

extern "C" b2_status b2_mlp_create(const b2_mlp_desc *desc, const float *w1, const float *w2,
                                   const float *w3, int weights_on_host, b2_stream stream_,
                                   b2_mlp **out) {
  if (!desc || !out || !w1 || !w2 || !w3) return B2_ERR_INVALID;
  *out = nullptr;
  const b2_mlp_desc &d = *desc;
  if (d.hidden <= 0 || d.hidden % 8 != 0 || d.inter <= 0 || d.max_tokens < 1 ||
      (d.dtype != B2_BF16 && d.dtype != B2_TF32))
    return B2_ERR_INVALID;
  DevInfo di;
  if (!dev_info(&di)) return B2_ERR_NO_DEVICE;
  if (di.cc_major != 10) return B2_ERR_NO_DEVICE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream_);

  b2_mlp *m = new b2_mlp();
  m->d = d;
  cudaGetDevice(&m->device);
  m->sms = di.sms;
  m->tf32 = d.dtype == B2_TF32;
  const int H = d.hidden, I = d.inter;
  m->Ip = (I + 127) / 128 * 128;
  const int Ip = m->Ip;
  const size_t es = m->tf32 ? 4 : 2, T = (size_t)d.max_tokens;
  auto bail = [&](b2_status st) {
    b2_mlp_destroy(m);
    return st;
  };
  if (mlp_alloc(m, &m->w13, es * 2 * Ip * H) != B2_OK ||
      mlp_alloc(m, &m->w2, es * (size_t)H * Ip) != B2_OK ||
      (!m->tf32 && mlp_alloc(m, &m->xc, es * T * H) != B2_OK) ||
      mlp_alloc(m, &m->inter, es * T * Ip) != B2_OK ||
      mlp_alloc(m, (void **)&m->status, sizeof(int)) != B2_OK)
    return bail(B2_ERR_CUDA);
  if (cudaMemsetAsync(m->status, 0, sizeof(int), s) != cudaSuccess ||
      cudaMemsetAsync(m->inter, 0, es * T * Ip, s) != cudaSuccess ||
      (m->xc && cudaMemsetAsync(m->xc, 0, es * T * H, s) != cudaSuccess))
    return bail(B2_ERR_CUDA);

  // weights: host matrices are staged through temporary device buffers
  const size_t mat = (size_t)I * H;
  float *st[3] = {nullptr, nullptr, nullptr};
  const float *src[3] = {w1, w3, w2};
  auto fail = [&](b2_status e) {
    for (float *p : st)
      if (p) cudaFree(p);
    return bail(e);
  };
  if (weights_on_host) {
    for (int i = 0; i < 3; ++i) {
      if (cudaMalloc(&st[i], mat * 4) != cudaSuccess) return fail(B2_ERR_CUDA);
      if (cudaMemcpyAsync(st[i], src[i], mat * 4, cudaMemcpyHostToDevice, s) != cudaSuccess)
        return fail(B2_ERR_CUDA);
      src[i] = st[i];
    }
  }
  if (m->tf32) {
    pack_w13_single<float><<<2 * Ip, 256, 0, s>>>(src[0], src[1], H, I, Ip,
                                                  reinterpret_cast<float *>(m->w13));
    pack_w2_single<float><<<H, 256, 0, s>>>(src[2], H, I, Ip, reinterpret_cast<float *>(m->w2));
  } else {
    pack_w13_single<__nv_bfloat16><<<2 * Ip, 256, 0, s>>>(
        src[0], src[1], H, I, Ip, reinterpret_cast<__nv_bfloat16 *>(m->w13));
    pack_w2_single<__nv_bfloat16><<<H, 256, 0, s>>>(src[2], H, I, Ip,
                                                     reinterpret_cast<__nv_bfloat16 *>(m->w2));
  }
  if (cudaGetLastError() != cudaSuccess) return fail(B2_ERR_CUDA);
  launch_counter().fetch_add(2, std::memory_order_relaxed);
  if (cudaStreamSynchronize(s) != cudaSuccess) return fail(B2_ERR_CUDA);
  for (float *&p : st)
    if (p) {
      cudaFree(p);
      p = nullptr;
    }

  const bool f = m->tf32;
  if ((m->xc && !make_tmap(&m->tm_xc, m->xc, f, H, T, (uint64_t)H * es, kBM)) ||
      !make_tmap(&m->tm_inter, m->inter, f, Ip, T, (uint64_t)Ip * es, kBM) ||
      !make_tmap(&m->tm_w13_128, m->w13, f, H, 2 * (uint64_t)Ip, (uint64_t)H * es, 128) ||
      !make_tmap(&m->tm_w13_256, m->w13, f, H, 2 * (uint64_t)Ip, (uint64_t)H * es, 256) ||
      !make_tmap(&m->tm_w2_64, m->w2, f, Ip, H, (uint64_t)Ip * es, 64) ||
      !make_tmap(&m->tm_w2_128, m->w2, f, Ip, H, (uint64_t)Ip * es, 128) ||
      !make_tmap(&m->tm_w2_256, m->w2, f, Ip, H, (uint64_t)Ip * es, 256))
    return bail(B2_ERR_CUDA);
  *out = m;
  return B2_OK;
}

extern "C" b2_status b2_mlp_forward(b2_mlp *m, const float *x, float *y, int T,
                                    b2_stream stream_) {
  return mlp_forward_impl(m, x, y, T, reinterpret_cast<cudaStream_t>(stream_), false);
}

b2_status b2::mlp_forward_impl(b2_mlp *m, const float *x, float *y, int T, cudaStream_t s,
                               bool accumulate) {
  if (!m || T < 0 || (T > 0 && (!x || !y || !aligned16(x) || !aligned16(y))))
    return B2_ERR_INVALID;
  if (T > m->d.max_tokens) return B2_ERR_CAPACITY;
  if (T == 0) return B2_OK;
  const int H = m->d.hidden, Ip = m->Ip;
  const bool f = m->tf32;
  const size_t es = f ? 4 : 2;

  // A operand of W1||W3: the bf16 copy of x, or x itself read as TF32
  CUtensorMap tm_x_call;
  const CUtensorMap *ta = &m->tm_xc;
  if (f) {
    if (!make_tmap(&tm_x_call, x, true, H, T, (uint64_t)H * 4, kBM)) return B2_ERR_INVALID;
    ta = &tm_x_call;
  } else {
    const size_t n = (size_t)T * H;
    const size_t blocks = std::min<size_t>((n / 8 + 255) / 256 + 1, (size_t)m->sms * 16);
    B2_RETURN_IF(launch_pdl(f32_to_bf16_kernel, dim3((unsigned)blocks), dim3(256), 0, s, x,
                            reinterpret_cast<__nv_bfloat16 *>(m->xc), n));
  }

  GemmArgs g1{};
  g1.M = T;
  g1.N = Ip;
  g1.num_k_blocks = (int)(((size_t)H * es + kBKBytes - 1) / kBKBytes);
  g1.out = m->inter;
  g1.ldo = Ip;
  g1.status = m->status;
  const DensePlan p1 = plan_dense(T, Ip, m->sms, true, g1.num_k_blocks, splitk_cluster_caps(true));
  const CUtensorMap &tb1 = p1.b_box_rows == 128 ? m->tm_w13_128 : m->tm_w13_256;
  if (f)
    B2_RETURN_IF((launch_dense<kEpiSwiGLU, true, float>(p1, *ta, tb1, g1, m->sms, s)));
  else
    B2_RETURN_IF((launch_dense<kEpiSwiGLU, false, __nv_bfloat16>(p1, *ta, tb1, g1, m->sms, s)));

  GemmArgs g2{};
  g2.M = T;
  g2.N = H;
  g2.num_k_blocks = (int)((size_t)Ip * es / kBKBytes);
  g2.out = y;
  g2.ldo = H;
  g2.status = m->status;
  g2.accumulate = accumulate ? 1 : 0;
  const DensePlan p2 = plan_dense(T, H, m->sms, false, g2.num_k_blocks, splitk_cluster_caps(false));
  const CUtensorMap &tb2 = p2.b_box_rows == 64    ? m->tm_w2_64
                           : p2.b_box_rows == 128 ? m->tm_w2_128
                                                  : m->tm_w2_256;
  if (f) return launch_dense<kEpiStore, true, float>(p2, m->tm_inter, tb2, g2, m->sms, s);
  return launch_dense<kEpiStore, false, float>(p2, m->tm_inter, tb2, g2, m->sms, s);
}

extern "C" b2_status b2_mlp_get_status(b2_mlp *m, b2_stream stream_, int *device_status) {
  if (!m || !device_status) return B2_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream_);
  int v = 0;
  B2_CUDA(cudaStreamSynchronize(s));
  B2_CUDA(cudaMemcpy(&v, m->status, sizeof(int), cudaMemcpyDeviceToHost));
  B2_CUDA(cudaMemset(m->status, 0, sizeof(int)));
  *device_status = v;
  return v ? B2_ERR_DEVICE : B2_OK;
}

extern "C" size_t b2_mlp_device_bytes(const b2_mlp *m) { return m ? m->bytes : 0; }
