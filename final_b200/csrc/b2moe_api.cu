// b2moe_api.cu -- implementation of the single-GPU C ABI in include/b2moe.h.
//
// Owns the packed weights, the scratch buffers and the TMA descriptors of an
// MoE layer object, and launches the kernel pipeline of moe_kernels.cuh and
// gemm_sm100.cuh.  Host code only: no torch types, no hidden host syncs on
// the forward path.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <vector>

#include "moe_internal.h"

using namespace b2;

namespace b2 {

std::atomic<uint64_t> &launch_counter() {
  static std::atomic<uint64_t> n{0};
  return n;
}

namespace {
template <typename Kern>
void query_caps(Kern kern, size_t smem, int sms, int *caps) {
  for (int sp = 0; sp <= kSplitMax; ++sp) caps[sp] = sp >= 2 ? static_max_clusters(sms, sp) : 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess) {
    cudaGetLastError();
    return;
  }
  for (int sp = 2; sp <= kSplitMax; ++sp) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sp * 64);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = sp;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0)
      caps[sp] = n;
    else
      cudaGetLastError();
  }
}
}  // namespace

const int *splitk_cluster_caps(bool swiglu_width) {
  // [device ordinal < 16][bn 128 / 256][size]
  static int caps[16][2][kSplitMax + 1];
  static std::atomic<uint32_t> done[16];
  int dev = 0;
  cudaGetDevice(&dev);
  DevInfo di;
  if (dev < 0 || dev >= 16 || !dev_info(&di)) return nullptr;
  const int w = swiglu_width ? 1 : 0;
  if (!(done[dev].load(std::memory_order_acquire) & (1u << w))) {
    if (w)
      query_caps(gemm_splitk_kernel<kEpiStore, false, float, 256>, splitk_smem_bytes(256), di.sms,
                 caps[dev][w]);
    else
      query_caps(gemm_splitk_kernel<kEpiStore, false, float, 128>, splitk_smem_bytes(128), di.sms,
                 caps[dev][w]);
    done[dev].fetch_or(1u << w, std::memory_order_acq_rel);
  }
  return caps[dev][w];
}

static cudaEvent_t prof_event(b2_moe *m) {
  if (!m->ev_pool.empty()) {
    cudaEvent_t e = m->ev_pool.back();
    m->ev_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

void prof_mark(b2_moe *m, cudaStream_t s) {
  if (!m->profile) return;
  cudaEvent_t e = prof_event(m);
  cudaEventRecord(e, s);
  m->ev_rec.push_back(e);
}

b2_status moe_alloc(b2_moe *m, void **p, size_t bytes) {
  if (bytes == 0) bytes = 16;
  B2_CUDA(cudaMalloc(p, bytes));
  m->allocs.push_back(*p);
  m->bytes += bytes;
  return B2_OK;
}

static void moe_free_all(b2_moe *m) {
  for (void *p : m->allocs) cudaFree(p);
  m->allocs.clear();
  for (cudaEvent_t e : m->ev_pool) cudaEventDestroy(e);
  for (cudaEvent_t e : m->ev_rec) cudaEventDestroy(e);
  m->ev_pool.clear();
  m->ev_rec.clear();
}

}  // namespace b2

extern "C" b2_status b2_moe_destroy(b2_moe *moe) {
  if (!moe) return B2_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(moe->device);
  moe_free_all(moe);
  cudaSetDevice(prev);
  delete moe;
  return B2_OK;
}

namespace b2 {

b2_status moe_create_impl(const b2_moe_desc *desc, int n_wexp, const float *const *w1,
                          const float *const *w2, const float *const *w3, const float *gate,
                          const float *bias, int weights_on_host, cudaStream_t stream,
                          bool local_gemm_buffers, b2_moe **out) {
  if (!desc || !out || !gate || (n_wexp > 0 && (!w1 || !w2 || !w3))) return B2_ERR_INVALID;
  *out = nullptr;
  const b2_moe_desc &d = *desc;
  if (d.hidden <= 0 || d.hidden % 64 != 0 || d.inter <= 0 || d.inter % 16 != 0 ||
      d.num_experts < 1 || d.num_experts > kMaxExperts || d.top_k < 1 || d.top_k > kMaxTopK ||
      d.top_k > d.num_experts || d.max_tokens < 1 || (d.dtype != B2_BF16 && d.dtype != B2_TF32) ||
      n_wexp < 0 || n_wexp > kMaxGroups)
    return B2_ERR_INVALID;
  if (d.use_bias && !bias) return B2_ERR_INVALID;
  DevInfo di;
  if (!dev_info(&di)) return B2_ERR_NO_DEVICE;
  if (di.cc_major != 10) return B2_ERR_NO_DEVICE;

  b2_moe *m = new b2_moe();
  m->d = d;
  m->n_wexp = n_wexp;
  cudaGetDevice(&m->device);
  m->sms = di.sms;
  m->tf32 = d.dtype == B2_TF32;
  const int E = d.num_experts, H = d.hidden, I = d.inter, K = d.top_k;
  const int W = n_wexp;
  m->Ip = (I + 127) / 128 * 128;
  const int Ip = m->Ip;
  const size_t es = m->tf32 ? 4 : 2;
  const size_t T = (size_t)d.max_tokens, R = T * K;
  const size_t nb = (T + kRouteTB - 1) / kRouteTB;

  auto bail = [&](b2_status s) {
    b2_moe_destroy(m);
    return s;
  };
#define B2_TRY(x)                     \
  do {                                \
    b2_status s_ = (x);               \
    if (s_ != B2_OK) return bail(s_); \
  } while (0)
  B2_TRY(moe_alloc(m, (void **)&m->gateT, sizeof(float) * H * kMaxExperts));
  B2_TRY(moe_alloc(m, (void **)&m->bias, sizeof(float) * kMaxExperts));
  B2_TRY(moe_alloc(m, &m->w13, es * (size_t)std::max(W, 1) * 2 * Ip * H));
  B2_TRY(moe_alloc(m, &m->w2, es * (size_t)std::max(W, 1) * H * Ip));
  B2_TRY(moe_alloc(m, (void **)&m->topk_idx, sizeof(int) * R));
  B2_TRY(moe_alloc(m, (void **)&m->topk_w, sizeof(float) * R));
  B2_TRY(moe_alloc(m, (void **)&m->block_counts, sizeof(int) * nb * kMaxExperts));
  B2_TRY(moe_alloc(m, (void **)&m->block_base, sizeof(int) * nb * kMaxExperts));
  B2_TRY(moe_alloc(m, (void **)&m->counts, sizeof(int) * kMaxExperts));
  B2_TRY(moe_alloc(m, (void **)&m->offsets, sizeof(int) * kMaxExperts));
  B2_TRY(moe_alloc(m, (void **)&m->mtile, sizeof(int) * (kMaxExperts + 1)));
  B2_TRY(moe_alloc(m, (void **)&m->token_slot, sizeof(int) * R));
  B2_TRY(moe_alloc(m, (void **)&m->sorted_token, sizeof(int) * R));
  B2_TRY(moe_alloc(m, (void **)&m->sorted_w, sizeof(float) * R));
  B2_TRY(moe_alloc(m, &m->sorted_x, es * R * H));
  if (local_gemm_buffers) B2_TRY(moe_alloc(m, &m->inter, es * R * Ip));
  B2_TRY(moe_alloc(m, &m->sout, es * R * H));
  B2_TRY(moe_alloc(m, (void **)&m->status, sizeof(int)));
  if (cudaMemsetAsync(m->status, 0, sizeof(int), stream) != cudaSuccess ||
      cudaMemsetAsync(m->bias, 0, sizeof(float) * kMaxExperts, stream) != cudaSuccess ||
      (m->inter && cudaMemsetAsync(m->inter, 0, es * R * Ip, stream) != cudaSuccess))
    return bail(B2_ERR_CUDA);

  // ---- weights: stage host matrices through one expert-sized device buffer
  float *st1 = nullptr, *st3 = nullptr, *st2 = nullptr, *stg = nullptr;
  auto fail = [&](b2_status s) {
    if (st1) cudaFree(st1);
    if (st3) cudaFree(st3);
    if (st2) cudaFree(st2);
    if (stg) cudaFree(stg);
    return bail(s);
  };
  const size_t mat = (size_t)I * H;
  if (weights_on_host) {
    if (cudaMalloc(&st1, mat * 4) != cudaSuccess || cudaMalloc(&st3, mat * 4) != cudaSuccess ||
        cudaMalloc(&st2, mat * 4) != cudaSuccess ||
        cudaMalloc(&stg, sizeof(float) * E * H) != cudaSuccess)
      return fail(B2_ERR_CUDA);
  }
  for (int e = 0; e < W; ++e) {
    const float *p1 = w1[e], *p3 = w3[e], *p2 = w2[e];
    if (!p1 || !p2 || !p3) return fail(B2_ERR_INVALID);
    if (weights_on_host) {
      if (cudaMemcpyAsync(st1, p1, mat * 4, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
          cudaMemcpyAsync(st3, p3, mat * 4, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
          cudaMemcpyAsync(st2, p2, mat * 4, cudaMemcpyHostToDevice, stream) != cudaSuccess)
        return fail(B2_ERR_CUDA);
      p1 = st1;
      p3 = st3;
      p2 = st2;
    }
    if (m->tf32) {
      float *o13 = reinterpret_cast<float *>(m->w13) + (size_t)e * 2 * Ip * H;
      float *o2 = reinterpret_cast<float *>(m->w2) + (size_t)e * H * Ip;
      pack_w13_single<float><<<2 * Ip, 256, 0, stream>>>(p1, p3, H, I, Ip, o13);
      pack_w2_single<float><<<H, 256, 0, stream>>>(p2, H, I, Ip, o2);
    } else {
      __nv_bfloat16 *o13 = reinterpret_cast<__nv_bfloat16 *>(m->w13) + (size_t)e * 2 * Ip * H;
      __nv_bfloat16 *o2 = reinterpret_cast<__nv_bfloat16 *>(m->w2) + (size_t)e * H * Ip;
      pack_w13_single<__nv_bfloat16><<<2 * Ip, 256, 0, stream>>>(p1, p3, H, I, Ip, o13);
      pack_w2_single<__nv_bfloat16><<<H, 256, 0, stream>>>(p2, H, I, Ip, o2);
    }
    if (cudaGetLastError() != cudaSuccess) return fail(B2_ERR_CUDA);
    launch_counter().fetch_add(2, std::memory_order_relaxed);
    if (weights_on_host && cudaStreamSynchronize(stream) != cudaSuccess)
      return fail(B2_ERR_CUDA);  // staging buffers are reused by the next expert
  }
  const float *gsrc = gate;
  if (weights_on_host) {
    if (cudaMemcpyAsync(stg, gate, sizeof(float) * E * H, cudaMemcpyHostToDevice, stream) !=
        cudaSuccess)
      return fail(B2_ERR_CUDA);
    gsrc = stg;
  }
  pack_gate_kernel<<<(H * kMaxExperts + 255) / 256, 256, 0, stream>>>(gsrc, E, H, m->gateT);
  if (cudaGetLastError() != cudaSuccess) return fail(B2_ERR_CUDA);
  launch_counter().fetch_add(1, std::memory_order_relaxed);
  if (d.use_bias &&
      cudaMemcpyAsync(m->bias, bias, sizeof(float) * E,
                      weights_on_host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice,
                      stream) != cudaSuccess)
    return fail(B2_ERR_CUDA);
  if (cudaStreamSynchronize(stream) != cudaSuccess) return fail(B2_ERR_CUDA);
  if (st1) cudaFree(st1);
  if (st3) cudaFree(st3);
  if (st2) cudaFree(st2);
  if (stg) cudaFree(stg);
  st1 = st3 = st2 = stg = nullptr;

  // ---- TMA descriptors (buffers are fixed for the object's lifetime)
  const bool f = m->tf32;
  const int Wm = std::max(W, 1);
  if (!make_tmap(&m->tm_x, m->sorted_x, f, H, R, (uint64_t)H * es, kBM) ||
      !make_tmap(&m->tm_w13, m->w13, f, H, (uint64_t)Wm * 2 * Ip, (uint64_t)H * es, kBN) ||
      (m->inter && !make_tmap(&m->tm_inter, m->inter, f, Ip, R, (uint64_t)Ip * es, kBM)) ||
      !make_tmap(&m->tm_w2, m->w2, f, Ip, (uint64_t)Wm * H, (uint64_t)Ip * es, kBN) ||
      !make_tmap(&m->tm_w13_half, m->w13, f, H, (uint64_t)Wm * 2 * Ip, (uint64_t)H * es, kBN / 2) ||
      !make_tmap(&m->tm_w2_half, m->w2, f, Ip, (uint64_t)Wm * H, (uint64_t)Ip * es, kBN / 2))
    return bail(B2_ERR_CUDA);
#undef B2_TRY
  *out = m;
  return B2_OK;
}

b2_status moe_route_stage(b2_moe *m, const float *x, int T, const b2_moe_trace *tr,
                          cudaStream_t s, bool with_scatter) {
  const int E = m->d.num_experts, K = m->d.top_k, H = m->d.hidden;
  const int nb = (T + kRouteTB - 1) / kRouteTB;
  prof_mark(m, s);
  B2_RETURN_IF(launch_pdl(route_kernel, dim3(nb), dim3(kRouteThreads), 0, s, x,
                          (const float *)m->gateT, (const float *)(m->d.use_bias ? m->bias : nullptr),
                          T, H, E, K, m->d.routed_scale, m->topk_idx, m->topk_w, m->block_counts,
                          tr ? tr->logits : (float *)nullptr));
  prof_mark(m, s);
  B2_RETURN_IF(launch_pdl(scan_kernel, dim3(1), dim3(1024), 0, s, (const int *)m->block_counts, nb,
                          E, (int)kPairBM, m->counts, m->offsets, m->mtile, m->block_base));
  prof_mark(m, s);
  return with_scatter ? moe_scatter_stage(m, x, T, s) : B2_OK;
}

b2_status moe_scatter_stage(b2_moe *m, const float *x, int T, cudaStream_t s) {
  const int E = m->d.num_experts, K = m->d.top_k, H = m->d.hidden;
  const int nb = (T + kRouteTB - 1) / kRouteTB;
  if (m->tf32)
    B2_RETURN_IF(launch_pdl(scatter_kernel<float>, dim3(nb), dim3(scatter_threads(K)), 0, s, x,
                            (const int *)m->topk_idx, (const float *)m->topk_w,
                            (const int *)m->block_base, T, H, E, K,
                            reinterpret_cast<float *>(m->sorted_x), m->token_slot, m->sorted_token,
                            m->sorted_w, m->status));
  else
    B2_RETURN_IF(launch_pdl(scatter_kernel<__nv_bfloat16>, dim3(nb), dim3(scatter_threads(K)), 0,
                            s, x, (const int *)m->topk_idx, (const float *)m->topk_w,
                            (const int *)m->block_base, T, H, E, K,
                            reinterpret_cast<__nv_bfloat16 *>(m->sorted_x), m->token_slot,
                            m->sorted_token, m->sorted_w, m->status));
  return B2_OK;
}

b2_status moe_gemm_stage(b2_moe *m, const CUtensorMap &tm_a1, const CUtensorMap &tm_a2,
                         void *inter, void *out, const GemmSched &sc, cudaStream_t s,
                         bool stage_marks) {
  const int H = m->d.hidden, Ip = m->Ip;
  const bool f = m->tf32;
  const int max_pairs = m->sms / 2;
  GemmArgs a1{};
  a1.counts = sc.counts;
  a1.offsets = sc.offsets;
  a1.mtile_offsets = sc.mtile_offsets;
  a1.group_b = sc.group_b;
  a1.num_groups = sc.num_groups;
  a1.b_rows_per_group = 2 * Ip;
  a1.N = Ip;
  a1.num_n_tiles = Ip / 128;
  a1.num_k_blocks = f ? H / 32 : H / 64;
  a1.out = inter;
  a1.ldo = Ip;
  a1.status = m->status;
  const int pairs1 = (int)std::min<long long>(max_pairs, sc.mtiles_upper_bound * a1.num_n_tiles);
  if (stage_marks) prof_mark(m, s);
  if (f)
    B2_RETURN_IF((launch_gemm_pair<kEpiSwiGLU, true, float>(tm_a1, m->tm_w13_half, a1, pairs1, s)));
  else
    B2_RETURN_IF(
        (launch_gemm_pair<kEpiSwiGLU, false, __nv_bfloat16>(tm_a1, m->tm_w13_half, a1, pairs1, s)));

  GemmArgs a2 = a1;
  a2.b_rows_per_group = H;
  a2.N = H;
  a2.num_n_tiles = (H + kBN - 1) / kBN;
  a2.num_k_blocks = f ? Ip / 32 : Ip / 64;
  a2.out = out;
  a2.ldo = H;
  const int pairs2 = (int)std::min<long long>(max_pairs, sc.mtiles_upper_bound * a2.num_n_tiles);
  if (stage_marks) prof_mark(m, s);
  if (f)
    B2_RETURN_IF((launch_gemm_pair<kEpiStore, true, float>(tm_a2, m->tm_w2_half, a2, pairs2, s)));
  else
    B2_RETURN_IF(
        (launch_gemm_pair<kEpiStore, false, __nv_bfloat16>(tm_a2, m->tm_w2_half, a2, pairs2, s)));
  return B2_OK;
}

b2_status moe_combine_stage(b2_moe *m, float *y, int T, cudaStream_t s, bool accumulate) {
  const int K = m->d.top_k, H = m->d.hidden;
  const int acc = accumulate ? 1 : 0;
  prof_mark(m, s);
  if (m->tf32)
    B2_RETURN_IF(launch_pdl(combine_kernel<float>, dim3(T), dim3(256), 0, s,
                            reinterpret_cast<const float *>(m->sout), (const int *)m->token_slot,
                            (const float *)m->topk_w, T, H, K, y, acc));
  else
    B2_RETURN_IF(launch_pdl(combine_kernel<__nv_bfloat16>, dim3(T), dim3(256), 0, s,
                            reinterpret_cast<const __nv_bfloat16 *>(m->sout),
                            (const int *)m->token_slot, (const float *)m->topk_w, T, H, K, y, acc));
  prof_mark(m, s);
  return B2_OK;
}

}  // namespace b2

// ---------------------------------------------------------------- C ABI
extern "C" b2_status b2_moe_create(const b2_moe_desc *desc, const float *const *w1,
                                   const float *const *w2, const float *const *w3,
                                   const float *gate, const float *bias, int weights_on_host,
                                   b2_stream stream, b2_moe **out) {
  if (!desc) return B2_ERR_INVALID;
  return moe_create_impl(desc, desc->num_experts, w1, w2, w3, gate, bias, weights_on_host,
                         reinterpret_cast<cudaStream_t>(stream), true, out);
}

static b2_status copy_trace(void *dst, const void *src, size_t bytes, cudaStream_t s) {
  if (!dst || bytes == 0) return B2_OK;
  B2_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s));
  return B2_OK;
}

extern "C" b2_status b2_moe_forward_ex(b2_moe *m, const float *x, float *y, int T,
                                       const b2_moe_trace *tr, b2_stream stream_) {
  return moe_forward_impl(m, x, y, T, tr, reinterpret_cast<cudaStream_t>(stream_), false);
}

b2_status b2::moe_forward_impl(b2_moe *m, const float *x, float *y, int T,
                               const b2_moe_trace *tr, cudaStream_t s, bool accumulate) {
  if (!m || T < 0 || (T > 0 && (!x || !y || !aligned16(x) || !aligned16(y))))
    return B2_ERR_INVALID;
  if (m->n_wexp != m->d.num_experts || !m->inter) return B2_ERR_INVALID;
  if (T > m->d.max_tokens) return B2_ERR_CAPACITY;
  if (T == 0) return B2_OK;
  const int E = m->d.num_experts, K = m->d.top_k;

  B2_RETURN_IF(moe_route_stage(m, x, T, tr, s));
  GemmSched sc;
  sc.counts = m->counts;
  sc.offsets = m->offsets;
  sc.mtile_offsets = m->mtile;
  sc.group_b = nullptr;
  sc.num_groups = E;
  sc.mtiles_upper_bound = ((long long)T * K + kPairBM - 1) / kPairBM + E;  // <= 1 partial tile per expert
  B2_RETURN_IF(moe_gemm_stage(m, m->tm_x, m->tm_inter, m->inter, m->sout, sc, s));
  B2_RETURN_IF(moe_combine_stage(m, y, T, s, accumulate));

  if (tr) {
    const size_t tk = (size_t)T * K;
    B2_RETURN_IF(copy_trace(tr->topk_idx, m->topk_idx, tk * 4, s));
    B2_RETURN_IF(copy_trace(tr->topk_w, m->topk_w, tk * 4, s));
    B2_RETURN_IF(copy_trace(tr->counts, m->counts, (size_t)E * 4, s));
    B2_RETURN_IF(copy_trace(tr->offsets, m->offsets, (size_t)E * 4, s));
    B2_RETURN_IF(copy_trace(tr->mtile_offsets, m->mtile, (size_t)(E + 1) * 4, s));
    B2_RETURN_IF(copy_trace(tr->token_slot, m->token_slot, tk * 4, s));
    B2_RETURN_IF(copy_trace(tr->sorted_token, m->sorted_token, tk * 4, s));
    B2_RETURN_IF(copy_trace(tr->sorted_w, m->sorted_w, tk * 4, s));
  }
  return B2_OK;
}

extern "C" b2_status b2_moe_forward(b2_moe *m, const float *x, float *y, int T,
                                    b2_stream stream) {
  return b2_moe_forward_ex(m, x, y, T, nullptr, stream);
}

extern "C" b2_status b2_moe_dispatch_slots(b2_moe *m, const int32_t *topk_idx, int T,
                                           int32_t *counts, int32_t *offsets,
                                           int32_t *token_slot, b2_stream stream_) {
  if (!m || T < 0 || (T > 0 && (!topk_idx || !token_slot))) return B2_ERR_INVALID;
  if (T > m->d.max_tokens) return B2_ERR_CAPACITY;
  const int E = m->d.num_experts, K = m->d.top_k;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream_);
  if (T == 0) {
    if (counts) B2_CUDA(cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, s));
    if (offsets) B2_CUDA(cudaMemsetAsync(offsets, 0, sizeof(int32_t) * E, s));
    return B2_OK;
  }
  const int nb = (T + kRouteTB - 1) / kRouteTB;
  B2_RETURN_IF(launch_pdl(hist_kernel, dim3(nb), dim3(128), 0, s, topk_idx, T, E, K,
                          m->block_counts));
  B2_RETURN_IF(launch_pdl(scan_kernel, dim3(1), dim3(1024), 0, s, (const int *)m->block_counts, nb,
                          E, (int)kPairBM, m->counts, m->offsets, m->mtile, m->block_base));
  // slot bookkeeping only (hidden 0: no row copy); bad ids are recorded here
  B2_RETURN_IF(launch_pdl(scatter_kernel<__nv_bfloat16>, dim3(nb), dim3(scatter_threads(K)), 0, s,
                          (const float *)nullptr, topk_idx, (const float *)nullptr,
                          (const int *)m->block_base, T, 0, E, K, (__nv_bfloat16 *)nullptr,
                          token_slot, (int *)nullptr, (float *)nullptr, m->status));
  if (counts)
    B2_CUDA(cudaMemcpyAsync(counts, m->counts, sizeof(int32_t) * E, cudaMemcpyDeviceToDevice, s));
  if (offsets)
    B2_CUDA(
        cudaMemcpyAsync(offsets, m->offsets, sizeof(int32_t) * E, cudaMemcpyDeviceToDevice, s));
  return B2_OK;
}

extern "C" b2_status b2_moe_get_status(b2_moe *m, b2_stream stream_, int *device_status) {
  if (!m || !device_status) return B2_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream_);
  int v = 0;
  B2_CUDA(cudaStreamSynchronize(s));
  B2_CUDA(cudaMemcpy(&v, m->status, sizeof(int), cudaMemcpyDeviceToHost));
  B2_CUDA(cudaMemset(m->status, 0, sizeof(int)));
  *device_status = v;
  return v ? B2_ERR_DEVICE : B2_OK;
}

extern "C" b2_status b2_moe_profile_enable(b2_moe *m, int enable) {
  if (!m) return B2_ERR_INVALID;
  m->profile = enable != 0;
  return B2_OK;
}

extern "C" b2_status b2_moe_profile_read(b2_moe *m, float *stage_ms, int *forwards) {
  if (!m || !stage_ms || !forwards) return B2_ERR_INVALID;
  for (int i = 0; i < kStageEvents - 1; ++i) stage_ms[i] = 0.0f;
  const size_t n = m->ev_rec.size() / kStageEvents;
  for (size_t f = 0; f < n; ++f) {
    cudaEvent_t *ev = &m->ev_rec[f * kStageEvents];
    B2_CUDA(cudaEventSynchronize(ev[kStageEvents - 1]));
    for (int i = 0; i < kStageEvents - 1; ++i) {
      float ms = 0.0f;
      B2_CUDA(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
      stage_ms[i] += ms;
    }
  }
  *forwards = (int)n;
  for (cudaEvent_t e : m->ev_rec) m->ev_pool.push_back(e);
  m->ev_rec.clear();
  return B2_OK;
}

extern "C" size_t b2_moe_device_bytes(const b2_moe *m) { return m ? m->bytes : 0; }

// ---------------------------------------------------------------- dense GEMM
// b2_gemm_nt with the plan given (kind < 0: the planner's choice).
static b2_status gemm_nt_impl(const void *A, const void *B, float *C, int M, int N, int K, int ldc,
                              int dtype, int kind, int bn, int split, int *status,
                              b2_stream stream_) {
  if (M < 0 || N <= 0 || K <= 0 || ldc < N || (M > 0 && (!A || !B || !C)))
    return B2_ERR_INVALID;
  if (dtype != B2_BF16 && dtype != B2_TF32) return B2_ERR_INVALID;
  const bool f = dtype == B2_TF32;
  if (K % (f ? 4 : 8) != 0) return B2_ERR_INVALID;
  if (M == 0) return B2_OK;
  DevInfo di;
  if (!dev_info(&di)) return B2_ERR_NO_DEVICE;
  const size_t es = f ? 4 : 2;
  const int kblocks = (int)(((size_t)K * es + kBKBytes - 1) / kBKBytes);
  DensePlan plan = plan_dense(M, N, di.sms, false, kblocks, splitk_cluster_caps(false));
  if (kind == 0) {
    if (bn != 64 && bn != 128 && bn != 256) return B2_ERR_INVALID;
    plan = {false, bn, bn, 1};
  } else if (kind == 1) {
    plan = {true, kBN, kBN / 2, 1};
  } else if (kind == 2) {
    if ((bn != 128 && bn != 256) || split < 2 || split > kSplitMax || split > kblocks)
      return B2_ERR_INVALID;
    plan = {false, bn, bn, split};
  } else if (kind == 3) {
    if (split < 2 || split > kPairSplitMax || split > kblocks) return B2_ERR_INVALID;
    plan = {true, kBN, kBN / 2, split};
  } else if (kind >= 0) {
    return B2_ERR_INVALID;
  }
  CUtensorMap ta, tb;
  if (!make_tmap(&ta, A, f, K, M, (uint64_t)K * es, kBM) ||
      !make_tmap(&tb, B, f, K, N, (uint64_t)K * es, plan.b_box_rows))
    return B2_ERR_INVALID;
  GemmArgs g{};
  g.M = M;
  g.N = N;
  g.num_k_blocks = kblocks;
  g.group_m = 16;
  g.out = C;
  g.ldo = ldc;
  g.status = status;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream_);
  if (f) return launch_dense<kEpiStore, true, float>(plan, ta, tb, g, di.sms, s);
  return launch_dense<kEpiStore, false, float>(plan, ta, tb, g, di.sms, s);
}

extern "C" b2_status b2_gemm_nt(const void *A, const void *B, float *C, int M, int N, int K,
                                int ldc, int dtype, int *status, b2_stream stream_) {
  return gemm_nt_impl(A, B, C, M, N, K, ldc, dtype, -1, 0, 0, status, stream_);
}

extern "C" b2_status b2_gemm_nt_config(const void *A, const void *B, float *C, int M, int N,
                                       int K, int ldc, int dtype, int kind, int bn, int split,
                                       int *status, b2_stream stream_) {
  if (kind < 0 || kind > 3) return B2_ERR_INVALID;
  return gemm_nt_impl(A, B, C, M, N, K, ldc, dtype, kind, bn, split, status, stream_);
}

extern "C" b2_status b2_gemm_plan(int M, int N, int K, int dtype, int sms, int *kind, int *bn,
                                  int *split) {
  if (M <= 0 || N <= 0 || K <= 0 || sms <= 0 || !kind || !bn || !split ||
      (dtype != B2_BF16 && dtype != B2_TF32))
    return B2_ERR_INVALID;
  const size_t es = dtype == B2_TF32 ? 4 : 2;
  const DensePlan p = plan_dense(M, N, sms, false, (int)(((size_t)K * es + kBKBytes - 1) / kBKBytes));
  *kind = p.pair ? (p.split > 1 ? 3 : 1) : p.split > 1 ? 2 : 0;
  *bn = p.bn;
  *split = p.split;
  return B2_OK;
}

extern "C" b2_status b2_convert_f32_to_bf16(const float *in, void *out, size_t n,
                                            b2_stream stream_) {
  if (n == 0) return B2_OK;
  if (!in || !out || (reinterpret_cast<uintptr_t>(in) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15))
    return B2_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream_);
  const size_t blocks = std::min<size_t>((n / 8 + 255) / 256 + 1, 148 * 16);
  f32_to_bf16_kernel<<<(unsigned)blocks, 256, 0, s>>>(in, reinterpret_cast<__nv_bfloat16 *>(out), n);
  B2_LAUNCHED();
  return B2_OK;
}

extern "C" uint64_t b2_kernel_launch_count(void) { return launch_counter().load(); }

extern "C" int b2_moe_tile_rows(void) { return kPairBM; }

extern "C" const char *b2_status_string(b2_status s) {
  switch (s) {
    case B2_OK: return "ok";
    case B2_ERR_INVALID: return "invalid argument";
    case B2_ERR_CUDA: return "CUDA error";
    case B2_ERR_CAPACITY: return "token count exceeds capacity";
    case B2_ERR_DEVICE: return "device-side error recorded";
    case B2_ERR_NO_DEVICE: return "no sm_100 device";
    case B2_ERR_COMM: return "communication error or timeout";
  }
  return "unknown";
}

extern "C" const char *b2_version(void) { return "b2moe sm_100a tcgen05 v0.2"; }

extern "C" b2_status b2_device_code_version(int *version) {
  if (!version) return B2_ERR_INVALID;
  cudaFuncAttributes a{};
  B2_CUDA(cudaFuncGetAttributes(&a, reinterpret_cast<const void *>(scan_kernel)));
  *version = a.binaryVersion;
  return B2_OK;
}
