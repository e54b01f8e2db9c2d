// moe_internal.h -- the MoE layer object and its pipeline stages, shared by
// the single-GPU entry points (b2moe_api.cu) and the expert-parallel ones
// (ep.cu).  Host code; not part of the public C ABI.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <utility>
#include <cstdio>
#include <vector>

#include "../../include/b2mlp.h"
#include "../../include/b2moe.h"
#include "../../include/b2moe_ep.h"
#include "gemm_sm100.cuh"
#include "gemm_sm100_pair.cuh"
#include "gemm_sm100_splitk.cuh"
#include "gemm_sm100_pair_splitk.cuh"
#include "host_tmap.h"
#include "moe_kernels.cuh"

namespace b2 {

// number of this library's kernel launches (all devices, whole process)
std::atomic<uint64_t> &launch_counter();

#define B2_CUDA(call)                                                                  \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess) {                                                           \
      fprintf(stderr, "[b2moe] %s failed at %s:%d: %s\n", #call, __FILE__, __LINE__,   \
              cudaGetErrorString(e_));                                                 \
      return B2_ERR_CUDA;                                                              \
    }                                                                                  \
  } while (0)

#define B2_LAUNCHED()                                                    \
  do {                                                                   \
    ::b2::launch_counter().fetch_add(1, std::memory_order_relaxed);      \
    B2_CUDA(cudaGetLastError());                                         \
  } while (0)

#define B2_RETURN_IF(x)     \
  do {                      \
    b2_status s_ = (x);     \
    if (s_ != B2_OK) return s_; \
  } while (0)

// 16-byte alignment of a caller's buffer: the kernels read and write x / y
// rows as 16-byte vectors (cp.async, float4 / uint4), so a misaligned
// pointer is refused before any launch instead of faulting on the device.
inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

struct DevInfo {
  int sms = 0;
  int cc_major = 0;
};

inline bool dev_info(DevInfo *d) {
  int dev;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&d->sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return false;
  if (cudaDeviceGetAttribute(&d->cc_major, cudaDevAttrComputeCapabilityMajor, dev) !=
      cudaSuccess)
    return false;
  return true;
}

// Launch with programmatic stream serialization: the kernel may begin while
// its predecessor in the stream drains; every kernel of this library calls
// pdl_wait() before it reads anything a predecessor produced.
template <typename... KArgs, typename... Args>
b2_status launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
  B2_LAUNCHED();
  return B2_OK;
}

// Raise a kernel's dynamic shared-memory limit once per device (the
// attribute is per device and per kernel; setting it costs a driver call).
// `done` belongs to the one kernel `kern`: one bit per device ordinal < 64.
template <typename Kern>
b2_status ensure_smem_limit(Kern kern, size_t smem, std::atomic<uint64_t> &done) {
  int dev = 0;
  B2_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = dev < 64 ? 1ull << dev : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return B2_OK;
  B2_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  done.fetch_or(bit, std::memory_order_acq_rel);
  return B2_OK;
}

template <int EPI, bool TF32, typename TOut, int BN = kBN>
b2_status launch_gemm(const CUtensorMap &ta, const CUtensorMap &tb, const GemmArgs &args,
                      int grid, cudaStream_t s) {
  auto kern = gemm_sm100_kernel<EPI, TF32, TOut, BN>;
  const size_t smem = gemm_smem_bytes(BN);
  static std::atomic<uint64_t> attr_done{0};  // per template instance = per kernel
  B2_RETURN_IF(ensure_smem_limit(kern, smem, attr_done));
  if (grid <= 0) return B2_OK;
  return launch_pdl(kern, dim3(grid), dim3(kGemmThreads), smem, s, ta, tb, args);
}

// The same GEMM run by CTA pairs (2-CTA clusters, cta_group::2 UMMA): `pairs`
// clusters of two CTAs.  The grouped schedule's m-tiles are kPairBM rows.
// ta2: A operand of the groups GemmArgs::group_src marks as remote (the
// expert-parallel receive buffer); ta when null.
template <int EPI, bool TF32, typename TOut>
b2_status launch_gemm_pair(const CUtensorMap &ta, const CUtensorMap &tb, const GemmArgs &args,
                           int pairs, cudaStream_t s, const CUtensorMap *ta2 = nullptr) {
  auto kern = gemm_pair_kernel<EPI, TF32, TOut>;
  const size_t smem = gemm_pair_smem_bytes();
  static std::atomic<uint64_t> attr_done{0};  // per template instance = per kernel
  B2_RETURN_IF(ensure_smem_limit(kern, smem, attr_done));
  if (pairs <= 0) return B2_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  B2_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, ta2 ? *ta2 : ta, args));
  B2_LAUNCHED();
  return B2_OK;
}

// Kernel configuration of a dense (single-group) GEMM over M rows and N
// output columns (for SwiGLU a 256-wide B tile gives 128 outputs), from
// measured B200 behaviour (every configuration timed on the same shapes):
//   pair   CTA-pair kernel (256x256 tiles) when they keep every pair busy;
//   else small products are bound by how fast each SM pulls its operands
//   from L2 (~70-100 GB/s per SM, ~9 TB/s in all) and by wave count, so:
//   single 128-column tiles when they fit one wave;
//   split  split-K over 128-column tiles (256 for SwiGLU) when those tiles
//          fill at most half the SMs: `split` CTAs (a cluster) per tile, the
//          most that still run as one wave of co-resident clusters
//          (max_clusters[s] = co-resident clusters of size s, from the
//          device; kSplitMax caps it), each with >= 4 k-blocks;
//   bn     else the single-CTA tile width (256, 128, 64) that needs the fewest
//          waves, the wider one on a tie.
// kb = 128-byte k-blocks of K (0: no split-K).
struct DensePlan {
  bool pair;
  int bn;
  int b_box_rows;  // rows of the B tensor map's box
  int split;       // K-slices per tile (1: no split): CTAs, or CTA pairs when `pair`
};

constexpr int kSplitPlanMax = 6;  // clusters of 7-8 rarely all fit one wave on 148 SMs

// Co-resident clusters of size s when the device was not asked: B200 GPCs
// hold ~18 SMs each, and a cluster must sit inside one GPC.
inline int static_max_clusters(int sms, int s) { return (sms / 18) * (18 / s); }

inline DensePlan plan_dense(long long M, int N, int sms, bool swiglu, int kb = 0,
                            const int *max_clusters = nullptr) {
  const long long nt256 = swiglu ? N / 128 : (N + kBN - 1) / kBN;
  if (((M + kPairBM - 1) / kPairBM) * nt256 >= sms / 2) return {true, kBN, kBN / 2, 1};
  const long long mt = (M + kBM - 1) / kBM;
  const int sbn = swiglu ? 256 : 128;  // split-K tile width
  const long long tiles = mt * (swiglu ? N / 128 : (N + 127) / 128);
  if (kb >= 8 && tiles * 2 <= sms) {
    for (int sp = std::min<long long>(kSplitPlanMax, std::min<long long>(sms / tiles, kb / 4));
         sp >= 2; --sp) {
      const int cap = max_clusters ? max_clusters[sp] : static_max_clusters(sms, sp);
      if (tiles <= cap) return {false, sbn, sbn, sp};
    }
  }
  if (swiglu) return {false, kBN, kBN, 1};
  if (tiles <= sms) return {false, 128, 128, 1};
  // more 128-column tiles than SMs: the width with the fewest waves, the
  // wider on a tie (at these sizes a 256-column tile costs ~1.1x a 128-column
  // one, a second wave ~1.7x: 2048 x 2048 x 2048 took 24.4 us in 1.73 waves
  // of 128-column tiles, 15.9 us in one wave of 256-column tiles)
  int best = 256;
  long long best_waves = (mt * ((N + 255) / 256) + sms - 1) / sms;
  for (int c : {128, 64}) {
    const long long w = (mt * ((N + c - 1) / c) + sms - 1) / sms;
    if (w < best_waves) {
      best = c;
      best_waves = w;
    }
  }
  return {false, best, best, 1};
}

// Co-resident clusters of each size 2..kSplitMax for the split-K kernels on
// the current device (cudaOccupancyMaxActiveClusters), queried once per
// device; [bn == 256][size].  Falls back to the static estimate.
const int *splitk_cluster_caps(bool swiglu_width);

// The split-K kernel over one wave of clusters (plan.split CTAs per tile).
template <int EPI, bool TF32, typename TOut>
b2_status launch_gemm_splitk(const DensePlan &plan, const CUtensorMap &ta, const CUtensorMap &tb,
                             const GemmArgs &g, cudaStream_t s) {
  SplitArgs a{};
  a.M = g.M;
  a.N = g.N;
  a.num_k_blocks = g.num_k_blocks;
  a.splits = plan.split;
  a.m_tiles = (g.M + kBM - 1) / kBM;
  a.out = g.out;
  a.ldo = g.ldo;
  a.status = g.status;
  a.accumulate = g.accumulate;
  const int n_tiles = EPI == kEpiSwiGLU ? g.N / 128 : (g.N + plan.bn - 1) / plan.bn;
  const int grid = a.m_tiles * n_tiles * plan.split;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = plan.split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (plan.bn == 256) {
    auto kern = gemm_splitk_kernel<EPI, TF32, TOut, 256>;
    static std::atomic<uint64_t> done{0};
    B2_RETURN_IF(ensure_smem_limit(kern, splitk_smem_bytes(256), done));
    cfg.dynamicSmemBytes = splitk_smem_bytes(256);
    if (grid > 0) B2_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, a));
  } else {
    if constexpr (EPI == kEpiStore) {
      auto kern = gemm_splitk_kernel<EPI, TF32, TOut, 128>;
      static std::atomic<uint64_t> done{0};
      B2_RETURN_IF(ensure_smem_limit(kern, splitk_smem_bytes(128), done));
      cfg.dynamicSmemBytes = splitk_smem_bytes(128);
      if (grid > 0) B2_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, a));
    } else {
      return B2_ERR_INVALID;
    }
  }
  if (grid > 0) B2_LAUNCHED();
  return B2_OK;
}

// Split-K over CTA pairs (gemm_sm100_pair_splitk.cuh): one cluster of
// 2 * plan.split CTAs per 256 x 256 tile; tb's box has 128 rows.
template <int EPI, bool TF32, typename TOut>
b2_status launch_gemm_pair_splitk(const DensePlan &plan, const CUtensorMap &ta,
                                  const CUtensorMap &tb, const GemmArgs &g, cudaStream_t s) {
  if (plan.split < 2 || plan.split > kPairSplitMax) return B2_ERR_INVALID;
  SplitArgs a{};
  a.M = g.M;
  a.N = g.N;
  a.num_k_blocks = g.num_k_blocks;
  a.splits = plan.split;
  a.m_tiles = (g.M + kPairBM - 1) / kPairBM;
  a.out = g.out;
  a.ldo = g.ldo;
  a.status = g.status;
  a.accumulate = g.accumulate;
  const int n_tiles = EPI == kEpiSwiGLU ? g.N / 128 : (g.N + kBN - 1) / kBN;
  const int grid = a.m_tiles * n_tiles * 2 * plan.split;
  auto kern = gemm_pair_splitk_kernel<EPI, TF32, TOut>;
  static std::atomic<uint64_t> done{0};
  B2_RETURN_IF(ensure_smem_limit(kern, pair_splitk_smem_bytes(), done));
  if (grid <= 0) return B2_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = pair_splitk_smem_bytes();
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2 * plan.split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  B2_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, a));
  B2_LAUNCHED();
  return B2_OK;
}

// Launches a dense GEMM planned by plan_dense.  g.M, g.N, g.num_k_blocks,
// g.out, g.ldo and g.status are set by the caller; tb's box has
// plan.b_box_rows rows.
template <int EPI, bool TF32, typename TOut>
b2_status launch_dense(const DensePlan &plan, const CUtensorMap &ta, const CUtensorMap &tb,
                       GemmArgs g, int sms, cudaStream_t s) {
  g.num_groups = 0;
  if (g.group_m <= 0) g.group_m = 16;
  const long long mt_pair = (g.M + kPairBM - 1) / kPairBM, mt = (g.M + kBM - 1) / kBM;
  if (EPI == kEpiSwiGLU) {
    g.num_n_tiles = g.N / 128;
  } else {
    g.num_n_tiles = (g.N + plan.bn - 1) / plan.bn;
  }
  if (plan.pair && plan.split > 1) return launch_gemm_pair_splitk<EPI, TF32, TOut>(plan, ta, tb, g, s);
  if (plan.pair) {
    const int pairs = (int)std::min<long long>(sms / 2, mt_pair * g.num_n_tiles);
    return launch_gemm_pair<EPI, TF32, TOut>(ta, tb, g, pairs, s);
  }
  if (plan.split > 1) return launch_gemm_splitk<EPI, TF32, TOut>(plan, ta, tb, g, s);
  const int grid = (int)std::min<long long>(sms, mt * g.num_n_tiles);
  if constexpr (EPI == kEpiSwiGLU) {
    return launch_gemm<EPI, TF32, TOut, 256>(ta, tb, g, grid, s);
  } else {
    switch (plan.bn) {
      case 256: return launch_gemm<EPI, TF32, TOut, 256>(ta, tb, g, grid, s);
      case 128: return launch_gemm<EPI, TF32, TOut, 128>(ta, tb, g, grid, s);
      default: return launch_gemm<EPI, TF32, TOut, 64>(ta, tb, g, grid, s);
    }
  }
}

// Row segments the two grouped GEMMs run over: group g covers rows
// [offsets[g], offsets[g] + counts[g]) of A and C and multiplies them with
// expert block group_b[g] (or g when group_b is null) of the weights.
struct GemmSched {
  const int *counts = nullptr;
  const int *offsets = nullptr;
  const int *mtile_offsets = nullptr;  // exclusive prefix of ceil(count/kPairBM), [groups+1]
  const int *group_b = nullptr;
  int num_groups = 0;
  long long mtiles_upper_bound = 0;    // sizes the persistent grid
};

}  // namespace b2

// ---------------------------------------------------------------- the layer
struct b2_moe {
  b2_moe_desc d;          // router / layer shape (num_experts = router experts)
  int n_wexp = 0;         // experts whose weights this object holds
  int device = 0;
  int Ip = 0;             // inter padded to 128
  int sms = 0;
  bool tf32 = false;
  size_t bytes = 0;
  // weights
  float *gateT = nullptr;
  float *bias = nullptr;
  void *w13 = nullptr;    // [n_wexp][2Ip][H]
  void *w2 = nullptr;     // [n_wexp][H][Ip]
  // scratch
  int *topk_idx = nullptr, *block_counts = nullptr, *block_base = nullptr;
  int *counts = nullptr, *offsets = nullptr, *mtile = nullptr;
  int *token_slot = nullptr, *sorted_token = nullptr;
  float *topk_w = nullptr, *sorted_w = nullptr;
  void *sorted_x = nullptr, *inter = nullptr, *sout = nullptr;
  int *status = nullptr;
  CUtensorMap tm_x, tm_w13, tm_inter, tm_w2;
  CUtensorMap tm_w13_half, tm_w2_half;  // B maps with 128-row boxes for the CTA-pair GEMM
  std::vector<void *> allocs;
  // stage profiling
  bool profile = false;
  std::vector<cudaEvent_t> ev_pool;
  std::vector<cudaEvent_t> ev_rec;
};

namespace b2 {

constexpr int kStageEvents = 7;

// Allocates and packs a layer object.  w1/w2/w3 hold n_wexp expert matrices
// (those this object computes); desc->num_experts is the router's expert count.
// local_gemm_buffers = false skips the intermediate buffer sized for the local
// rows (an expert-parallel owner keeps its intermediates elsewhere).
b2_status moe_create_impl(const b2_moe_desc *desc, int n_wexp, const float *const *w1,
                          const float *const *w2, const float *const *w3, const float *gate,
                          const float *bias, int weights_on_host, cudaStream_t stream,
                          bool local_gemm_buffers, b2_moe **out);
b2_status moe_alloc(b2_moe *m, void **p, size_t bytes);
void prof_mark(b2_moe *m, cudaStream_t s);

// route + scan (+ scatter unless with_scatter is false) of T local tokens;
// after the scan m->counts holds the per-expert row counts
b2_status moe_route_stage(b2_moe *m, const float *x, int T, const b2_moe_trace *tr,
                          cudaStream_t s, bool with_scatter = true);
// scatter of the routed tokens into m->sorted_x (expert order)
b2_status moe_scatter_stage(b2_moe *m, const float *x, int T, cudaStream_t s);
// W1||W3 + SwiGLU and W2 over the scheduled row segments of A (rows of tm_a1)
b2_status moe_gemm_stage(b2_moe *m, const CUtensorMap &tm_a1, const CUtensorMap &tm_a2,
                         void *inter, void *out, const GemmSched &sched, cudaStream_t s,
                         bool stage_marks = true);
// y[t] = sum_k w[t,k] * m->sout[slot(t,k)]  (accumulate: y[t] += that sum)
b2_status moe_combine_stage(b2_moe *m, float *y, int T, cudaStream_t s, bool accumulate = false);
// The dense MLP's forward (mlp.cu); accumulate adds the MLP output into y.
b2_status mlp_forward_impl(b2_mlp *m, const float *x, float *y, int T, cudaStream_t s,
                           bool accumulate);
// The whole single-GPU forward; accumulate adds the layer output into y.
b2_status moe_forward_impl(b2_moe *m, const float *x, float *y, int T, const b2_moe_trace *tr,
                           cudaStream_t s, bool accumulate);

// Expert-parallel layer (ep.cu).  With `share` the new layer uses share's
// communicator instead of creating one from unique_id (collective either way);
// the communicator lives until the last layer using it is destroyed.
b2_status ep_create_impl(const b2_moe_desc *desc, int world, int rank, const void *unique_id,
                         b2_ep *share, int mode, const float *const *w1,
                         const float *const *w2, const float *const *w3, const float *gate,
                         const float *bias, int weights_on_host, b2_stream stream,
                         b2_ep **out);
// b2_ep_forward; accumulate adds the layer output into y.
b2_status ep_forward_impl(b2_ep *ep, const float *x, float *y, int T, cudaStream_t s,
                          bool accumulate);

}  // namespace b2
