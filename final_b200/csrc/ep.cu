// ep.cu -- expert-parallel MoE layer (include/b2moe_ep.h).
//
// Per forward on every rank:
//   1. route / scan the local tokens (moe_route_stage): per-expert counts on
//      the device; the scatter of the rows into expert order (sorted_x) is
//      launched next and runs while
//   2. the [world][E] count matrix is all-gathered on the dispatch stream and
//      copied to the host; one bounded host wait on it, then every rank
//      computes the same exchange plan (b2_ep_plan_compute);
//   3. dispatch: the copy engine pushes each peer's contiguous chunk of bf16
//      rows straight into that peer's receive buffer (CUDA IPC mapping over
//      NVLink), followed by a sequence-number flag -- no SMs are used;
//   4. fused pipeline (default): ONE W1||W3 launch over the rank's own rows
//      and every source's rows -- the TMA producer of a tile from source s
//      waits (bounded) on s's arrival flag before loading it, so the GEMM
//      starts on the own rows at once and takes each source as it lands --
//      and ONE W2 launch that stores every result locally and counts the
//      stored tiles per return chunk; the copy engine sends each chunk to its
//      source as soon as its counter is complete (a stream wait on the
//      counter), then raises this rank's return flag there.
//      Staged pipeline: the own rows in place, then per source a bounded flag
//      wait and a W1||W3 + W2 launch pair, results returned by the copy
//      engine;
//   5. after every source has signalled, the local k-ordered combine
//      (moe_combine_stage) reads sout unchanged.
// NCCL (loaded at run time: the process's libnccl.so.2, normally PyTorch's, so
// the library has no link-time NCCL dependency) carries only the per-forward
// all-gather of the expert counts and the start-up exchange of IPC handles.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>

#include "../../include/b2moe_ep.h"
#include "moe_internal.h"
#include "ep_sched.cuh"

using namespace b2;

namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
#define B2_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name))
    B2_SYM(GetUniqueId, "ncclGetUniqueId");
    B2_SYM(CommInitRank, "ncclCommInitRank");
    B2_SYM(CommDestroy, "ncclCommDestroy");
    B2_SYM(CommAbort, "ncclCommAbort");
    B2_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    B2_SYM(GroupStart, "ncclGroupStart");
    B2_SYM(GroupEnd, "ncclGroupEnd");
    B2_SYM(Send, "ncclSend");
    B2_SYM(Recv, "ncclRecv");
    B2_SYM(AllGather, "ncclAllGather");
    B2_SYM(GetErrorString, "ncclGetErrorString");
#undef B2_SYM
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.CommAbort &&
             api.CommGetAsyncError && api.GroupStart && api.GroupEnd && api.Send && api.Recv &&
             api.AllGather && api.GetErrorString;
  });
  return api;
}

#define B2_NCCL(call)                                                                  \
  do {                                                                                 \
    ncclResult_t r_ = (call);                                                          \
    if (r_ != ncclSuccess) {                                                           \
      fprintf(stderr, "[b2moe] %s failed: %s\n", #call, nccl().GetErrorString(r_));    \
      return B2_ERR_COMM;                                                              \
    }                                                                                  \
  } while (0)

// Estimated grouped-GEMM cost beyond the rows themselves, in rows (balanced
// plan): a row segment ends in a partly filled 256-row pair tile (128 rows
// wasted on average), and every distinct expert a rank computes costs its
// weight reads and tile-schedule ramp (~320 rows' time, from 2-GPU timelines
// of skewed routing on B200).
constexpr int64_t kEpSegmentCost = 128;
constexpr int64_t kEpExpertCost = 320;

// rows of source s (its expert-sorted order) whose global slot is < g
int64_t rows_below(const int32_t *cnt_s, const int64_t *gpos_s, int E, int64_t g) {
  int64_t n = 0;
  for (int e = 0; e < E; ++e) {
    const int64_t v = g - gpos_s[e];
    n += v <= 0 ? 0 : (v < cnt_s[e] ? v : cnt_s[e]);
  }
  return n;
}

}  // namespace

// ---------------------------------------------------------------- plan
extern "C" b2_status b2_ep_plan_compute(int G, int r, int E, int mode, const int32_t *cnt,
                                        b2_ep_plan *p) {
  if (G < 1 || G > B2_EP_MAX_WORLD || r < 0 || r >= G || E < 1 || !cnt || !p)
    return B2_ERR_INVALID;
  if (mode != B2_EP_OWNER && mode != B2_EP_BALANCED) return B2_ERR_INVALID;
  if (mode == B2_EP_OWNER && E % G != 0) return B2_ERR_INVALID;
  for (int i = 0; i < G * E; ++i)
    if (cnt[i] < 0) return B2_ERR_INVALID;
  memset(p, 0, sizeof(*p));
  const int32_t *mine = cnt + (size_t)r * E;
  if (mode == B2_EP_OWNER) {
    const int EL = E / G;
    int64_t off = 0;
    for (int d = 0; d < G; ++d) {  // my rows of rank d's experts are contiguous
      int64_t c = 0;
      for (int e = d * EL; e < (d + 1) * EL; ++e) c += mine[e];
      p->send_off[d] = off;
      p->send_cnt[d] = c;
      off += c;
    }
    int64_t roff = 0;
    for (int s = 0; s < G; ++s) {
      int64_t c = 0;
      for (int e = r * EL; e < (r + 1) * EL; ++e) c += cnt[(size_t)s * E + e];
      p->recv_off[s] = roff;
      p->recv_cnt[s] = c;
      roff += c;
    }
    p->recv_rows = roff;
    int n = 0;
    for (int el = 0; el < EL; ++el)  // expert-major, then source
      for (int s = 0; s < G; ++s) {
        const int e = r * EL + el;
        const int32_t c = cnt[(size_t)s * E + e];
        if (c == 0) continue;
        int64_t within = 0;
        for (int e2 = r * EL; e2 < e; ++e2) within += cnt[(size_t)s * E + e2];
        if (n >= B2_EP_MAX_SEGMENTS) return B2_ERR_INVALID;
        p->seg_off[n] = (int32_t)(p->recv_off[s] + within);
        p->seg_cnt[n] = c;
        p->seg_expert[n] = el;
        p->seg_source[n] = s;
        ++n;
      }
    p->num_segments = n;
    return B2_OK;
  }
  // ---- balanced: global order is expert-major, then source rank, then the
  // source's own order; rank d computes global rows [bound[d], bound[d+1]).
  std::vector<int64_t> tot(E, 0), gpos((size_t)G * E);
  int64_t R = 0;
  for (int e = 0; e < E; ++e) {
    for (int s = 0; s < G; ++s) tot[e] += cnt[(size_t)s * E + e];
  }
  int64_t gstart = 0;
  for (int e = 0; e < E; ++e) {
    int64_t run = gstart;
    for (int s = 0; s < G; ++s) {
      gpos[(size_t)s * E + e] = run;
      run += cnt[(size_t)s * E + e];
    }
    gstart += tot[e];
  }
  R = gstart;
  // Rank boundaries split the estimated GEMM cost evenly: every row costs 1,
  // every non-empty (expert, source) block of the global order kEpSegmentCost
  // more (it becomes a row segment of the grouped GEMMs) and every expert
  // kEpExpertCost more.  Splitting rows evenly instead leaves the rank with
  // the many light experts of a skewed routing well behind the rank with the
  // few heavy ones.  Each boundary stays within R/(4G) rows of the even row
  // split, so every rank computes between 1/2 and 3/2 of the mean rows (the
  // receive buffers hold 3/2).
  int64_t C = R;
  for (int e = 0; e < E; ++e) {
    bool any = false;
    for (int s = 0; s < G; ++s)
      if (cnt[(size_t)s * E + e] > 0) {
        C += kEpSegmentCost;
        any = true;
      }
    if (any) C += kEpExpertCost;
  }
  std::vector<int64_t> bound(G + 1);
  bound[0] = 0;
  bound[G] = R;
  {
    int d = 1;
    int64_t row = 0, cost = 0;  // position and cost before the current block
    for (int e = 0; e < E && d < G; ++e) {
      bool first = true;
      for (int s = 0; s < G && d < G; ++s) {
        const int64_t c = cnt[(size_t)s * E + e];
        if (c == 0) continue;
        const int64_t ov = kEpSegmentCost + (first ? kEpExpertCost : 0);
        first = false;
        // boundaries whose target cost falls inside this block
        while (d < G && C * d / G <= cost + ov + c) {
          const int64_t over = C * d / G - cost - ov;
          bound[d] = row + std::min<int64_t>(std::max<int64_t>(over, 0), c);
          ++d;
        }
        row += c;
        cost += ov + c;
      }
    }
    for (; d < G; ++d) bound[d] = R;
    const int64_t slack = R / (4 * G);
    for (int q = 1; q < G; ++q)
      bound[q] = std::min(std::max(bound[q], R * q / G - slack), R * q / G + slack);
  }
  const int64_t *gpos_r = &gpos[(size_t)r * E];
  for (int d = 0; d < G; ++d) {
    const int64_t lo = rows_below(mine, gpos_r, E, bound[d]);
    const int64_t hi = rows_below(mine, gpos_r, E, bound[d + 1]);
    p->send_off[d] = lo;
    p->send_cnt[d] = hi - lo;
  }
  int64_t roff = 0;
  std::vector<int64_t> first(G);
  for (int s = 0; s < G; ++s) {
    const int32_t *cs = cnt + (size_t)s * E;
    const int64_t *gs = &gpos[(size_t)s * E];
    first[s] = rows_below(cs, gs, E, bound[r]);
    const int64_t c = rows_below(cs, gs, E, bound[r + 1]) - first[s];
    p->recv_off[s] = roff;
    p->recv_cnt[s] = c;
    roff += c;
  }
  p->recv_rows = roff;
  int n = 0;
  for (int e = 0; e < E; ++e)
    for (int s = 0; s < G; ++s) {
      const int32_t *cs = cnt + (size_t)s * E;
      const int64_t *gs = &gpos[(size_t)s * E];
      const int64_t a = std::max(gs[e], bound[r]);
      const int64_t b = std::min(gs[e] + cs[e], bound[r + 1]);
      if (a >= b) continue;
      if (n >= B2_EP_MAX_SEGMENTS) return B2_ERR_INVALID;
      p->seg_off[n] = (int32_t)(p->recv_off[s] + rows_below(cs, gs, E, a) - first[s]);
      p->seg_cnt[n] = (int32_t)(b - a);
      p->seg_expert[n] = e;
      p->seg_source[n] = s;
      ++n;
    }
  p->num_segments = n;
  return B2_OK;
}

// ---------------------------------------------------------------- object
// Flags each rank receives: slot [kFlagDispatch*G + s] is written by rank s's
// copy engine after its rows landed in our receive buffer; slot
// [kFlagReturn*G + d] after rank d returned our rows into our sout.  Values are
// the forward's sequence number, so they never need resetting.
static constexpr int kFlagDispatch = 0, kFlagReturn = 1;

// The communicator of one or more layers.  A model's MoE layers share one:
// all of their collectives are issued on the model's stream in layer order,
// so every rank meets them in the same order.  When a layer aborts it (a lost
// peer), every layer that shares it sees `ok == false`.
struct EpComm {
  ncclComm_t comm = nullptr;  // count all-gather (the per-forward barrier) and set-up
  bool ok = false;
  int refs = 1;
};

struct b2_ep {
  b2_moe *moe = nullptr;
  int world = 1, rank = 0, mode = 0, E = 0, n_wexp = 0;
  EpComm *cm = nullptr;
  cudaStream_t st_d = nullptr, st_r = nullptr;  // copy-engine streams: dispatch / return
  std::vector<cudaEvent_t> ev_out;               // per exchange step
  cudaEvent_t ev_ready = nullptr, ev_ret = nullptr;
  cudaEvent_t ev_scan = nullptr, ev_cnt = nullptr;  // counts ready / count matrix on the host
  int64_t cap_rows = 0;
  void *recv_x = nullptr, *inter = nullptr, *out_recv = nullptr;
  uint64_t *flags = nullptr;                     // [2][world]
  uint64_t *d_seq = nullptr, *h_seq = nullptr;   // value the copy engines write into flags
  uint64_t seq = 0;
  std::vector<char *> peer_recv, peer_sout;      // IPC mappings of the peers' buffers
  std::vector<uint64_t *> peer_flags;
  int *d_wait_idx = nullptr, *h_wait_idx = nullptr;
  CUtensorMap tm_recv, tm_inter;
  int64_t inter_rows = 0;
  int pipeline = B2_EP_PIPE_FUSED;
  bool fused_ok = false;               // the device supports the fused pipeline's waits
  void **d_out_ptrs = nullptr;         // [world]: W2 destination by source rank: this
                                       // rank -> sout, a peer -> out_recv
  unsigned long long *d_chunk_done = nullptr;  // [kMaxGroups]: return-chunk counters
  std::vector<ReturnChunk> chunks;     // return chunks of the last forward
  cudaEvent_t ev_w2go = nullptr, ev_dsp = nullptr;
  cudaEvent_t ev_ag = nullptr;         // the count all-gather done (device side)
  int *d_ngroups = nullptr;            // [2]: group counts of a schedule built on the GPU
  int32_t *d_fsched = nullptr, *h_fsched = nullptr;  // fused schedules: W1||W3, then W2
  int32_t *d_cnt_all = nullptr, *h_cnt_all = nullptr;
  int32_t *d_sched = nullptr, *h_sched = nullptr;  // per source: counts|offsets|mtile|group_b
  std::vector<b2_ep_plan> plans;                   // every rank's plan of the last forward
  double timeout_s = 60.0;
  // timeline of the last forward while the layer's profiling is on
  std::vector<cudaEvent_t> tl_ev;
  std::vector<int> tl_tag;
  int tl_n = 0;
  double host_wait_ms = 0.0, host_enqueue_ms = 0.0;  // host side of the last forward
};

static constexpr int kSchedInts = 4 * (kMaxGroups + 1);
// a fused schedule: counts | C rows | m-tile prefix | expert | A rows | source | destination
static constexpr int kFusedSchedInts = kPairSchedArrays * (kMaxGroups + 1);
static_assert(kPairSchedArrays == kFusedSchedArrays && kSchedTileRows == kPairBM,
              "the fused schedule's layout is the CTA-pair kernel's");

// Sets every return-chunk counter far past any target (after W2 on the same
// stream), so that a copy-engine wait on a counter always ends even if W2
// aborted before counting all of its tiles.
static __global__ void release_counters_kernel(unsigned long long *counters, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) counters[i] = 1ull << 62;
}

// The fused pipeline's schedule in owner placement, built on the GPU from the
// all-gathered count matrix as soon as the all-gather completes, so W1||W3
// starts on the own rows without the host's round trip: W1||W3's and W2's
// group lists and counts (owner_fused_schedule, the function the host runs
// for its copies), the return-chunk counters reset, and the forward's
// sequence number for the copy engines' flag writes.  One block; one thread
// builds the lists from the matrix in shared memory.
static __global__ void owner_plan_kernel(const int32_t *cnt_all, int G, int r, int E, int nt2,
                                         int32_t *sched, int *ngroups,
                                         unsigned long long *chunk_done, uint64_t *seq_out,
                                         uint64_t seq) {
  __shared__ int32_t c[B2_EP_MAX_WORLD * kMaxExperts];
  for (int i = threadIdx.x; i < G * E; i += blockDim.x) c[i] = cnt_all[i];
  for (int i = threadIdx.x; i < kMaxGroups; i += blockDim.x) chunk_done[i] = 0ull;
  __syncthreads();
  if (threadIdx.x == 0) {
    int mt = 0;
    ngroups[0] = owner_fused_schedule(G, r, E, c, false, 0, kMaxGroups + 1, sched, &mt, nullptr,
                                      nullptr);
    ngroups[1] = owner_fused_schedule(G, r, E, c, true, nt2, kMaxGroups + 1,
                                      sched + kPairSchedArrays * (kMaxGroups + 1), &mt, nullptr,
                                      nullptr);
    *seq_out = seq;
  }
}

// Bounded wait until every rank d in `mask` has raised this rank's return
// flag (flags[ret0 + d] >= target), one thread per rank; gives up after
// timeout_ns recording kDevTimeoutPeer.  The ranks come as a bit mask (the
// world is at most 64), so nothing has to be uploaded for it.
static __global__ void wait_return_flags_kernel(const volatile uint64_t *flags, int ret0,
                                                uint64_t mask, uint64_t target,
                                                uint64_t timeout_ns, int *status) {
  const int d = threadIdx.x;
  if (d < 64 && ((mask >> d) & 1)) {
    const uint64_t t0 = globaltimer();
    while (flags[ret0 + d] < target) {
      if (globaltimer() - t0 > timeout_ns) {
        atomicCAS(status, 0, (int)kDevTimeoutPeer);
        break;
      }
      __nanosleep(200);
    }
  }
  __threadfence_system();
}

// cuStreamWaitValue64 / cuDeviceGetAttribute from the driver, looked up once
// through the runtime (the library links no driver library).
typedef CUresult (*WaitValue64Fn)(CUstream, CUdeviceptr, cuuint64_t, unsigned int);
typedef CUresult (*DevAttrFn)(int *, CUdevice_attribute, CUdevice);
static WaitValue64Fn ep_wait_value64() {
  static WaitValue64Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWaitValue64", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<WaitValue64Fn>(p);
  });
  return fn;
}
// Whether the current device can wait on 64-bit values in a stream (the
// fused pipeline's return copies need it).
static bool stream_wait64_supported() {
  if (!ep_wait_value64()) return false;
  void *p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuDeviceGetAttribute", &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return false;
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (reinterpret_cast<DevAttrFn>(p)(&v, CU_DEVICE_ATTRIBUTE_CAN_USE_64_BIT_STREAM_MEM_OPS,
                                     (CUdevice)dev) != CUDA_SUCCESS)
    return false;
  return v != 0;
}

// Bounded wait, on this GPU, for flags[idx[i]] >= target (one lane per flag).
// Gives up after timeout_ns, recording kDevTimeoutPeer in *status.  Launched
// with programmatic dependent launch between two GEMM stages, it lets the next
// stage's GEMM launch (and run its prologue) at once, and completes only after
// the flags and its predecessor in the stream: the GEMM's griddepcontrol.wait
// therefore orders it after both.
static __global__ void wait_flags_kernel(const volatile uint64_t *flags, const int *idx, int n,
                                         uint64_t target, uint64_t timeout_ns, int *status) {
  pdl_trigger();
  const int i = threadIdx.x;
  if (i < n) {
    const uint64_t t0 = globaltimer();
    while (flags[idx[i]] < target) {
      if (globaltimer() - t0 > timeout_ns) {
        atomicCAS(status, 0, (int)kDevTimeoutPeer);
        break;
      }
      __nanosleep(200);
    }
  }
  __threadfence_system();
  pdl_wait();
}

extern "C" b2_status b2_flag_wait(const uint64_t *flags, const int *idx, int n, uint64_t target,
                                  double timeout_s, int *status, b2_stream stream) {
  if (n < 0 || n > 1024 || (n > 0 && (!flags || !idx || !status)) || !(timeout_s > 0) ||
      timeout_s > 600)
    return B2_ERR_INVALID;
  if (n == 0) return B2_OK;
  wait_flags_kernel<<<1, 32 * ((n + 31) / 32), 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      flags, idx, n, target, (uint64_t)(timeout_s * 1e9), status);
  B2_LAUNCHED();
  return B2_OK;
}

extern "C" b2_status b2_ep_unique_id(void *id_out) {
  if (!id_out) return B2_ERR_INVALID;
  if (!nccl().ok) return B2_ERR_COMM;
  ncclUniqueId id;
  B2_NCCL(nccl().GetUniqueId(&id));
  memcpy(id_out, &id, sizeof(id));
  return B2_OK;
}

static void ep_abort(b2_ep *ep) {
  if (ep->cm->comm) nccl().CommAbort(ep->cm->comm);
  ep->cm->comm = nullptr;
  ep->cm->ok = false;
}

// Wait for `query` (a stream or an event) to report completion, with a
// bound; abort the communicator if a peer is lost.
template <typename Query>
static b2_status bounded_wait(b2_ep *ep, Query query) {
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    const cudaError_t q = query();
    if (q == cudaSuccess) return B2_OK;
    if (q != cudaErrorNotReady) {
      fprintf(stderr, "[b2moe] stream error: %s\n", cudaGetErrorString(q));
      return B2_ERR_CUDA;
    }
    ncclResult_t ae = ncclSuccess;
    if (nccl().CommGetAsyncError(ep->cm->comm, &ae) != ncclSuccess || ae != ncclSuccess) {
      ep_abort(ep);
      return B2_ERR_COMM;
    }
    const double el =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > ep->timeout_s) {
      fprintf(stderr, "[b2moe] rank %d: peers did not answer within %.1f s; aborting\n",
              ep->rank, ep->timeout_s);
      ep_abort(ep);
      return B2_ERR_COMM;
    }
    // The per-forward wait (count all-gather) normally ends within tens of
    // microseconds and the GPU may idle until it does: poll without sleeping
    // for the first milliseconds (a 20 us sleep costs 60-80 us with the
    // kernel's timer slack), then back off.
    if (el > 5e-3) std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

static b2_status bounded_sync(b2_ep *ep, cudaStream_t s) {
  return bounded_wait(ep, [s] { return cudaStreamQuery(s); });
}

extern "C" b2_status b2_ep_destroy(b2_ep *ep) {
  if (!ep) return B2_OK;
  if (ep->cm && ep->cm->ok && ep->world > 1 && ep->moe && ep->d_cnt_all) {
    // every rank stops using the others' memory before anyone unmaps it
    cudaStream_t s = ep->st_d;
    if (nccl().AllGather(ep->moe->counts, ep->d_cnt_all, ep->E, ncclInt32, ep->cm->comm, s) ==
        ncclSuccess)
      bounded_sync(ep, s);
  }
  if (ep->st_d) cudaStreamSynchronize(ep->st_d);
  if (ep->st_r) cudaStreamSynchronize(ep->st_r);
  for (char *p : ep->peer_recv)
    if (p) cudaIpcCloseMemHandle(p);
  for (char *p : ep->peer_sout)
    if (p) cudaIpcCloseMemHandle(p);
  for (uint64_t *p : ep->peer_flags)
    if (p) cudaIpcCloseMemHandle(p);
  if (ep->cm && --ep->cm->refs == 0) {
    if (ep->cm->comm) {
      if (ep->cm->ok)
        nccl().CommDestroy(ep->cm->comm);
      else
        nccl().CommAbort(ep->cm->comm);
    }
    delete ep->cm;
  }
  for (cudaEvent_t e : ep->ev_out) cudaEventDestroy(e);
  if (ep->ev_ready) cudaEventDestroy(ep->ev_ready);
  if (ep->ev_ret) cudaEventDestroy(ep->ev_ret);
  if (ep->ev_scan) cudaEventDestroy(ep->ev_scan);
  for (cudaEvent_t e : ep->tl_ev) cudaEventDestroy(e);
  if (ep->ev_cnt) cudaEventDestroy(ep->ev_cnt);
  if (ep->ev_w2go) cudaEventDestroy(ep->ev_w2go);
  if (ep->ev_dsp) cudaEventDestroy(ep->ev_dsp);
  if (ep->ev_ag) cudaEventDestroy(ep->ev_ag);
  if (ep->st_d) cudaStreamDestroy(ep->st_d);
  if (ep->st_r) cudaStreamDestroy(ep->st_r);
  if (ep->h_cnt_all) cudaFreeHost(ep->h_cnt_all);
  if (ep->h_sched) cudaFreeHost(ep->h_sched);
  if (ep->h_seq) cudaFreeHost(ep->h_seq);
  if (ep->h_wait_idx) cudaFreeHost(ep->h_wait_idx);
  if (ep->h_fsched) cudaFreeHost(ep->h_fsched);
  b2_moe_destroy(ep->moe);  // also frees the buffers registered with it
  delete ep;
  return B2_OK;
}

b2_status b2::ep_create_impl(const b2_moe_desc *desc, int world, int rank,
                            const void *unique_id, b2_ep *share, int mode,
                            const float *const *w1, const float *const *w2,
                            const float *const *w3, const float *gate, const float *bias,
                            int weights_on_host, b2_stream stream_, b2_ep **out) {
  if (!desc || (!unique_id && !share) || !out || world < 1 || world > B2_EP_MAX_WORLD ||
      rank < 0 || rank >= world)
    return B2_ERR_INVALID;
  if (share && (share->world != world || share->rank != rank)) return B2_ERR_INVALID;
  if (mode != B2_EP_OWNER && mode != B2_EP_BALANCED) return B2_ERR_INVALID;
  const int E = desc->num_experts;
  if (mode == B2_EP_OWNER && E % world != 0) return B2_ERR_INVALID;
  if (!nccl().ok) return B2_ERR_COMM;
  *out = nullptr;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  b2_ep *ep = new b2_ep();
  ep->world = world;
  ep->rank = rank;
  ep->mode = mode;
  ep->E = E;
  ep->n_wexp = mode == B2_EP_OWNER ? E / world : E;
  b2_status st = moe_create_impl(desc, ep->n_wexp, w1, w2, w3, gate, bias, weights_on_host,
                                 stream, false, &ep->moe);
  if (st != B2_OK) {
    delete ep;
    return st;
  }
  b2_moe *m = ep->moe;
  const int H = desc->hidden, Ip = m->Ip;
  const size_t es = m->tf32 ? 4 : 2;
  const int64_t local_rows = (int64_t)desc->max_tokens * desc->top_k;
  // receive-side rows; the inter buffer also holds the rank's own rows, which
  // are computed in place at their expert-sorted positions
  ep->cap_rows =
      mode == B2_EP_OWNER ? local_rows * world : local_rows + local_rows / 2 + world + 1;
  const int64_t inter_rows = std::max<int64_t>(ep->cap_rows, local_rows);
  ep->inter_rows = inter_rows;
  auto fail = [&](b2_status s) {
    b2_ep_destroy(ep);
    return s;
  };
  if ((st = moe_alloc(m, &ep->recv_x, es * ep->cap_rows * H)) != B2_OK) return fail(st);
  if ((st = moe_alloc(m, &ep->inter, es * inter_rows * Ip)) != B2_OK) return fail(st);
  if ((st = moe_alloc(m, &ep->out_recv, es * ep->cap_rows * H)) != B2_OK) return fail(st);
  if ((st = moe_alloc(m, (void **)&ep->flags, sizeof(uint64_t) * 2 * world)) != B2_OK)
    return fail(st);
  if ((st = moe_alloc(m, (void **)&ep->d_seq, sizeof(uint64_t))) != B2_OK) return fail(st);
  if ((st = moe_alloc(m, (void **)&ep->d_wait_idx, sizeof(int) * 2 * world)) != B2_OK)
    return fail(st);
  if ((st = moe_alloc(m, (void **)&ep->d_cnt_all, sizeof(int32_t) * world * kMaxExperts)) != B2_OK)
    return fail(st);
  if ((st = moe_alloc(m, (void **)&ep->d_sched, sizeof(int32_t) * kSchedInts * (world + 1))) !=
      B2_OK)
    return fail(st);
  if ((st = moe_alloc(m, (void **)&ep->d_fsched, sizeof(int32_t) * 2 * kFusedSchedInts)) != B2_OK)
    return fail(st);
  if ((st = moe_alloc(m, (void **)&ep->d_out_ptrs, sizeof(void *) * world)) != B2_OK)
    return fail(st);
  if ((st = moe_alloc(m, (void **)&ep->d_chunk_done, sizeof(unsigned long long) * kMaxGroups)) !=
      B2_OK)
    return fail(st);
  if ((st = moe_alloc(m, (void **)&ep->d_ngroups, sizeof(int) * 2)) != B2_OK) return fail(st);
  ep->fused_ok = stream_wait64_supported();
  if (!ep->fused_ok) ep->pipeline = B2_EP_PIPE_STAGED;
  if (cudaMallocHost(&ep->h_cnt_all, sizeof(int32_t) * world * kMaxExperts) != cudaSuccess ||
      cudaMallocHost(&ep->h_sched, sizeof(int32_t) * kSchedInts * (world + 1)) != cudaSuccess ||
      cudaMallocHost(&ep->h_seq, sizeof(uint64_t)) != cudaSuccess ||
      cudaMallocHost(&ep->h_wait_idx, sizeof(int) * 2 * world) != cudaSuccess ||
      cudaMallocHost(&ep->h_fsched, sizeof(int32_t) * 2 * kFusedSchedInts) != cudaSuccess)
    return fail(B2_ERR_CUDA);
  if (cudaMemsetAsync(ep->inter, 0, es * inter_rows * Ip, stream) != cudaSuccess ||
      cudaMemsetAsync(ep->flags, 0, sizeof(uint64_t) * 2 * world, stream) != cudaSuccess)
    return fail(B2_ERR_CUDA);
  const bool f = m->tf32;
  if (!make_tmap(&ep->tm_recv, ep->recv_x, f, H, ep->cap_rows, (uint64_t)H * es, kBM) ||
      !make_tmap(&ep->tm_inter, ep->inter, f, Ip, inter_rows, (uint64_t)Ip * es, kBM))
    return fail(B2_ERR_CUDA);
  if (cudaStreamCreateWithFlags(&ep->st_d, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ep->st_r, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&ep->ev_ready, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&ep->ev_ret, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&ep->ev_scan, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&ep->ev_cnt, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&ep->ev_w2go, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&ep->ev_dsp, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&ep->ev_ag, cudaEventDisableTiming) != cudaSuccess)
    return fail(B2_ERR_CUDA);
  ep->ev_out.resize(world, nullptr);
  for (int k = 0; k < world; ++k)
    if (cudaEventCreateWithFlags(&ep->ev_out[k], cudaEventDisableTiming) != cudaSuccess)
      return fail(B2_ERR_CUDA);
  if (cudaStreamSynchronize(stream) != cudaSuccess) return fail(B2_ERR_CUDA);
  if (share) {
    ep->cm = share->cm;
    ++ep->cm->refs;
    if (!ep->cm->ok) return fail(B2_ERR_COMM);
  } else {
    ep->cm = new EpComm();
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof(id));
    if (nccl().CommInitRank(&ep->cm->comm, world, id, rank) != ncclSuccess) {
      ep->cm->comm = nullptr;
      return fail(B2_ERR_COMM);
    }
    ep->cm->ok = true;
  }
  ep->plans.resize(world);
  // share IPC handles of the receive buffer, sout and the flag words
  ep->peer_recv.assign(world, nullptr);
  ep->peer_sout.assign(world, nullptr);
  ep->peer_flags.assign(world, nullptr);
  if (world > 1) {
    constexpr size_t kH = sizeof(cudaIpcMemHandle_t);
    std::vector<char> mine(3 * kH), all(3 * kH * world);
    if (cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t *>(&mine[0]), ep->recv_x) !=
            cudaSuccess ||
        cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t *>(&mine[kH]), m->sout) !=
            cudaSuccess ||
        cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t *>(&mine[2 * kH]), ep->flags) !=
            cudaSuccess)
      return fail(B2_ERR_CUDA);
    void *d_h = nullptr;
    if ((st = moe_alloc(m, &d_h, 3 * kH * world)) != B2_OK) return fail(st);
    if (cudaMemcpyAsync(static_cast<char *>(d_h) + 3 * kH * rank, mine.data(), 3 * kH,
                        cudaMemcpyHostToDevice, stream) != cudaSuccess)
      return fail(B2_ERR_CUDA);
    if (nccl().AllGather(static_cast<char *>(d_h) + 3 * kH * rank, d_h, 3 * kH, ncclUint8,
                         ep->cm->comm, stream) != ncclSuccess)
      return fail(B2_ERR_COMM);
    if (cudaMemcpyAsync(all.data(), d_h, 3 * kH * world, cudaMemcpyDeviceToHost, stream) !=
        cudaSuccess)
      return fail(B2_ERR_CUDA);
    if ((st = bounded_sync(ep, stream)) != B2_OK) return fail(st);
    for (int p = 0; p < world; ++p) {
      if (p == rank) continue;
      cudaIpcMemHandle_t h;
      void *ptr = nullptr;
      memcpy(&h, &all[3 * kH * p], kH);
      if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
        return fail(B2_ERR_CUDA);
      ep->peer_recv[p] = static_cast<char *>(ptr);
      memcpy(&h, &all[3 * kH * p + kH], kH);
      if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
        return fail(B2_ERR_CUDA);
      ep->peer_sout[p] = static_cast<char *>(ptr);
      memcpy(&h, &all[3 * kH * p + 2 * kH], kH);
      if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
        return fail(B2_ERR_CUDA);
      ep->peer_flags[p] = static_cast<uint64_t *>(ptr);
    }
  }
  // W2 destinations of the fused pipeline, by source rank: this rank's own
  // rows go to sout, a peer's rows to out_recv (returned by the copy engine)
  {
    std::vector<void *> outs(world);
    for (int p = 0; p < world; ++p) outs[p] = p == rank ? m->sout : ep->out_recv;
    if (cudaMemcpy(ep->d_out_ptrs, outs.data(), sizeof(void *) * world,
                   cudaMemcpyHostToDevice) != cudaSuccess)
      return fail(B2_ERR_CUDA);
  }
  *out = ep;
  return B2_OK;
}

extern "C" b2_status b2_ep_create(const b2_moe_desc *desc, int world, int rank,
                                  const void *unique_id, int mode, const float *const *w1,
                                  const float *const *w2, const float *const *w3,
                                  const float *gate, const float *bias, int weights_on_host,
                                  b2_stream stream, b2_ep **out) {
  if (!unique_id) return B2_ERR_INVALID;
  return ep_create_impl(desc, world, rank, unique_id, nullptr, mode, w1, w2, w3, gate, bias,
                        weights_on_host, stream, out);
}

// GEMM schedule of the segments that came from `src` (rows of the receive
// buffer), restricted to the source-relative rows [lo, hi); with `self_rows`
// the rank's own rows are addressed at their expert-sorted positions
// (self_base + row) instead.  Returns the number of segments.
static int fill_sched(const b2_ep_plan &p, int src, bool self_rows, int64_t self_base,
                      int64_t lo, int64_t hi, int32_t *h, int *mtiles) {
  int32_t *hc = h, *ho = h + (kMaxGroups + 1), *hm = ho + (kMaxGroups + 1),
          *hg = hm + (kMaxGroups + 1);
  int n = 0, mt = 0;
  for (int g = 0; g < p.num_segments; ++g) {
    if (p.seg_source[g] != src) continue;
    const int64_t a = std::max<int64_t>(p.seg_off[g] - p.recv_off[src], lo);
    const int64_t b = std::min<int64_t>(p.seg_off[g] - p.recv_off[src] + p.seg_cnt[g], hi);
    if (a >= b) continue;
    hc[n] = (int32_t)(b - a);
    ho[n] = (int32_t)(self_rows ? self_base + a : p.recv_off[src] + a);
    hg[n] = p.seg_expert[g];
    hm[n] = mt;
    mt += (int)((b - a + kPairBM - 1) / kPairBM);
    ++n;
  }
  hm[n] = mt;
  *mtiles = mt;
  return n;
}

// Schedule of one fused launch (every source's rows), into h (kFusedSchedInts
// ints).  W1||W3 (w2 = false): the own rows first -- A = sorted_x at their
// expert-sorted rows, so the GEMM starts at once -- then the sources in the
// order their rows arrive (rank s pushes to s+1 first, so r-1, r-2, ...), A =
// the receive buffer behind that source's flag; C = the receive-layout row
// (inter).  W2 (w2 = true): the remote sources first and the own rows last;
// A = the inter row; the own rows' results go to sout at their expert-sorted
// row (destination r), a peer's rows' results to out_recv at their
// receive-layout row (destination: the peer), grouped into return chunks of
// consecutive groups of one source (about kReturnChunkRows rows each) that
// the copy engine sends home as soon as their tiles are stored.  Within a
// source the groups keep the plan's expert order.  Returns the number of
// groups; *mtiles the 256-row tiles; `chunks` (may be null) the return chunks
// with their counter targets for W2's n_tiles output tiles per row block.
static int fill_fused(int G, int r, const b2_ep_plan *plans, bool w2, int n_tiles, int32_t *h,
                      int *mtiles, std::vector<ReturnChunk> *chunks) {
  constexpr int N1 = kMaxGroups + 1;
  const b2_ep_plan &p = plans[r];
  int32_t *hc = h, *ho = h + N1, *hm = h + 2 * N1, *hg = h + 3 * N1, *ha = h + 4 * N1,
          *hs = h + 5 * N1, *hd = h + 6 * N1, *hk = h + 7 * N1;
  if (chunks) chunks->clear();
  int n = 0, mt = 0, nchunk = 0;
  for (int k = 0; k < G; ++k) {
    const int src = w2 ? (k < G - 1 ? (r - 1 - k + 2 * G) % G : r) : (r - k + G) % G;
    ReturnChunk cur{-1, 0, 0, 0, 0};
    for (int g = 0; g < p.num_segments; ++g) {
      if (p.seg_source[g] != src) continue;
      const int64_t within = p.seg_off[g] - p.recv_off[src];
      const int64_t home = plans[src].send_off[r] + within;  // its row at the source
      const int tiles = (p.seg_cnt[g] + kPairBM - 1) / kPairBM;
      hc[n] = p.seg_cnt[g];
      hg[n] = p.seg_expert[g];
      hk[n] = -1;
      if (!w2) {
        ho[n] = p.seg_off[g];
        ha[n] = (int32_t)(src == r ? home : p.seg_off[g]);
        hs[n] = src == r ? -1 : src;
        hd[n] = 0;
      } else {
        ho[n] = (int32_t)(src == r ? home : p.seg_off[g]);
        ha[n] = p.seg_off[g];
        hs[n] = -1;
        hd[n] = src;
        if (src != r) {
          // a new chunk when none is open, the open one is full, or the rows
          // are not contiguous with it
          if (cur.src < 0 || cur.rows >= kReturnChunkRows || cur.row + cur.rows != p.seg_off[g]) {
            if (cur.src >= 0) {
              if (chunks) chunks->push_back(cur);
              ++nchunk;
            }
            cur = ReturnChunk{src, p.seg_off[g], home, 0, 0};
          }
          cur.rows += p.seg_cnt[g];
          cur.target += 8ull * (uint64_t)tiles * (uint64_t)n_tiles;  // 8 epilogue warps per tile
          hk[n] = nchunk;
        }
      }
      hm[n] = mt;
      mt += tiles;
      ++n;
    }
    if (cur.src >= 0) {
      if (chunks) chunks->push_back(cur);
      ++nchunk;
    }
  }
  hm[n] = mt;
  *mtiles = mt;
  return n;
}

extern "C" b2_status b2_ep_fused_schedule(int world, int rank, int num_experts, int mode,
                                          const int32_t *counts, int w2, int32_t *sched,
                                          int *groups, int *mtiles) {
  if (world < 1 || world > B2_EP_MAX_WORLD || rank < 0 || rank >= world || !counts || !sched ||
      !groups || !mtiles)
    return B2_ERR_INVALID;
  std::vector<b2_ep_plan> plans(world);
  for (int q = 0; q < world; ++q)
    B2_RETURN_IF(b2_ep_plan_compute(world, q, num_experts, mode, counts, &plans[q]));
  if (mode == B2_EP_OWNER) {
    *groups = owner_fused_schedule(world, rank, num_experts, counts, w2 != 0, 1, kMaxGroups + 1,
                                   sched, mtiles, nullptr, nullptr);
    return *groups < 0 ? B2_ERR_INVALID : B2_OK;
  }
  *groups = fill_fused(world, rank, plans.data(), w2 != 0, 1, sched, mtiles, nullptr);
  return B2_OK;
}

// W1||W3 of one fused launch over every source's rows.  ngroups_dev: the
// group count on the GPU (a schedule built there) instead of n1.
static b2_status launch_fused_w13(b2_ep *ep, cudaStream_t s, uint64_t timeout_ns, int n1,
                                  int mt1, const int *ngroups_dev) {
  b2_moe *m = ep->moe;
  const int G = ep->world, H = m->d.hidden, Ip = m->Ip;
  const bool f = m->tf32;
  constexpr int N1 = kMaxGroups + 1;
  const int32_t *d1 = ep->d_fsched;
  const int max_pairs = m->sms / 2;
  GemmArgs a1{};
  a1.counts = d1;
  a1.offsets = d1 + N1;
  a1.mtile_offsets = d1 + 2 * N1;
  a1.group_b = d1 + 3 * N1;
  a1.a_offsets = d1 + 4 * N1;
  a1.group_src = d1 + 5 * N1;
  a1.num_groups = n1;
  a1.num_groups_dev = ngroups_dev;
  a1.b_rows_per_group = 2 * Ip;
  a1.N = Ip;
  a1.num_n_tiles = Ip / 128;
  a1.num_k_blocks = f ? H / 32 : H / 64;
  a1.out = ep->inter;
  a1.ldo = Ip;
  a1.status = m->status;
  a1.flags = ep->flags + kFlagDispatch * G;
  a1.flag_target = ep->seq;
  a1.c_rows = ep->inter_rows;
  // every wait of the launch may last as long as a source's flag wait
  a1.wait_ns = timeout_ns + kWaitTimeoutNs;
  // a schedule built on the GPU: as many pairs as the device has (extra pairs
  // find no tile and leave at once)
  const int pairs1 =
      ngroups_dev ? max_pairs
                  : (int)std::min<long long>(max_pairs, (long long)mt1 * a1.num_n_tiles);
  if (!ngroups_dev && n1 == 0) return B2_OK;
  if (f)
    return launch_gemm_pair<kEpiSwiGLU, true, float>(m->tm_x, m->tm_w13_half, a1, pairs1, s,
                                                     &ep->tm_recv);
  return launch_gemm_pair<kEpiSwiGLU, false, __nv_bfloat16>(m->tm_x, m->tm_w13_half, a1, pairs1,
                                                            s, &ep->tm_recv);
}

// Owner placement, fused pipeline: once the count all-gather has completed
// on the GPU, one small kernel builds this rank's schedule (owner_plan_kernel)
// and W1||W3 starts on the own rows -- the host has not seen the counts yet.
static b2_status fused_w13_device_plan(b2_ep *ep, cudaStream_t s, uint64_t timeout_ns,
                                       const std::function<b2_status(int)> &tl) {
  b2_moe *m = ep->moe;
  const int nt2 = (m->d.hidden + kBN - 1) / kBN;
  B2_CUDA(cudaStreamWaitEvent(s, ep->ev_ag, 0));
  owner_plan_kernel<<<1, 128, 0, s>>>(ep->d_cnt_all, ep->world, ep->rank, ep->E, nt2,
                                      ep->d_fsched, ep->d_ngroups, ep->d_chunk_done, ep->d_seq,
                                      ep->seq);
  B2_LAUNCHED();
  // schedule, chunk counters and sequence number are in place
  B2_CUDA(cudaEventRecord(ep->ev_w2go, s));
  B2_RETURN_IF(tl(B2_EP_TL_PLANNED));
  return launch_fused_w13(ep, s, timeout_ns, 0, 0, ep->d_ngroups);
}

// The fused exchange + expert GEMMs (B2_EP_PIPE_FUSED), from the host's plan
// to the moment every source has returned this rank's rows.  dplan: the
// schedule was built on the GPU and W1||W3 launched already
// (fused_w13_device_plan); the host builds the same lists for its copies.
static b2_status fused_gemms(b2_ep *ep, cudaStream_t s, uint64_t timeout_ns,
                             const std::function<b2_status(int)> &tl, bool dplan) {
  b2_moe *m = ep->moe;
  const int G = ep->world, r = ep->rank, H = m->d.hidden, Ip = m->Ip;
  const bool f = m->tf32;
  const b2_ep_plan &p = ep->plans[r];
  const size_t rb = (f ? 4 : 2) * (size_t)H;
  const int nt2 = (H + kBN - 1) / kBN;
  int mt1 = 0, mt2 = 0, n1 = 0, n2 = 0;
  if (ep->mode == B2_EP_OWNER) {
    int nch = 0;
    ep->chunks.resize(kMaxGroups);
    n1 = owner_fused_schedule(G, r, ep->E, ep->h_cnt_all, false, 0, kMaxGroups + 1,
                              ep->h_fsched, &mt1, nullptr, nullptr);
    n2 = owner_fused_schedule(G, r, ep->E, ep->h_cnt_all, true, nt2, kMaxGroups + 1,
                              ep->h_fsched + kFusedSchedInts, &mt2, ep->chunks.data(), &nch);
    if (n1 < 0 || n2 < 0) return B2_ERR_INVALID;
    ep->chunks.resize(nch);
  } else {
    n1 = fill_fused(G, r, ep->plans.data(), false, 0, ep->h_fsched, &mt1, nullptr);
    n2 = fill_fused(G, r, ep->plans.data(), true, nt2, ep->h_fsched + kFusedSchedInts, &mt2,
                    &ep->chunks);
  }
  const int nchunks = (int)ep->chunks.size();
  uint64_t ret_mask = 0;  // ranks that return rows of ours
  for (int d = 0; d < G; ++d)
    if (d != r && p.send_cnt[d] > 0) ret_mask |= 1ull << d;
  if (!dplan) {
    B2_CUDA(cudaMemcpyAsync(ep->d_fsched, ep->h_fsched, sizeof(int32_t) * 2 * kFusedSchedInts,
                            cudaMemcpyHostToDevice, s));
    B2_CUDA(cudaMemcpyAsync(ep->d_seq, ep->h_seq, sizeof(uint64_t), cudaMemcpyHostToDevice, s));
    // every return chunk's counter starts at zero (before W1||W3, so that
    // W1||W3 and W2 follow each other directly and overlap by programmatic
    // launch)
    if (nchunks > 0)
      B2_CUDA(cudaMemsetAsync(ep->d_chunk_done, 0, sizeof(unsigned long long) * nchunks, s));
    B2_CUDA(cudaEventRecord(ep->ev_w2go, s));
    B2_RETURN_IF(tl(B2_EP_TL_PLANNED));
    B2_RETURN_IF(launch_fused_w13(ep, s, timeout_ns, n1, mt1, nullptr));
  }
  // dispatch on the copy engine (the GEMM is running on the own rows
  // meanwhile): step k pushes the rows for rank r+k into its receive buffer,
  // then our sequence number into its flag slot.  ev_w2go follows the scatter
  // and the sequence number's update.
  const char *sx = reinterpret_cast<const char *>(m->sorted_x);
  B2_CUDA(cudaStreamWaitEvent(ep->st_d, ep->ev_w2go, 0));
  for (int k = 1; k < G; ++k) {
    const int to = (r + k) % G;
    if (p.send_cnt[to])
      B2_CUDA(cudaMemcpyAsync(ep->peer_recv[to] + ep->plans[to].recv_off[r] * rb,
                              sx + p.send_off[to] * rb, p.send_cnt[to] * rb,
                              cudaMemcpyDeviceToDevice, ep->st_d));
    B2_CUDA(cudaMemcpyAsync(ep->peer_flags[to] + kFlagDispatch * G + r, ep->d_seq,
                            sizeof(uint64_t), cudaMemcpyDeviceToDevice, ep->st_d));
  }
  B2_RETURN_IF(tl(B2_EP_TL_W13_DONE));
  prof_mark(m, s);  // W2 starts

  // W2: own rows into sout, a peer's rows into out_recv (local stores only)
  constexpr int N1 = kMaxGroups + 1;
  const int32_t *d2 = ep->d_fsched + kFusedSchedInts;
  GemmArgs a2{};
  a2.counts = d2;
  a2.offsets = d2 + N1;
  a2.mtile_offsets = d2 + 2 * N1;
  a2.group_b = d2 + 3 * N1;
  a2.a_offsets = d2 + 4 * N1;
  a2.group_dst = d2 + 6 * N1;
  a2.group_chunk = d2 + 7 * N1;
  a2.chunk_done = ep->d_chunk_done;
  a2.out_ptrs = ep->d_out_ptrs;
  a2.num_groups = n2;
  a2.num_groups_dev = dplan ? ep->d_ngroups + 1 : nullptr;
  a2.b_rows_per_group = H;
  a2.N = H;
  a2.num_n_tiles = nt2;
  a2.num_k_blocks = f ? Ip / 32 : Ip / 64;
  a2.out = m->sout;
  a2.ldo = H;
  a2.status = m->status;
  // rows of the larger destination: out_recv (a peer's rows, receive layout)
  // or sout (own rows, expert-sorted)
  a2.c_rows = std::max<int64_t>(ep->cap_rows, (int64_t)m->d.max_tokens * m->d.top_k);
  const int pairs2 = (int)std::min<long long>(m->sms / 2, (long long)mt2 * a2.num_n_tiles);
  if (n2 > 0) {
    if (f)
      B2_RETURN_IF(
          (launch_gemm_pair<kEpiStore, true, float>(ep->tm_inter, m->tm_w2_half, a2, pairs2, s)));
    else
      B2_RETURN_IF((launch_gemm_pair<kEpiStore, false, __nv_bfloat16>(ep->tm_inter,
                                                                      m->tm_w2_half, a2, pairs2,
                                                                      s)));
  }
  if (nchunks > 0) {
    // once W2 has finished -- normally or by an abort that left tiles
    // uncounted -- every chunk counter is past its target, so no wait of the
    // return stream below can outlive this forward's kernels
    release_counters_kernel<<<1, 256, 0, s>>>(ep->d_chunk_done, nchunks);
    B2_LAUNCHED();
  }
  B2_RETURN_IF(tl(B2_EP_TL_W2_DONE));

  // return: each chunk goes home on the copy engine as soon as its counter
  // says its rows are stored; a source's flag follows its last chunk
  const char *ro = reinterpret_cast<const char *>(ep->out_recv);
  B2_CUDA(cudaStreamWaitEvent(ep->st_r, ep->ev_w2go, 0));
  for (int d = 0; d < G; ++d) {  // sources without rows here: nothing to wait for
    if (d == r || p.recv_cnt[d] > 0) continue;
    B2_CUDA(cudaMemcpyAsync(ep->peer_flags[d] + kFlagReturn * G + r, ep->d_seq, sizeof(uint64_t),
                            cudaMemcpyDeviceToDevice, ep->st_r));
  }
  for (int c = 0; c < nchunks; ++c) {
    const ReturnChunk &ch = ep->chunks[c];
    CUresult cr = ep_wait_value64()(reinterpret_cast<CUstream>(ep->st_r),
                                     reinterpret_cast<CUdeviceptr>(ep->d_chunk_done + c),
                                     ch.target, CU_STREAM_WAIT_VALUE_GEQ);
    if (cr != CUDA_SUCCESS) {
      fprintf(stderr, "[b2moe] cuStreamWaitValue64 failed (%d)\n", (int)cr);
      return B2_ERR_CUDA;
    }
    B2_CUDA(cudaMemcpyAsync(ep->peer_sout[ch.src] + ch.home * rb, ro + ch.row * rb, ch.rows * rb,
                            cudaMemcpyDeviceToDevice, ep->st_r));
    if (c + 1 == nchunks || ep->chunks[c + 1].src != ch.src)
      B2_CUDA(cudaMemcpyAsync(ep->peer_flags[ch.src] + kFlagReturn * G + r, ep->d_seq,
                              sizeof(uint64_t), cudaMemcpyDeviceToDevice, ep->st_r));
  }
  if (ret_mask) {
    wait_return_flags_kernel<<<1, 64, 0, s>>>(ep->flags, kFlagReturn * G, ret_mask, ep->seq,
                                             timeout_ns, m->status);
    B2_LAUNCHED();
  }
  if (G > 1) {
    // the copy streams are done before the next forward rewrites sorted_x,
    // out_recv or the chunk counters
    B2_CUDA(cudaEventRecord(ep->ev_ret, ep->st_r));
    B2_CUDA(cudaStreamWaitEvent(s, ep->ev_ret, 0));
    B2_CUDA(cudaEventRecord(ep->ev_dsp, ep->st_d));
    B2_CUDA(cudaStreamWaitEvent(s, ep->ev_dsp, 0));
  }
  B2_RETURN_IF(tl(B2_EP_TL_RETURNED));
  return B2_OK;
}

b2_status b2::ep_forward_impl(b2_ep *ep, const float *x, float *y, int T, cudaStream_t s,
                             bool accumulate) {
  if (!ep || T < 0 || (T > 0 && (!x || !y || !aligned16(x) || !aligned16(y))))
    return B2_ERR_INVALID;
  if (!ep->cm->ok) return B2_ERR_COMM;
  b2_moe *m = ep->moe;
  if (T > m->d.max_tokens) return B2_ERR_CAPACITY;
  const int E = ep->E, G = ep->world, r = ep->rank, H = m->d.hidden;
  const size_t rb = (m->tf32 ? 4 : 2) * (size_t)H;  // bytes per row
  const uint64_t timeout_ns = (uint64_t)(ep->timeout_s * 1e9);
  const std::function<b2_status(int)> tl = [&](int tag) -> b2_status {
    if (!m->profile) return B2_OK;
    if (ep->tl_n >= (int)ep->tl_ev.size()) {
      cudaEvent_t e = nullptr;
      B2_CUDA(cudaEventCreate(&e));
      ep->tl_ev.push_back(e);
      ep->tl_tag.push_back(0);
    }
    ep->tl_tag[ep->tl_n] = tag;
    B2_CUDA(cudaEventRecord(ep->tl_ev[ep->tl_n++], s));
    return B2_OK;
  };
  ep->tl_n = 0;
  B2_RETURN_IF(tl(B2_EP_TL_START));

  // 1. local routing and scan (also for T == 0: the rank still takes part in
  // the exchange)
  if (T > 0) {
    B2_RETURN_IF(moe_route_stage(m, x, T, nullptr, s, false));
  } else {
    for (int i = 0; i < 3; ++i) prof_mark(m, s);  // keep the stage-event layout
    B2_CUDA(cudaMemsetAsync(m->counts, 0, sizeof(int) * E, s));
  }
  // 2. count matrix -> host on the dispatch stream while `s` runs the scatter,
  // so the host round trip hides behind it.  The all-gather starts after this
  // rank's scan, which follows its previous forward on `s`; so once it has
  // completed, every rank's previous forward is done and every peer buffer
  // written below is free for this forward.
  B2_CUDA(cudaEventRecord(ep->ev_scan, s));
  B2_CUDA(cudaStreamWaitEvent(ep->st_d, ep->ev_scan, 0));
  B2_NCCL(nccl().AllGather(m->counts, ep->d_cnt_all, E, ncclInt32, ep->cm->comm, ep->st_d));
  B2_CUDA(cudaEventRecord(ep->ev_ag, ep->st_d));
  B2_CUDA(cudaMemcpyAsync(ep->h_cnt_all, ep->d_cnt_all, sizeof(int32_t) * G * E,
                          cudaMemcpyDeviceToHost, ep->st_d));
  B2_CUDA(cudaEventRecord(ep->ev_cnt, ep->st_d));
  if (T > 0) B2_RETURN_IF(moe_scatter_stage(m, x, T, s));
  prof_mark(m, s);  // exchange + expert GEMMs start
  B2_RETURN_IF(tl(B2_EP_TL_SCATTERED));
  // fused pipeline, owner placement: W1||W3 is scheduled on the GPU and
  // launched now; the host's round trip below only sizes the copies
  const bool dplan = ep->pipeline == B2_EP_PIPE_FUSED && ep->fused_ok && ep->mode == B2_EP_OWNER;
  if (dplan) {
    ep->seq += 1;
    *ep->h_seq = ep->seq;
    B2_RETURN_IF(fused_w13_device_plan(ep, s, timeout_ns, tl));
  }
  const auto h0 = std::chrono::steady_clock::now();
  {
    cudaEvent_t ev = ep->ev_cnt;
    B2_RETURN_IF(bounded_wait(ep, [ev] { return cudaEventQuery(ev); }));
  }
  const auto h1 = std::chrono::steady_clock::now();
  for (int q = 0; q < G; ++q)
    B2_RETURN_IF(b2_ep_plan_compute(G, q, E, ep->mode, ep->h_cnt_all, &ep->plans[q]));
  const b2_ep_plan &p = ep->plans[r];
  if (p.recv_rows > ep->cap_rows) return B2_ERR_CAPACITY;
  if (!dplan) {
    ep->seq += 1;
    *ep->h_seq = ep->seq;
  }
  if (ep->pipeline == B2_EP_PIPE_FUSED && ep->fused_ok) {
    B2_RETURN_IF(fused_gemms(ep, s, timeout_ns, tl, dplan));
    // 6. local k-ordered combine
    if (T > 0) {
      B2_RETURN_IF(moe_combine_stage(m, y, T, s, accumulate));
    } else {
      for (int i = 0; i < 2; ++i) prof_mark(m, s);
    }
    ep->host_wait_ms = std::chrono::duration<double, std::milli>(h1 - h0).count();
    ep->host_enqueue_ms =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - h1).count();
    return tl(B2_EP_TL_DONE);
  }
  // schedule slots: one per source; the rank's own rows are split in two
  // (slot r before the remote steps, slot G after them) so that the return of
  // the last remote step overlaps the second half
  const int64_t self_rows = p.recv_cnt[r];
  const int64_t self_b = G > 1 ? std::min<int64_t>(self_rows / 2, p.recv_cnt[(r + 1) % G]) : 0;
  std::vector<int> nseg(G + 1), mtiles(G + 1);
  for (int src = 0; src < G; ++src) {
    const int64_t hi = src == r ? self_rows - self_b : INT64_MAX;
    nseg[src] = fill_sched(p, src, src == r, p.send_off[r], 0, hi,
                           ep->h_sched + (size_t)src * kSchedInts, &mtiles[src]);
  }
  nseg[G] = fill_sched(p, r, true, p.send_off[r], self_rows - self_b, self_rows,
                       ep->h_sched + (size_t)G * kSchedInts, &mtiles[G]);
  int nwait_ret = 0;
  for (int d = 0; d < G; ++d)
    if (d != r && p.send_cnt[d] > 0) ep->h_wait_idx[G + nwait_ret++] = kFlagReturn * G + d;
  B2_CUDA(cudaMemcpyAsync(ep->d_sched, ep->h_sched, sizeof(int32_t) * kSchedInts * (G + 1),
                          cudaMemcpyHostToDevice, s));
  B2_CUDA(cudaMemcpyAsync(ep->d_seq, ep->h_seq, sizeof(uint64_t), cudaMemcpyHostToDevice, s));
  for (int src = 0; src < G; ++src) ep->h_wait_idx[src] = kFlagDispatch * G + src;
  B2_CUDA(cudaMemcpyAsync(ep->d_wait_idx, ep->h_wait_idx, sizeof(int) * 2 * G,
                          cudaMemcpyHostToDevice, s));
  B2_CUDA(cudaEventRecord(ep->ev_ready, s));
  B2_RETURN_IF(tl(B2_EP_TL_PLANNED));

  auto sched_of = [&](int src) {
    GemmSched sc;
    int32_t *d = ep->d_sched + (size_t)src * kSchedInts;
    sc.counts = d;
    sc.offsets = d + (kMaxGroups + 1);
    sc.mtile_offsets = d + 2 * (kMaxGroups + 1);
    sc.group_b = d + 3 * (kMaxGroups + 1);
    sc.num_groups = nseg[src];
    sc.mtiles_upper_bound = mtiles[src];
    return sc;
  };

  // 3. first part of the own rows, in place (sorted_x -> inter -> sout), while
  // rows travel.  Launched before the host enqueues the 2(G-1) dispatch
  // copies, which wait on ev_ready either way, so the GPU does not idle while
  // the host issues them.
  if (nseg[r] > 0)
    B2_RETURN_IF(moe_gemm_stage(m, m->tm_x, ep->tm_inter, ep->inter, m->sout, sched_of(r), s,
                                false));
  B2_RETURN_IF(tl(B2_EP_TL_OWN_FIRST));
  // 4. dispatch on the copy engine: step k pushes the rows for rank r+k into
  // its receive buffer, then our sequence number into its flag slot
  const char *sx = reinterpret_cast<const char *>(m->sorted_x);
  B2_CUDA(cudaStreamWaitEvent(ep->st_d, ep->ev_ready, 0));
  for (int k = 1; k < G; ++k) {
    const int to = (r + k) % G;
    if (p.send_cnt[to])
      B2_CUDA(cudaMemcpyAsync(ep->peer_recv[to] + ep->plans[to].recv_off[r] * rb,
                              sx + p.send_off[to] * rb, p.send_cnt[to] * rb,
                              cudaMemcpyDeviceToDevice, ep->st_d));
    B2_CUDA(cudaMemcpyAsync(ep->peer_flags[to] + kFlagDispatch * G + r, ep->d_seq,
                            sizeof(uint64_t), cudaMemcpyDeviceToDevice, ep->st_d));
  }
  // 5. per step: wait for the rows of rank r-k, expert GEMMs, return them
  const char *ro = reinterpret_cast<const char *>(ep->out_recv);
  for (int k = 1; k < G; ++k) {
    const int from = (r - k + G) % G;
    if (p.recv_cnt[from] > 0) {
      B2_RETURN_IF(launch_pdl(wait_flags_kernel, dim3(1), dim3(32), 0, s,
                              (const volatile uint64_t *)ep->flags,
                              (const int *)(ep->d_wait_idx + from), 1, ep->seq, timeout_ns,
                              m->status));
      B2_RETURN_IF(tl(B2_EP_TL_ARRIVED));
      B2_RETURN_IF(moe_gemm_stage(m, ep->tm_recv, ep->tm_inter, ep->inter, ep->out_recv,
                                  sched_of(from), s, false));
      B2_RETURN_IF(tl(B2_EP_TL_REMOTE_DONE));
    }
    B2_CUDA(cudaEventRecord(ep->ev_out[k], s));
    B2_CUDA(cudaStreamWaitEvent(ep->st_r, ep->ev_out[k], 0));
    if (p.recv_cnt[from])
      B2_CUDA(cudaMemcpyAsync(ep->peer_sout[from] + ep->plans[from].send_off[r] * rb,
                              ro + p.recv_off[from] * rb, p.recv_cnt[from] * rb,
                              cudaMemcpyDeviceToDevice, ep->st_r));
    B2_CUDA(cudaMemcpyAsync(ep->peer_flags[from] + kFlagReturn * G + r, ep->d_seq,
                            sizeof(uint64_t), cudaMemcpyDeviceToDevice, ep->st_r));
  }
  // second part of the own rows while the last results travel back
  if (nseg[G] > 0)
    B2_RETURN_IF(moe_gemm_stage(m, m->tm_x, ep->tm_inter, ep->inter, m->sout, sched_of(G), s,
                                false));
  B2_RETURN_IF(tl(B2_EP_TL_OWN_SECOND));
  prof_mark(m, s);  // expert GEMMs done; waiting for returns
  if (nwait_ret > 0) {
    wait_flags_kernel<<<1, 32 * ((nwait_ret + 31) / 32), 0, s>>>(
        ep->flags, ep->d_wait_idx + G, nwait_ret, ep->seq, timeout_ns, m->status);
    B2_LAUNCHED();
  }
  if (G > 1) {
    // our own copy streams are done before the next forward reuses the sources
    B2_CUDA(cudaEventRecord(ep->ev_ret, ep->st_r));
    B2_CUDA(cudaStreamWaitEvent(s, ep->ev_ret, 0));
  }
  B2_RETURN_IF(tl(B2_EP_TL_RETURNED));
  // 6. local k-ordered combine
  if (T > 0) {
    B2_RETURN_IF(moe_combine_stage(m, y, T, s, accumulate));
  } else {
    for (int i = 0; i < 2; ++i) prof_mark(m, s);
  }
  ep->host_wait_ms = std::chrono::duration<double, std::milli>(h1 - h0).count();
  ep->host_enqueue_ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - h1).count();
  return tl(B2_EP_TL_DONE);
}

extern "C" b2_status b2_ep_forward(b2_ep *ep, const float *x, float *y, int T,
                                   b2_stream stream) {
  return ep_forward_impl(ep, x, y, T, reinterpret_cast<cudaStream_t>(stream), false);
}

extern "C" b2_status b2_ep_profile_timeline(b2_ep *ep, int max, int *tags, float *ms, int *n) {
  if (!ep || max < 0 || !n || (max > 0 && (!tags || !ms))) return B2_ERR_INVALID;
  int k = std::min(max, ep->tl_n);
  if (ep->tl_n > 0) B2_CUDA(cudaEventSynchronize(ep->tl_ev[ep->tl_n - 1]));
  for (int i = 0; i < k; ++i) {
    tags[i] = ep->tl_tag[i];
    ms[i] = 0.0f;
    if (i > 0) B2_CUDA(cudaEventElapsedTime(&ms[i], ep->tl_ev[0], ep->tl_ev[i]));
  }
  if (ep->tl_n > 0 && k + 2 <= max) {
    tags[k] = B2_EP_TL_HOST_WAIT;
    ms[k++] = (float)ep->host_wait_ms;
    tags[k] = B2_EP_TL_HOST_ENQUEUE;
    ms[k++] = (float)ep->host_enqueue_ms;
  }
  *n = k;
  return B2_OK;
}

extern "C" b2_status b2_ep_set_pipeline(b2_ep *ep, int pipeline) {
  if (!ep || (pipeline != B2_EP_PIPE_FUSED && pipeline != B2_EP_PIPE_STAGED))
    return B2_ERR_INVALID;
  if (pipeline == B2_EP_PIPE_FUSED && !ep->fused_ok) {
    fprintf(stderr, "[b2moe] the fused pipeline needs 64-bit stream waits, which this device "
                    "does not offer\n");
    return B2_ERR_NO_DEVICE;
  }
  ep->pipeline = pipeline;
  return B2_OK;
}

extern "C" b2_status b2_ep_set_timeout(b2_ep *ep, double seconds) {
  if (!ep || !(seconds > 0)) return B2_ERR_INVALID;
  ep->timeout_s = seconds;
  return B2_OK;
}

extern "C" b2_status b2_ep_last_plan(const b2_ep *ep, b2_ep_plan *plan) {
  if (!ep || !plan) return B2_ERR_INVALID;
  *plan = ep->plans.empty() ? b2_ep_plan{} : ep->plans[ep->rank];
  return B2_OK;
}

extern "C" b2_moe *b2_ep_layer(b2_ep *ep) { return ep ? ep->moe : nullptr; }
