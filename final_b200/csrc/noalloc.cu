// noalloc.cu -- the routing step of the MoE layer for callers that cannot
// allocate device memory.
//
// Some callers of this library may not call cudaMalloc on the path that routes
// tokens: an inference server that plans every device byte at start-up and
// must not allocate afterwards (cudaMalloc and cudaFree synchronise the device
// and can fail under memory pressure in the middle of a request), or a host
// integration whose allocator is owned by someone else.  b2_moe_route_noalloc
// gives them the routing step (router logits, sigmoid top-k, expert counts and
// offsets, token -> slot map) with all of its scratch in a file-scope
// __device__ array instead of cudaMalloc'ed buffers.  The caller still passes
// its inputs and outputs.
//
// The scratch array is a fixed 1 MiB that every GPU which loads the library
// holds until the process exits; calls whose sizes exceed it are rejected.
// All calls share the one array, so calls that overlap on the GPU (on two
// streams at once, or from two host threads) race and must not be issued.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/b2moe.h"
#include "moe_kernels.cuh"

using namespace b2;

namespace {

constexpr int kNoAllocMaxHidden = 4096;
constexpr int kNoAllocMaxTokens = 65536;
constexpr int kNoAllocMaxBlocks = kNoAllocMaxTokens / kRouteTB;  // 2048

// layout of the scratch array (bytes)
constexpr size_t kGateTBytes = sizeof(float) * kNoAllocMaxHidden * kMaxExperts;        // 512 KB
constexpr size_t kBlockCountsBytes = sizeof(int) * kNoAllocMaxBlocks * kMaxExperts;    // 256 KB
constexpr size_t kBlockBaseBytes = kBlockCountsBytes;                                   // 256 KB
constexpr size_t kTileOffBytes = 256;
constexpr size_t kScratchBytes = kGateTBytes + kBlockCountsBytes + kBlockBaseBytes + kTileOffBytes;

constexpr int kMaxDevices = 64;

}  // namespace

// The scratch itself.  In host code this name is only a host-side stand-in:
// its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_route_scratch[kScratchBytes];

namespace {

std::mutex g_setup_mu;
void *g_scratch_ptr[kMaxDevices] = {};

// First call on a device (with that device current): look up the device
// address of g_route_scratch.  Returns nullptr on failure.  The address is
// cached for the life of the process: a cudaDeviceReset unloads the module
// and invalidates it (documented in include/b2moe.h).
unsigned char *scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    cudaError_t rc = cudaGetSymbolAddress(&p, g_route_scratch);
    if (rc != cudaSuccess) {
      fprintf(stderr, "[b2moe] cudaGetSymbolAddress(route scratch) failed on device %d: %s\n",
              dev, cudaGetErrorString(rc));
      return nullptr;
    }
    g_scratch_ptr[dev] = p;
  }
  return static_cast<unsigned char *>(g_scratch_ptr[dev]);
}

}  // namespace

extern "C" b2_status b2_moe_route_noalloc(const float *x, const float *gate, const float *bias,
                                          int num_tokens, int hidden, int num_experts,
                                          int top_k, float routed_scale, int32_t *topk_idx,
                                          float *topk_w, int32_t *counts, int32_t *offsets,
                                          int32_t *token_slot, b2_stream stream_) {
  const int T = num_tokens, H = hidden, E = num_experts, K = top_k;
  if (T < 0 || H <= 0 || H % 64 != 0 || E < 1 || E > kMaxExperts || K < 1 || K > kMaxTopK ||
      K > E || !gate || (T > 0 && (!x || !topk_idx || !topk_w || !token_slot)) || !counts ||
      !offsets)
    return B2_ERR_INVALID;
  // route_kernel reads x rows in 16-byte cp.async pieces
  if (T > 0 && (reinterpret_cast<uintptr_t>(x) & 15)) return B2_ERR_INVALID;
  if (T > kNoAllocMaxTokens || H > kNoAllocMaxHidden) {
    fprintf(stderr,
            "[b2moe] b2_moe_route_noalloc: %d tokens x hidden %d exceeds the fixed scratch "
            "(at most %d tokens, hidden at most %d)\n",
            T, H, kNoAllocMaxTokens, kNoAllocMaxHidden);
    return B2_ERR_CAPACITY;
  }
  unsigned char *base = scratch_for_current_device();
  if (!base) return B2_ERR_CUDA;
  float *gateT = reinterpret_cast<float *>(base);
  int *block_counts = reinterpret_cast<int *>(base + kGateTBytes);
  int *block_base = reinterpret_cast<int *>(base + kGateTBytes + kBlockCountsBytes);
  int *tile_off = reinterpret_cast<int *>(base + kGateTBytes + kBlockCountsBytes + kBlockBaseBytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream_);

  // Every scratch word a kernel reads is written earlier in the same call
  // (gateT by the pack, block_counts by route, block_base / tile_off by scan),
  // so nothing left over from the previous call is ever read.
  if (T == 0) {
    if (cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, s) != cudaSuccess ||
        cudaMemsetAsync(offsets, 0, sizeof(int32_t) * E, s) != cudaSuccess)
      return B2_ERR_CUDA;
    return B2_OK;
  }
  pack_gate_kernel<<<(H * kMaxExperts + 255) / 256, 256, 0, s>>>(gate, E, H, gateT);
  if (cudaGetLastError() != cudaSuccess) return B2_ERR_CUDA;
  const int nb = (T + kRouteTB - 1) / kRouteTB;
  route_kernel<<<nb, kRouteThreads, 0, s>>>(x, gateT, bias, T, H, E, K, routed_scale, topk_idx,
                                            topk_w, block_counts, nullptr);
  if (cudaGetLastError() != cudaSuccess) return B2_ERR_CUDA;
  scan_kernel<<<1, 1024, 0, s>>>(block_counts, nb, E, 128, counts, offsets, tile_off, block_base);
  if (cudaGetLastError() != cudaSuccess) return B2_ERR_CUDA;
  // slot bookkeeping only: hidden 0 skips the row copy
  scatter_kernel<__nv_bfloat16><<<nb, scatter_threads(K), 0, s>>>(x, topk_idx, topk_w, block_base, T, 0, E, K,
                                                      nullptr, token_slot, nullptr, nullptr,
                                                      nullptr);
  if (cudaGetLastError() != cudaSuccess) return B2_ERR_CUDA;
  return B2_OK;
}
