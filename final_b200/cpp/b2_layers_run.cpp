// b2_layers_run.cpp -- drives the C++ drop-in layers the way the reference's
// DecoderLayer::forward_gpu does (src/layer.cu:1908-1914): construct by layer
// index / tensor names, init_gpu(), forward_gpu() on device fp32 buffers.
// Used by the parity tests to exercise the C++ boundary end to end.
//
//   b2_layers_run moe <weights_dir> <layer_idx> <tokens> <x.f32> <y.f32> [bf16|tf32]
//   b2_layers_run mlp <weights_dir> <layer_idx> <tokens> <x.f32> <y.f32> [bf16|tf32]
//
// Weights come from a DirWeightStore over <weights_dir> under the reference's
// tensor names; x is read from <x.f32> ([tokens][2048-or-stored hidden] fp32)
// and y written to <y.f32>.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "b2_layers.h"

#define RUN_CHECK(call)                                                               \
  do {                                                                                \
    cudaError_t e_ = (call);                                                          \
    if (e_ != cudaSuccess) {                                                          \
      fprintf(stderr, "CUDA error (%s:%d): %s\n", __FILE__, __LINE__,                 \
              cudaGetErrorString(e_));                                                \
      return 1;                                                                       \
    }                                                                                 \
  } while (0)

static void usage() {
  fprintf(stderr,
          "usage: b2_layers_run <moe|mlp> <weights_dir> <layer_idx> <tokens> <x.f32> <y.f32> "
          "[bf16|tf32]\n");
}

int main(int argc, char **argv) {
  if (argc == 2 && (!strcmp(argv[1], "--help") || !strcmp(argv[1], "-h"))) {
    usage();
    return 0;
  }
  if (argc < 7) {
    usage();
    return 2;
  }
  const std::string kind = argv[1], dir = argv[2];
  const int layer = atoi(argv[3]), T = atoi(argv[4]);
  const int dtype = (argc > 7 && !strcmp(argv[7], "tf32")) ? B2_TF32 : B2_BF16;
  b2layer::DirWeightStore store(dir);
  b2layer::set_weight_store(&store);
  b2layer::set_max_tokens(T > 0 ? T : 1);
  b2layer::set_gemm_dtype(dtype);

  const std::string pre = "layers." + std::to_string(layer) + ".feed_forward.";
  b2layer::SparseMoeBlock *moe = nullptr;
  b2layer::MLP *mlp = nullptr;
  int H = 0;
  if (kind == "moe") {
    moe = new b2layer::SparseMoeBlock(layer);
    moe->init_gpu();
  } else if (kind == "mlp") {
    mlp = new b2layer::MLP(pre + "w1.weight", pre + "w2.weight", pre + "w3.weight");
    mlp->init_gpu();
  } else {
    usage();
    return 2;
  }
  {
    std::vector<float> d;
    std::vector<size_t> s;
    store.load(kind == "moe" ? pre + "gate.weight" : pre + "w1.weight", &d, &s);
    H = (int)s[1];
  }
  std::vector<float> x((size_t)T * H), y((size_t)T * H);
  std::ifstream fx(argv[5], std::ios::binary);
  fx.read(reinterpret_cast<char *>(x.data()), (std::streamsize)(x.size() * 4));
  if ((size_t)fx.gcount() != x.size() * 4) {
    fprintf(stderr, "short read of %s\n", argv[5]);
    return 1;
  }
  float *dx = nullptr, *dy = nullptr;
  cudaStream_t st;
  RUN_CHECK(cudaStreamCreate(&st));
  RUN_CHECK(cudaMalloc(&dx, x.size() * 4 + 16));
  RUN_CHECK(cudaMalloc(&dy, y.size() * 4 + 16));
  RUN_CHECK(cudaMemcpyAsync(dx, x.data(), x.size() * 4, cudaMemcpyHostToDevice, st));
  if (moe) moe->forward_gpu(dx, dy, 1, T, H, st);
  if (mlp) mlp->forward_gpu(dx, dy, 1, T, H, st);
  RUN_CHECK(cudaMemcpyAsync(y.data(), dy, y.size() * 4, cudaMemcpyDeviceToHost, st));
  RUN_CHECK(cudaStreamSynchronize(st));
  int dev_status = 0;
  if (moe && b2_moe_get_status(moe->handle(), st, &dev_status) != B2_OK) {
    fprintf(stderr, "device status 0x%x\n", dev_status);
    return 1;
  }
  if (mlp && b2_mlp_get_status(mlp->handle(), st, &dev_status) != B2_OK) {
    fprintf(stderr, "device status 0x%x\n", dev_status);
    return 1;
  }
  std::ofstream fy(argv[6], std::ios::binary);
  fy.write(reinterpret_cast<const char *>(y.data()), (std::streamsize)(y.size() * 4));
  delete moe;
  delete mlp;
  cudaFree(dx);
  cudaFree(dy);
  cudaStreamDestroy(st);
  printf("ok %s T=%d H=%d\n", kind.c_str(), T, H);
  return 0;
}
