// b2_layers_run.cpp -- drives the C++ drop-in classes the way the reference
// engine drives its own (construct by layer index / tensor names, init_gpu(),
// forward_gpu() on device fp32 buffers; DecoderLayer::forward_gpu,
// src/layer.cu:1895-1919; LFM2Model::forward + sync, src/main.cpp).  The
// parity tests use it to exercise the C++ boundary end to end.
//
//   b2_layers_run moe     <weights> <layer> <tokens> <x.f32> <y.f32> [bf16|tf32]
//   b2_layers_run mlp     <weights> <layer> <tokens> <x.f32> <y.f32> [bf16|tf32]
//   b2_layers_run attn    <weights> <layer> <batch> <seq> <x.f32> <y.f32>
//   b2_layers_run conv    <weights> <layer> <batch> <seq> <x.f32> <y.f32>
//   b2_layers_run decoder <weights> <layer> <is_attention> <batch> <seq> <x.f32> <y.f32>
//   b2_layers_run model   <model.bin> <batch> <seq> <ids.i32> <logits.f32>
//   b2_layers_run model_ep <model.bin> <batch> <seq> <ids.i32> <logits.f32>
//                          <world> <rank> <id file> [balanced|owner]
//
// model_ep is one rank of the expert-parallel model: rank 0 writes the NCCL
// unique id to <id file>, the other ranks wait for it (60 s at most).
//
// <weights> is a directory of <name>.f32 / <name>.shape files or a model file
// in the reference's format.  x is [tokens][hidden] fp32; y the same.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <fstream>
#include <memory>
#include <string>
#include <sys/stat.h>
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
          "usage: b2_layers_run moe|mlp <weights> <layer> <tokens> <x.f32> <y.f32> [bf16|tf32]\n"
          "       b2_layers_run attn|conv <weights> <layer> <batch> <seq> <x.f32> <y.f32>\n"
          "       b2_layers_run decoder <weights> <layer> <is_attention> <batch> <seq> <x.f32> "
          "<y.f32>\n"
          "       b2_layers_run model <model.bin> <batch> <seq> <ids.i32> <logits.f32>\n"
          "       b2_layers_run model_ep <model.bin> <batch> <seq> <ids.i32> <logits.f32> "
          "<world> <rank> <id file> [balanced|owner]\n");
}

template <typename T>
static bool read_file(const char *path, std::vector<T> *v) {
  std::ifstream f(path, std::ios::binary);
  f.read(reinterpret_cast<char *>(v->data()), (std::streamsize)(v->size() * sizeof(T)));
  return (size_t)f.gcount() == v->size() * sizeof(T);
}

template <typename T>
static void write_file(const char *path, const std::vector<T> &v) {
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char *>(v.data()), (std::streamsize)(v.size() * sizeof(T)));
}

static std::unique_ptr<b2layer::WeightStore> open_store(const std::string &src) {
  struct stat st;
  if (stat(src.c_str(), &st) == 0 && S_ISDIR(st.st_mode))
    return std::unique_ptr<b2layer::WeightStore>(new b2layer::DirWeightStore(src));
  return std::unique_ptr<b2layer::WeightStore>(new b2layer::ModelLoader(src));
}

static int run_model(int argc, char **argv) {
  if (argc < 7) {
    usage();
    return 2;
  }
  const int B = atoi(argv[3]), S = atoi(argv[4]);
  b2layer::set_model_limits(B, S);
  b2layer::LFM2Model model(argv[2]);
  std::vector<int> ids((size_t)B * S);
  if (!read_file(argv[5], &ids)) {
    fprintf(stderr, "short read of %s\n", argv[5]);
    return 1;
  }
  std::vector<float> logits((size_t)B * model.vocab()), again(logits.size());
  model.forward(0, B, ids.data(), S, logits.data());
  model.forward(B, B, ids.data(), S, again.data());  // the next batch slot (next replica)
  model.sync();
  if (memcmp(logits.data(), again.data(), logits.size() * sizeof(float)) != 0) {
    fprintf(stderr, "two forwards of the same ids differ\n");
    return 1;
  }
  write_file(argv[6], logits);
  printf("ok model B=%d S=%d V=%d\n", B, S, model.vocab());
  return 0;
}

// Rank 0 publishes the id (write, then rename: readers never see half a
// file); the others poll for it.
static bool share_unique_id(const std::string &path, int rank, std::string *id) {
  if (rank == 0) {
    *id = b2layer::LFM2Model::unique_id();
    const std::string tmp = path + ".tmp";
    {
      std::ofstream f(tmp, std::ios::binary);
      f.write(id->data(), (std::streamsize)id->size());
      if (!f) return false;
    }
    return rename(tmp.c_str(), path.c_str()) == 0;
  }
  for (int i = 0; i < 6000; ++i) {
    std::ifstream f(path, std::ios::binary);
    if (f) {
      id->assign(B2_EP_UNIQUE_ID_BYTES, '\0');
      f.read(&(*id)[0], B2_EP_UNIQUE_ID_BYTES);
      if (f.gcount() == B2_EP_UNIQUE_ID_BYTES) return true;
    }
    struct timespec ts = {0, 10 * 1000 * 1000};
    nanosleep(&ts, nullptr);
  }
  return false;
}

static int run_model_ep(int argc, char **argv) {
  if (argc < 10) {
    usage();
    return 2;
  }
  const int B = atoi(argv[3]), S = atoi(argv[4]);
  const int world = atoi(argv[7]), rank = atoi(argv[8]);
  const bool owner = argc > 10 && !strcmp(argv[10], "owner");
  std::string id;
  if (!share_unique_id(argv[9], rank, &id)) {
    fprintf(stderr, "rank %d: no unique id in %s\n", rank, argv[9]);
    return 1;
  }
  b2layer::set_model_limits(B, S);
  b2layer::LFM2Model model(argv[2], world, rank, id, owner);
  std::vector<int> ids((size_t)B * S);
  if (!read_file(argv[5], &ids)) {
    fprintf(stderr, "short read of %s\n", argv[5]);
    return 1;
  }
  std::vector<float> logits((size_t)B * model.vocab()), again(logits.size());
  model.forward(0, B, ids.data(), S, logits.data());
  model.forward(B, B, ids.data(), S, again.data());
  model.sync();
  if (memcmp(logits.data(), again.data(), logits.size() * sizeof(float)) != 0) {
    fprintf(stderr, "two forwards of the same ids differ\n");
    return 1;
  }
  write_file(argv[6], logits);
  printf("ok model_ep rank %d of %d B=%d S=%d V=%d\n", rank, world, B, S, model.vocab());
  return 0;
}

int main(int argc, char **argv) {
  if (argc == 2 && (!strcmp(argv[1], "--help") || !strcmp(argv[1], "-h"))) {
    usage();
    return 0;
  }
  if (argc < 2) {
    usage();
    return 2;
  }
  const std::string kind = argv[1];
  if (kind == "model") return run_model(argc, argv);
  if (kind == "model_ep") return run_model_ep(argc, argv);
  const bool seq_form = kind == "attn" || kind == "conv" || kind == "decoder";
  const int need = kind == "decoder" ? 9 : seq_form ? 8 : 7;
  if (argc < need) {
    usage();
    return 2;
  }
  std::unique_ptr<b2layer::WeightStore> store = open_store(argv[2]);
  b2layer::set_weight_store(store.get());
  const int layer = atoi(argv[3]);
  int a = 4;
  const bool is_attn = kind == "decoder" ? atoi(argv[a++]) != 0 : kind == "attn";
  int B = 1, S = 0;
  if (seq_form) {
    B = atoi(argv[a++]);
    S = atoi(argv[a++]);
  } else {
    S = atoi(argv[a++]);
  }
  const char *xin = argv[a++], *yout = argv[a++];
  const int T = B * S;
  const int dtype = (!seq_form && argc > 7 && !strcmp(argv[7], "tf32")) ? B2_TF32 : B2_BF16;
  b2layer::set_max_tokens(T > 0 ? T : 1);
  b2layer::set_gemm_dtype(dtype);

  const std::string pre = "layers." + std::to_string(layer) + ".";
  int H = 0;
  {
    std::vector<float> d;
    std::vector<size_t> s;
    const std::string probe = kind == "moe" ? pre + "feed_forward.gate.weight"
                              : kind == "mlp" ? pre + "feed_forward.w1.weight"
                                              : pre + "operator_norm.weight";
    if (!store->load(probe, &d, &s)) {
      fprintf(stderr, "missing tensor %s\n", probe.c_str());
      return 1;
    }
    H = (int)s.back();
  }
  std::unique_ptr<b2layer::SparseMoeBlock> moe;
  std::unique_ptr<b2layer::MLP> mlp;
  std::unique_ptr<b2layer::Attention> att;
  std::unique_ptr<b2layer::ShortConv> conv;
  std::unique_ptr<b2layer::DecoderLayer> dec;
  std::unique_ptr<b2layer::RotaryEmbedding> rope;
  if (kind == "moe") {
    moe.reset(new b2layer::SparseMoeBlock(layer));
    moe->init_gpu();
  } else if (kind == "mlp") {
    const std::string ff = pre + "feed_forward.";
    mlp.reset(new b2layer::MLP(ff + "w1.weight", ff + "w2.weight", ff + "w3.weight"));
    mlp->init_gpu();
  } else if (kind == "attn") {
    att.reset(new b2layer::Attention(layer));
    att->init_gpu();
  } else if (kind == "conv") {
    conv.reset(new b2layer::ShortConv(layer));
    conv->init_gpu();
  } else if (kind == "decoder") {
    dec.reset(new b2layer::DecoderLayer(layer, is_attn));
    dec->init_gpu(0);
  } else {
    usage();
    return 2;
  }
  if (is_attn) {
    rope.reset(new b2layer::RotaryEmbedding());
    rope->init_gpu();
  }
  std::vector<float> x((size_t)T * H), y((size_t)T * H);
  if (!read_file(xin, &x)) {
    fprintf(stderr, "short read of %s\n", xin);
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
  if (att) att->forward_gpu(dx, rope->cos_gpu_, rope->sin_gpu_, dy, B, S, H, st);
  if (conv) conv->forward_gpu(dx, dy, B, S, H, st);
  if (dec) dec->forward_gpu(dx, rope ? rope->cos_gpu_ : nullptr, rope ? rope->sin_gpu_ : nullptr,
                            dy, B, S, H, st);
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
  write_file(yout, y);
  cudaFree(dx);
  cudaFree(dy);
  cudaStreamDestroy(st);
  printf("ok %s B=%d S=%d H=%d\n", kind.c_str(), B, S, H);
  return 0;
}
