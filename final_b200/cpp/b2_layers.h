// b2_layers.h -- C++ drop-in for the reference engine's MoE and dense-MLP
// layer classes (include/layer.h:48-123 of the reference), running on the
// B200 C ABI (include/b2moe.h, include/b2mlp.h).
//
// Same class names, constructors and GPU entry points as the reference:
//
//   SparseMoeBlock(int layer_idx);  init_gpu();
//   forward_gpu(float *x, float *y, int batch, int seq_len, int hidden_size,
//               cudaStream_t stream = 0);
//   MLP(w1_name, w2_name, w3_name); init_gpu(); forward_gpu(...same...);
//
// Weights are fetched by the reference's tensor names
// ("layers.<i>.feed_forward.gate.weight", "...experts.<e>.w1.weight", ...,
// src/layer.cu:1274-1297) from the process-wide WeightStore, the counterpart
// of the reference's g_model_loader / Tensor::load_from_file
// (src/tensor.cu:175-187).  Failures print a message and exit the process,
// as the reference's CHECK_CUDA does (include/tensor.h:9-17); the C ABI
// underneath returns status codes instead.
//
// The classes live in namespace b2layer so that they can be linked next to
// the reference's own; an integration selects them with
//   using b2layer::SparseMoeBlock; using b2layer::MLP;
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <map>
#include <string>
#include <vector>

#include "../../include/b2mlp.h"
#include "../../include/b2moe.h"

namespace b2layer {

// Model constants of the reference (include/config.h:3-20).
constexpr int kHiddenSize = 2048;
constexpr int kIntermediateSize = 7168;     // dense MLP (layers 0-1)
constexpr int kNumExperts = 32;
constexpr int kNumExpertsPerTok = 4;
constexpr int kMoeIntermediateSize = 1792;
constexpr float kRoutedScalingFactor = 1.0f;
constexpr bool kUseExpertBias = true;

// Source of host fp32 weights by tensor name (row-major, shape as stored).
class WeightStore {
 public:
  virtual ~WeightStore() = default;
  // Returns false if the tensor does not exist.
  virtual bool load(const std::string &name, std::vector<float> *data,
                    std::vector<size_t> *shape) = 0;
};

// Process-wide store the layer constructors read from (not owned).
void set_weight_store(WeightStore *store);
WeightStore *weight_store();

// In-memory store (tests, callers that already hold the tensors).
class MapWeightStore : public WeightStore {
 public:
  void put(const std::string &name, std::vector<float> data, std::vector<size_t> shape);
  bool load(const std::string &name, std::vector<float> *data,
            std::vector<size_t> *shape) override;

 private:
  std::map<std::string, std::pair<std::vector<float>, std::vector<size_t>>> t_;
};

// Directory store: <dir>/<name>.f32 (raw little-endian fp32) and
// <dir>/<name>.shape (dimensions as text).
class DirWeightStore : public WeightStore {
 public:
  explicit DirWeightStore(std::string dir) : dir_(std::move(dir)) {}
  bool load(const std::string &name, std::vector<float> *data,
            std::vector<size_t> *shape) override;

 private:
  std::string dir_;
};

// Token capacity of the layers created after this call (the reference's
// fixed scratch holds 4096 tokens, src/layer.cu:1399).  Default 16384.
void set_max_tokens(int max_tokens);
// Expert / MLP GEMM operand type for layers created after this call:
// B2_BF16 (default) or B2_TF32.
void set_gemm_dtype(int dtype);

class MLP {
 public:
  MLP(const std::string &w1_file, const std::string &w2_file, const std::string &w3_file);
  ~MLP();
  MLP(MLP &&other) noexcept;
  MLP(const MLP &) = delete;
  MLP &operator=(const MLP &) = delete;

  void init_gpu();
  void forward_gpu(float *x, float *y, int batch, int seq_len, int hidden_size,
                   cudaStream_t stream = 0);

  b2_mlp *handle() const { return h_; }

 private:
  std::vector<float> w1_, w2_, w3_;  // host copies, as the reference keeps its Tensors
  int inter_ = 0, hidden_ = 0;
  int max_tokens_ = 0, dtype_ = 0;
  b2_mlp *h_ = nullptr;
};

class SparseMoeBlock {
 public:
  explicit SparseMoeBlock(int layer_idx);
  ~SparseMoeBlock();
  SparseMoeBlock(const SparseMoeBlock &) = delete;
  SparseMoeBlock &operator=(const SparseMoeBlock &) = delete;

  void init_gpu();
  void forward_gpu(float *x, float *y, int batch, int seq_len, int hidden_size,
                   cudaStream_t stream = 0);

  b2_moe *handle() const { return h_; }

 private:
  int layer_idx_;
  std::vector<float> gate_, bias_;
  std::vector<std::vector<float>> w1_, w2_, w3_;  // per expert
  int inter_ = 0, hidden_ = 0, experts_ = 0;
  int max_tokens_ = 0, dtype_ = 0;
  b2_moe *h_ = nullptr;
};

}  // namespace b2layer
