// b2_layers.h -- C++ drop-in for the reference engine's layer and model
// classes (include/layer.h, include/model.h, include/model_loader.h of the
// reference), running on the B200 C ABI (include/b2moe.h, b2mlp.h, b2lfm2.h,
// b2loader.h).
//
// Same class names, constructors and GPU entry points as the reference:
//
//   SparseMoeBlock(int layer_idx);  init_gpu();
//   forward_gpu(float *x, float *y, int batch, int seq_len, int hidden_size,
//               cudaStream_t stream = 0);
//   MLP(w1_name, w2_name, w3_name); init_gpu(); forward_gpu(...same...);
//   RMSNorm(weight_name); init_gpu(); forward_gpu(x, y, rows, hidden_dim, stream);
//   RotaryEmbedding(); init_gpu(); cos_gpu_ / sin_gpu_;
//   Attention(int layer_idx); init_gpu();
//   forward_gpu(x, cos, sin, output, batch, seq_len, hidden_size, stream);
//   ShortConv(int layer_idx); init_gpu(); forward_gpu(x, y, batch, seq_len, hidden, stream);
//   DecoderLayer(int layer_idx, bool is_attention_layer); init_gpu(int device_id);
//   forward_gpu(x, cos, sin, output, batch, seq_len, hidden_size, stream);
//   ModelLoader(model_file): has_tensor / get_shape / load (the weight store);
//   LFM2Model(model_file); forward(sample_idx, batch_size, ids, seq_len, out); sync();
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

#include "../../include/b2lfm2.h"
#include "../../include/b2loader.h"
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
  // Whether the tensor exists (default: by loading it).
  virtual bool has(const std::string &name);
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

// The reference's model file (ModelLoader, include/model_loader.h:10-34),
// memory-mapped: a missing file or a corrupt index prints and exits, as the
// reference's constructor throws out of main.
class ModelLoader : public WeightStore {
 public:
  explicit ModelLoader(const std::string &model_file);
  ~ModelLoader() override;
  ModelLoader(const ModelLoader &) = delete;
  ModelLoader &operator=(const ModelLoader &) = delete;
  bool has_tensor(const std::string &name) const;
  std::vector<size_t> get_shape(const std::string &name) const;
  bool load(const std::string &name, std::vector<float> *data,
            std::vector<size_t> *shape) override;
  bool has(const std::string &name) override { return has_tensor(name); }
  b2_loader *handle() const { return l_; }

 private:
  b2_loader *l_ = nullptr;
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

// Model constants (include/config.h:8-9, 22-26).
constexpr float kRmsNormEps = 1e-5f;
constexpr float kRopeTheta = 1000000.0f;
constexpr size_t kMaxPositionEmbeddings = 128000;
constexpr int kHeadDim = 64;

class RMSNorm {
 public:
  explicit RMSNorm(const std::string &weight_file);
  ~RMSNorm();
  RMSNorm(const RMSNorm &) = delete;
  RMSNorm &operator=(const RMSNorm &) = delete;
  void init_gpu();
  void forward_gpu(float *x, float *y, int rows, int hidden_dim, cudaStream_t stream = 0);
  const float *weight_gpu() const { return weight_gpu_; }

 private:
  std::vector<float> weight_;
  float *weight_gpu_ = nullptr;
};

class RotaryEmbedding {
 public:
  RotaryEmbedding();
  ~RotaryEmbedding();
  RotaryEmbedding(const RotaryEmbedding &) = delete;
  RotaryEmbedding &operator=(const RotaryEmbedding &) = delete;
  void init_gpu();
  float *cos_gpu_ = nullptr;  // [max_seq_len][64]
  float *sin_gpu_ = nullptr;

 private:
  size_t max_seq_len_;
};

class Attention {
 public:
  explicit Attention(int layer_idx);
  ~Attention();
  Attention(const Attention &) = delete;
  Attention &operator=(const Attention &) = delete;
  void init_gpu();
  void forward_gpu(float *x, float *cos, float *sin, float *output, int batch, int seq_len,
                   int hidden_size, cudaStream_t stream = 0);

 private:
  int layer_idx_;
  std::vector<float> q_, k_, v_, o_, q_ln_, k_ln_;
  int hidden_ = 0, heads_ = 0, kv_heads_ = 0, max_tokens_ = 0;
  b2_attn *h_ = nullptr;
};

class ShortConv {
 public:
  explicit ShortConv(int layer_idx);
  ~ShortConv();
  ShortConv(const ShortConv &) = delete;
  ShortConv &operator=(const ShortConv &) = delete;
  void init_gpu();
  void forward_gpu(float *x, float *y, int batch, int seq_len, int hidden_size,
                   cudaStream_t stream = 0);

 private:
  int layer_idx_;
  std::vector<float> conv_, in_, out_;
  int hidden_ = 0, kernel_ = 0, max_tokens_ = 0;
  b2_conv *h_ = nullptr;
};

class DecoderLayer {
 public:
  DecoderLayer(int layer_idx, bool is_attention_layer);
  ~DecoderLayer();
  DecoderLayer(const DecoderLayer &) = delete;
  DecoderLayer &operator=(const DecoderLayer &) = delete;
  void init_gpu(int device_id);
  void forward_gpu(float *x, float *cos, float *sin, float *output, int batch, int seq_len,
                   int hidden_size, cudaStream_t stream = 0);
  bool is_attention_layer() const { return is_attention_layer_; }

 private:
  int layer_idx_;
  bool is_attention_layer_;
  int max_tokens_;
  RMSNorm input_layernorm_, post_attention_layernorm_;
  Attention *self_attn_ = nullptr;
  ShortConv *short_conv_ = nullptr;
  SparseMoeBlock *moe_block_ = nullptr;
  MLP *dense_mlp_ = nullptr;
  float *normed_input_gpu_ = nullptr, *attn_output_gpu_ = nullptr;
  float *normed_hidden_gpu_ = nullptr, *ffn_output_gpu_ = nullptr;
};

// Sequences per forward and positions per sequence the models created after
// this call accept (the reference fixes 64 x 32 for its pipeline buffers,
// include/model.h:58, include/config.h:52).  Default 64 x 512.
void set_model_limits(int max_batch, int max_seq);

// The whole model from a model file.  Every visible GPU holds a replica
// (weights fit one B200 many times over); forward() sends batch
// sample_idx / batch_size to GPU (sample_idx / batch_size) % num_gpus, so
// consecutive batches run on different GPUs concurrently, replacing the
// reference's 24-stage pipeline over 4 GPUs (src/model.cu:235-562).
// output_buffer receives [batch_size][vocab] fp32 logits of each sequence's
// last position once sync() returns.
class LFM2Model {
 public:
  explicit LFM2Model(const std::string &model_file);
  // The expert-parallel model, one process per GPU (b2_lfm2_create_ep): this
  // process is `rank` of `world` and uses device rank % (visible devices);
  // every MoE layer exchanges expert rows with the other ranks over NVLink
  // instead of the reference's stages passing the whole residual stream.
  // unique_id is LFM2Model::unique_id() of rank 0, shared by the caller (MPI,
  // a file, ...).  Construction, forward(), sync() and destruction are
  // collective: every rank calls them in the same order, each forward() with
  // its own batch.  Logits are bit-identical to the single-GPU model's.
  LFM2Model(const std::string &model_file, int world, int rank, const std::string &unique_id,
            bool owner_placement = false);
  // A fresh NCCL unique id (B2_EP_UNIQUE_ID_BYTES bytes) for the constructor above.
  static std::string unique_id();
  ~LFM2Model();
  LFM2Model(const LFM2Model &) = delete;
  LFM2Model &operator=(const LFM2Model &) = delete;
  void forward(int sample_idx, int batch_size, const int *input_ids_ptr, size_t seq_len,
               float *output_buffer);
  void sync();
  int vocab() const { return desc_.vocab; }

 private:
  struct Replica {
    int device = 0;
    b2_lfm2 *model = nullptr;
    cudaStream_t stream = nullptr;
    int *ids = nullptr;
    float *logits = nullptr;
  };
  ModelLoader loader_;
  b2_lfm2_desc desc_{};
  std::vector<Replica> replicas_;
};

}  // namespace b2layer
