// b2_layers.cpp -- the reference-shaped C++ layer classes over the C ABI.
#include "b2_layers.h"

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <sstream>

namespace b2layer {

namespace {

WeightStore *g_store = nullptr;
int g_max_tokens = 16384;
int g_dtype = B2_BF16;

[[noreturn]] void die(const char *what, const std::string &detail) {
  fprintf(stderr, "b2layer error: %s: %s\n", what, detail.c_str());
  exit(EXIT_FAILURE);
}

// CHECK_CUDA-style wrapper for the C ABI's status codes.
void check(b2_status s, const char *what) {
  if (s != B2_OK) die(what, b2_status_string(s));
}

std::vector<float> fetch(const std::string &name, std::vector<size_t> *shape_out) {
  if (!g_store) die("no weight store set", name);
  std::vector<float> data;
  std::vector<size_t> shape;
  if (!g_store->load(name, &data, &shape)) die("missing tensor", name);
  size_t n = 1;
  for (size_t d : shape) n *= d;
  if (n != data.size()) die("tensor size does not match its shape", name);
  if (shape_out) *shape_out = shape;
  return data;
}

}  // namespace

void set_weight_store(WeightStore *store) { g_store = store; }
WeightStore *weight_store() { return g_store; }
void set_max_tokens(int max_tokens) { g_max_tokens = max_tokens; }
void set_gemm_dtype(int dtype) { g_dtype = dtype; }

void MapWeightStore::put(const std::string &name, std::vector<float> data,
                         std::vector<size_t> shape) {
  t_[name] = {std::move(data), std::move(shape)};
}

bool MapWeightStore::load(const std::string &name, std::vector<float> *data,
                          std::vector<size_t> *shape) {
  auto it = t_.find(name);
  if (it == t_.end()) return false;
  *data = it->second.first;
  *shape = it->second.second;
  return true;
}

bool DirWeightStore::load(const std::string &name, std::vector<float> *data,
                          std::vector<size_t> *shape) {
  std::ifstream sh(dir_ + "/" + name + ".shape");
  if (!sh) return false;
  shape->clear();
  size_t d, n = 1;
  while (sh >> d) {
    shape->push_back(d);
    n *= d;
  }
  std::ifstream f(dir_ + "/" + name + ".f32", std::ios::binary);
  if (!f) return false;
  data->resize(n);
  f.read(reinterpret_cast<char *>(data->data()), (std::streamsize)(n * sizeof(float)));
  return (size_t)f.gcount() == n * sizeof(float);
}

// ------------------------------------------------------------------- MLP
MLP::MLP(const std::string &w1_file, const std::string &w2_file, const std::string &w3_file)
    : max_tokens_(g_max_tokens), dtype_(g_dtype) {
  std::vector<size_t> s1, s2, s3;
  w1_ = fetch(w1_file, &s1);
  w2_ = fetch(w2_file, &s2);
  w3_ = fetch(w3_file, &s3);
  if (s1.size() != 2 || s1 != s3 || s2.size() != 2 || s2[0] != s1[1] || s2[1] != s1[0])
    die("MLP weight shapes", w1_file);
  inter_ = (int)s1[0];
  hidden_ = (int)s1[1];
}

MLP::MLP(MLP &&o) noexcept
    : w1_(std::move(o.w1_)), w2_(std::move(o.w2_)), w3_(std::move(o.w3_)), inter_(o.inter_),
      hidden_(o.hidden_), max_tokens_(o.max_tokens_), dtype_(o.dtype_), h_(o.h_) {
  o.h_ = nullptr;
}

MLP::~MLP() {
  if (h_) b2_mlp_destroy(h_);
}

void MLP::init_gpu() {
  if (h_) return;
  b2_mlp_desc d{hidden_, inter_, max_tokens_, dtype_};
  check(b2_mlp_create(&d, w1_.data(), w2_.data(), w3_.data(), /*weights_on_host=*/1, nullptr,
                      &h_),
        "b2_mlp_create");
}

void MLP::forward_gpu(float *x, float *y, int batch, int seq_len, int hidden_size,
                      cudaStream_t stream) {
  if (!h_) die("MLP::forward_gpu", "init_gpu() was not called");
  if (hidden_size != hidden_) die("MLP::forward_gpu", "hidden_size mismatch");
  check(b2_mlp_forward(h_, x, y, batch * seq_len, reinterpret_cast<b2_stream>(stream)),
        "b2_mlp_forward");
}

// --------------------------------------------------------- SparseMoeBlock
SparseMoeBlock::SparseMoeBlock(int layer_idx)
    : layer_idx_(layer_idx), max_tokens_(g_max_tokens), dtype_(g_dtype) {
  const std::string pre = "layers." + std::to_string(layer_idx) + ".feed_forward.";
  std::vector<size_t> sg;
  gate_ = fetch(pre + "gate.weight", &sg);
  if (sg.size() != 2) die("router shape", pre + "gate.weight");
  experts_ = (int)sg[0];
  hidden_ = (int)sg[1];
  w1_.resize(experts_);
  w2_.resize(experts_);
  w3_.resize(experts_);
  for (int e = 0; e < experts_; ++e) {
    const std::string ep = pre + "experts." + std::to_string(e) + ".";
    std::vector<size_t> s1, s2, s3;
    w1_[e] = fetch(ep + "w1.weight", &s1);
    w2_[e] = fetch(ep + "w2.weight", &s2);
    w3_[e] = fetch(ep + "w3.weight", &s3);
    if (s1.size() != 2 || s1 != s3 || s1[1] != (size_t)hidden_ || s2.size() != 2 ||
        s2[0] != (size_t)hidden_ || s2[1] != s1[0])
      die("expert weight shapes", ep + "w1.weight");
    if (e == 0) inter_ = (int)s1[0];
    if ((int)s1[0] != inter_) die("expert inter sizes differ", ep + "w1.weight");
  }
  if (kUseExpertBias) {
    std::vector<size_t> sb;
    bias_ = fetch(pre + "expert_bias", &sb);
    if (bias_.size() != (size_t)experts_) die("expert_bias size", pre + "expert_bias");
  }
}

SparseMoeBlock::~SparseMoeBlock() {
  if (h_) b2_moe_destroy(h_);
}

void SparseMoeBlock::init_gpu() {
  if (h_) return;
  b2_moe_desc d{hidden_, inter_, experts_, kNumExpertsPerTok, max_tokens_,
                kRoutedScalingFactor, kUseExpertBias ? 1 : 0, dtype_};
  std::vector<const float *> p1(experts_), p2(experts_), p3(experts_);
  for (int e = 0; e < experts_; ++e) {
    p1[e] = w1_[e].data();
    p2[e] = w2_[e].data();
    p3[e] = w3_[e].data();
  }
  check(b2_moe_create(&d, p1.data(), p2.data(), p3.data(), gate_.data(),
                      kUseExpertBias ? bias_.data() : nullptr, /*weights_on_host=*/1, nullptr,
                      &h_),
        "b2_moe_create");
}

void SparseMoeBlock::forward_gpu(float *x, float *y, int batch, int seq_len, int hidden_size,
                                 cudaStream_t stream) {
  if (!h_) die("SparseMoeBlock::forward_gpu", "init_gpu() was not called");
  if (hidden_size != hidden_) die("SparseMoeBlock::forward_gpu", "hidden_size mismatch");
  check(b2_moe_forward(h_, x, y, batch * seq_len, reinterpret_cast<b2_stream>(stream)),
        "b2_moe_forward");
}

}  // namespace b2layer
