// b2_layers.cpp -- the reference-shaped C++ layer classes over the C ABI.
#include "b2_layers.h"

#include <algorithm>
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

// ======================================================================
// decoder glue, model and model file
namespace b2layer {

namespace {
int g_max_batch = 64;
int g_max_seq = 512;

void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess) die(what, cudaGetErrorString(e));
}

float *upload(const std::vector<float> &h) {
  float *d = nullptr;
  cuda_check(cudaMalloc(&d, h.size() * sizeof(float)), "cudaMalloc");
  cuda_check(cudaMemcpy(d, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice),
             "cudaMemcpy");
  return d;
}
}  // namespace

bool WeightStore::has(const std::string &name) {
  std::vector<float> d;
  std::vector<size_t> s;
  return load(name, &d, &s);
}

void set_model_limits(int max_batch, int max_seq) {
  g_max_batch = max_batch;
  g_max_seq = max_seq;
}

// ------------------------------------------------------------ ModelLoader
ModelLoader::ModelLoader(const std::string &model_file) {
  if (b2_loader_open(model_file.c_str(), &l_) != B2_OK)
    die("cannot open model file (missing, or not in the LFM2 format)", model_file);
}

ModelLoader::~ModelLoader() { b2_loader_close(l_); }

bool ModelLoader::has_tensor(const std::string &name) const {
  return b2_loader_tensor(l_, name.c_str(), nullptr, nullptr, nullptr, nullptr) == B2_OK;
}

std::vector<size_t> ModelLoader::get_shape(const std::string &name) const {
  int64_t shp[8];
  int nd = 0;
  if (b2_loader_tensor(l_, name.c_str(), nullptr, nullptr, shp, &nd) != B2_OK)
    die("tensor not found", name);
  return std::vector<size_t>(shp, shp + nd);
}

bool ModelLoader::load(const std::string &name, std::vector<float> *data,
                       std::vector<size_t> *shape) {
  const float *p = nullptr;
  int64_t n = 0, shp[8];
  int nd = 0;
  if (b2_loader_tensor(l_, name.c_str(), &p, &n, shp, &nd) != B2_OK) return false;
  data->assign(p, p + n);
  shape->assign(shp, shp + nd);
  return true;
}

// ---------------------------------------------------------------- RMSNorm
RMSNorm::RMSNorm(const std::string &weight_file) { weight_ = fetch(weight_file, nullptr); }

RMSNorm::~RMSNorm() {
  if (weight_gpu_) cudaFree(weight_gpu_);
}

void RMSNorm::init_gpu() {
  if (!weight_gpu_) weight_gpu_ = upload(weight_);
}

void RMSNorm::forward_gpu(float *x, float *y, int rows, int hidden_dim, cudaStream_t stream) {
  if (!weight_gpu_) die("RMSNorm::forward_gpu", "init_gpu() was not called");
  if ((size_t)hidden_dim != weight_.size()) die("RMSNorm::forward_gpu", "hidden_dim mismatch");
  check(b2_rmsnorm(x, weight_gpu_, y, rows, hidden_dim, kRmsNormEps,
                   reinterpret_cast<b2_stream>(stream)),
        "b2_rmsnorm");
}

// ------------------------------------------------------- RotaryEmbedding
RotaryEmbedding::RotaryEmbedding() : max_seq_len_(kMaxPositionEmbeddings) {}

RotaryEmbedding::~RotaryEmbedding() {
  if (cos_gpu_) cudaFree(cos_gpu_);
  if (sin_gpu_) cudaFree(sin_gpu_);
}

void RotaryEmbedding::init_gpu() {
  if (cos_gpu_) return;
  std::vector<float> c(max_seq_len_ * kHeadDim), s(max_seq_len_ * kHeadDim);
  check(b2_rope_tables(c.data(), s.data(), (int)max_seq_len_, kHeadDim, kRopeTheta),
        "b2_rope_tables");
  cos_gpu_ = upload(c);
  sin_gpu_ = upload(s);
}

// -------------------------------------------------------------- Attention
Attention::Attention(int layer_idx) : layer_idx_(layer_idx), max_tokens_(g_max_tokens) {
  const std::string a = "layers." + std::to_string(layer_idx) + ".self_attn.";
  std::vector<size_t> sq, sk, sv, so;
  q_ = fetch(a + "q_proj.weight", &sq);
  k_ = fetch(a + "k_proj.weight", &sk);
  v_ = fetch(a + "v_proj.weight", &sv);
  o_ = fetch(a + "out_proj.weight", &so);
  q_ln_ = fetch(a + "q_layernorm.weight", nullptr);
  k_ln_ = fetch(a + "k_layernorm.weight", nullptr);
  if (sq.size() != 2 || sk.size() != 2 || sk != sv || so.size() != 2 || sq[1] != sk[1] ||
      so[0] != sq[1] || so[1] != sq[0] || sq[0] % kHeadDim || sk[0] % kHeadDim ||
      q_ln_.size() != (size_t)kHeadDim || k_ln_.size() != (size_t)kHeadDim)
    die("attention weight shapes", a + "q_proj.weight");
  hidden_ = (int)sq[1];
  heads_ = (int)sq[0] / kHeadDim;
  kv_heads_ = (int)sk[0] / kHeadDim;
}

Attention::~Attention() {
  if (h_) b2_attn_destroy(h_);
}

void Attention::init_gpu() {
  if (h_) return;
  b2_attn_desc d{hidden_, heads_, kv_heads_, kHeadDim, max_tokens_, kRmsNormEps};
  check(b2_attn_create(&d, q_.data(), k_.data(), v_.data(), o_.data(), q_ln_.data(),
                       k_ln_.data(), /*weights_on_host=*/1, nullptr, &h_),
        "b2_attn_create");
}

void Attention::forward_gpu(float *x, float *cos, float *sin, float *output, int batch,
                            int seq_len, int hidden_size, cudaStream_t stream) {
  if (!h_) die("Attention::forward_gpu", "init_gpu() was not called");
  if (hidden_size != hidden_) die("Attention::forward_gpu", "hidden_size mismatch");
  check(b2_attn_forward(h_, x, cos, sin, output, batch, seq_len,
                        reinterpret_cast<b2_stream>(stream)),
        "b2_attn_forward");
}

// -------------------------------------------------------------- ShortConv
ShortConv::ShortConv(int layer_idx) : layer_idx_(layer_idx), max_tokens_(g_max_tokens) {
  const std::string c = "layers." + std::to_string(layer_idx) + ".conv.";
  std::vector<size_t> sc, si, so;
  conv_ = fetch(c + "conv.weight", &sc);
  in_ = fetch(c + "in_proj.weight", &si);
  out_ = fetch(c + "out_proj.weight", &so);
  if (so.size() != 2 || so[0] != so[1] || si.size() != 2 || si[0] != 3 * so[0] ||
      si[1] != so[0] || sc.empty() || sc[0] != so[0])
    die("short-conv weight shapes", c + "in_proj.weight");
  hidden_ = (int)so[0];
  kernel_ = (int)sc.back();
}

ShortConv::~ShortConv() {
  if (h_) b2_conv_destroy(h_);
}

void ShortConv::init_gpu() {
  if (h_) return;
  b2_conv_desc d{hidden_, kernel_, max_tokens_};
  check(b2_conv_create(&d, conv_.data(), in_.data(), out_.data(), /*weights_on_host=*/1, nullptr,
                       &h_),
        "b2_conv_create");
}

void ShortConv::forward_gpu(float *x, float *y, int batch, int seq_len, int hidden_size,
                            cudaStream_t stream) {
  if (!h_) die("ShortConv::forward_gpu", "init_gpu() was not called");
  if (hidden_size != hidden_) die("ShortConv::forward_gpu", "hidden_size mismatch");
  check(b2_conv_forward(h_, x, y, batch, seq_len, reinterpret_cast<b2_stream>(stream)),
        "b2_conv_forward");
}

// ----------------------------------------------------------- DecoderLayer
DecoderLayer::DecoderLayer(int layer_idx, bool is_attention_layer)
    : layer_idx_(layer_idx),
      is_attention_layer_(is_attention_layer),
      max_tokens_(g_max_tokens),
      input_layernorm_("layers." + std::to_string(layer_idx) + ".operator_norm.weight"),
      post_attention_layernorm_("layers." + std::to_string(layer_idx) + ".ffn_norm.weight") {
  if (is_attention_layer)
    self_attn_ = new Attention(layer_idx);
  else
    short_conv_ = new ShortConv(layer_idx);
  // MoE where the model has a router for this layer (the reference: layer
  // index >= NUM_DENSE_LAYERS, src/layer.cu:1797-1812)
  const std::string ff = "layers." + std::to_string(layer_idx) + ".feed_forward.";
  if (!g_store) die("no weight store set", ff);
  if (g_store->has(ff + "gate.weight"))
    moe_block_ = new SparseMoeBlock(layer_idx);
  else
    dense_mlp_ = new MLP(ff + "w1.weight", ff + "w2.weight", ff + "w3.weight");
}

DecoderLayer::~DecoderLayer() {
  delete self_attn_;
  delete short_conv_;
  delete moe_block_;
  delete dense_mlp_;
  for (float *p : {normed_input_gpu_, attn_output_gpu_, normed_hidden_gpu_, ffn_output_gpu_})
    if (p) cudaFree(p);
}

void DecoderLayer::init_gpu(int device_id) {
  cuda_check(cudaSetDevice(device_id), "cudaSetDevice");
  input_layernorm_.init_gpu();
  post_attention_layernorm_.init_gpu();
  if (self_attn_) self_attn_->init_gpu();
  if (short_conv_) short_conv_->init_gpu();
  if (moe_block_) moe_block_->init_gpu();
  if (dense_mlp_) dense_mlp_->init_gpu();
  if (normed_input_gpu_) return;
  size_t hidden = 0;
  {
    std::vector<size_t> s;
    std::vector<float> d;
    const std::string n = "layers." + std::to_string(layer_idx_) + ".ffn_norm.weight";
    if (!g_store->load(n, &d, &s)) die("missing tensor", n);
    hidden = d.size();
  }
  const size_t bytes = (size_t)max_tokens_ * hidden * sizeof(float);
  for (float **p : {&normed_input_gpu_, &attn_output_gpu_, &normed_hidden_gpu_, &ffn_output_gpu_})
    cuda_check(cudaMalloc(p, bytes), "cudaMalloc");
}

void DecoderLayer::forward_gpu(float *x, float *cos, float *sin, float *output, int batch,
                               int seq_len, int hidden_size, cudaStream_t stream) {
  if (!normed_input_gpu_) die("DecoderLayer::forward_gpu", "init_gpu() was not called");
  const int T = batch * seq_len;
  if (T > max_tokens_) die("DecoderLayer::forward_gpu", "batch * seq_len exceeds capacity");
  b2_stream s = reinterpret_cast<b2_stream>(stream);
  // 1. input norm  2. attention / conv
  input_layernorm_.forward_gpu(x, normed_input_gpu_, T, hidden_size, stream);
  if (self_attn_)
    self_attn_->forward_gpu(normed_input_gpu_, cos, sin, attn_output_gpu_, batch, seq_len,
                            hidden_size, stream);
  else
    short_conv_->forward_gpu(normed_input_gpu_, attn_output_gpu_, batch, seq_len, hidden_size,
                             stream);
  // 3. output = x + attn_out   4. normed_hidden = post-attention norm(output)
  if (output != x)
    cuda_check(cudaMemcpyAsync(output, x, (size_t)T * hidden_size * sizeof(float),
                               cudaMemcpyDeviceToDevice, stream),
               "cudaMemcpyAsync");
  check(b2_add_rmsnorm(output, attn_output_gpu_, post_attention_layernorm_.weight_gpu(),
                       normed_hidden_gpu_, nullptr, T, hidden_size, kRmsNormEps, s),
        "b2_add_rmsnorm");
  // 5. FFN   6. output += ffn_out (the norm of this call is not used)
  if (moe_block_)
    moe_block_->forward_gpu(normed_hidden_gpu_, ffn_output_gpu_, batch, seq_len, hidden_size,
                            stream);
  else
    dense_mlp_->forward_gpu(normed_hidden_gpu_, ffn_output_gpu_, batch, seq_len, hidden_size,
                            stream);
  check(b2_add_rmsnorm(output, ffn_output_gpu_, post_attention_layernorm_.weight_gpu(), nullptr,
                       nullptr, T, hidden_size, kRmsNormEps, s),
        "b2_add_rmsnorm");
}

// -------------------------------------------------------------- LFM2Model
namespace {
// Model shape from the tensors in the file (the reference compiles it in,
// include/config.h).
b2_lfm2_desc infer_desc(ModelLoader &f) {
  b2_lfm2_desc d{};
  const std::vector<size_t> emb = f.get_shape("embed_tokens.weight");
  if (emb.size() != 2) die("embedding shape", "embed_tokens.weight");
  d.vocab = (int)emb[0];
  d.hidden = (int)emb[1];
  int L = 0;
  while (f.has_tensor("layers." + std::to_string(L) + ".operator_norm.weight")) ++L;
  if (L < 1 || L > 64) die("number of layers", std::to_string(L));
  d.num_layers = L;
  d.num_heads = d.hidden / kHeadDim;
  d.num_kv_heads = std::max(1, d.num_heads / 4);
  for (int i = 0; i < L; ++i) {
    const std::string a = "layers." + std::to_string(i) + ".self_attn.";
    d.layer_types[i] = f.has_tensor(a + "q_proj.weight") ? 0 : 1;
    if (d.layer_types[i] == 0) {
      d.num_heads = (int)f.get_shape(a + "q_proj.weight")[0] / kHeadDim;
      d.num_kv_heads = (int)f.get_shape(a + "k_proj.weight")[0] / kHeadDim;
    }
  }
  while (d.num_dense_layers < L &&
         f.has_tensor("layers." + std::to_string(d.num_dense_layers) + ".feed_forward.w1.weight"))
    ++d.num_dense_layers;
  if (d.num_dense_layers > 0) d.dense_inter = (int)f.get_shape("layers.0.feed_forward.w1.weight")[0];
  if (d.num_dense_layers < L) {
    const std::string m = "layers." + std::to_string(d.num_dense_layers) + ".feed_forward.";
    d.num_experts = (int)f.get_shape(m + "gate.weight")[0];
    d.moe_inter = (int)f.get_shape(m + "experts.0.w1.weight")[0];
    d.use_expert_bias = f.has_tensor(m + "expert_bias") ? 1 : 0;
  }
  d.top_k = kNumExpertsPerTok;
  d.max_batch = g_max_batch;
  d.max_seq = g_max_seq;
  d.eps = kRmsNormEps;
  d.rope_theta = kRopeTheta;
  d.routed_scale = kRoutedScalingFactor;
  d.dtype = g_dtype;
  return d;
}
}  // namespace

LFM2Model::LFM2Model(const std::string &model_file) : loader_(model_file) {
  desc_ = infer_desc(loader_);
  int n = 0;
  cuda_check(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
  if (n < 1) die("LFM2Model", "no CUDA device");
  replicas_.resize(n);
  for (int d = 0; d < n; ++d) {
    Replica &r = replicas_[d];
    r.device = d;
    cuda_check(cudaSetDevice(d), "cudaSetDevice");
    cuda_check(cudaStreamCreateWithFlags(&r.stream, cudaStreamNonBlocking), "cudaStreamCreate");
    check(b2_lfm2_create(&desc_, b2_loader_weight, loader_.handle(), /*weights_on_host=*/1,
                         reinterpret_cast<b2_stream>(r.stream), &r.model),
          "b2_lfm2_create");
    cuda_check(cudaMalloc(&r.ids, (size_t)desc_.max_batch * desc_.max_seq * sizeof(int)),
               "cudaMalloc");
    cuda_check(cudaMalloc(&r.logits, (size_t)desc_.max_batch * desc_.vocab * sizeof(float)),
               "cudaMalloc");
  }
  cuda_check(cudaSetDevice(0), "cudaSetDevice");
}

LFM2Model::LFM2Model(const std::string &model_file, int world, int rank,
                     const std::string &unique_id, bool owner_placement)
    : loader_(model_file) {
  desc_ = infer_desc(loader_);
  if (unique_id.size() != B2_EP_UNIQUE_ID_BYTES) die("LFM2Model", "unique id of the wrong size");
  int n = 0;
  cuda_check(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
  if (n < 1) die("LFM2Model", "no CUDA device");
  replicas_.resize(1);
  Replica &r = replicas_[0];
  r.device = rank % n;
  cuda_check(cudaSetDevice(r.device), "cudaSetDevice");
  cuda_check(cudaStreamCreateWithFlags(&r.stream, cudaStreamNonBlocking), "cudaStreamCreate");
  check(b2_lfm2_create_ep(&desc_, b2_loader_weight, loader_.handle(), /*weights_on_host=*/1,
                          world, rank, unique_id.data(),
                          owner_placement ? B2_EP_OWNER : B2_EP_BALANCED,
                          reinterpret_cast<b2_stream>(r.stream), &r.model),
        "b2_lfm2_create_ep");
  cuda_check(cudaMalloc(&r.ids, (size_t)desc_.max_batch * desc_.max_seq * sizeof(int)),
             "cudaMalloc");
  cuda_check(cudaMalloc(&r.logits, (size_t)desc_.max_batch * desc_.vocab * sizeof(float)),
             "cudaMalloc");
}

std::string LFM2Model::unique_id() {
  std::string id(B2_EP_UNIQUE_ID_BYTES, '\0');
  check(b2_ep_unique_id(&id[0]), "b2_ep_unique_id");
  return id;
}

LFM2Model::~LFM2Model() {
  for (Replica &r : replicas_) {
    cudaSetDevice(r.device);
    if (r.stream) cudaStreamSynchronize(r.stream);
    if (r.model) b2_lfm2_destroy(r.model);
    if (r.ids) cudaFree(r.ids);
    if (r.logits) cudaFree(r.logits);
    if (r.stream) cudaStreamDestroy(r.stream);
  }
}

void LFM2Model::forward(int sample_idx, int batch_size, const int *input_ids_ptr, size_t seq_len,
                        float *output_buffer) {
  if (batch_size < 1 || batch_size > desc_.max_batch || seq_len < 1 ||
      seq_len > (size_t)desc_.max_seq)
    die("LFM2Model::forward", "batch or sequence length outside the model's limits");
  Replica &r = replicas_[(size_t)(sample_idx / batch_size) % replicas_.size()];
  cuda_check(cudaSetDevice(r.device), "cudaSetDevice");
  const size_t T = (size_t)batch_size * seq_len;
  cuda_check(cudaMemcpyAsync(r.ids, input_ids_ptr, T * sizeof(int), cudaMemcpyHostToDevice,
                             r.stream),
             "cudaMemcpyAsync");
  check(b2_lfm2_forward(r.model, r.ids, batch_size, (int)seq_len, r.logits,
                        reinterpret_cast<b2_stream>(r.stream)),
        "b2_lfm2_forward");
  cuda_check(cudaMemcpyAsync(output_buffer, r.logits,
                             (size_t)batch_size * desc_.vocab * sizeof(float),
                             cudaMemcpyDeviceToHost, r.stream),
             "cudaMemcpyAsync");
}

void LFM2Model::sync() {
  for (Replica &r : replicas_) {
    cuda_check(cudaSetDevice(r.device), "cudaSetDevice");
    int st = 0;
    if (b2_lfm2_get_status(r.model, reinterpret_cast<b2_stream>(r.stream), &st) != B2_OK)
      die("LFM2Model::sync", "device-side error " + std::to_string(st));
  }
}

}  // namespace b2layer
