// rustane.hpp — C++17 host API over the C ABI of cuda_bridge.h, for callers in
// compiled code. It keeps the reference engine's model-config and forward/loss API
// (whiskeypolitik/rustane, crates/engine) with the same names, argument meaning and
// error behaviour:
//   ModelConfig                 crates/engine/src/model.rs:5-17 (presets :21-151,
//                               param_count :109-114)
//   LayerWeights, ModelWeights  layer.rs:52-63, full_model.rs:19-23 (random :132-141)
//   CompiledKernels             layer.rs:909,967 (compile, compile_forward_only)
//   ModelForwardWorkspace       full_model.rs:206-264 (new, new_lean)
//   forward_only_ws, forward_ws full_model.rs:378,494
//   forward, ForwardResult      full_model.rs:915, :121-129
//   forward_losses              full_model.rs:1603
//   ForwardScheduler            multistream.rs:54-161 (one worker per device and
//                               host thread, whole sequences, results in order)
//   load_checkpoint             bin/train.rs:238-346 (RSTK files, cb_load_rstk)
//   DeviceTokens, eval_windows  data.rs:11-91, bin/train.rs:197-236 (uint16 token
//                               files in HBM, validation sums for val_loss/val_bpb)
//   forward_backward, ModelGrads full_model.rs:592-702, :26-30, :143-160 (training step)
//   prefill, decode_step        single-token decode with a KV cache
//   ParallelBenchRunner         parallel_bench.rs:24-364 (shard requests from the
//                               environment, resolution as sharding.rs:162-307,
//                               mode labels, forward_loss :239)
// The reference panics when an ANE evaluation fails (layer.rs:1678); here every failed
// call throws CudaBridgeError carrying the cb_status and the library's message.
// Header-only: link -lcudabridge.
#ifndef RUSTANE_HPP
#define RUSTANE_HPP

#include <algorithm>
#include <array>
#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstdlib>
#include <exception>
#include <memory>
#include <mutex>
#include <numeric>
#include <optional>
#include <stdexcept>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "cuda_bridge.h"

namespace rustane {

class CudaBridgeError : public std::runtime_error {
 public:
  CudaBridgeError(cb_status status, const std::string& what)
      : std::runtime_error(what + " (status " + std::to_string(status) + ")"), status_(status) {}
  cb_status status() const { return status_; }

 private:
  cb_status status_;
};

struct ModelConfig {
  int32_t dim, hidden, heads, kv_heads, hd, seq, nlayers, vocab;

  int32_t q_dim() const { return heads * hd; }
  int32_t kv_dim() const { return kv_heads * hd; }
  int32_t gqa_ratio() const { return heads / kv_heads; }
  // Same estimate as ModelConfig::param_count (model.rs:109-114).
  int64_t param_count() const {
    const int64_t per_layer = 4LL * dim * dim + 3LL * dim * hidden;
    return nlayers * per_layer + (int64_t)vocab * dim + (int64_t)dim * (2 * nlayers + 1);
  }
  cb_model_config c() const { return {dim, hidden, heads, kv_heads, hd, seq, nlayers, vocab}; }
  bool operator==(const ModelConfig& o) const {
    return dim == o.dim && hidden == o.hidden && heads == o.heads && kv_heads == o.kv_heads &&
           hd == o.hd && seq == o.seq && nlayers == o.nlayers && vocab == o.vocab;
  }
  bool operator!=(const ModelConfig& o) const { return !(*this == o); }

  // Reference presets (model.rs).
  static ModelConfig gpt_karpathy() { return {768, 2048, 6, 6, 128, 512, 6, 8192}; }
  static ModelConfig gpt_1024() { return {1024, 2816, 8, 8, 128, 512, 8, 8192}; }
  static ModelConfig target_600m() { return {1536, 4096, 12, 12, 128, 512, 20, 8192}; }
  static ModelConfig target_800m() { return {1792, 4864, 14, 14, 128, 512, 24, 8192}; }
  static ModelConfig target_1b() { return {2048, 5632, 16, 16, 128, 512, 28, 8192}; }
  static ModelConfig target_1_5b() { return {2304, 6144, 18, 18, 128, 512, 32, 8192}; }
  static ModelConfig mha_28l() { return {1024, 3072, 8, 8, 128, 256, 28, 8192}; }
};

// MHA config with hd = 128 (custom_config, tests/bench_fwd_only_scale.rs:24-44).
inline ModelConfig custom_config(int32_t dim, int32_t hidden, int32_t heads, int32_t nlayers,
                                 int32_t seq, int32_t vocab = 8192) {
  return {dim, hidden, heads, heads, 128, seq, nlayers, vocab};
}

// Host f32 layer weights in the reference orientation (x @ W): wq [dim, q_dim],
// wk/wv [dim, kv_dim], wo [q_dim, dim], w1/w3/w2 [dim, hidden], gamma1/gamma2 [dim].
struct LayerWeights {
  std::vector<float> wq, wk, wv, wo, w1, w3, w2, gamma1, gamma2;
};

// Either host arrays or a device-side generator spec (no host copy of the model).
// A context uploads a ModelWeights once and skips later loads of the same generation;
// after changing the arrays in place, call touch() so the next load uploads them.
struct ModelWeights {
  std::vector<float> embed;        // [vocab, dim]
  std::vector<LayerWeights> layers;
  std::vector<float> gamma_final;  // [dim]
  bool generated = false;
  int32_t scheme = CB_INIT_NORMAL;
  uint64_t seed = 0;
  float sigma = 0.02f;
  uint64_t generation = next_generation();

  // The reference's own init (ModelWeights::random, full_model.rs:132-141).
  static ModelWeights random(const ModelConfig&) {
    ModelWeights w;
    w.generated = true;
    w.scheme = CB_INIT_REFERENCE;
    return w;
  }
  // All matrices ~N(0, sigma), gains 1.0 (the benchmark init).
  static ModelWeights normal(const ModelConfig&, uint64_t seed = 0, float sigma = 0.02f) {
    ModelWeights w;
    w.generated = true;
    w.scheme = CB_INIT_NORMAL;
    w.seed = seed;
    w.sigma = sigma;
    return w;
  }
  // A new generation: the next load_weights uploads these arrays again.
  void touch() { generation = next_generation(); }

 private:
  static uint64_t next_generation() {
    static std::atomic<uint64_t> counter{0};
    return ++counter;
  }
};

// The reference's forward workspace; device buffers live in the context here, so it
// carries no state.
struct ModelForwardWorkspace {
  static ModelForwardWorkspace new_(const ModelConfig&) { return {}; }
  static ModelForwardWorkspace new_lean(const ModelConfig&) { return {}; }
};

struct ForwardResult {
  float loss = 0.f;
  std::vector<float> per_token_loss;
};

// Gradients in the reference orientation, laid out like the weights (ModelGrads,
// full_model.rs:26-30, :143-160).
struct ModelGrads {
  std::vector<float> embed, gamma_final;
  std::vector<LayerWeights> layers;

  static ModelGrads zeros(const ModelConfig& c) {
    const size_t d = c.dim, h = c.hidden, qd = c.q_dim(), kvd = c.kv_dim();
    ModelGrads g;
    g.embed.assign((size_t)c.vocab * d, 0.f);
    g.gamma_final.assign(d, 0.f);
    g.layers.resize(c.nlayers);
    for (LayerWeights& l : g.layers) {
      l.wq.assign(d * qd, 0.f), l.wk.assign(d * kvd, 0.f), l.wv.assign(d * kvd, 0.f);
      l.wo.assign(qd * d, 0.f), l.w1.assign(d * h, 0.f), l.w3.assign(d * h, 0.f);
      l.w2.assign(d * h, 0.f), l.gamma1.assign(d, 0.f), l.gamma2.assign(d, 0.f);
    }
    return g;
  }
};

// Sums of an evaluation pass; val_loss and val_bpb as validate forms them
// (train.rs:197-236, compute_bpb data.rs:75-91).
struct EvalTotals {
  double loss_sum = 0, nats = 0;
  int64_t bytes = 0, tokens = 0;
  double val_loss() const { return tokens ? loss_sum / tokens : 0.0; }
  double val_bpb() const { return bytes ? nats / (0.6931471805599453 * bytes) : 0.0; }
  EvalTotals& operator+=(const EvalTotals& o) {
    loss_sum += o.loss_sum, nats += o.nats, bytes += o.bytes, tokens += o.tokens;
    return *this;
  }
};

inline void check(cb_status s, const cb_ctx* ctx, const char* call) {
  if (s == CB_OK) return;
  const char* msg = ctx ? cb_last_error(ctx) : cb_create_error();
  throw CudaBridgeError(s, std::string(call) + ": " + (msg && *msg ? msg : "failed"));
}

// A uint16 token array resident in one device's HBM (TokenData, data.rs:11-44, which
// memory-maps the file; 1e9 tokens take 2 GB).
class DeviceTokens {
 public:
  static DeviceTokens open(const std::string& path, int32_t device = 0) {
    cb_tokens* t = nullptr;
    check(cb_tokens_open(path.c_str(), device, &t), nullptr, "cb_tokens_open");
    return DeviceTokens(t);
  }
  static DeviceTokens from_host(const std::vector<uint16_t>& tokens, int32_t device = 0) {
    cb_tokens* t = nullptr;
    check(cb_tokens_from_host(tokens.data(), (int64_t)tokens.size(), device, &t), nullptr,
          "cb_tokens_from_host");
    return DeviceTokens(t);
  }
  int64_t len() const {
    int64_t n = 0;
    check(cb_tokens_len(t_.get(), &n), nullptr, "cb_tokens_len");
    return n;
  }
  const cb_tokens* handle() const { return t_.get(); }

 private:
  struct Close {
    void operator()(cb_tokens* t) const { cb_tokens_close(t); }
  };
  explicit DeviceTokens(cb_tokens* t) : t_(t) {}
  std::unique_ptr<cb_tokens, Close> t_;
};

// One cb_ctx: device weights, workspace and captured forward graphs for up to
// max_batch sequences on one GPU. Not thread-safe (one per host thread).
class CompiledKernels {
 public:
  CompiledKernels(const ModelConfig& cfg, int32_t device = 0, int32_t max_batch = 1)
      : cfg_(cfg), device_(device), max_batch_(max_batch) {
    const cb_model_config c = cfg.c();
    cb_ctx* h = nullptr;
    check(cb_create(&c, device, max_batch, &h), nullptr, "cb_create");
    ctx_.reset(h);
  }
  static CompiledKernels compile_forward_only(const ModelConfig& cfg, int32_t device = 0,
                                              int32_t max_batch = 1) {
    return CompiledKernels(cfg, device, max_batch);
  }
  static CompiledKernels compile(const ModelConfig& cfg, int32_t device = 0,
                                 int32_t max_batch = 1) {
    return CompiledKernels(cfg, device, max_batch);
  }

  // Tensor parallelism (cb_create_tp; the reference's head- and hidden-sharded layer,
  // layer.rs:1906-2053,4943-5139): rank tp_rank of tp_world, one process or thread per
  // GPU, every rank with the same NCCL unique id (nccl_unique_id() on one rank, handed to
  // the others by the caller). Every rank returns the same losses.
  using NcclId = std::array<uint8_t, 128>;
  CompiledKernels(const ModelConfig& cfg, int32_t device, int32_t max_batch, int32_t tp_rank,
                  int32_t tp_world, const NcclId& nccl_id)
      : cfg_(cfg), device_(device), max_batch_(max_batch) {
    const cb_model_config c = cfg.c();
    cb_ctx* h = nullptr;
    check(cb_create_tp(&c, device, max_batch, tp_rank, tp_world, nccl_id.data(), &h), nullptr,
          "cb_create_tp");
    ctx_.reset(h);
  }
  static NcclId nccl_unique_id() {
    NcclId id{};
    check(cb_nccl_unique_id(id.data()), nullptr, "cb_nccl_unique_id");
    return id;
  }

  // This rank's share: heads, kv heads and hidden columns, and where they start.
  struct TpShare {
    int32_t rank, world, heads, kv_heads, hidden, head0, kv_head0, hidden0;
  };
  static TpShare share_of(const int32_t (&a)[8]) {
    return TpShare{a[0], a[1], a[2], a[3], a[4], a[5], a[6], a[7]};
  }
  TpShare tp_info() const {
    int32_t a[8];
    check(cb_tp_info(ctx_.get(), a), ctx_.get(), "cb_tp_info");
    return share_of(a);
  }
  // The split cb_create_tp would give rank tp_rank, without a context or a GPU.
  static TpShare tp_partition(const ModelConfig& cfg, int32_t tp_world, int32_t tp_rank) {
    const cb_model_config c = cfg.c();
    int32_t a[8];
    check(cb_tp_partition(&c, tp_world, tp_rank, a), nullptr, "cb_tp_partition");
    return share_of(a);
  }
  // Between steps: a peer rank has left (learned by the caller's heartbeat or store); no
  // collective is launched toward it, later calls throw (CB_ERR_NCCL), and the process
  // should destroy the context and exit.
  void tp_peer_lost(const std::string& why) {
    check(cb_tp_peer_lost(ctx_.get(), why.c_str()), ctx_.get(), "cb_tp_peer_lost");
  }

  const ModelConfig& cfg() const { return cfg_; }
  int32_t device() const { return device_; }
  int32_t max_batch() const { return max_batch_; }
  cb_ctx* handle() const { return ctx_.get(); }

  void init_weights(uint64_t seed, int32_t scheme = CB_INIT_NORMAL, float sigma = 0.02f) {
    loaded_generation_ = 0;
    check(cb_init_weights(ctx_.get(), seed, scheme, sigma), ctx_.get(), "cb_init_weights");
  }

  // Uploads (or generates) `w` unless this context already holds it.
  void load_weights(const ModelWeights& w) {
    if (loaded_generation_ == w.generation) return;
    if (w.generated) {
      init_weights(w.seed, w.scheme, w.sigma);
    } else {
      if ((int32_t)w.layers.size() != cfg_.nlayers)
        throw std::invalid_argument("layer count does not match the config");
      // cb_load_weights_f32 reads a fixed number of floats from every pointer: a short
      // vector would be read past its end, so each size is checked against the config.
      const size_t d = cfg_.dim, h = cfg_.hidden, qd = cfg_.q_dim(), kvd = cfg_.kv_dim();
      auto need = [](const std::vector<float>& v, size_t n, const std::string& what) {
        if (v.size() != n)
          throw std::invalid_argument(what + " holds " + std::to_string(v.size()) +
                                      " floats, the config needs " + std::to_string(n));
      };
      need(w.embed, (size_t)cfg_.vocab * d, "embed");
      need(w.gamma_final, d, "gamma_final");
      for (size_t i = 0; i < w.layers.size(); ++i) {
        const LayerWeights& l = w.layers[i];
        const std::string p = "layer " + std::to_string(i) + " ";
        need(l.wq, d * qd, p + "wq"), need(l.wk, d * kvd, p + "wk"), need(l.wv, d * kvd, p + "wv");
        need(l.wo, qd * d, p + "wo"), need(l.w1, d * h, p + "w1"), need(l.w3, d * h, p + "w3");
        need(l.w2, d * h, p + "w2"), need(l.gamma1, d, p + "gamma1");
        need(l.gamma2, d, p + "gamma2");
      }
      // A failed upload leaves the device weights half written: forget the old generation
      // first, so a retry with the same ModelWeights uploads again.
      loaded_generation_ = 0;
      std::vector<cb_layer_weights_f32> arr(w.layers.size());
      for (size_t i = 0; i < w.layers.size(); ++i) {
        const LayerWeights& l = w.layers[i];
        arr[i] = {l.wq.data(), l.wk.data(), l.wv.data(), l.wo.data(), l.w1.data(),
                  l.w3.data(), l.w2.data(), l.gamma1.data(), l.gamma2.data()};
      }
      check(cb_load_weights_f32(ctx_.get(), w.embed.data(), w.gamma_final.data(), arr.data()),
            ctx_.get(), "cb_load_weights_f32");
    }
    loaded_generation_ = w.generation;
  }

  // Mean next-token loss of whole sequences held back to back in tokens/targets;
  // per_token (nullable) receives every position's loss.
  float forward_loss(const std::vector<uint32_t>& tokens, const std::vector<uint32_t>& targets,
                     float softcap = 0.f, std::vector<float>* per_token = nullptr) {
    if (tokens.size() != targets.size() || tokens.empty() || tokens.size() % cfg_.seq != 0)
      throw std::invalid_argument("tokens/targets must hold whole sequences of cfg.seq");
    const int32_t batch = (int32_t)(tokens.size() / cfg_.seq);
    float loss = 0.f;
    if (per_token) per_token->assign(tokens.size(), 0.f);
    check(cb_forward_loss(ctx_.get(), tokens.data(), targets.data(), batch, softcap, &loss,
                          per_token ? per_token->data() : nullptr),
          ctx_.get(), "cb_forward_loss");
    return loss;
  }

  // RSTK checkpoint straight into the device weights; returns the header's step.
  uint32_t load_checkpoint(const std::string& path) {
    uint32_t step = 0;
    check(cb_load_rstk(ctx_.get(), path.c_str(), &step), ctx_.get(), "cb_load_rstk");
    loaded_generation_ = 0;
    return step;
  }

  // One forward over windows of a device token array: sequence b reads tokens
  // data[positions[b] .. + seq) and targets one position later (train.rs:556-558).
  float forward_loss_windows(const DeviceTokens& data, const std::vector<int64_t>& positions,
                             float softcap = 0.f, std::vector<float>* per_token = nullptr) {
    float loss = 0.f;
    if (per_token) per_token->assign(positions.size() * (size_t)cfg_.seq, 0.f);
    check(cb_forward_loss_windows(ctx_.get(), data.handle(), positions.data(),
                                  (int32_t)positions.size(), softcap, &loss,
                                  per_token ? per_token->data() : nullptr),
          ctx_.get(), "cb_forward_loss_windows");
    return loss;
  }

  // Device sums of validation steps [step_begin, step_end); token_bytes (nullable) are
  // the byte lengths of the token ids (TokenBytes, data.rs:47-73).
  EvalTotals eval_windows(const DeviceTokens& data, const std::vector<int32_t>* token_bytes,
                          int64_t step_begin, int64_t step_end, float softcap = 0.f) {
    cb_eval_totals t{};
    check(cb_eval_windows(ctx_.get(), data.handle(), token_bytes ? token_bytes->data() : nullptr,
                          token_bytes ? (int32_t)token_bytes->size() : 0, step_begin, step_end,
                          softcap, &t),
          ctx_.get(), "cb_eval_windows");
    EvalTotals r;
    r.loss_sum = t.loss_sum, r.nats = t.nats, r.bytes = t.bytes, r.tokens = t.tokens;
    return r;
  }

  // ---- training step (full_model.rs:592-702): gradients accumulate on the device
  void enable_training() {
    check(cb_enable_training(ctx_.get()), ctx_.get(), "cb_enable_training");
  }
  void zero_grads() { check(cb_zero_grads(ctx_.get()), ctx_.get(), "cb_zero_grads"); }
  float forward_backward(const std::vector<uint32_t>& tokens,
                         const std::vector<uint32_t>& targets, float softcap = 0.f,
                         float loss_scale = 1.f) {
    if (tokens.size() != targets.size() || tokens.empty() || tokens.size() % cfg_.seq != 0)
      throw std::invalid_argument("tokens/targets must hold whole sequences of cfg.seq");
    float loss = 0.f;
    check(cb_forward_backward(ctx_.get(), tokens.data(), targets.data(),
                              (int32_t)(tokens.size() / cfg_.seq), softcap, loss_scale, &loss),
          ctx_.get(), "cb_forward_backward");
    return loss;
  }
  // Host copy of the accumulated gradients.
  ModelGrads grads() {
    ModelGrads g = ModelGrads::zeros(cfg_);
    std::vector<cb_layer_grads_f32> arr(g.layers.size());
    for (size_t i = 0; i < g.layers.size(); ++i) {
      LayerWeights& l = g.layers[i];
      arr[i] = {l.wq.data(), l.wk.data(), l.wv.data(), l.wo.data(), l.w1.data(),
                l.w3.data(), l.w2.data(), l.gamma1.data(), l.gamma2.data()};
    }
    check(cb_get_grads_f32(ctx_.get(), g.embed.data(), g.gamma_final.data(), arr.data()),
          ctx_.get(), "cb_get_grads_f32");
    return g;
  }

  // ---- single-token decode with a KV cache
  // Prefills `batch` prompts of equal length held back to back; returns each prompt's
  // last-position logits [batch * vocab].
  std::vector<float> prefill(const std::vector<uint32_t>& prompts, int32_t batch,
                             float softcap = 0.f) {
    if (batch <= 0 || prompts.empty() || prompts.size() % (size_t)batch != 0)
      throw std::invalid_argument("prompts must hold batch prompts of equal length");
    std::vector<float> logits((size_t)batch * cfg_.vocab);
    check(cb_prefill(ctx_.get(), prompts.data(), batch, (int32_t)(prompts.size() / batch),
                     softcap, logits.data()),
          ctx_.get(), "cb_prefill");
    return logits;
  }
  // Advances every sequence by one token; returns the greedy next tokens, and the
  // next-token logits [batch * vocab] into `logits` when given.
  std::vector<uint32_t> decode_step(const std::vector<uint32_t>& tokens,
                                    std::vector<float>* logits = nullptr) {
    std::vector<uint32_t> next(tokens.size());
    if (logits) logits->assign(tokens.size() * (size_t)cfg_.vocab, 0.f);
    check(cb_decode_step(ctx_.get(), tokens.data(), (int32_t)tokens.size(),
                         logits ? logits->data() : nullptr, next.data()),
          ctx_.get(), "cb_decode_step");
    return next;
  }
  int32_t decode_position() const {
    int32_t pos = 0;
    check(cb_decode_position(ctx_.get(), &pos), ctx_.get(), "cb_decode_position");
    return pos;
  }

  // Logits of rows (b * seq + s) of the last forward, [rows.size() * vocab].
  std::vector<float> sampled_logits(const std::vector<int32_t>& rows) {
    std::vector<float> out(rows.size() * (size_t)cfg_.vocab);
    check(cb_sampled_logits(ctx_.get(), rows.data(), (int32_t)rows.size(), out.data()),
          ctx_.get(), "cb_sampled_logits");
    return out;
  }

 private:
  struct Destroy {
    void operator()(cb_ctx* c) const { cb_destroy(c); }
  };
  ModelConfig cfg_;
  int32_t device_, max_batch_;
  std::unique_ptr<cb_ctx, Destroy> ctx_;
  uint64_t loaded_generation_ = 0;
};

// full_model.rs:378 / :494: mean next-token cross-entropy.
inline float forward_only_ws(const ModelConfig& cfg, CompiledKernels& kernels,
                             const ModelWeights& weights, const std::vector<uint32_t>& tokens,
                             const std::vector<uint32_t>& targets, float softcap,
                             ModelForwardWorkspace&) {
  if (kernels.cfg() != cfg) throw std::invalid_argument("kernels were compiled for another config");
  kernels.load_weights(weights);
  return kernels.forward_loss(tokens, targets, softcap);
}

inline float forward_ws(const ModelConfig& cfg, CompiledKernels& kernels,
                        const ModelWeights& weights, const std::vector<uint32_t>& tokens,
                        const std::vector<uint32_t>& targets, float softcap,
                        ModelForwardWorkspace& ws) {
  return forward_only_ws(cfg, kernels, weights, tokens, targets, softcap, ws);
}

// full_model.rs:915: loss and the per-position losses.
inline ForwardResult forward(const ModelConfig& cfg, CompiledKernels& kernels,
                             const ModelWeights& weights, const std::vector<uint32_t>& tokens,
                             const std::vector<uint32_t>& targets, float softcap = 0.f) {
  if (kernels.cfg() != cfg) throw std::invalid_argument("kernels were compiled for another config");
  kernels.load_weights(weights);
  ForwardResult r;
  r.loss = kernels.forward_loss(tokens, targets, softcap, &r.per_token_loss);
  return r;
}

// full_model.rs:1603: per-position losses.
inline std::vector<float> forward_losses(const ModelConfig& cfg, CompiledKernels& kernels,
                                         const ModelWeights& weights,
                                         const std::vector<uint32_t>& tokens,
                                         const std::vector<uint32_t>& targets,
                                         float softcap = 0.f) {
  return forward(cfg, kernels, weights, tokens, targets, softcap).per_token_loss;
}

// Sequence-parallel forward workers (multistream.rs:54-161): one CompiledKernels per
// entry of `devices`, each driven by its own host thread, pulling whole sequences;
// losses come back in request order. No communication between workers.
class ForwardScheduler {
 public:
  using Request = std::pair<std::vector<uint32_t>, std::vector<uint32_t>>;

  ForwardScheduler(const ModelConfig& cfg, const ModelWeights& weights,
                   const std::vector<int32_t>& devices, int32_t max_batch = 1) {
    for (int32_t d : devices) {
      workers_.emplace_back(new CompiledKernels(cfg, d, max_batch));
      workers_.back()->load_weights(weights);
    }
  }

  std::vector<float> run_batch(const std::vector<Request>& requests, float softcap = 0.f) {
    std::vector<float> out(requests.size(), 0.f);
    std::atomic<size_t> next{0};
    std::mutex err_mu;
    std::exception_ptr err;
    auto work = [&](CompiledKernels* k) {
      for (;;) {
        const size_t i = next.fetch_add(1);
        if (i >= requests.size()) return;
        try {
          out[i] = k->forward_loss(requests[i].first, requests[i].second, softcap);
        } catch (...) {
          std::lock_guard<std::mutex> lk(err_mu);
          if (!err) err = std::current_exception();
          return;
        }
      }
    };
    std::vector<std::thread> threads;
    for (auto& w : workers_) threads.emplace_back(work, w.get());
    for (auto& t : threads) t.join();
    if (err) std::rethrow_exception(err);
    return out;
  }

 private:
  std::vector<std::unique_ptr<CompiledKernels>> workers_;
};

// ---------------------------------------------------------------- ParallelBenchRunner

class ParallelBenchError : public std::invalid_argument {
 public:
  using std::invalid_argument::invalid_argument;
};

enum class ShardPolicy { FailFast, AutoAdjustNearest };

// Sorted divisors (sharding.rs:286-300).
inline std::vector<int32_t> divisors(int32_t value) {
  std::vector<int32_t> out;
  for (int32_t i = 1; (int64_t)i * i <= value; ++i)
    if (value % i == 0) {
      out.push_back(i);
      if (i != value / i) out.push_back(value / i);
    }
  std::sort(out.begin(), out.end());
  return out;
}

// The divisor closest to `requested`; the smaller one on a tie (sharding.rs:302-307).
inline int32_t nearest_divisor(const std::vector<int32_t>& divs, int32_t requested) {
  return *std::min_element(divs.begin(), divs.end(), [&](int32_t a, int32_t b) {
    const int64_t da = std::llabs((int64_t)requested - a), db = std::llabs((int64_t)requested - b);
    return da != db ? da < db : a < b;
  });
}

inline std::string join(const std::vector<int32_t>& v) {
  std::string s;
  for (size_t i = 0; i < v.size(); ++i) s += (i ? ", " : "") + std::to_string(v[i]);
  return s;
}

// One forward axis (sharding.rs:227-260): unset -> 1 shard; a divisor -> itself;
// otherwise FailFast throws and AutoAdjustNearest takes the nearest divisor.
inline int32_t resolve_axis(const std::string& axis, const std::string& shape_name,
                            int32_t shape_value, std::optional<int32_t> requested,
                            ShardPolicy policy, std::vector<std::string>* notes) {
  if (!requested) return 1;
  if (*requested <= 0) throw ParallelBenchError(axis + " must be positive");
  const std::vector<int32_t> valid = divisors(shape_value);
  if (std::find(valid.begin(), valid.end(), *requested) != valid.end()) return *requested;
  const std::string where = shape_name + "=" + std::to_string(shape_value);
  if (policy == ShardPolicy::FailFast)
    throw ParallelBenchError(axis + "=" + std::to_string(*requested) + " is invalid for " +
                             where + "; valid divisors: " + join(valid));
  const int32_t applied = nearest_divisor(valid, *requested);
  notes->push_back("requested " + axis + "=" + std::to_string(*requested) + ", applied " +
                   std::to_string(applied) + " (nearest valid divisor for " + where + ")");
  return applied;
}

inline std::optional<int32_t> env_count(const char* var) {
  const char* raw = std::getenv(var);
  if (!raw) return std::nullopt;
  char* end = nullptr;
  const long v = std::strtol(raw, &end, 10);
  if (end == raw || *end != '\0')
    throw ParallelBenchError(std::string(var) + " must be an integer, got '" + raw + "'");
  if (v <= 0) throw ParallelBenchError(std::string(var) + " must be positive");
  return (int32_t)v;
}

// Requested forward shard counts (parallel_bench.rs:24-39).
struct ParallelBenchRequest {
  std::optional<int32_t> attn_request, ffn_request;
  ShardPolicy policy = ShardPolicy::FailFast;

  // ATTN_FWD_SHARDS / FFN_FWD_SHARDS, or the ATTN_SHARDS / FFN_SHARDS shorthand (not
  // both for one axis), as ShardRequest::from_env (sharding.rs:64-100) reads them.
  static ParallelBenchRequest from_env(ShardPolicy policy = ShardPolicy::FailFast) {
    ParallelBenchRequest r;
    r.policy = policy;
    const char* names[2][4] = {{"ATTN_SHARDS", "ATTN_FWD_SHARDS", "ATTN_BWD_SHARDS", "attention"},
                               {"FFN_SHARDS", "FFN_FWD_SHARDS", "FFN_BWD_SHARDS", "FFN"}};
    for (int a = 0; a < 2; ++a) {
      const auto shorthand = env_count(names[a][0]);
      const auto fwd = env_count(names[a][1]);
      const auto bwd = env_count(names[a][2]);
      if (shorthand && (fwd || bwd))
        throw ParallelBenchError(std::string(names[a][0]) + "=" + std::to_string(*shorthand) +
                                 " conflicts with per-direction " + names[a][3] +
                                 " shard vars; use per-direction vars or the shorthand, "
                                 "not both");
      (a == 0 ? r.attn_request : r.ffn_request) = shorthand ? shorthand : fwd;
    }
    return r;
  }
};

// What a request resolved to (parallel_bench.rs:57-88).
struct ResolvedParallelBenchConfig {
  std::optional<int32_t> requested_attn, requested_ffn;
  int32_t applied_attn = 1, applied_ffn = 1;
  std::vector<std::string> notes;

  std::string mode_label() const {
    const bool a = applied_attn > 1, f = applied_ffn > 1;
    if (a && f) return "attn" + std::to_string(applied_attn) + "_ffn" + std::to_string(applied_ffn);
    if (a) return "attn" + std::to_string(applied_attn);
    if (f) return "ffn" + std::to_string(applied_ffn);
    return "baseline";
  }
  std::string benchmark_suffix() const {
    const std::string l = mode_label();
    return l == "baseline" ? "" : "_" + l;
  }
};

// resolve_parallel_bench_config (parallel_bench.rs:316-364): attention splits into
// groups of kv heads (gcd(heads, kv_heads) of them), the FFN along the hidden width.
inline ResolvedParallelBenchConfig resolve_parallel_bench_config(
    const ModelConfig& cfg, const ParallelBenchRequest& req) {
  ResolvedParallelBenchConfig r;
  r.requested_attn = req.attn_request;
  r.requested_ffn = req.ffn_request;
  r.applied_attn = resolve_axis("ATTN_FWD_SHARDS", "attention group count",
                                std::gcd(cfg.heads, cfg.kv_heads), req.attn_request, req.policy,
                                &r.notes);
  r.applied_ffn = resolve_axis("FFN_FWD_SHARDS", "hidden width", cfg.hidden, req.ffn_request,
                               req.policy, &r.notes);
  return r;
}

// ParallelBenchRunner (parallel_bench.rs:110-290) on one B200: every resolved mode runs
// the same single-context forward, since each kernel already covers all heads and hidden
// columns of a layer that the reference splits into side-by-side ANE programs.
class ParallelBenchRunner {
 public:
  // (runner, compile seconds); an invalid request throws ParallelBenchError before
  // anything is compiled (parallel_bench.rs:165-233).
  static std::pair<ParallelBenchRunner, float> compile(const ModelConfig& cfg,
                                                       const ParallelBenchRequest& request = {},
                                                       bool use_lean_workspace = true,
                                                       int32_t device = 0,
                                                       int32_t max_batch = 1) {
    ResolvedParallelBenchConfig resolved = resolve_parallel_bench_config(cfg, request);
    const auto t0 = std::chrono::steady_clock::now();
    CompiledKernels k(cfg, device, max_batch);
    const float s = std::chrono::duration<float>(std::chrono::steady_clock::now() - t0).count();
    return {ParallelBenchRunner(cfg, std::move(resolved), std::move(k), use_lean_workspace), s};
  }

  const ResolvedParallelBenchConfig& resolved() const { return resolved_; }
  CompiledKernels& kernels() { return kernels_; }
  bool use_lean_workspace() const { return lean_; }

  // Mean next-token loss of the sequences in tokens/targets (parallel_bench.rs:239-289).
  float forward_loss(const ModelWeights& weights, const std::vector<uint32_t>& tokens,
                     const std::vector<uint32_t>& targets, float softcap,
                     ModelForwardWorkspace& ws) {
    return forward_only_ws(cfg_, kernels_, weights, tokens, targets, softcap, ws);
  }

 private:
  ParallelBenchRunner(const ModelConfig& cfg, ResolvedParallelBenchConfig resolved,
                      CompiledKernels kernels, bool lean)
      : cfg_(cfg), resolved_(std::move(resolved)), kernels_(std::move(kernels)), lean_(lean) {}
  ModelConfig cfg_;
  ResolvedParallelBenchConfig resolved_;
  CompiledKernels kernels_;
  bool lean_;
};

}  // namespace rustane

#endif  // RUSTANE_HPP
