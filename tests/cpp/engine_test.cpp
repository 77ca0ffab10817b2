// C++ tests of the host API in include/rustane.hpp, written like the reference engine's
// own Rust tests of the same calls. Built and run by tests/test_host_cpp.py:
//   engine_test cpu   host-only checks (configs, errors), no device needed
//   engine_test gpu   forward through CompiledKernels / forward_only_ws / forward /
//                     forward_losses / ForwardScheduler on device 0, checked against
//                     the CPU oracle (oracle/liboracle.so, test infrastructure) with
//                     the tolerances of the Python parity tests
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include <unistd.h>

#include "rustane.hpp"

// The CPU oracle's C interface (oracle/forward_ref.cpp).
extern "C" {
struct orc_config {
  int32_t dim, hidden, heads, kv_heads, hd, seq, nlayers, vocab;
};
struct orc_layer {
  float *wq, *wk, *wv, *wo, *w1, *w3, *w2, *gamma1, *gamma2;
};
int orc_gen_weights(const orc_config* cfg, uint64_t seed, int scheme, float sigma, float* embed,
                    float* gamma_final, const orc_layer* layers);
int orc_forward(const orc_config* cfg, const float* embed, const float* gamma_final,
                const orc_layer* layers, const uint32_t* tokens, const uint32_t* targets,
                int batch, float softcap, float* loss, float* per_token_loss,
                const int32_t* sample_rows, int n_sample, float* sampled_logits);
}

using namespace rustane;

static int failures = 0;
#define EXPECT(cond)                                              \
  do {                                                            \
    if (!(cond)) {                                                \
      std::fprintf(stderr, "FAILED line %d: %s\n", __LINE__, #cond); \
      ++failures;                                                 \
    }                                                             \
  } while (0)

template <class F>
static bool throws_status(F f, cb_status want, const char* text) {
  try {
    f();
  } catch (const CudaBridgeError& e) {
    return e.status() == want && std::strstr(e.what(), text) != nullptr;
  }
  return false;
}

template <class F>
static bool throws_bench_error(F f, const char* text) {
  try {
    f();
  } catch (const ParallelBenchError& e) {
    return std::strstr(e.what(), text) != nullptr;
  }
  return false;
}

// parallel_bench.rs / sharding.rs host logic (request parsing, resolution, labels).
static void bench_runner_tests() {
  // sharding.rs:326-368: divisors sorted; the smaller divisor wins a tie
  EXPECT(divisors(12) == std::vector<int32_t>({1, 2, 3, 4, 6, 12}));
  EXPECT(divisors(52) == std::vector<int32_t>({1, 2, 4, 13, 26, 52}));
  EXPECT(nearest_divisor(divisors(12), 5) == 4 && nearest_divisor(divisors(52), 8) == 4);

  const char* vars[] = {"ATTN_SHARDS", "FFN_SHARDS", "ATTN_FWD_SHARDS", "FFN_FWD_SHARDS",
                        "ATTN_BWD_SHARDS", "FFN_BWD_SHARDS"};
  for (const char* v : vars) unsetenv(v);
  ParallelBenchRequest r = ParallelBenchRequest::from_env();
  EXPECT(!r.attn_request && !r.ffn_request);
  setenv("ATTN_FWD_SHARDS", "4", 1);
  setenv("FFN_SHARDS", "8", 1);
  r = ParallelBenchRequest::from_env(ShardPolicy::AutoAdjustNearest);
  EXPECT(r.attn_request == 4 && r.ffn_request == 8 && r.policy == ShardPolicy::AutoAdjustNearest);
  setenv("ATTN_FWD_SHARDS", "x", 1);
  EXPECT(throws_bench_error([] { ParallelBenchRequest::from_env(); }, "must be an integer"));
  setenv("ATTN_FWD_SHARDS", "0", 1);
  EXPECT(throws_bench_error([] { ParallelBenchRequest::from_env(); }, "must be positive"));
  unsetenv("ATTN_FWD_SHARDS");
  setenv("FFN_BWD_SHARDS", "2", 1);
  EXPECT(throws_bench_error([] { ParallelBenchRequest::from_env(); }, "conflicts"));
  for (const char* v : vars) unsetenv(v);

  const ModelConfig cfg = ModelConfig::target_600m();  // 12 heads, hidden 4096
  ParallelBenchRequest q;
  EXPECT(resolve_parallel_bench_config(cfg, q).mode_label() == "baseline");
  EXPECT(resolve_parallel_bench_config(cfg, q).benchmark_suffix().empty());
  q.attn_request = 4;
  q.ffn_request = 8;
  EXPECT(resolve_parallel_bench_config(cfg, q).benchmark_suffix() == "_attn4_ffn8");
  q.ffn_request.reset();
  q.attn_request = 5;
  EXPECT(throws_bench_error([&] { resolve_parallel_bench_config(cfg, q); }, "valid divisors"));
  EXPECT(throws_bench_error([&] { ParallelBenchRunner::compile(cfg, q); }, "valid divisors"));
  q.policy = ShardPolicy::AutoAdjustNearest;
  const ResolvedParallelBenchConfig adj = resolve_parallel_bench_config(cfg, q);
  EXPECT(adj.applied_attn == 4 && adj.requested_attn == 5 && adj.mode_label() == "attn4");
  EXPECT(adj.notes.size() == 1 && adj.notes[0].find("applied 4") != std::string::npos);
  // test_combined_forward_correctness.rs:245-268: one attention group, 8 requested -> baseline
  const ModelConfig odd = {256, 768, 1, 1, 128, 16, 2, 256};
  ParallelBenchRequest o;
  o.attn_request = 8;
  o.policy = ShardPolicy::AutoAdjustNearest;
  EXPECT(resolve_parallel_bench_config(odd, o).mode_label() == "baseline");
  int32_t n = 0;
  cb_device_count(&n);
  if (n == 0)
    EXPECT(throws_status([&] { ParallelBenchRunner::compile(cfg, q); }, CB_ERR_UNSUPPORTED,
                         "no CUDA device"));
}

static void host_type_tests() {
  const ModelConfig c = custom_config(256, 512, 2, 2, 128, 1024);
  const ModelGrads g = ModelGrads::zeros(c);
  EXPECT(g.embed.size() == 1024u * 256 && g.layers.size() == 2);
  EXPECT(g.layers[1].wq.size() == 256u * 256 && g.layers[1].w2.size() == 256u * 512);
  EvalTotals t;
  t.loss_sum = 20.0, t.tokens = 10, t.nats = 6.931471805599453, t.bytes = 5;
  EvalTotals u = t;
  u += t;
  EXPECT(std::fabs(t.val_loss() - 2.0) < 1e-12 && std::fabs(u.val_bpb() - 2.0) < 1e-12);
  bool threw = false;
  try {
    DeviceTokens::open("/nonexistent/tokens.bin", 0);
  } catch (const CudaBridgeError& e) {
    threw = e.status() != CB_OK;
  }
  EXPECT(threw);
}

// The tensor-parallel split as the C++ API reports it (no context, no GPU): 52 heads and
// 17920 hidden columns (280 blocks of 64) over 8 ranks, every head and column once.
static void tp_split_tests() {
  const ModelConfig c = custom_config(6656, 17920, 52, 60, 2048);
  int32_t heads = 0, hidden = 0, next_head = 0, next_col = 0;
  for (int32_t r = 0; r < 8; ++r) {
    const CompiledKernels::TpShare s = CompiledKernels::tp_partition(c, 8, r);
    EXPECT(s.rank == r && s.world == 8);
    EXPECT(s.heads == (r < 4 ? 7 : 6) && s.kv_heads == s.heads);
    EXPECT(s.head0 == next_head && s.hidden0 == next_col && s.hidden % 64 == 0);
    heads += s.heads, hidden += s.hidden;
    next_head += s.heads, next_col += s.hidden;
  }
  EXPECT(heads == 52 && hidden == 17920);
  EXPECT(throws_status([&] { CompiledKernels::tp_partition(c, 53, 0); }, CB_ERR_INVALID_ARG,
                       "larger than the kv heads"));
}

static void cpu_tests() {
  bench_runner_tests();
  host_type_tests();
  tp_split_tests();
  // model.rs doc comment: 600M preset ~579M parameters
  EXPECT(std::fabs(ModelConfig::target_600m().param_count() / 1e6 - 579.0) < 1.0);
  const ModelConfig c = custom_config(1536, 4096, 12, 20, 512);
  EXPECT(c == ModelConfig::target_600m() && c.q_dim() == 1536 && c.gqa_ratio() == 1);
  ModelConfig bad = c;
  bad.hd = 64;
  EXPECT(throws_status([&] { CompiledKernels k(bad); }, CB_ERR_INVALID_ARG, "hd must be 128"));
  int32_t n = 0;
  EXPECT(cb_device_count(&n) == CB_OK);
  ModelWeights a = ModelWeights::normal(c, 1), b = a;
  EXPECT(a.generation == b.generation);
  b.touch();
  EXPECT(b.generation != a.generation);
  if (n == 0)
    EXPECT(throws_status([&] { CompiledKernels::compile_forward_only(c); }, CB_ERR_UNSUPPORTED,
                         "no CUDA device"));
}

struct Oracle {
  orc_config c;
  std::vector<float> embed, gamma_final;
  std::vector<LayerWeights> layers;
  std::vector<orc_layer> ptrs;
  Oracle(const ModelConfig& m, uint64_t seed, float sigma)
      : c{m.dim, m.hidden, m.heads, m.kv_heads, m.hd, m.seq, m.nlayers, m.vocab} {
    const size_t d = m.dim, h = m.hidden, qd = m.q_dim(), kvd = m.kv_dim();
    embed.resize((size_t)m.vocab * d);
    gamma_final.resize(d);
    layers.resize(m.nlayers);
    for (auto& l : layers) {
      l.wq.resize(d * qd), l.wk.resize(d * kvd), l.wv.resize(d * kvd), l.wo.resize(qd * d);
      l.w1.resize(d * h), l.w3.resize(d * h), l.w2.resize(d * h);
      l.gamma1.resize(d), l.gamma2.resize(d);
      ptrs.push_back({l.wq.data(), l.wk.data(), l.wv.data(), l.wo.data(), l.w1.data(),
                      l.w3.data(), l.w2.data(), l.gamma1.data(), l.gamma2.data()});
    }
    orc_gen_weights(&c, seed, CB_INIT_NORMAL, sigma, embed.data(), gamma_final.data(),
                    ptrs.data());
  }
  float loss(const std::vector<uint32_t>& t, const std::vector<uint32_t>& g) const {
    float l = 0.f;
    orc_forward(&c, embed.data(), gamma_final.data(), ptrs.data(), t.data(), g.data(),
                (int)(t.size() / c.seq), 0.f, &l, nullptr, nullptr, 0, nullptr);
    return l;
  }
};

static std::vector<uint32_t> random_tokens(size_t n, uint32_t vocab, uint32_t seed) {
  std::mt19937 rng(seed);
  std::vector<uint32_t> v(n);
  for (auto& x : v) x = rng() % vocab;
  return v;
}

// RSTK file (bin/train.rs:238-273): "RSTK", u32 version 1, step, dim, nlayers, vocab,
// seq, then the f32 tensors in checkpoint order.
static std::string write_rstk(const ModelConfig& c, const Oracle& o, uint32_t step) {
  char tmpl[] = "/tmp/engine_test_XXXXXX";
  const int fd = mkstemp(tmpl);
  if (fd < 0) throw std::runtime_error("mkstemp failed");
  FILE* f = fdopen(fd, "wb");
  const uint32_t h[6] = {1u, step, (uint32_t)c.dim, (uint32_t)c.nlayers, (uint32_t)c.vocab,
                         (uint32_t)c.seq};
  std::fwrite("RSTK", 1, 4, f);
  std::fwrite(h, 4, 6, f);
  auto put = [&](const std::vector<float>& v) { std::fwrite(v.data(), 4, v.size(), f); };
  put(o.embed);
  put(o.gamma_final);
  for (const LayerWeights& l : o.layers) {
    put(l.wq), put(l.wk), put(l.wv), put(l.wo), put(l.w1), put(l.w3), put(l.w2);
    put(l.gamma1), put(l.gamma2);
  }
  std::fclose(f);
  return tmpl;
}

// The wrappers of the later rows on a GPU: weight-size checks, checkpoint load, device
// token windows and evaluation sums, the training step with its gradients, prefill and
// decode. Each is compared with the forward the earlier checks pinned to the oracle.
static void later_row_tests(const ModelConfig& cfg, const Oracle& ora, const ModelWeights& w,
                            const std::vector<uint32_t>& tok, const std::vector<uint32_t>& tgt,
                            float loss) {
  CompiledKernels k(cfg, 0, 2);
  ModelForwardWorkspace ws = ModelForwardWorkspace::new_lean(cfg);
  EXPECT(forward_only_ws(cfg, k, w, tok, tgt, 0.f, ws) == loss);

  // a short weight vector is refused before any copy; the loaded weights stay usable
  ModelWeights bad;
  bad.embed = ora.embed;
  bad.layers = ora.layers;
  bad.gamma_final = ora.gamma_final;
  bad.layers[1].wq.resize(bad.layers[1].wq.size() - 1);
  bool refused = false;
  try {
    k.load_weights(bad);
  } catch (const std::invalid_argument& e) {
    refused = std::strstr(e.what(), "layer 1 wq") != nullptr;
  }
  EXPECT(refused);
  EXPECT(k.forward_loss(tok, tgt) == loss);

  // checkpoint: the file of the oracle's arrays loads to the same bits as the device init
  const std::string path = write_rstk(cfg, ora, 1234);
  EXPECT(k.load_checkpoint(path) == 1234u);
  EXPECT(k.forward_loss(tok, tgt) == loss);
  std::remove(path.c_str());

  // token windows from a device-resident array equal the host-token forward
  std::vector<uint16_t> stream(3 * cfg.seq + 1);
  for (size_t i = 0; i < stream.size(); ++i) stream[i] = (uint16_t)((i * 7919u + 13u) % cfg.vocab);
  const DeviceTokens data = DeviceTokens::from_host(stream, 0);
  EXPECT(data.len() == (int64_t)stream.size());
  const std::vector<int64_t> pos = {0, (int64_t)cfg.seq + 5};
  std::vector<uint32_t> wt, wg;
  for (int64_t p0 : pos)
    for (int32_t i = 0; i < cfg.seq; ++i) {
      wt.push_back(stream[p0 + i]);
      wg.push_back(stream[p0 + i + 1]);
    }
  std::vector<float> ptl_win, ptl_host;
  const float l_win = k.forward_loss_windows(data, pos, 0.f, &ptl_win);
  const float l_host = k.forward_loss(wt, wg, 0.f, &ptl_host);
  EXPECT(l_win == l_host && ptl_win == ptl_host);
  // validation steps 0 and 1 evaluate the windows at (vs * seq) % (n - seq - 1) = 0 and
  // seq: their sums equal the per-token losses of those windows (train.rs:197-236)
  const EvalTotals tot = k.eval_windows(data, nullptr, 0, 2);
  std::vector<float> ptl_val;
  k.forward_loss_windows(data, {0, (int64_t)cfg.seq}, 0.f, &ptl_val);
  double want_sum = 0;
  for (float x : ptl_val) want_sum += x;
  EXPECT(tot.tokens == 2 * (int64_t)cfg.seq);
  EXPECT(std::fabs(tot.loss_sum - want_sum) <= 1e-6 * want_sum);

  // training step: the loss equals the forward's, gradients accumulate and zero
  k.enable_training();
  k.zero_grads();
  const float l_train = k.forward_backward(tok, tgt);
  EXPECT(std::fabs(l_train - loss) <= 1e-4f * loss);
  ModelGrads g1 = k.grads();
  double n1 = 0;
  for (float x : g1.layers[0].wq) n1 += (double)x * x;
  EXPECT(n1 > 0 && std::isfinite(n1));
  k.forward_backward(tok, tgt);
  ModelGrads g2 = k.grads();
  double d2 = 0;
  for (size_t i = 0; i < g1.layers[0].wq.size(); ++i) {
    const double e = g2.layers[0].wq[i] - 2.0 * g1.layers[0].wq[i];
    d2 += e * e;
  }
  EXPECT(d2 <= 1e-8 * 4 * n1);
  k.zero_grads();
  ModelGrads g0 = k.grads();
  EXPECT(std::all_of(g0.embed.begin(), g0.embed.end(), [](float x) { return x == 0.f; }));

  // prefill + one decode step against the forward's logits at the same positions
  const int32_t plen = 40;
  std::vector<uint32_t> prompt(tok.begin(), tok.begin() + plen);
  const std::vector<float> last = k.prefill(prompt, 1);
  std::vector<float> step_logits;
  const std::vector<uint32_t> nxt = k.decode_step({tok[plen]}, &step_logits);
  EXPECT(k.decode_position() == plen + 1 && nxt.size() == 1);
  const std::vector<uint32_t> one_tok(tok.begin(), tok.begin() + cfg.seq);
  const std::vector<uint32_t> one_tgt(tgt.begin(), tgt.begin() + cfg.seq);
  k.forward_loss(one_tok, one_tgt);
  const std::vector<float> z = k.sampled_logits({plen - 1, plen});
  float dz = 0.f;
  for (int32_t v = 0; v < cfg.vocab; ++v) {
    dz = std::max(dz, std::fabs(last[v] - z[v]));
    dz = std::max(dz, std::fabs(step_logits[v] - z[cfg.vocab + v]));
  }
  EXPECT(dz <= 2e-2f);  // the parity tests' logit tolerance
  const uint32_t argmax = (uint32_t)(std::max_element(step_logits.begin(), step_logits.end()) -
                                     step_logits.begin());
  EXPECT(nxt[0] == argmax);
  std::printf("gpu: later rows ok (decode logits max|d| %.2e)\n", dz);
}

static void gpu_tests() {
  const ModelConfig cfg = custom_config(256, 512, 2, 2, 128, 1024);
  const ModelWeights w = ModelWeights::normal(cfg, 1, 0.05f);
  const auto tok = random_tokens(2 * cfg.seq, cfg.vocab, 5);
  const auto tgt = random_tokens(2 * cfg.seq, cfg.vocab, 6);
  const Oracle ora(cfg, 1, 0.05f);
  const float want = ora.loss(tok, tgt);

  CompiledKernels k = CompiledKernels::compile_forward_only(cfg, 0, 2);
  ModelForwardWorkspace ws = ModelForwardWorkspace::new_lean(cfg);
  const float loss = forward_only_ws(cfg, k, w, tok, tgt, 0.f, ws);
  EXPECT(std::fabs(loss - want) / want <= 1e-3f);  // the parity tests' loss tolerance

  const ForwardResult r = forward(cfg, k, w, tok, tgt);
  double mean = 0;
  for (float x : r.per_token_loss) mean += x;
  mean /= r.per_token_loss.size();
  EXPECT(r.loss == loss && std::fabs(mean - loss) < 1e-5);
  EXPECT(forward_losses(cfg, k, w, tok, tgt) == r.per_token_loss);

  // host arrays in the reference orientation give the device generator's bits
  ModelWeights host;
  host.embed = ora.embed;
  host.layers = ora.layers;
  host.gamma_final = ora.gamma_final;
  EXPECT(forward_only_ws(cfg, k, host, tok, tgt, 0.f, ws) == loss);
  // changed in place: the same generation is not uploaded again until touch()
  for (float& x : host.embed) x *= 2.f;
  EXPECT(forward_only_ws(cfg, k, host, tok, tgt, 0.f, ws) == loss);
  host.touch();
  EXPECT(forward_only_ws(cfg, k, host, tok, tgt, 0.f, ws) != loss);

  bool rejected = false;
  try {
    k.forward_loss(std::vector<uint32_t>(cfg.seq + 1), std::vector<uint32_t>(cfg.seq + 1));
  } catch (const std::invalid_argument&) {
    rejected = true;
  }
  EXPECT(rejected);

  // two workers (both on device 0 here) return every loss in request order
  std::vector<ForwardScheduler::Request> reqs;
  std::vector<float> single;
  for (uint32_t i = 0; i < 4; ++i) {
    reqs.push_back({random_tokens(cfg.seq, cfg.vocab, 20 + i),
                    random_tokens(cfg.seq, cfg.vocab, 30 + i)});
  }
  CompiledKernels one(cfg, 0, 1);
  for (const auto& q : reqs) single.push_back(forward_only_ws(cfg, one, w, q.first, q.second, 0.f, ws));
  ForwardScheduler sched(cfg, w, {0, 0});
  const std::vector<float> got = sched.run_batch(reqs);
  for (size_t i = 0; i < reqs.size(); ++i) EXPECT(std::fabs(got[i] - single[i]) <= 1e-6f);
  std::printf("gpu: loss %.6f oracle %.6f\n", loss, want);
  later_row_tests(cfg, ora, w, tok, tgt, loss);
}

int main(int argc, char** argv) {
  const std::string mode = argc > 1 ? argv[1] : "cpu";
  try {
    if (mode == "cpu") cpu_tests();
    else gpu_tests();
  } catch (const std::exception& e) {
    std::fprintf(stderr, "exception: %s\n", e.what());
    ++failures;
  }
  std::printf(failures ? "engine_test %s: %d failure(s)\n" : "engine_test %s: ok\n",
              mode.c_str(), failures);
  return failures ? 1 : 0;
}
