// CPU ORACLE — test infrastructure only. Never linked into or called by the
// product path (rustane_b200/libcudabridge.so); only tests/, the smoke check in
// __graft_entry__.py and bench.py's CPU-baseline/reference legs load it.
//
// A same-math fp32 restatement of the reference engine's forward pass + loss
// (whiskeypolitik/rustane, crates/engine), written from the reference's math:
//   model flow         full_model.rs:378-472 (forward_only_ws), :283-329 (finalize)
//   layer flow         layer.rs:4409-4624 (forward), alpha = 1/sqrt(2L) at :4420,
//                      residual x2 = x + alpha*o at :4471 (vDSP_vsma)
//   embedding          cpu/embedding.rs:8-17
//   RMSNorm            cpu/rmsnorm.rs:149-183, EPS = 1e-5 (:10)
//   QKV + RoPE + SDPA  kernels/sdpa_fwd.rs:24-60 (RoPE table, interleaved pairs),
//                      :117-150 (x @ Wq/Wk/Wv), :213-258 (scale 1/sqrt(hd),
//                      causal mask, softmax, P @ V)
//   O projection       kernels/dyn_matmul.rs:15-75, layer.rs:4918-4930
//   SwiGLU FFN         kernels/ffn_fused.rs:79-80 (h1, h3), :105-107 (silu gate),
//                      :130 (gate @ W2^T), :144-154 (residual)
//   LM head            full_model.rs:436-454 (tied: logits = x_final @ embed^T,
//                      cpu/vdsp.rs:354-376 sgemm_at)
//   softcap            full_model.rs:456-461
//   cross-entropy      cpu/cross_entropy.rs:58-96, mean over positions full_model.rs:471
// The reference is channel-first [dim, seq]; this restatement is token-major
// [tokens, dim]; the arithmetic per element is the same.
//
// Weights come from rustane_b200/csrc/weight_init.h, the generator the CUDA
// bridge also uses, so both sides see bit-identical fp16-valued weights.
// Accumulations that the reference does in f32 (norm sums, CE log-sum-exp) are
// done in double here: the oracle is the accuracy reference.
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "../rustane_b200/csrc/weight_init.h"

extern "C" {

typedef struct orc_config {
  int32_t dim, hidden, heads, kv_heads, hd, seq, nlayers, vocab;
} orc_config;

typedef struct orc_layer {
  float *wq, *wk, *wv, *wo, *w1, *w3, *w2, *gamma1, *gamma2;
} orc_layer;

}  // extern "C"

namespace {

// ------------------------------------------------------------ packed SGEMM
// C[M,N] (=|+=) A[M,K] * op(B), op(B) = B[K,N] (b_trans = 0) or B[N,K]^T (b_trans = 1).
typedef float v8 __attribute__((vector_size(32)));
typedef float v8u __attribute__((vector_size(32), aligned(4)));

constexpr int MR = 6, NR = 16, MC = 48, NC = 128, KC = 256;

inline v8 ld8(const float* p) { return *reinterpret_cast<const v8u*>(p); }
inline void st8(float* p, v8 v) { *reinterpret_cast<v8u*>(p) = v; }

// a: packed [kc][MR], b: packed [kc][NR]; writes an MR x NR tile into c (ldc).
void micro_6x16(int kc, const float* a, const float* b, float* c, int ldc, int mr, int nr,
                bool accumulate) {
  v8 acc[MR][2];
  for (int i = 0; i < MR; ++i) acc[i][0] = acc[i][1] = (v8){0, 0, 0, 0, 0, 0, 0, 0};
  for (int k = 0; k < kc; ++k) {
    v8 b0 = ld8(b + k * NR), b1 = ld8(b + k * NR + 8);
    const float* ak = a + k * MR;
    for (int i = 0; i < MR; ++i) {
      v8 ai = (v8){ak[i], ak[i], ak[i], ak[i], ak[i], ak[i], ak[i], ak[i]};
      acc[i][0] += ai * b0;
      acc[i][1] += ai * b1;
    }
  }
  if (mr == MR && nr == NR) {
    for (int i = 0; i < MR; ++i) {
      float* ci = c + (size_t)i * ldc;
      if (accumulate) {
        st8(ci, ld8(ci) + acc[i][0]);
        st8(ci + 8, ld8(ci + 8) + acc[i][1]);
      } else {
        st8(ci, acc[i][0]);
        st8(ci + 8, acc[i][1]);
      }
    }
  } else {
    float tmp[MR][NR];
    for (int i = 0; i < MR; ++i) {
      st8(tmp[i], acc[i][0]);
      st8(tmp[i] + 8, acc[i][1]);
    }
    for (int i = 0; i < mr; ++i)
      for (int j = 0; j < nr; ++j) {
        float* cij = c + (size_t)i * ldc + j;
        *cij = accumulate ? *cij + tmp[i][j] : tmp[i][j];
      }
  }
}

void sgemm(int M, int N, int K, const float* A, const float* B, bool b_trans, float* C) {
  const int mb = (M + MC - 1) / MC, nb = (N + NC - 1) / NC;
  for (int k0 = 0; k0 < K; k0 += KC) {
    const int kc = std::min(KC, K - k0);
    const bool acc = k0 > 0;
#pragma omp parallel
    {
      std::vector<float> pa((size_t)MC * KC), pb((size_t)NC * KC);
#pragma omp for schedule(dynamic, 1) collapse(2)
      for (int ib = 0; ib < mb; ++ib)
        for (int jb = 0; jb < nb; ++jb) {
          const int m0 = ib * MC, n0 = jb * NC;
          const int mc = std::min(MC, M - m0), nc = std::min(NC, N - n0);
          // pack A: panels of MR rows, [kc][MR]
          for (int p = 0; p < mc; p += MR) {
            float* dst = pa.data() + (size_t)p * kc;
            const int mr = std::min(MR, mc - p);
            for (int k = 0; k < kc; ++k)
              for (int i = 0; i < MR; ++i)
                dst[k * MR + i] = i < mr ? A[(size_t)(m0 + p + i) * K + k0 + k] : 0.f;
          }
          // pack B: panels of NR columns, [kc][NR]
          for (int q = 0; q < nc; q += NR) {
            float* dst = pb.data() + (size_t)q * kc;
            const int nr = std::min(NR, nc - q);
            for (int k = 0; k < kc; ++k)
              for (int j = 0; j < NR; ++j) {
                float v = 0.f;
                if (j < nr)
                  v = b_trans ? B[(size_t)(n0 + q + j) * K + k0 + k]
                              : B[(size_t)(k0 + k) * N + n0 + q + j];
                dst[k * NR + j] = v;
              }
          }
          for (int p = 0; p < mc; p += MR)
            for (int q = 0; q < nc; q += NR)
              micro_6x16(kc, pa.data() + (size_t)p * kc, pb.data() + (size_t)q * kc,
                         C + (size_t)(m0 + p) * N + n0 + q, N, std::min(MR, mc - p),
                         std::min(NR, nc - q), acc);
        }
    }
  }
}

// ------------------------------------------------------------ row ops
const float RMS_EPS = 1e-5f;  // cpu/rmsnorm.rs:10

void rmsnorm(const float* x, const float* gamma, float* out, int T, int d) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const float* xr = x + (size_t)t * d;
    double ss = 0.0;
    for (int i = 0; i < d; ++i) ss += (double)xr[i] * xr[i];
    const float rinv = (float)(1.0 / sqrt(ss / d + (double)RMS_EPS));
    float* o = out + (size_t)t * d;
    for (int i = 0; i < d; ++i) o[i] = xr[i] * rinv * gamma[i];
  }
}

// RoPE table [seq][64] (cos, sin), theta = p * 10000^(-2i/128) (sdpa_fwd.rs:24-39).
std::vector<float> rope_table(int seq) {
  std::vector<float> tab((size_t)seq * 128);
  for (int p = 0; p < seq; ++p)
    for (int i = 0; i < 64; ++i) {
      double th = (double)p * pow(10000.0, -2.0 * i / 128.0);
      tab[(size_t)p * 128 + 2 * i] = (float)cos(th);
      tab[(size_t)p * 128 + 2 * i + 1] = (float)sin(th);
    }
  return tab;
}

// In-place RoPE on [T, ncols] (heads of 128), pairs (2i, 2i+1):
// (a, b) -> (a cos - b sin, b cos + a sin)   (sdpa_fwd.rs:53-60,213-221)
void apply_rope(float* m, int T, int ncols, int seq, const std::vector<float>& tab) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const int p = t % seq;
    float* r = m + (size_t)t * ncols;
    for (int c = 0; c < ncols; c += 2) {
      const int i = (c & 127) >> 1;
      const float cs = tab[(size_t)p * 128 + 2 * i], sn = tab[(size_t)p * 128 + 2 * i + 1];
      const float a = r[c], b = r[c + 1];
      r[c] = a * cs - b * sn;
      r[c + 1] = b * cs + a * sn;
    }
  }
}

// Causal attention per (sequence, head): softmax(q k^T / sqrt(128)) v over keys u <= t.
void attention(const float* Q, const float* K, const float* V, float* out, int batch, int seq,
               int heads, int kv_heads) {
  const int qd = heads * 128, kvd = kv_heads * 128, grp = heads / kv_heads;
  const float scale = 1.0f / sqrtf(128.0f);
#pragma omp parallel
  {
    std::vector<float> sc(seq);
#pragma omp for schedule(dynamic, 4) collapse(3)
    for (int b = 0; b < batch; ++b)
      for (int h = 0; h < heads; ++h)
        for (int t = 0; t < seq; ++t) {
          const int hk = h / grp;
          const float* q = Q + ((size_t)b * seq + t) * qd + h * 128;
          float mx = -INFINITY;
          for (int u = 0; u <= t; ++u) {
            const float* k = K + ((size_t)b * seq + u) * kvd + hk * 128;
            float s = 0.f;
            for (int i = 0; i < 128; ++i) s += q[i] * k[i];
            s *= scale;
            sc[u] = s;
            mx = std::max(mx, s);
          }
          double den = 0.0;
          for (int u = 0; u <= t; ++u) {
            sc[u] = expf(sc[u] - mx);
            den += sc[u];
          }
          const float inv = (float)(1.0 / den);
          float acc[128];
          for (int i = 0; i < 128; ++i) acc[i] = 0.f;
          for (int u = 0; u <= t; ++u) {
            const float* v = V + ((size_t)b * seq + u) * kvd + hk * 128;
            const float p = sc[u] * inv;
            for (int i = 0; i < 128; ++i) acc[i] += p * v[i];
          }
          float* o = out + ((size_t)b * seq + t) * qd + h * 128;
          for (int i = 0; i < 128; ++i) o[i] = acc[i];
        }
  }
}

}  // namespace

extern "C" {

void orc_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}

int orc_max_threads(void) { return omp_get_max_threads(); }

// Fill host f32 buffers (reference orientation) with the fp16-valued weights the
// CUDA bridge generates for the same (seed, scheme, sigma). Gains are 1.0.
int orc_gen_weights(const orc_config* cfg, uint64_t seed, int scheme, float sigma, float* embed,
                    float* gamma_final, const orc_layer* layers) {
  if (!cfg || !embed || !gamma_final || !layers) return 1;
  const int d = cfg->dim, hid = cfg->hidden, V = cfg->vocab;
  const int qd = cfg->heads * cfg->hd, kvd = cfg->kv_heads * cfg->hd;
  const float mul = (float)((double)sigma / CB_IRWIN_HALL4_STD);
  const float s_embed = 0.005f;
  const float s_qkv = 1.0f / sqrtf((float)d);
  const float s_ffn = 1.0f / sqrtf((float)hid);
  auto fill = [&](float* dst, uint64_t n, int layer, int kind, float ref_scale) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) {
      uint16_t bits;
      if (scheme == 0)
        bits = cb_normal_f16(seed, cb_tensor_id(layer, kind), (uint64_t)i, mul);
      else
        bits = ref_scale == 0.f ? (uint16_t)0 : cb_lcg_f16(n, (uint64_t)i, ref_scale);
      dst[i] = cb_f16_bits_to_f32(bits);
    }
  };
  fill(embed, (uint64_t)V * d, -1, 0, s_embed);
  for (int i = 0; i < d; ++i) gamma_final[i] = 1.0f;
  for (int l = 0; l < cfg->nlayers; ++l) {
    const orc_layer& w = layers[l];
    fill(w.wq, (uint64_t)d * qd, l, CB_T_WQ, s_qkv);
    fill(w.wk, (uint64_t)d * kvd, l, CB_T_WK, s_qkv);
    fill(w.wv, (uint64_t)d * kvd, l, CB_T_WV, s_qkv);
    fill(w.wo, (uint64_t)qd * d, l, CB_T_WO, 0.f);
    fill(w.w1, (uint64_t)d * hid, l, CB_T_W1, s_ffn);
    fill(w.w3, (uint64_t)d * hid, l, CB_T_W3, s_ffn);
    fill(w.w2, (uint64_t)d * hid, l, CB_T_W2, 0.f);
    for (int i = 0; i < d; ++i) w.gamma1[i] = w.gamma2[i] = 1.0f;
  }
  return 0;
}

// fp16 round trip helpers exposed for tests.
uint16_t orc_f32_to_f16_bits(float f) { return cb_f32_to_f16_bits(f); }
float orc_f16_bits_to_f32(uint16_t h) { return cb_f16_bits_to_f32(h); }
uint64_t orc_lcg_jump(uint64_t s0, uint64_t k) { return cb_lcg_jump(s0, k); }
float orc_lcg_value(uint64_t s, float scale) { return cb_lcg_value(s, scale); }

// Full forward + loss for `batch` sequences back to back.
//   loss:            mean CE over batch*seq positions
//   per_token_loss:  nullable [batch*seq]
//   sampled_logits:  nullable [n_sample, vocab] for rows sample_rows[i] (= b*seq + s)
int orc_forward(const orc_config* cfg, const float* embed, const float* gamma_final,
                const orc_layer* layers, const uint32_t* tokens, const uint32_t* targets,
                int batch, float softcap, float* loss, float* per_token_loss,
                const int32_t* sample_rows, int n_sample, float* sampled_logits) {
  if (!cfg || !embed || !gamma_final || !layers || !tokens || !targets || batch <= 0 || !loss)
    return 1;
  const int d = cfg->dim, hid = cfg->hidden, V = cfg->vocab, S = cfg->seq, L = cfg->nlayers;
  const int qd = cfg->heads * cfg->hd, kvd = cfg->kv_heads * cfg->hd;
  if (cfg->hd != 128) return 2;
  const int T = batch * S;
  for (int t = 0; t < T; ++t)
    if (tokens[t] >= (uint32_t)V || targets[t] >= (uint32_t)V) return 3;
  const float alpha = 1.0f / sqrtf(2.0f * (float)L);  // layer.rs:4420
  const std::vector<float> rope = rope_table(S);

  std::vector<float> X((size_t)T * d), Xn((size_t)T * d), Q((size_t)T * qd), Kb((size_t)T * kvd),
      Vb((size_t)T * kvd), A((size_t)T * qd), O((size_t)T * d), H1((size_t)T * hid),
      H3((size_t)T * hid);

  // embedding (cpu/embedding.rs:8-17)
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) memcpy(&X[(size_t)t * d], embed + (size_t)tokens[t] * d, d * 4);

  for (int l = 0; l < L; ++l) {
    const orc_layer& w = layers[l];
    rmsnorm(X.data(), w.gamma1, Xn.data(), T, d);
    sgemm(T, qd, d, Xn.data(), w.wq, false, Q.data());
    sgemm(T, kvd, d, Xn.data(), w.wk, false, Kb.data());
    sgemm(T, kvd, d, Xn.data(), w.wv, false, Vb.data());
    apply_rope(Q.data(), T, qd, S, rope);
    apply_rope(Kb.data(), T, kvd, S, rope);
    attention(Q.data(), Kb.data(), Vb.data(), A.data(), batch, S, cfg->heads, cfg->kv_heads);
    sgemm(T, d, qd, A.data(), w.wo, false, O.data());
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)T * d; ++i) X[i] = X[i] + alpha * O[i];
    rmsnorm(X.data(), w.gamma2, Xn.data(), T, d);
    sgemm(T, hid, d, Xn.data(), w.w1, false, H1.data());
    sgemm(T, hid, d, Xn.data(), w.w3, false, H3.data());
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)T * hid; ++i) {
      const float h1 = H1[i];
      H1[i] = h1 / (1.0f + expf(-h1)) * H3[i];  // silu(h1) * h3 (cpu/silu.rs:37-46)
    }
    sgemm(T, d, hid, H1.data(), w.w2, true, O.data());  // gate @ W2^T
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)T * d; ++i) X[i] = X[i] + alpha * O[i];
  }

  rmsnorm(X.data(), gamma_final, Xn.data(), T, d);
  // free what is no longer needed before the [T, V] logits
  std::vector<float>().swap(Q);
  std::vector<float>().swap(Kb);
  std::vector<float>().swap(Vb);
  std::vector<float>().swap(A);
  std::vector<float>().swap(H1);
  std::vector<float>().swap(H3);

  // LM head + CE in row chunks so the logits buffer stays bounded.
  const int CH = 512;
  std::vector<float> Z((size_t)CH * V);
  std::vector<double> tok_loss(T);
  for (int t0 = 0; t0 < T; t0 += CH) {
    const int n = std::min(CH, T - t0);
    sgemm(n, V, d, Xn.data() + (size_t)t0 * d, embed, true, Z.data());
    if (softcap > 0.f) {
#pragma omp parallel for schedule(static)
      for (int64_t i = 0; i < (int64_t)n * V; ++i) Z[i] = softcap * tanhf(Z[i] / softcap);
    }
#pragma omp parallel for schedule(static)
    for (int r = 0; r < n; ++r) {
      const float* z = Z.data() + (size_t)r * V;
      float mx = -INFINITY;
      for (int i = 0; i < V; ++i) mx = std::max(mx, z[i]);
      double se = 0.0;
      for (int i = 0; i < V; ++i) se += exp((double)z[i] - mx);
      tok_loss[t0 + r] = log(se) + mx - z[targets[t0 + r]];
    }
    if (sampled_logits && sample_rows) {
      for (int i = 0; i < n_sample; ++i) {
        const int r = sample_rows[i];
        if (r >= t0 && r < t0 + n)
          memcpy(sampled_logits + (size_t)i * V, Z.data() + (size_t)(r - t0) * V, (size_t)V * 4);
      }
    }
  }
  double sum = 0.0;
  for (int t = 0; t < T; ++t) {
    sum += tok_loss[t];
    if (per_token_loss) per_token_loss[t] = (float)tok_loss[t];
  }
  *loss = (float)(sum / T);
  return 0;
}

}  // extern "C"
