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
// orc_forward_backward adds the backward pass (the training step's gradients):
//   model backward     full_model.rs:592-702 (backward_ws): dlogits = (softmax -
//                      onehot) * loss_scale / seq (cross_entropy.rs:58-96), softcap
//                      derivative (1 - tanh^2), dembed += dl^T x_final, dx_final =
//                      dl embed, final RMSNorm backward, layers in reverse, embedding
//                      backward (embedding.rs:34-44)
//   layer backward     layer.rs:6747-7037 (backward): dffn = alpha dy, dsilu = dffn W2,
//                      SiLU derivative, dx_ffn = dh1 W1^T + dh3 W3^T, RMSNorm2
//                      backward + dy, dx2s = alpha dx2, da = dx2s Wo^T, SDPA backward,
//                      RoPE backward (:7391-7408), dx = dq Wq^T + dk Wk^T + dv Wv^T,
//                      RMSNorm1 backward + dx2; weight gradients as accumulate_dw
//   RMSNorm backward   cpu/rmsnorm.rs:190-238
//
// The single ops (embedding, RMSNorm, SwiGLU gate, CE, SGEMM) are also exported as
// orc_op_* so that ports of the reference's CPU-op unit tests run against the very
// functions the forward and backward use.
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

void rmsnorm_save(const float* x, const float* gamma, float* out, float* rinv_out, int T, int d) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const float* xr = x + (size_t)t * d;
    double ss = 0.0;
    for (int i = 0; i < d; ++i) ss += (double)xr[i] * xr[i];
    const float rinv = (float)(1.0 / sqrt(ss / d + (double)RMS_EPS));
    rinv_out[t] = rinv;
    float* o = out + (size_t)t * d;
    for (int i = 0; i < d; ++i) o[i] = xr[i] * rinv * gamma[i];
  }
}

// cpu/rmsnorm.rs:190-238: x_hat = x rinv; dgamma += sum_t dy x_hat;
// dx = rinv (dy gamma - x_hat mean_d(dy gamma x_hat)). dx = or += (accumulate).
void rmsnorm_backward(const float* dy, const float* x, const float* gamma, const float* rinv,
                      float* dx, bool accumulate, float* dgamma, int T, int d) {
  std::vector<double> dg((size_t)d, 0.0);
#pragma omp parallel
  {
    std::vector<double> dg_local((size_t)d, 0.0);
#pragma omp for schedule(static)
    for (int t = 0; t < T; ++t) {
      const float* dyr = dy + (size_t)t * d;
      const float* xr = x + (size_t)t * d;
      double dot = 0.0;
      for (int i = 0; i < d; ++i) {
        const double xh = (double)xr[i] * rinv[t];
        dot += (double)dyr[i] * gamma[i] * xh;
        dg_local[i] += (double)dyr[i] * xh;
      }
      dot /= d;
      float* o = dx + (size_t)t * d;
      for (int i = 0; i < d; ++i) {
        const double xh = (double)xr[i] * rinv[t];
        const float v = (float)(rinv[t] * ((double)dyr[i] * gamma[i] - xh * dot));
        o[i] = accumulate ? o[i] + v : v;
      }
    }
#pragma omp critical
    for (int i = 0; i < d; ++i) dg[i] += dg_local[i];
  }
  for (int i = 0; i < d; ++i) dgamma[i] += (float)dg[i];
}

// out[c][r] = in[r][c]
void transpose(const float* in, int rows, int cols, float* out) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < cols; ++c) out[(size_t)c * rows + r] = in[(size_t)r * cols + c];
}

// ------------------------------------------------------------ embedding, SwiGLU, CE
// out[t, :] = table[ids[t], :] (cpu/embedding.rs:8-17).
void embedding_forward(const float* table, int d, const uint32_t* ids, int n, float* out) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < n; ++t)
    memcpy(out + (size_t)t * d, table + (size_t)ids[t] * d, (size_t)d * 4);
}

// dtable[ids[t], :] += dout[t, :], in position order (cpu/embedding.rs:20-44).
void embedding_backward(const float* dout, int d, const uint32_t* ids, int n, float* dtable) {
  for (int t = 0; t < n; ++t) {
    float* dst = dtable + (size_t)ids[t] * d;
    const float* src = dout + (size_t)t * d;
    for (int i = 0; i < d; ++i) dst[i] += src[i];
  }
}

// g = silu(h1) * h3 with silu(z) = z / (1 + e^-z) (cpu/silu.rs:8-46,
// kernels/ffn_fused.rs:105-107).
inline float silu_gate1(float h1, float h3) { return h1 / (1.0f + expf(-h1)) * h3; }

// Backward of g = silu(h1) * h3: dh3 = dg silu(h1), dh1 = dg h3 silu'(h1) with
// silu'(z) = s (1 + z (1 - s)), s = sigmoid(z) (cpu/silu.rs:23-34).
inline void silu_gate_backward1(float dg, float h1, float h3, float* dh1, float* dh3) {
  const float sig = 1.0f / (1.0f + expf(-h1));
  const float silu = h1 * sig;
  const float dsil = sig * (1.0f + h1 * (1.0f - sig));
  *dh3 = dg * silu;
  *dh1 = dg * h3 * dsil;
}

// Cross-entropy of one row of logits z [V] (cpu/cross_entropy.rs:13-41, 58-96):
// loss = log sum_v exp(z_v - m) + m - z_tgt, m = max_v z_v; the sum in double. With
// dl != nullptr also dl_v = (softmax_v - [v == tgt]) * scale (cross_entropy.rs:43-56,
// scaled as forward_backward_batch scales by inv_seq), times the softcap derivative
// 1 - (z_v / softcap)^2 when softcap > 0 (z holds the capped logits, so
// z / softcap = tanh(raw / softcap)). dl may alias z.
double ce_row(const float* z, int V, int tgt, float softcap, double scale, float* dl) {
  float mx = -INFINITY;
  for (int i = 0; i < V; ++i) mx = std::max(mx, z[i]);
  double se = 0.0;
  for (int i = 0; i < V; ++i) se += exp((double)z[i] - mx);
  const double loss = log(se) + mx - z[tgt];
  if (dl) {
    for (int i = 0; i < V; ++i) {
      const double pr = exp((double)z[i] - mx) / se;
      double g = (pr - (i == tgt ? 1.0 : 0.0)) * scale;
      if (softcap > 0.f) {
        const double th = z[i] / softcap;
        g *= 1.0 - th * th;
      }
      dl[i] = (float)g;
    }
  }
  return loss;
}

// z = softcap * tanh(z / softcap) when softcap > 0 (full_model.rs:456-461).
inline void softcap_row(float* z, int V, float softcap) {
  if (softcap > 0.f)
    for (int i = 0; i < V; ++i) z[i] = softcap * tanhf(z[i] / softcap);
}

// dW[R, N] += X^T dY for X [T, R], dY [T, N] (accumulate_dw of the reference).
void accumulate_dw(const float* X, int R, const float* dY, int N, int T, float* dW) {
  std::vector<float> xt((size_t)R * T), tmp((size_t)R * N);
  transpose(X, T, R, xt.data());
  sgemm(R, N, T, xt.data(), dY, false, tmp.data());
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)R * N; ++i) dW[i] += tmp[i];
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

// Inverse RoPE (rotation by -theta), layer.rs:7391-7408:
// (d0, d1) -> (c d0 + s d1, -s d0 + c d1)
void rope_backward(float* m, int T, int ncols, int seq, const std::vector<float>& tab) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const int p = t % seq;
    float* r = m + (size_t)t * ncols;
    for (int c = 0; c < ncols; c += 2) {
      const int i = (c & 127) >> 1;
      const float cs = tab[(size_t)p * 128 + 2 * i], sn = tab[(size_t)p * 128 + 2 * i + 1];
      const float a = r[c], b = r[c + 1];
      r[c] = cs * a + sn * b;
      r[c + 1] = -sn * a + cs * b;
    }
  }
}

// Backward of causal attention for one forward: dO [T, qd] -> dQ [T, qd], dK, dV
// [T, kvd] (written, not accumulated). Scores are recomputed:
//   P = softmax(S), dV_u += P_u dO_t, dP_u = dO_t . V_u, D_t = sum_u P_u dP_u,
//   dS_u = P_u (dP_u - D_t), dQ_t = scale sum_u dS_u K_u, dK_u += scale dS_u Q_t.
void attention_backward(const float* Q, const float* K, const float* V, const float* dO,
                        float* dQ, float* dK, float* dV, int batch, int seq, int heads,
                        int kv_heads) {
  const int qd = heads * 128, kvd = kv_heads * 128, grp = heads / kv_heads;
  const float scale = 1.0f / sqrtf(128.0f);
  memset(dK, 0, (size_t)batch * seq * kvd * 4);
  memset(dV, 0, (size_t)batch * seq * kvd * 4);
#pragma omp parallel
  {
    std::vector<float> p(seq), dp(seq);
#pragma omp for schedule(dynamic, 1) collapse(2)
    for (int b = 0; b < batch; ++b)
      for (int hk = 0; hk < kv_heads; ++hk)
        for (int h = hk * grp; h < (hk + 1) * grp; ++h)
          for (int t = 0; t < seq; ++t) {
            const float* q = Q + ((size_t)b * seq + t) * qd + h * 128;
            const float* go = dO + ((size_t)b * seq + t) * qd + h * 128;
            float mx = -INFINITY;
            for (int u = 0; u <= t; ++u) {
              const float* k = K + ((size_t)b * seq + u) * kvd + hk * 128;
              float s = 0.f;
              for (int i = 0; i < 128; ++i) s += q[i] * k[i];
              p[u] = s * scale;
              mx = std::max(mx, p[u]);
            }
            double den = 0.0;
            for (int u = 0; u <= t; ++u) {
              p[u] = expf(p[u] - mx);
              den += p[u];
            }
            const float inv = (float)(1.0 / den);
            double Dt = 0.0;
            for (int u = 0; u <= t; ++u) {
              p[u] *= inv;
              const float* v = V + ((size_t)b * seq + u) * kvd + hk * 128;
              float s = 0.f;
              for (int i = 0; i < 128; ++i) s += go[i] * v[i];
              dp[u] = s;
              Dt += (double)p[u] * s;
            }
            float* gq = dQ + ((size_t)b * seq + t) * qd + h * 128;
            float accq[128];
            for (int i = 0; i < 128; ++i) accq[i] = 0.f;
            for (int u = 0; u <= t; ++u) {
              const float ds = p[u] * (dp[u] - (float)Dt);
              const float* k = K + ((size_t)b * seq + u) * kvd + hk * 128;
              float* gk = dK + ((size_t)b * seq + u) * kvd + hk * 128;
              float* gv = dV + ((size_t)b * seq + u) * kvd + hk * 128;
              for (int i = 0; i < 128; ++i) {
                accq[i] += ds * k[i];
                gk[i] += scale * ds * q[i];
                gv[i] += p[u] * go[i];
              }
            }
            for (int i = 0; i < 128; ++i) gq[i] = scale * accq[i];
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

// ---- the oracle's row and element ops, exposed one by one so that the reference's
// CPU-op unit tests (cpu/{embedding,rmsnorm,silu,cross_entropy,vdsp}.rs test modules)
// run against the same functions the oracle forward and backward use. Rows are
// token-major [n, d]. Return 1 on a null or bad argument, 3 on an id >= vocab.

int orc_op_embedding(const float* table, int vocab, int d, const uint32_t* ids, int n,
                     float* out) {
  if (!table || !ids || !out || vocab <= 0 || d <= 0 || n < 0) return 1;
  for (int t = 0; t < n; ++t)
    if (ids[t] >= (uint32_t)vocab) return 3;
  embedding_forward(table, d, ids, n, out);
  return 0;
}

int orc_op_embedding_backward(const float* dout, int vocab, int d, const uint32_t* ids, int n,
                              float* dtable) {
  if (!dout || !ids || !dtable || vocab <= 0 || d <= 0 || n < 0) return 1;
  for (int t = 0; t < n; ++t)
    if (ids[t] >= (uint32_t)vocab) return 3;
  embedding_backward(dout, d, ids, n, dtable);
  return 0;
}

int orc_op_rmsnorm(const float* x, const float* gamma, float* out, float* rinv, int n, int d) {
  if (!x || !gamma || !out || !rinv || n < 0 || d <= 0) return 1;
  rmsnorm_save(x, gamma, out, rinv, n, d);
  return 0;
}

// dx is written; dgamma accumulates over the rows.
int orc_op_rmsnorm_backward(const float* dy, const float* x, const float* gamma,
                            const float* rinv, float* dx, float* dgamma, int n, int d) {
  if (!dy || !x || !gamma || !rinv || !dx || !dgamma || n < 0 || d <= 0) return 1;
  rmsnorm_backward(dy, x, gamma, rinv, dx, false, dgamma, n, d);
  return 0;
}

int orc_op_silu_gate(const float* gate, const float* up, float* out, int64_t n) {
  if (!gate || !up || !out || n < 0) return 1;
  for (int64_t i = 0; i < n; ++i) out[i] = silu_gate1(gate[i], up[i]);
  return 0;
}

int orc_op_silu_gate_backward(const float* dout, const float* gate, const float* up,
                              float* dgate, float* dup, int64_t n) {
  if (!dout || !gate || !up || !dgate || !dup || n < 0) return 1;
  for (int64_t i = 0; i < n; ++i) silu_gate_backward1(dout[i], gate[i], up[i], &dgate[i], &dup[i]);
  return 0;
}

// Per-row CE of raw logits [n, V] (softcapped first when softcap > 0): losses [n];
// dlogits [n, V] (nullable) = d(loss_row * scale) / d(raw logits).
int orc_op_cross_entropy(const float* logits, const uint32_t* targets, int n, int V,
                         float softcap, float scale, float* losses, float* dlogits) {
  if (!logits || !targets || !losses || n < 0 || V <= 0) return 1;
  for (int t = 0; t < n; ++t)
    if (targets[t] >= (uint32_t)V) return 3;
  std::vector<float> z((size_t)V);
  for (int t = 0; t < n; ++t) {
    memcpy(z.data(), logits + (size_t)t * V, (size_t)V * 4);
    softcap_row(z.data(), V, softcap);
    losses[t] = (float)ce_row(z.data(), V, (int)targets[t], softcap, scale,
                              dlogits ? dlogits + (size_t)t * V : nullptr);
  }
  return 0;
}

// C[M, N] = A[M, K] op(B): op(B) = B [K, N], or B [N, K] transposed when b_trans
// (the LM head's x_final embed^T, cpu/vdsp.rs:354-376 sgemm_at, is the b_trans form).
int orc_op_sgemm(int M, int N, int K, const float* A, const float* B, int b_trans, float* C) {
  if (!A || !B || !C || M < 0 || N < 0 || K <= 0) return 1;
  sgemm(M, N, K, A, B, b_trans != 0, C);
  return 0;
}

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

  embedding_forward(embed, d, tokens, T, X.data());

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
    for (int64_t i = 0; i < (int64_t)T * hid; ++i) H1[i] = silu_gate1(H1[i], H3[i]);
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
#pragma omp parallel for schedule(static)
    for (int r = 0; r < n; ++r) {
      float* z = Z.data() + (size_t)r * V;
      softcap_row(z, V, softcap);
      tok_loss[t0 + r] = ce_row(z, V, (int)targets[t0 + r], softcap, 0.0, nullptr);
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

// Forward + backward of `batch` sequences back to back (the training step's
// gradients). Gradients ADD into the grad buffers (reference orientation, laid out like
// the weights), as ModelGrads accumulates over micro-batches; dlogits carry
// loss_scale / seq per position, i.e. each sequence contributes the gradient of its own
// mean loss, as `batch` separate reference calls would.
int orc_forward_backward(const orc_config* cfg, const float* embed, const float* gamma_final,
                         const orc_layer* layers, const uint32_t* tokens,
                         const uint32_t* targets, int batch, float softcap, float loss_scale,
                         float* loss, float* d_embed, float* d_gamma_final,
                         const orc_layer* grads) {
  if (!cfg || !embed || !gamma_final || !layers || !tokens || !targets || batch <= 0 || !loss ||
      !d_embed || !d_gamma_final || !grads)
    return 1;
  const int d = cfg->dim, hid = cfg->hidden, V = cfg->vocab, S = cfg->seq, L = cfg->nlayers;
  const int qd = cfg->heads * cfg->hd, kvd = cfg->kv_heads * cfg->hd;
  if (cfg->hd != 128) return 2;
  const int T = batch * S;
  for (int t = 0; t < T; ++t)
    if (tokens[t] >= (uint32_t)V || targets[t] >= (uint32_t)V) return 3;
  const float alpha = 1.0f / sqrtf(2.0f * (float)L);
  const std::vector<float> rope = rope_table(S);
  const size_t Td = (size_t)T * d;

  struct Cache {
    std::vector<float> x, xn, r1, q, k, v, a, x2, x2n, r2, h1, h3, g;
  };
  std::vector<Cache> cache(L);
  std::vector<float> X(Td), O(Td);
  embedding_forward(embed, d, tokens, T, X.data());
  for (int l = 0; l < L; ++l) {
    const orc_layer& w = layers[l];
    Cache& c = cache[l];
    c.x = X;
    c.xn.resize(Td);
    c.r1.resize(T);
    rmsnorm_save(X.data(), w.gamma1, c.xn.data(), c.r1.data(), T, d);
    c.q.resize((size_t)T * qd);
    c.k.resize((size_t)T * kvd);
    c.v.resize((size_t)T * kvd);
    sgemm(T, qd, d, c.xn.data(), w.wq, false, c.q.data());
    sgemm(T, kvd, d, c.xn.data(), w.wk, false, c.k.data());
    sgemm(T, kvd, d, c.xn.data(), w.wv, false, c.v.data());
    apply_rope(c.q.data(), T, qd, S, rope);
    apply_rope(c.k.data(), T, kvd, S, rope);
    c.a.resize((size_t)T * qd);
    attention(c.q.data(), c.k.data(), c.v.data(), c.a.data(), batch, S, cfg->heads,
              cfg->kv_heads);
    sgemm(T, d, qd, c.a.data(), w.wo, false, O.data());
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)Td; ++i) X[i] = X[i] + alpha * O[i];
    c.x2 = X;
    c.x2n.resize(Td);
    c.r2.resize(T);
    rmsnorm_save(X.data(), w.gamma2, c.x2n.data(), c.r2.data(), T, d);
    c.h1.resize((size_t)T * hid);
    c.h3.resize((size_t)T * hid);
    c.g.resize((size_t)T * hid);
    sgemm(T, hid, d, c.x2n.data(), w.w1, false, c.h1.data());
    sgemm(T, hid, d, c.x2n.data(), w.w3, false, c.h3.data());
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)T * hid; ++i) c.g[i] = silu_gate1(c.h1[i], c.h3[i]);
    sgemm(T, d, hid, c.g.data(), w.w2, true, O.data());
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)Td; ++i) X[i] = X[i] + alpha * O[i];
  }
  std::vector<float> Xf(Td), rf(T);
  rmsnorm_save(X.data(), gamma_final, Xf.data(), rf.data(), T, d);

  // LM head + CE + dlogits, in row chunks; dx_final = dl embed, dembed += dl^T Xf
  std::vector<float> dXf(Td);
  const float inv_seq = loss_scale / (float)S;
  double loss_sum = 0.0;
  const int CH = 512;
  std::vector<float> Z((size_t)CH * V), dZt((size_t)V * CH), tmp((size_t)V * d);
  for (int t0 = 0; t0 < T; t0 += CH) {
    const int n = std::min(CH, T - t0);
    sgemm(n, V, d, Xf.data() + (size_t)t0 * d, embed, true, Z.data());
    std::vector<double> part(n);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < n; ++r) {
      float* z = Z.data() + (size_t)r * V;
      softcap_row(z, V, softcap);
      part[r] = ce_row(z, V, (int)targets[t0 + r], softcap, inv_seq, z);  // z now holds dl
    }
    for (int r = 0; r < n; ++r) loss_sum += part[r];
    sgemm(n, d, V, Z.data(), embed, false, dXf.data() + (size_t)t0 * d);
    transpose(Z.data(), n, V, dZt.data());
    sgemm(V, d, n, dZt.data(), Xf.data() + (size_t)t0 * d, false, tmp.data());
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)V * d; ++i) d_embed[i] += tmp[i];
  }
  *loss = (float)(loss_sum / T);

  std::vector<float> dY(Td), dffn(Td), dx2(Td), dx2s(Td), dxa(Td);
  rmsnorm_backward(dXf.data(), X.data(), gamma_final, rf.data(), dY.data(), false,
                   d_gamma_final, T, d);
  std::vector<float> dsilu((size_t)T * hid), dh1((size_t)T * hid), dh3((size_t)T * hid);
  std::vector<float> da((size_t)T * qd), dq((size_t)T * qd), dk((size_t)T * kvd),
      dv((size_t)T * kvd);
  for (int l = L - 1; l >= 0; --l) {
    const orc_layer& w = layers[l];
    const orc_layer& gw = grads[l];
    Cache& c = cache[l];
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)Td; ++i) dffn[i] = alpha * dY[i];
    sgemm(T, hid, d, dffn.data(), w.w2, false, dsilu.data());  // dffn @ W2
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)T * hid; ++i)
      silu_gate_backward1(dsilu[i], c.h1[i], c.h3[i], &dh1[i], &dh3[i]);
    sgemm(T, d, hid, dh1.data(), w.w1, true, dxa.data());  // dh1 @ W1^T
    {
      std::vector<float> t3(Td);
      sgemm(T, d, hid, dh3.data(), w.w3, true, t3.data());
#pragma omp parallel for schedule(static)
      for (int64_t i = 0; i < (int64_t)Td; ++i) dxa[i] += t3[i];
    }
    accumulate_dw(c.x2n.data(), d, dh1.data(), hid, T, gw.w1);
    accumulate_dw(c.x2n.data(), d, dh3.data(), hid, T, gw.w3);
    accumulate_dw(dffn.data(), d, c.g.data(), hid, T, gw.w2);
    rmsnorm_backward(dxa.data(), c.x2.data(), w.gamma2, c.r2.data(), dx2.data(), false,
                     gw.gamma2, T, d);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)Td; ++i) {
      dx2[i] += dY[i];
      dx2s[i] = alpha * dx2[i];
    }
    sgemm(T, qd, d, dx2s.data(), w.wo, true, da.data());  // dx2s @ Wo^T
    accumulate_dw(c.a.data(), qd, dx2s.data(), d, T, gw.wo);
    attention_backward(c.q.data(), c.k.data(), c.v.data(), da.data(), dq.data(), dk.data(),
                       dv.data(), batch, S, cfg->heads, cfg->kv_heads);
    rope_backward(dq.data(), T, qd, S, rope);
    rope_backward(dk.data(), T, kvd, S, rope);
    sgemm(T, d, qd, dq.data(), w.wq, true, dxa.data());
    {
      std::vector<float> t3(Td);
      sgemm(T, d, kvd, dk.data(), w.wk, true, t3.data());
#pragma omp parallel for schedule(static)
      for (int64_t i = 0; i < (int64_t)Td; ++i) dxa[i] += t3[i];
      sgemm(T, d, kvd, dv.data(), w.wv, true, t3.data());
#pragma omp parallel for schedule(static)
      for (int64_t i = 0; i < (int64_t)Td; ++i) dxa[i] += t3[i];
    }
    accumulate_dw(c.xn.data(), d, dq.data(), qd, T, gw.wq);
    accumulate_dw(c.xn.data(), d, dk.data(), kvd, T, gw.wk);
    accumulate_dw(c.xn.data(), d, dv.data(), kvd, T, gw.wv);
    rmsnorm_backward(dxa.data(), c.x.data(), w.gamma1, c.r1.data(), dY.data(), false,
                     gw.gamma1, T, d);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)Td; ++i) dY[i] += dx2[i];
  }
  embedding_backward(dY.data(), d, tokens, T, d_embed);
  return 0;
}

}  // extern "C"
