// Training step: forward with saved activations + backward into fp32 gradients.
//
// Included at the end of bridge.cu (it uses the context, the GEMM launchers and the
// forward's kernels). The math follows the reference's backward (full_model.rs:592-702
// backward_ws; layer.rs:6747-7037 backward; cpu/rmsnorm.rs:190-238;
// cpu/embedding.rs:34-44; cpu/cross_entropy.rs:58-96):
//   dl      = softmax(z) - onehot(target) (x (1 - tanh^2) with softcap)
//   dXf     = dl E,              dE  += s dl^T Xf            (tied head)
//   dX      = RMSNorm_f backward(dXf)
//   per layer, top down (alpha = 1/sqrt(2L)):
//     dG    = (alpha dX) W2      -> SwiGLU backward -> dH13 = (dh1, dh3)
//     dW2  += s (alpha dX)^T G
//     dX2n  = dH13 W13,          dW13 += s dH13^T X2n
//     dX2   = RMSNorm_2 backward(dX2n) + dX
//     dA    = (alpha dX2) Wo^T,  dWo  += s A^T (alpha dX2)
//     dQ, dK, dV = attention backward(dA), RoPE undone
//     dXn   = [dQ dK dV] Wqkv,   dWqkv += s [dQ dK dV]^T Xn
//     dX    = RMSNorm_1 backward(dXn) + dX2
//   dE[token] += s dX (embedding backward)
// Activation gradients are carried in units of the SUM of token losses (they stay
// O(1e-2 .. 1e-4), inside the fp16 range of the GEMM operands); s = loss_scale / seq is
// applied where weight gradients are accumulated, so each sequence of a batch
// contributes the gradient of its own mean loss, exactly as `batch` calls of the
// reference's forward_ws + backward_ws would (ModelGrads accumulates across calls).
//
// Every weight-gradient GEMM has K = tokens. When its tiles fill the GPU poorly it is
// split along K into separate fp32 partial buffers that a fixed-order reduction adds
// into the gradient, so gradients are bit-reproducible run to run.

namespace cb {

// ------------------------------------------------------------------ row kernels

// RMSNorm backward of one row (cpu/rmsnorm.rs:190-238), one warp per row:
//   x_hat = x rinv, dot = mean_d(dy gamma x_hat), dx = rinv (dy gamma - x_hat dot) + dres
// dx_h (nullable) receives fp16(alpha_h * dx): the A operand of the next backward GEMMs.
__global__ void rmsnorm_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                   const float* __restrict__ gamma,
                                   const float* __restrict__ rinv,
                                   const float* __restrict__ dres, float* __restrict__ dx,
                                   __half* __restrict__ dx_h, float alpha_h, int T, int dim) {
  const int row = blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const float* dr = dy + (size_t)row * dim;
  const float* xr = x + (size_t)row * dim;
  const float ri = rinv[row];
  float dot = 0.f;
  for (int c = lane * 8; c < dim; c += 256) {
    float a[8], b[8], gm[8];
    load8(dr + c, a);
    load8(xr + c, b);
    load8(gamma + c, gm);
#pragma unroll
    for (int i = 0; i < 8; ++i) dot += a[i] * gm[i] * b[i];
  }
  dot = warp_sum(dot) * ri / (float)dim;  // mean of dy gamma x_hat
  float* o = dx + (size_t)row * dim;
  const float* rr = dres ? dres + (size_t)row * dim : nullptr;
  for (int c = lane * 8; c < dim; c += 256) {
    float a[8], b[8], gm[8], r[8];
    load8(dr + c, a);
    load8(xr + c, b);
    load8(gamma + c, gm);
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = ri * (a[i] * gm[i] - b[i] * ri * dot);
    if (rr) {
      float e[8];
      load8(rr + c, e);
#pragma unroll
      for (int i = 0; i < 8; ++i) r[i] += e[i];
    }
    *reinterpret_cast<float4*>(o + c) = make_float4(r[0], r[1], r[2], r[3]);
    *reinterpret_cast<float4*>(o + c + 4) = make_float4(r[4], r[5], r[6], r[7]);
    if (dx_h) {
      float h[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = alpha_h * r[i];
      *reinterpret_cast<uint4*>(dx_h + (size_t)row * dim + c) = f8_to_h8(h);
    }
  }
}

// RMSNorm backward with the gain gradient fused (rows of up to NREG * 256 elements):
// each block handles RB_ROWS rows (8 per warp); every lane keeps the dy * x_hat sums of
// its columns in registers, the block adds its warps' sums in warp order through shared
// memory and writes one partial row part[blockIdx.x][dim] (reduced by
// dgamma_reduce_kernel in block order: deterministic).
constexpr int RB_ROWS = 64;

template <int NREG>
__global__ void __launch_bounds__(ROW_WARPS * 32)
    rmsnorm_bwd_dg_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                          const float* __restrict__ gamma, const float* __restrict__ rinv,
                          const float* __restrict__ dres, float* __restrict__ dx,
                          __half* __restrict__ dx_h, float alpha_h, int T, int dim,
                          float* __restrict__ part) {
  __shared__ float red[NREG * 256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float dg[NREG][8];
#pragma unroll
  for (int it = 0; it < NREG; ++it)
#pragma unroll
    for (int i = 0; i < 8; ++i) dg[it][i] = 0.f;
  for (int rr = 0; rr < RB_ROWS / ROW_WARPS; ++rr) {
    const int row = blockIdx.x * RB_ROWS + rr * ROW_WARPS + warp;
    if (row >= T) break;
    const float* dr = dy + (size_t)row * dim;
    const float* xr = x + (size_t)row * dim;
    const float ri = rinv[row];
    float dot = 0.f;
#pragma unroll
    for (int it = 0; it < NREG; ++it) {  // pass 1: dot and the gain gradient
      const int c = it * 256 + lane * 8;
      if (c < dim) {
        float a[8], b[8], gm[8];
        load8(dr + c, a);
        load8(xr + c, b);
        load8(gamma + c, gm);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float xh = b[i] * ri;
          dot += a[i] * gm[i] * xh;
          dg[it][i] += a[i] * xh;
        }
      }
    }
    dot = warp_sum(dot) / (float)dim;
#pragma unroll
    for (int it = 0; it < NREG; ++it) {  // pass 2 (the row is L1-hot): dx
      const int c = it * 256 + lane * 8;
      if (c < dim) {
        float a[8], b[8], gm[8], r[8];
        load8(dr + c, a);
        load8(xr + c, b);
        load8(gamma + c, gm);
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = ri * (a[i] * gm[i] - b[i] * ri * dot);
        if (dres) {
          float e[8];
          load8(dres + (size_t)row * dim + c, e);
#pragma unroll
          for (int i = 0; i < 8; ++i) r[i] += e[i];
        }
        float* o = dx + (size_t)row * dim + c;
        *reinterpret_cast<float4*>(o) = make_float4(r[0], r[1], r[2], r[3]);
        *reinterpret_cast<float4*>(o + 4) = make_float4(r[4], r[5], r[6], r[7]);
        if (dx_h) {
          float h[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) h[i] = alpha_h * r[i];
          *reinterpret_cast<uint4*>(dx_h + (size_t)row * dim + c) = f8_to_h8(h);
        }
      }
    }
  }
  // block sum of the warps' dgamma partials, in warp order
  for (int w = 0; w < ROW_WARPS; ++w) {
    if (warp == w) {
#pragma unroll
      for (int it = 0; it < NREG; ++it) {
        const int c = it * 256 + lane * 8;
        if (c < dim)
#pragma unroll
          for (int i = 0; i < 8; ++i) red[c + i] = (w == 0 ? 0.f : red[c + i]) + dg[it][i];
      }
    }
    __syncthreads();
  }
  for (int c = threadIdx.x; c < dim; c += blockDim.x) part[(size_t)blockIdx.x * dim + c] = red[c];
}

// out[c] += scale * sum_b part[b][c] over `nb` partial rows, in order.
__global__ void dgamma_reduce_rows_kernel(const float* __restrict__ part, int nb,
                                          float* __restrict__ out, int dim, float scale) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= dim) return;
  float acc = 0.f;
  for (int b = 0; b < nb; ++b) acc += part[(size_t)b * dim + c];
  out[c] += scale * acc;
}

constexpr int DGAMMA_SPLITS = 64;

// dgamma[c] = sum_t dy[t][c] x[t][c] rinv[t], first pass: DGAMMA_SPLITS row ranges,
// one thread per column (coalesced), partial sums in part[split][dim].
__global__ void dgamma_partial_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                      const float* __restrict__ rinv, float* __restrict__ part,
                                      int T, int dim) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int split = blockIdx.y;
  if (c >= dim) return;
  const int per = (T + DGAMMA_SPLITS - 1) / DGAMMA_SPLITS;
  const int t0 = split * per, t1 = min(T, t0 + per);
  float acc = 0.f;
  for (int t = t0; t < t1; ++t) acc += dy[(size_t)t * dim + c] * x[(size_t)t * dim + c] * rinv[t];
  part[(size_t)split * dim + c] = acc;
}

// out[c] += scale * sum_s part[s][c] (fixed order).
__global__ void dgamma_reduce_kernel(const float* __restrict__ part, float* __restrict__ out,
                                     int dim, float scale) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= dim) return;
  float acc = 0.f;
  for (int s = 0; s < DGAMMA_SPLITS; ++s) acc += part[(size_t)s * dim + c];
  out[c] += scale * acc;
}

// grad[i] += sum_s part[s * n + i] (fixed order): the split-K reduction.
__global__ void grad_reduce_kernel(float* __restrict__ grad, const float* __restrict__ part,
                                   int splits, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n / 4;
       i += (size_t)gridDim.x * blockDim.x) {
    float4 g = reinterpret_cast<const float4*>(grad)[i];
    for (int s = 0; s < splits; ++s) {
      const float4 p = reinterpret_cast<const float4*>(part + (size_t)s * n)[i];
      g.x += p.x;
      g.y += p.y;
      g.z += p.z;
      g.w += p.w;
    }
    reinterpret_cast<float4*>(grad)[i] = g;
  }
}

// Embedding backward (embedding.rs:34-44): dE[v] += scale * sum of dX rows whose token
// is v, in position order. One warp per vocabulary row scans the token list (ballots of
// 32) and accumulates its matches in registers, 32 columns per lane per pass.
__global__ void embed_bwd_kernel(const uint32_t* __restrict__ tokens, int T,
                                 const float* __restrict__ dx, int dim, int vocab,
                                 float* __restrict__ dembed, float scale) {
  const int v = blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (v >= vocab) return;
  for (int c0 = 0; c0 < dim; c0 += 1024) {  // 32 columns per lane per pass
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
    bool any = false;
    for (int t0 = 0; t0 < T; t0 += 32) {
      const int t = t0 + lane;
      unsigned m = __ballot_sync(0xffffffffu, t < T && tokens[t] == (uint32_t)v);
      while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1;
        any = true;
        const float* src = dx + (size_t)(t0 + j) * dim + c0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int c = i * 32 + lane;
          if (c0 + c < dim) acc[i] += src[c];
        }
      }
    }
    if (!any) continue;
    float* dst = dembed + (size_t)v * dim + c0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int c = i * 32 + lane;
      if (c0 + c < dim) dst[c] += scale * acc[i];
    }
  }
}

// Reference-orientation copy of one storage-layout gradient (the inverse of
// load_weight_kernel): out[ref index] = grad[storage element] for the elements of
// reference tensor `sub`.
__global__ void grad_to_ref_kernel(const float* __restrict__ grad, int st, int rows, int cols,
                                   ShapeInfo s, int sub, float* __restrict__ out) {
  const uint64_t total = (uint64_t)rows * cols;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    const RefElem e = ref_of_storage(st, r, c, s);
    if (e.kind != sub) continue;
    out[e.idx] = grad[i];
  }
}

}  // namespace cb

// ------------------------------------------------------------------ host side

struct TrainState {
  size_t T = 0;
  // saved activations, per layer
  float* x_in = nullptr;   // [L][T][d] layer inputs
  __half* xn = nullptr;    // [L][T][d]
  float* r1 = nullptr;     // [L][T]
  __half* q = nullptr;     // [L][B,H,S,128]
  __half* k = nullptr;     // [L][B,Hkv,S,128]
  __half* v = nullptr;
  __half* attn = nullptr;  // [L][T][qd]
  float* lse = nullptr;    // [L][B,H,S]
  float* x2 = nullptr;     // [L][T][d]
  __half* x2n = nullptr;   // [L][T][d]
  float* r2 = nullptr;     // [L][T]
  __half* h13 = nullptr;   // [L][T][2h]
  __half* g = nullptr;     // [L][T][h]
  float* x_last = nullptr; // [T][d] final residual (before the final norm)
  float* rf = nullptr;     // [T]
  // backward scratch
  __half* dl = nullptr;    // [T][V]
  float* dtmp = nullptr;   // [T][d]
  float* dxa = nullptr;    // [T][d]
  float* dxb = nullptr;    // [T][d]
  __half* dxh = nullptr;   // [T][d]
  __half* dh13 = nullptr;  // [T][2h]
  __half* da = nullptr;    // [T][qd]
  __half* dqkv = nullptr;  // [T][n_qkv]
  float* dq32 = nullptr;   // [T][qd]
  float* dsum = nullptr;   // [B,H,S]
  float* dgam = nullptr;   // [DGAMMA_SPLITS][d]
  float* gpart = nullptr;  // split-K partials
  size_t gpart_elems = 0;
  // gradients (fp32, storage layout of the weights)
  float* g_embed = nullptr;
  float* g_wqkv = nullptr;
  float* g_wo = nullptr;
  float* g_w13 = nullptr;
  float* g_w2 = nullptr;
  float* g_gamma = nullptr;        // [L][2][d]
  float* g_gamma_final = nullptr;  // [d]
  std::vector<void*> allocs;
  std::map<std::tuple<int, uint32_t, uint32_t>, cudaGraphExec_t> graphs;
};

namespace {

// Tile mode and K split of a weight-gradient GEMM (M x N output, K = tokens): every
// (mode, splits) candidate gets an estimated time, the FLOPs at a tensor rate scaled by
// its last-wave fill (and by how fast each tile mode runs these MN-major GEMMs: the CTA
// pair fastest) plus the split-K partials' DRAM round trip; each split keeps >= 1024
// k-rows.
void pick_grad_gemm(int M, int N, int K, const DeviceInfo& di, size_t max_partial, int* mode,
                    int* splits) {
  auto fill = [](long tiles, long units) {
    const long waves = (tiles + units - 1) / units;
    return (double)tiles / (double)(waves * units);
  };
  const bool n256 = N % 256 == 0;
  const double flops = 2.0 * M * N * K, tensor = 1.3e15, hbm = 5.0e12;
  double best = 1e30;
  *mode = GM_SINGLE128;
  *splits = 1;
  for (int sp = 1; sp <= 8; sp *= 2) {
    if (sp > 1 && (K / sp < 1024 || (size_t)sp * M * N > max_partial)) break;
    const double extra = sp > 1 ? (double)sp * M * N * 4 * 2 + (double)M * N * 8 : 0.0;
    struct Cand { int mode; double rate; };
    const Cand cands[3] = {
        {GM_PAIR, n256 ? fill((long)((M + 255) / 256) * (N / 256) * sp, di.pair_clusters) : 0.0},
        {GM_SINGLE256, n256 ? 0.85 * fill((long)((M + 127) / 128) * (N / 256) * sp, di.sms) : 0.0},
        {GM_SINGLE128, 0.65 * fill((long)((M + 127) / 128) * ((N + 127) / 128) * sp, di.sms)}};
    for (const Cand& c : cands) {
      if (c.rate <= 0.0) continue;
      const double t = flops / (tensor * c.rate) + extra / hbm;
      if (t < best) {
        best = t;
        *mode = c.mode;
        *splits = sp;
      }
    }
  }
}

}  // namespace

void free_train_state(TrainState* t) {
  if (!t) return;
  for (auto& kv : t->graphs) cudaGraphExecDestroy(kv.second);
  for (void* p : t->allocs) cudaFree(p);
  delete t;
}

static cb_status alloc_train(cb_ctx* c) {
  if (c->train) return CB_OK;
  const cb_model_config& cfg = c->cfg;
  const size_t T = c->T_max(), d = cfg.dim, L = cfg.nlayers, V = cfg.vocab;
  const size_t h = c->hidden_l, qd = c->q_dim, kvd = c->kv_dim, nq = c->n_qkv;
  TrainState* t = new TrainState;
  t->T = T;
  bool ok = true;
  auto get = [&](auto** p, size_t n) {
    if (!ok) return;
    void* q = nullptr;
    if (cudaMalloc(&q, std::max<size_t>(n * sizeof(**p), 16)) != cudaSuccess) {
      ok = false;
      return;
    }
    t->allocs.push_back(q);
    *p = static_cast<std::remove_reference_t<decltype(*p)>>(q);
  };
  get(&t->x_in, L * T * d);
  get(&t->xn, L * T * d);
  get(&t->r1, L * T);
  get(&t->q, L * T * qd);
  get(&t->k, L * T * kvd);
  get(&t->v, L * T * kvd);
  get(&t->attn, L * T * qd);
  get(&t->lse, L * T * c->heads_l);
  get(&t->x2, L * T * d);
  get(&t->x2n, L * T * d);
  get(&t->r2, L * T);
  get(&t->h13, L * T * 2 * h);
  get(&t->g, L * T * h);
  get(&t->x_last, T * d);
  get(&t->rf, T);
  get(&t->dl, T * V);
  get(&t->dtmp, T * d);
  get(&t->dxa, T * d);
  get(&t->dxb, T * d);
  get(&t->dxh, T * d);
  get(&t->dh13, T * 2 * h);
  get(&t->da, T * qd);
  get(&t->dqkv, T * nq);
  get(&t->dq32, T * qd);
  get(&t->dsum, T * c->heads_l);
  get(&t->dgam, std::max<size_t>(DGAMMA_SPLITS, (T + RB_ROWS - 1) / RB_ROWS) * d);
  const size_t maxw = std::max(std::max(V * d, 2 * h * d), std::max(nq * d, d * qd));
  t->gpart_elems = 8 * maxw;
  get(&t->gpart, t->gpart_elems);
  get(&t->g_embed, V * d);
  get(&t->g_wqkv, L * nq * d);
  get(&t->g_wo, L * d * qd);
  get(&t->g_w13, L * 2 * h * d);
  get(&t->g_w2, L * d * h);
  get(&t->g_gamma, L * 2 * d);
  get(&t->g_gamma_final, d);
  if (!ok) {
    free_train_state(t);
    return fail(c, CB_ERR_OUT_OF_MEMORY, "training buffers do not fit in device memory");
  }
  c->train = t;
  return CB_OK;
}

static cudaError_t zero_grads(cb_ctx* c, cudaStream_t st) {
  TrainState* t = c->train;
  const cb_model_config& cfg = c->cfg;
  const size_t d = cfg.dim, L = cfg.nlayers, V = cfg.vocab;
  const size_t h = c->hidden_l, qd = c->q_dim, nq = c->n_qkv;
  const std::pair<void*, size_t> bufs[] = {
      {t->g_embed, V * d}, {t->g_wqkv, L * nq * d}, {t->g_wo, L * d * qd},
      {t->g_w13, L * 2 * h * d}, {t->g_w2, L * d * h}, {t->g_gamma, L * 2 * d},
      {t->g_gamma_final, d}};
  for (const auto& b : bufs) {
    cudaError_t e = cudaMemsetAsync(b.first, 0, b.second * sizeof(float), st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// One training step (forward with saved activations + backward) on `st`.
static cudaError_t enqueue_train_step(cb_ctx* c, int batch, float softcap, float loss_scale,
                                      cudaStream_t st) {
  TrainState* t = c->train;
  const cb_model_config& cfg = c->cfg;
  const int S = cfg.seq, d = cfg.dim, hid = c->hidden_l, V = cfg.vocab, L = cfg.nlayers;
  const int T = batch * S, H = c->heads_l, Hk = c->kv_heads_l;
  const int qd = c->q_dim, nq = c->n_qkv;
  const size_t Ts = c->T_max();  // per-layer stride of the saved buffers
  const float alpha = 1.0f / sqrtf(2.0f * (float)L);
  const float s_w = loss_scale / (float)S;
  const int row_blocks = (T + ROW_WARPS - 1) / ROW_WARPS;
  const DeviceInfo& di = device_info(c->device);
  cudaError_t e;
  bool maps_ok = true;
  auto kmap = [&](const void* p, int K, int rows) {  // K-major A operand [rows][K]
    CUtensorMap m;
    maps_ok &= make_tmap(&m, p, K, rows, 1, 128);
    return m;
  };
  auto mnmap = [&](const void* p, int mn, int K, int depth = 1) {  // MN-major [depth][K][mn]
    CUtensorMap m;
    maps_ok &= make_tmap_mn(&m, p, mn, K, depth);
    return m;
  };
#define TRY(...)                                      \
  do {                                                \
    if ((e = (__VA_ARGS__)) != cudaSuccess) return e; \
  } while (0)
#define TRY_LAUNCH() TRY(cudaGetLastError())

  // ---------------- forward (saved activations)
  embed_rmsnorm_kernel<<<row_blocks, ROW_WARPS * 32, 0, st>>>(
      c->tokens, c->embed, c->gamma, t->x_in, t->xn, T, d, V, c->dev_err, t->r1);
  TRY_LAUNCH();
  const int m_qkv = pick_mode(T, nq, di), m_o = pick_mode(T, d, di);
  const int m_13 = pick_mode(T, 2 * hid, di), m_2 = pick_mode(T, d, di);
  for (int l = 0; l < L; ++l) {
    const size_t lo = (size_t)l * Ts;
    float* x_in = t->x_in + lo * d;
    __half* xn = t->xn + lo * d;
    __half *q = t->q + lo * qd, *k = t->k + lo * c->kv_dim, *v = t->v + lo * c->kv_dim;
    __half* attn = t->attn + lo * qd;
    {
      EpiQkvRope ep{q, k, v, c->rope, S, H, Hk};
      const CUtensorMap ta = kmap(xn, d, T);
      TRY(launch_gemm(m_qkv, ta, c->tm_wqkv[0], c->tm_wqkv[1], T, nq, d, l, ep, c->dev_err, di,
                      st, 1, nullptr, nullptr, true));
    }
    {
      CUtensorMap tq, tk, tv;
      const bool tc = S % FA_BQ == 0 && make_tmap_qkv(&tq, q, (uint64_t)T * H, FA_BQ) &&
                      make_tmap_qkv(&tk, k, (uint64_t)T * Hk, FA_BKV) &&
                      make_tmap_qkv(&tv, v, (uint64_t)T * Hk, FA_BKV);
      TRY(launch_attention(tc ? &tq : nullptr, &tk, &tv, q, k, v, attn, batch, H, Hk, S,
                           c->dev_err, st, t->lse + lo * H));
    }
    {
      EpiScaledF16 ep{c->delta, d, alpha};
      const CUtensorMap ta = kmap(attn, qd, T);
      TRY(launch_gemm(m_o, ta, c->tm_wo[0], c->tm_wo[1], T, d, qd, l, ep, c->dev_err, di, st, 1, nullptr, nullptr, true));
    }
    float* x2 = t->x2 + lo * d;
    __half* x2n = t->x2n + lo * d;
    TRY(launch_add_rmsnorm(x_in, x2, c->delta, c->gamma + (size_t)l * 2 * d + d, x2n, T, d, st,
                           t->r2 + lo));
    __half* g = t->g + lo * hid;
    {
      EpiSwigluSave ep{g, hid, t->h13 + lo * 2 * hid, 2 * hid};
      const CUtensorMap ta = kmap(x2n, d, T);
      TRY(launch_gemm(m_13, ta, c->tm_w13[0], c->tm_w13[1], T, 2 * hid, d, l, ep, c->dev_err,
                      di, st, 1, nullptr, nullptr, true));
    }
    {
      EpiScaledF16 ep{c->delta, d, alpha};
      const CUtensorMap ta = kmap(g, hid, T);
      TRY(launch_gemm(m_2, ta, c->tm_w2[0], c->tm_w2[1], T, d, hid, l, ep, c->dev_err, di, st, 1, nullptr, nullptr, true));
    }
    const bool last = l + 1 == L;
    TRY(launch_add_rmsnorm(x2, last ? t->x_last : t->x_in + (lo + Ts) * d, c->delta,
                           last ? c->gamma_final : c->gamma + (size_t)(l + 1) * 2 * d,
                           last ? c->xn : t->xn + (lo + Ts) * d, T, d, st,
                           last ? t->rf : t->r1 + lo + Ts));
  }
  if (!maps_ok) return cudaErrorInvalidValue;
  const int m_head = pick_mode(T, V, di);
  const int nparts = (V + mode_block_n(m_head) - 1) / mode_block_n(m_head);
  {
    EpiCrossEntropy ep{};
    ep.part = c->ce_part;
    ep.nparts = nparts;
    ep.targets = c->targets;
    ep.tgt_logit = c->tgt_logit;
    ep.softcap = softcap;
    TRY(launch_gemm(m_head, c->tm_xn, c->tm_embed[0], c->tm_embed[1], T, V, d, 0, ep,
                    c->dev_err, di, st, 1, nullptr, nullptr, true));
  }
  ce_finalize_kernel<<<row_blocks, ROW_WARPS * 32, 0, st>>>(c->ce_part, nparts, c->tgt_logit,
                                                            c->tok_loss, c->block_sums, T);
  TRY_LAUNCH();
  loss_mean_kernel<<<1, 256, 0, st>>>(c->block_sums, row_blocks, T, c->loss);
  TRY_LAUNCH();

  // ---------------- backward
  // weight-gradient GEMM: grad[M][N] += s_w * A^T B over the T tokens (A, B MN-major)
  auto grad_gemm = [&](const CUtensorMap& ta, const CUtensorMap& tb, int M, int N,
                       float* grad) -> cudaError_t {
    int mode, splits;
    pick_grad_gemm(M, N, T, di, t->gpart_elems, &mode, &splits);
    if (splits == 1) {
      EpiScaledF32Add ep{grad, N, s_w};  // one add per element: order-independent
      return launch_gemm<EpiScaledF32Add, GEMM_A_MN | GEMM_B_MN>(mode, ta, tb, tb, M, N, T, 0,
                                                                 ep, c->dev_err, di, st, 1, nullptr, nullptr, true);
    }
    if ((size_t)splits * M * N > t->gpart_elems) return cudaErrorInvalidValue;
    EpiPartialF32 ep{t->gpart, N, s_w, (size_t)M * N};
    cudaError_t r = launch_gemm<EpiPartialF32, GEMM_A_MN | GEMM_B_MN>(
        mode, ta, tb, tb, M, N, T, 0, ep, c->dev_err, di, st, splits, nullptr, nullptr, true);
    if (r != cudaSuccess) return r;
    const size_t n = (size_t)M * N;
    const int blocks = (int)std::min<size_t>((n / 4 + 255) / 256, (size_t)di.sms * 16);
    grad_reduce_kernel<<<blocks, 256, 0, st>>>(grad, t->gpart, splits, n);
    return cudaGetLastError();
  };
  auto dgamma = [&](const float* dy, const float* x, const float* rinv, float* out) {
    dim3 grid((d + 255) / 256, DGAMMA_SPLITS);
    dgamma_partial_kernel<<<grid, 256, 0, st>>>(dy, x, rinv, t->dgam, T, d);
    dgamma_reduce_kernel<<<(d + 255) / 256, 256, 0, st>>>(t->dgam, out, d, s_w);
    return cudaGetLastError();
  };
  // RMSNorm backward + residual, with the gain gradient (+= s_w sum_t dy x_hat) into dgam_out
  // Every GEMM of the step is launched with programmatic dependent launch (its CTAs set
  // up while the kernel before drains and wait in pdl_enter() before touching memory).
  auto norm_bwd = [&](const float* dy, const float* x, const float* gamma, const float* rinv,
                      const float* dres, float* dx, __half* dxh, float* dgam_out) {
    const int nb = (T + RB_ROWS - 1) / RB_ROWS, th = ROW_WARPS * 32;
    bool fused = true;
    if (d <= 512)
      rmsnorm_bwd_dg_kernel<2><<<nb, th, 0, st>>>(dy, x, gamma, rinv, dres, dx, dxh, alpha, T, d,
                                                  t->dgam);
    else if (d <= 1024)
      rmsnorm_bwd_dg_kernel<4><<<nb, th, 0, st>>>(dy, x, gamma, rinv, dres, dx, dxh, alpha, T, d,
                                                  t->dgam);
    else if (d <= 1536)
      rmsnorm_bwd_dg_kernel<6><<<nb, th, 0, st>>>(dy, x, gamma, rinv, dres, dx, dxh, alpha, T, d,
                                                  t->dgam);
    else if (d <= 2048)
      rmsnorm_bwd_dg_kernel<8><<<nb, th, 0, st>>>(dy, x, gamma, rinv, dres, dx, dxh, alpha, T, d,
                                                  t->dgam);
    else
      fused = false;
    if (fused) {
      dgamma_reduce_rows_kernel<<<(d + 255) / 256, 256, 0, st>>>(t->dgam, nb, dgam_out, d, s_w);
      return cudaGetLastError();
    }
    cudaError_t r = dgamma(dy, x, rinv, dgam_out);
    if (r != cudaSuccess) return r;
    rmsnorm_bwd_kernel<<<row_blocks, ROW_WARPS * 32, 0, st>>>(dy, x, gamma, rinv, dres, dx, dxh,
                                                              alpha, T, d);
    return cudaGetLastError();
  };

  // logits gradient, then dXf = dl E and dE += s dl^T Xf
  {
    EpiCeBwd ep{};
    ep.dl = t->dl;
    ep.ldo = V;
    ep.targets = c->targets;
    ep.tok_loss = c->tok_loss;
    ep.tgt_logit = c->tgt_logit;
    ep.softcap = softcap;
    TRY(launch_gemm(m_head, c->tm_xn, c->tm_embed[0], c->tm_embed[1], T, V, d, 0, ep,
                    c->dev_err, di, st, 1, nullptr, nullptr, true));
  }
  {
    EpiScaledF32 ep{t->dtmp, d, 1.0f};
    const CUtensorMap ta = kmap(t->dl, V, T), tb = mnmap(c->embed, d, V);
    TRY(launch_gemm<EpiScaledF32, GEMM_B_MN>(pick_mode(T, d, di), ta, tb, tb, T, d, V, 0, ep,
                                             c->dev_err, di, st, 1, nullptr, nullptr, true));
    TRY(grad_gemm(mnmap(t->dl, V, T), mnmap(c->xn, d, T), V, d, t->g_embed));
  }
  float* dX = t->dxa;
  float* dX2 = t->dxb;
  TRY(norm_bwd(t->dtmp, t->x_last, c->gamma_final, t->rf, nullptr, dX, t->dxh, t->g_gamma_final));

  const CUtensorMap tb_w2 = mnmap(c->w2, hid, d, L);
  const CUtensorMap tb_w13 = mnmap(c->w13, d, 2 * hid, L);
  const CUtensorMap tb_wo = mnmap(c->wo, qd, d, L);
  const CUtensorMap tb_wqkv = mnmap(c->wqkv, d, nq, L);
  const CUtensorMap ta_dxh = kmap(t->dxh, d, T), tg_dxh = mnmap(t->dxh, d, T);
  const CUtensorMap ta_dh13 = kmap(t->dh13, 2 * hid, T), tg_dh13 = mnmap(t->dh13, 2 * hid, T);
  const CUtensorMap ta_dqkv = kmap(t->dqkv, nq, T), tg_dqkv = mnmap(t->dqkv, nq, T);
  for (int l = L - 1; l >= 0; --l) {
    const size_t lo = (size_t)l * Ts;
    // FFN: dG = (alpha dX) W2 -> SwiGLU backward; dW2 += s (alpha dX)^T G
    {
      EpiSwigluBwd ep{t->dh13, t->h13 + lo * 2 * hid, 2 * hid};
      TRY(launch_gemm<EpiSwigluBwd, GEMM_B_MN>(pick_mode(T, hid, di), ta_dxh, tb_w2, tb_w2, T,
                                               hid, d, l, ep, c->dev_err, di, st, 1, nullptr, nullptr, true));
    }
    TRY(grad_gemm(tg_dxh, mnmap(t->g + lo * hid, hid, T), d, hid,
                  t->g_w2 + (size_t)l * d * hid));
    {
      EpiScaledF32 ep{t->dtmp, d, 1.0f};
      TRY(launch_gemm<EpiScaledF32, GEMM_B_MN>(m_2, ta_dh13, tb_w13, tb_w13, T, d, 2 * hid, l,
                                               ep, c->dev_err, di, st, 1, nullptr, nullptr, true));
    }
    TRY(grad_gemm(tg_dh13, mnmap(t->x2n + lo * d, d, T), 2 * hid, d,
                  t->g_w13 + (size_t)l * 2 * hid * d));
    float* g2 = t->g_gamma + (size_t)l * 2 * d + d;
    TRY(norm_bwd(t->dtmp, t->x2 + lo * d, c->gamma + (size_t)l * 2 * d + d, t->r2 + lo, dX, dX2,
                 t->dxh, g2));
    // attention: dA = (alpha dX2) Wo^T; dWo += s (alpha dX2)^T A
    {
      EpiStoreF16Dsum ep{t->da, qd, t->attn + lo * qd, t->dsum, S, H, 0.f};
      TRY(launch_gemm<EpiStoreF16Dsum, GEMM_B_MN>(pick_mode(T, qd, di), ta_dxh, tb_wo, tb_wo, T,
                                                  qd, d, l, ep, c->dev_err, di, st, 1, nullptr, nullptr, true));
    }
    TRY(grad_gemm(tg_dxh, mnmap(t->attn + lo * qd, qd, T), d, qd, t->g_wo + (size_t)l * d * qd));
    TRY(launch_attention_bwd(t->q + lo * qd, t->k + lo * c->kv_dim, t->v + lo * c->kv_dim,
                             t->attn + lo * qd, t->da, t->lse + lo * H, t->dsum, t->dq32, c->rope,
                             c->rope_pm, t->dqkv, batch, H, Hk, S, di.sms, st, c->dev_err,
                             /*dsum_ready=*/true));
    {
      EpiScaledF32 ep{t->dtmp, d, 1.0f};
      TRY(launch_gemm<EpiScaledF32, GEMM_B_MN>(m_o, ta_dqkv, tb_wqkv, tb_wqkv, T, d, nq, l, ep,
                                               c->dev_err, di, st, 1, nullptr, nullptr, true));
    }
    TRY(grad_gemm(tg_dqkv, mnmap(t->xn + lo * d, d, T), nq, d,
                  t->g_wqkv + (size_t)l * nq * d));
    float* g1 = t->g_gamma + (size_t)l * 2 * d;
    TRY(norm_bwd(t->dtmp, t->x_in + lo * d, c->gamma + (size_t)l * 2 * d, t->r1 + lo, dX2, dX,
                 t->dxh, g1));
  }
  if (!maps_ok) return cudaErrorInvalidValue;
  embed_bwd_kernel<<<(V + ROW_WARPS - 1) / ROW_WARPS, ROW_WARPS * 32, 0, st>>>(
      c->tokens, T, dX, d, V, t->g_embed, s_w);
  TRY_LAUNCH();
#undef TRY
#undef TRY_LAUNCH
  return cudaSuccess;
}

extern "C" {

cb_status cb_enable_training(cb_ctx* ctx) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  if (ctx->tp_world > 1)
    return fail(ctx, CB_ERR_UNSUPPORTED, "training on a tensor-parallel context is not supported");
  CB_CUDA(cudaSetDevice(ctx->device));
  cb_status rc = alloc_train(ctx);
  if (rc != CB_OK) return rc;
  CB_CUDA(zero_grads(ctx, ctx->stream));
  CB_CUDA(cudaStreamSynchronize(ctx->stream));
  return CB_OK;
}

cb_status cb_zero_grads(cb_ctx* ctx) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  if (!ctx->train) return fail(ctx, CB_ERR_NOT_READY, "training is not enabled");
  CB_CUDA(cudaSetDevice(ctx->device));
  CB_CUDA(zero_grads(ctx, ctx->stream));
  CB_CUDA(cudaStreamSynchronize(ctx->stream));
  return CB_OK;
}

cb_status cb_forward_backward(cb_ctx* ctx, const uint32_t* tokens, const uint32_t* targets,
                              int32_t batch, float softcap, float loss_scale, float* loss_out) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  if (!ctx->train) return fail(ctx, CB_ERR_NOT_READY, "training is not enabled");
  cb_status rc = check_forward_args(ctx, tokens, targets, batch);
  if (rc != CB_OK) return rc;
  if (!loss_out) return fail(ctx, CB_ERR_INVALID_ARG, "null loss_out");
  const size_t T = (size_t)batch * ctx->cfg.seq;
  const uint32_t V = (uint32_t)ctx->cfg.vocab;
  for (size_t i = 0; i < T; ++i)
    if (tokens[i] >= V || targets[i] >= V)
      return fail(ctx, CB_ERR_INVALID_ARG, "token id out of range at position " + std::to_string(i));
  CB_CUDA(cudaSetDevice(ctx->device));
  cudaStream_t st = ctx->stream;
  CB_CUDA(cudaMemcpyAsync(ctx->tokens, tokens, T * 4, cudaMemcpyHostToDevice, st));
  CB_CUDA(cudaMemcpyAsync(ctx->targets, targets, T * 4, cudaMemcpyHostToDevice, st));
  uint32_t sc_bits, ls_bits;
  std::memcpy(&sc_bits, &softcap, 4);
  std::memcpy(&ls_bits, &loss_scale, 4);
  const auto key = std::make_tuple((int)batch, sc_bits, ls_bits);
  TrainState* t = ctx->train;
  auto it = t->graphs.find(key);
  if (it == t->graphs.end()) {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    CB_CUDA(prepare_attention(ctx, batch));
    CB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = enqueue_train_step(ctx, batch, softcap, loss_scale, st);
    cudaError_t e2 = cudaStreamEndCapture(st, &graph);
    if (e != cudaSuccess || e2 != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();
      return fail(ctx, CB_ERR_CUDA, std::string("training step capture: ") +
                                        cudaGetErrorString(e != cudaSuccess ? e : e2));
    }
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess)
      return fail(ctx, CB_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    it = t->graphs.emplace(key, exec).first;
  }
  CB_CUDA(cudaGraphLaunch(it->second, st));
  ctx->last_batch = batch;
  ctx->last_softcap = softcap;
  ctx->x_final = t->x_last;
  CB_CUDA(cudaMemcpyAsync(ctx->h_loss, ctx->loss, sizeof(float), cudaMemcpyDeviceToHost, st));
  rc = read_device_error(ctx);
  if (rc != CB_OK) return rc;
  *loss_out = *ctx->h_loss;
  return CB_OK;
}

cb_status cb_get_grads_f32(cb_ctx* ctx, float* d_embed, float* d_gamma_final,
                           const cb_layer_grads_f32* layers) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  if (!ctx->train) return fail(ctx, CB_ERR_NOT_READY, "training is not enabled");
  if (!d_embed || !d_gamma_final || !layers)
    return fail(ctx, CB_ERR_INVALID_ARG, "null gradient pointer");
  const cb_model_config& cfg = ctx->cfg;
  for (int l = 0; l < cfg.nlayers; ++l) {
    const cb_layer_grads_f32& w = layers[l];
    if (!w.wq || !w.wk || !w.wv || !w.wo || !w.w1 || !w.w3 || !w.w2 || !w.gamma1 || !w.gamma2)
      return fail(ctx, CB_ERR_INVALID_ARG, "null pointer in layer " + std::to_string(l));
  }
  CB_CUDA(cudaSetDevice(ctx->device));
  TrainState* t = ctx->train;
  const ShapeInfo s = shape_of(ctx);
  const size_t d = cfg.dim, hid = cfg.hidden, V = cfg.vocab;
  const size_t qd = (size_t)cfg.heads * 128, kvd = (size_t)cfg.kv_heads * 128;
  const size_t stage_n = std::max(std::max(V * d, d * hid), d * qd);
  float* stage = nullptr;
  CB_CUDA(cudaMalloc(&stage, stage_n * sizeof(float)));
  cudaStream_t st = ctx->stream;
  const int grid = ctx->num_sms * 8, block = 256;
  bool ok = true;
  auto out = [&](const float* g, int kind, int rows, int cols, int sub, float* host, size_t n) {
    if (!ok) return;
    grad_to_ref_kernel<<<grid, block, 0, st>>>(g, kind, rows, cols, s, sub, stage);
    ok = cudaGetLastError() == cudaSuccess &&
         cudaMemcpyAsync(host, stage, n * sizeof(float), cudaMemcpyDeviceToHost, st) ==
             cudaSuccess &&
         cudaStreamSynchronize(st) == cudaSuccess;
  };
  out(t->g_embed, ST_EMBED, (int)V, (int)d, -1, d_embed, V * d);
  ok = ok && cudaMemcpy(d_gamma_final, t->g_gamma_final, d * 4, cudaMemcpyDeviceToHost) ==
                 cudaSuccess;
  for (int l = 0; ok && l < cfg.nlayers; ++l) {
    const cb_layer_grads_f32& w = layers[l];
    const float* gq = t->g_wqkv + (size_t)l * ctx->n_qkv * d;
    out(gq, ST_QKV, ctx->n_qkv, (int)d, CB_T_WQ, w.wq, d * qd);
    out(gq, ST_QKV, ctx->n_qkv, (int)d, CB_T_WK, w.wk, d * kvd);
    out(gq, ST_QKV, ctx->n_qkv, (int)d, CB_T_WV, w.wv, d * kvd);
    out(t->g_wo + (size_t)l * d * ctx->q_dim, ST_WO, (int)d, ctx->q_dim, CB_T_WO, w.wo, qd * d);
    const float* g13 = t->g_w13 + (size_t)l * 2 * ctx->hidden_l * d;
    out(g13, ST_W13, 2 * ctx->hidden_l, (int)d, CB_T_W1, w.w1, d * hid);
    out(g13, ST_W13, 2 * ctx->hidden_l, (int)d, CB_T_W3, w.w3, d * hid);
    out(t->g_w2 + (size_t)l * d * ctx->hidden_l, ST_W2, (int)d, ctx->hidden_l, CB_T_W2, w.w2,
        d * hid);
    ok = ok &&
         cudaMemcpy(w.gamma1, t->g_gamma + (size_t)l * 2 * d, d * 4, cudaMemcpyDeviceToHost) ==
             cudaSuccess &&
         cudaMemcpy(w.gamma2, t->g_gamma + (size_t)l * 2 * d + d, d * 4,
                    cudaMemcpyDeviceToHost) == cudaSuccess;
  }
  cudaFree(stage);
  if (!ok) return fail(ctx, CB_ERR_CUDA, "gradient read-back failed");
  return CB_OK;
}

}  // extern "C"
