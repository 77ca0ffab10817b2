// Single-token decode with a KV cache (the intent of the reference's metal-decode crate,
// crates/metal-decode/src/lib.rs:1-4, a placeholder there).
//
// Included at the end of bridge.cu. A prefill runs the ordinary forward over the prompt
// (padded to seq; causal attention makes the padding invisible to earlier positions)
// with every layer's roped K and V kept in the cache [L][max_batch][kv_heads][seq][128].
// Each decode step then advances all `batch` sequences by one token at the shared
// position `pos`:
//   embedding + RMSNorm -> per layer: QKV (tcgen05 GEMM, split-K) -> RoPE at pos, K/V
//   appended to the cache -> attention of the new query over keys 0..pos -> O projection
//   (split-K) -> residual + RMSNorm -> W1/W3 (split-K) -> SwiGLU -> W2 (split-K) ->
//   residual + RMSNorm -> final norm -> tied LM head (split-K) -> logits (softcap) and
//   the greedy next token.
// With M = batch <= 128 rows a GEMM has one row of tiles; K is split so that about one
// work unit per SM streams its slice of the weights (decode reads every weight once per
// step: the step is bound by HBM, weights plus the KV cache). The partial sums land in
// separate fp32 slices that the following element-wise kernel adds in a fixed order.
// The position lives in device memory, so one CUDA graph per batch size serves every
// step.

namespace cb {

// Sum of the split-K partials of element (row b, column c): part[s][b][n], added in split
// order. All loads go out before the first add (predicated up to DEC_MAX_SPLITS): the
// partials were just written and sit in L2, and one dependent load per split made these
// kernels latency-bound.
// MAXS (>= splits) bounds the predicated loads: the element-wise kernels are instantiated
// for up to 4 splits (QKV, W1/W3, LM head) and up to DEC_MAX_SPLITS (O, down).
constexpr int DEC_MAX_SPLITS = 16;
template <int MAXS = DEC_MAX_SPLITS>
__device__ __forceinline__ float sum_parts(const float* __restrict__ part, int splits,
                                           size_t slice, size_t idx) {
  float a[MAXS];
#pragma unroll
  for (int s = 0; s < MAXS; ++s)
    a[s] = s < splits ? __ldg(part + (size_t)s * slice + idx) : 0.f;
  float acc = 0.f;
#pragma unroll
  for (int s = 0; s < MAXS; ++s)
    if (s < splits) acc += a[s];
  return acc;
}

// QKV of the new token: RoPE at `pos` on Q and K (sdpa_fwd.rs:53-60), Q to qbuf [B][qd],
// K and V into cache slot `pos` ([B][kv_heads][seq][128] of this layer).
template <int MAXS>
__global__ void decode_qkv_kernel(const float* __restrict__ part, int splits, int B, int n_qkv,
                                  int heads, int kv_heads, const int* __restrict__ pos_ptr,
                                  const float2* __restrict__ cs_pos, int seq,
                                  __half* __restrict__ qbuf, __half* __restrict__ kc,
                                  __half* __restrict__ vc) {
  pdl_enter();
  const int pos = *pos_ptr;
  const int qd = heads * 128, kvd = kv_heads * 128;
  const size_t slice = (size_t)B * n_qkv;
  const int pairs = n_qkv / 2;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < B * pairs; i += gridDim.x * blockDim.x) {
    const int b = i / pairs, col = 2 * (i % pairs);
    float a0 = sum_parts<MAXS>(part, splits, slice, (size_t)b * n_qkv + col);
    float a1 = sum_parts<MAXS>(part, splits, slice, (size_t)b * n_qkv + col + 1);
    if (col < qd + kvd) {  // rotate Q and K
      const float2 cs = cs_pos[(col & 127) >> 1];  // no dependency on pos: one round trip
      const float r0 = a0 * cs.x - a1 * cs.y, r1 = a1 * cs.x + a0 * cs.y;
      a0 = r0;
      a1 = r1;
    }
    const uint32_t w = pack_half2(a0, a1);
    if (col < qd) {
      *reinterpret_cast<uint32_t*>(qbuf + (size_t)b * qd + col) = w;
    } else {
      const bool is_k = col < qd + kvd;
      const int c = is_k ? col - qd : col - qd - kvd;
      const int hk = c >> 7, dim = c & 127;
      __half* dst = (is_k ? kc : vc) + (((size_t)b * kv_heads + hk) * seq + pos) * 128 + dim;
      *reinterpret_cast<uint32_t*>(dst) = w;
    }
  }
}

// Attention of one new query per (sequence, head) over cached keys 0..pos, split along
// the keys into `nsplit` CTAs (blockIdx.z) of DEC_ATTN_WARPS warps; lanes split the 128
// dims (4 each), each warp takes 4 keys per step (independent dot-product reductions)
// with an online softmax in base 2. The kernel is bound by memory latency (the K and V
// rows a warp waits on), so a CTA has 8 warps at 40 registers: at 64 sequences the 768
// CTAs of one wave hold ~40 warps per SM. A split writes its (max, sum, unnormalised
// output) to `acc` for decode_attn_combine_kernel; with one split the kernel writes the
// output directly.
constexpr int DEC_ATTN_WARPS = 8;
struct DecAttnPart {
  float m, l;
  float o[128];
};

__global__ void __launch_bounds__(DEC_ATTN_WARPS * 32)
    decode_attn_kernel(const __half* __restrict__ q, const __half* __restrict__ kc,
                       const __half* __restrict__ vc, const int* __restrict__ pos_ptr,
                       int seq, int heads, int kv_heads, float scale_log2,
                       __half* __restrict__ out, DecAttnPart* __restrict__ acc) {
  pdl_enter();
  __shared__ float sm_m[DEC_ATTN_WARPS], sm_l[DEC_ATTN_WARPS];
  __shared__ float sm_o[DEC_ATTN_WARPS][128];
  const int h = blockIdx.x, b = blockIdx.y, split = blockIdx.z, nsplit = gridDim.z;
  const int hk = h / (heads / kv_heads);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = *pos_ptr + 1;
  const int per = (n + nsplit - 1) / nsplit;
  const int k0 = split * per, k1 = min(n, k0 + per);
  float qv[4];
  {
    const uint2 u = *reinterpret_cast<const uint2*>(q + ((size_t)b * heads + h) * 128 + lane * 4);
    const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    qv[0] = f0.x * scale_log2;
    qv[1] = f0.y * scale_log2;
    qv[2] = f1.x * scale_log2;
    qv[3] = f1.y * scale_log2;
  }
  const __half* kb = kc + ((size_t)b * kv_heads + hk) * seq * 128 + lane * 4;
  const __half* vb = vc + ((size_t)b * kv_heads + hk) * seq * 128 + lane * 4;
  float m = -CUDART_INF_F, l = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
  for (int key = k0 + warp * 4; key < k1; key += 4 * DEC_ATTN_WARPS) {
    float s[4];
    uint2 vu[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kk = min(key + j, k1 - 1);
      const uint2 ku = __ldg(reinterpret_cast<const uint2*>(kb + (size_t)kk * 128));
      vu[j] = __ldg(reinterpret_cast<const uint2*>(vb + (size_t)kk * 128));
      const float2 a0 = __half22float2(*reinterpret_cast<const __half2*>(&ku.x));
      const float2 a1 = __half22float2(*reinterpret_cast<const __half2*>(&ku.y));
      s[j] = qv[0] * a0.x + qv[1] * a0.y + qv[2] * a1.x + qv[3] * a1.y;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[j] += __shfl_xor_sync(0xffffffffu, s[j], off);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (key + j >= k1) s[j] = -CUDART_INF_F;
    const float mn = fmaxf(fmaxf(fmaxf(m, s[0]), fmaxf(s[1], s[2])), s[3]);
    const float corr = exp2_mufu(m - mn);  // 2^-inf = 0 on the first step
    m = mn;
    l *= corr;
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] *= corr;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float p = exp2_mufu(s[j] - mn);
      l += p;
      const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&vu[j].x));
      const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&vu[j].y));
      o[0] += p * v0.x;
      o[1] += p * v0.y;
      o[2] += p * v1.x;
      o[3] += p * v1.y;
    }
  }
  if (lane == 0) {
    sm_m[warp] = m;
    sm_l[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) sm_o[warp][lane * 4 + i] = o[i];
  __syncthreads();
  if (warp == 0) {
    float mx = -CUDART_INF_F;
    for (int w = 0; w < DEC_ATTN_WARPS; ++w) mx = fmaxf(mx, sm_m[w]);
    float lt = 0.f, r[4] = {0.f, 0.f, 0.f, 0.f};
    for (int w = 0; w < DEC_ATTN_WARPS; ++w) {
      if (sm_m[w] == -CUDART_INF_F) continue;  // a warp that saw no key
      const float f = exp2_mufu(sm_m[w] - mx);
      lt += sm_l[w] * f;
#pragma unroll
      for (int i = 0; i < 4; ++i) r[i] += sm_o[w][lane * 4 + i] * f;
    }
    if (nsplit == 1) {
      const float inv = 1.0f / lt;
      uint2 w;
      w.x = pack_half2(r[0] * inv, r[1] * inv);
      w.y = pack_half2(r[2] * inv, r[3] * inv);
      *reinterpret_cast<uint2*>(out + ((size_t)b * heads + h) * 128 + lane * 4) = w;
    } else {
      DecAttnPart* a = acc + ((size_t)b * heads + h) * nsplit + split;
      if (lane == 0) {
        a->m = mx;
        a->l = lt;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) a->o[lane * 4 + i] = r[i];
    }
  }
}

// Merge the key splits of one (sequence, head): one warp, lanes over the dims.
__global__ void decode_attn_combine_kernel(const DecAttnPart* __restrict__ acc, int nsplit,
                                           int heads, int total, __half* __restrict__ out) {
  pdl_enter();
  const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= total) return;
  const DecAttnPart* a = acc + (size_t)i * nsplit;
  float mx = -CUDART_INF_F;
  for (int s = 0; s < nsplit; ++s)
    if (a[s].l > 0.f) mx = fmaxf(mx, a[s].m);
  float lt = 0.f, r[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < nsplit; ++s) {
    if (!(a[s].l > 0.f)) continue;  // a split past the last key
    const float f = exp2f(a[s].m - mx);
    lt += a[s].l * f;
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] += a[s].o[lane * 4 + j] * f;
  }
  const float inv = 1.0f / lt;
  uint2 w;
  w.x = pack_half2(r[0] * inv, r[1] * inv);
  w.y = pack_half2(r[2] * inv, r[3] * inv);
  *reinterpret_cast<uint2*>(out + (size_t)i * 128 + lane * 4) = w;
}

// x[b] += alpha * (sum of the partials of row b); xn[b] = RMSNorm(x[b]) * gamma. One
// block per row (the partial sums are many short independent loads: spread them).
constexpr int DEC_NORM_THREADS = 512;
constexpr int DEC_NORM_PER_THREAD = 16;  // rows up to 8192 wide

__global__ void __launch_bounds__(DEC_NORM_THREADS)
    decode_residual_norm_kernel(const float* __restrict__ part, int splits, int B, int dim,
                                float alpha, float* __restrict__ x,
                                const float* __restrict__ gamma, __half* __restrict__ xn) {
  pdl_enter();
  __shared__ float red[DEC_NORM_THREADS / 32];
  const int b = blockIdx.x;
  const size_t slice = (size_t)B * dim;
  float* xr = x + (size_t)b * dim;
  // The row stays in registers (dim <= DEC_NORM_THREADS * DEC_NORM_PER_THREAD), and gamma
  // is loaded with the residual, so the kernel makes one round trip to memory before the
  // reduction instead of three.
  float v[DEC_NORM_PER_THREAD], gm[DEC_NORM_PER_THREAD];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < DEC_NORM_PER_THREAD; ++i) {
    const int c = threadIdx.x + i * DEC_NORM_THREADS;
    v[i] = 0.f;
    gm[i] = 0.f;
    if (c < dim) {
      gm[i] = __ldg(gamma + c);
      v[i] = xr[c] + alpha * sum_parts(part, splits, slice, (size_t)b * dim + c);
      xr[c] = v[i];
      ss += v[i] * v[i];
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < DEC_NORM_THREADS / 32; ++w) tot += red[w];
  const float rinv = 1.0f / sqrtf(tot / (float)dim + RMS_EPS);
#pragma unroll
  for (int i = 0; i < DEC_NORM_PER_THREAD; ++i) {
    const int c = threadIdx.x + i * DEC_NORM_THREADS;
    if (c < dim) xn[(size_t)b * dim + c] = __float2half_rn(v[i] * rinv * gm[i]);
  }
}

// g[b][j] = silu(h1) * h3 from the interleaved W1/W3 partial sums.
template <int MAXS>
__global__ void decode_swiglu_kernel(const float* __restrict__ part, int splits, int B, int hid,
                                     __half* __restrict__ g) {
  pdl_enter();
  const size_t slice = (size_t)B * 2 * hid;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < B * hid; i += gridDim.x * blockDim.x) {
    const int b = i / hid, j = i % hid;
    const float h1 = sum_parts<MAXS>(part, splits, slice, (size_t)b * 2 * hid + 2 * j);
    const float h3 = sum_parts<MAXS>(part, splits, slice, (size_t)b * 2 * hid + 2 * j + 1);
    g[i] = __float2half_rn(__fdividef(h1, 1.0f + __expf(-h1)) * h3);
  }
}

// Logits of row b (softcapped when softcap > 0, full_model.rs:456-461) and the greedy
// next token (largest logit, lowest id on ties). One block per row.
template <int MAXS>
__global__ void decode_logits_kernel(const float* __restrict__ part, int splits, int B, int V,
                                     float softcap, float* __restrict__ logits,
                                     uint32_t* __restrict__ next) {
  pdl_enter();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int b = blockIdx.x;
  const size_t slice = (size_t)B * V;
  float best = -CUDART_INF_F;
  int bi = 0x7fffffff;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    float z = sum_parts<MAXS>(part, splits, slice, (size_t)b * V + v);
    if (softcap > 0.f) z = softcap * tanhf(z / softcap);
    logits[(size_t)b * V + v] = z;
    if (z > best) {  // v increases along the loop: ties keep the lower id
      best = z;
      bi = v;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i)
      if (sv[i] > best || (sv[i] == best && si[i] < bi)) {
        best = sv[i];
        bi = si[i];
      }
    next[b] = (uint32_t)bi;
  }
}

// Position bookkeeping of the decode graph, one block of 64 threads: with advance the
// position moves to pos + 1 (end of a step), otherwise it stays; either way cs_pos
// receives the (cos, sin) of every frequency pair at the new position (pair-major table
// [64][seq]), so the next step's QKV kernel loads its rotation without first reading
// the position.
__global__ void decode_set_pos_kernel(int* pos_ptr, int advance, const float2* __restrict__ rope,
                                      int seq, float2* __restrict__ cs_pos) {
  pdl_enter();
  const int pos = *pos_ptr + advance;
  __syncthreads();  // every thread has read the old position
  if (threadIdx.x == 0) *pos_ptr = pos;
  const int p = pos < seq ? pos : seq - 1;  // a full sequence takes no further step
  if (threadIdx.x < 64) cs_pos[threadIdx.x] = rope[(size_t)threadIdx.x * seq + p];
}

}  // namespace cb

// ------------------------------------------------------------------ host side

constexpr int DEC_MAX_KV_SPLITS = 16;

struct DecodeState {
  __half* kc = nullptr;   // [L][max_batch][kv_heads][seq][128]
  __half* vc = nullptr;
  size_t layer_stride = 0;
  float* x = nullptr;     // [max_batch][d] residual of the new token
  __half* xn = nullptr;   // [max_batch][d]
  __half* q = nullptr;    // [max_batch][qd]
  __half* o = nullptr;    // [max_batch][qd]
  __half* g = nullptr;    // [max_batch][hidden]
  float* part = nullptr;  // split-K partial sums
  size_t part_elems = 0;
  DecAttnPart* attn_acc = nullptr;  // [max_batch][heads][DEC_MAX_KV_SPLITS]
  float* logits = nullptr;    // [max_batch][V]
  uint32_t* next = nullptr;   // [max_batch]
  uint32_t* tok = nullptr;    // [max_batch]
  int* d_pos = nullptr;
  float2* d_cs = nullptr;     // [64] (cos, sin) of each RoPE pair at d_pos
  int pos = 0;                // host copy: position of the next token
  int batch = 0;              // sequences of the last prefill
  float softcap = 0.f;
  CUtensorMap tm_xn, tm_o, tm_g;
  std::vector<void*> allocs;
  std::map<std::pair<int, uint32_t>, cudaGraphExec_t> graphs;
  // pinned staging of a step's outputs (a device-to-host copy into pageable memory runs
  // through the driver's own staging at a fraction of the pinned rate)
  float* h_logits = nullptr;   // [max_batch][V]
  uint32_t* h_next = nullptr;  // [max_batch]
};

void free_decode_state(DecodeState* s) {
  if (!s) return;
  for (auto& kv : s->graphs) cudaGraphExecDestroy(kv.second);
  for (void* p : s->allocs) cudaFree(p);
  if (s->h_logits) cudaFreeHost(s->h_logits);
  if (s->h_next) cudaFreeHost(s->h_next);
  delete s;
}

static cb_status alloc_decode(cb_ctx* c) {
  if (c->decode) return CB_OK;
  const cb_model_config& cfg = c->cfg;
  if (cfg.dim > DEC_NORM_THREADS * DEC_NORM_PER_THREAD)
    return fail(c, CB_ERR_UNSUPPORTED, "decode supports dim <= " +
                                           std::to_string(DEC_NORM_THREADS * DEC_NORM_PER_THREAD));
  const size_t B = c->max_batch, S = cfg.seq, L = cfg.nlayers, d = cfg.dim, V = cfg.vocab;
  const size_t h = c->hidden_l, qd = c->q_dim, nq = c->n_qkv;
  DecodeState* s = new DecodeState;
  bool ok = true;
  auto get = [&](auto** p, size_t n) {
    if (!ok) return;
    void* q = nullptr;
    if (cudaMalloc(&q, std::max<size_t>(n * sizeof(**p), 256)) != cudaSuccess) {
      ok = false;
      return;
    }
    s->allocs.push_back(q);
    *p = static_cast<std::remove_reference_t<decltype(*p)>>(q);
  };
  s->layer_stride = B * c->kv_heads_l * S * 128;
  get(&s->kc, L * s->layer_stride);
  get(&s->vc, L * s->layer_stride);
  get(&s->x, B * d);
  get(&s->xn, B * d);
  get(&s->q, B * qd);
  get(&s->o, B * qd);
  get(&s->g, B * h);
  s->part_elems = 16 * B * std::max(std::max(nq, 2 * h), std::max(d, V));
  get(&s->part, s->part_elems);
  get(&s->attn_acc, B * c->heads_l * DEC_MAX_KV_SPLITS);
  get(&s->logits, B * V);
  get(&s->next, B);
  get(&s->tok, B);
  get(&s->d_pos, 1);
  get(&s->d_cs, 64);
  if (ok) {
    ok = make_tmap(&s->tm_xn, s->xn, d, B, 1, 128) && make_tmap(&s->tm_o, s->o, qd, B, 1, 128) &&
         make_tmap(&s->tm_g, s->g, h, B, 1, 128);
  }
  if (ok)
    ok = cudaMallocHost(reinterpret_cast<void**>(&s->h_logits), B * V * sizeof(float)) ==
             cudaSuccess &&
         cudaMallocHost(reinterpret_cast<void**>(&s->h_next), B * sizeof(uint32_t)) == cudaSuccess;
  if (!ok) {
    free_decode_state(s);
    return fail(c, CB_ERR_OUT_OF_MEMORY, "decode buffers do not fit in device memory");
  }
  c->decode = s;
  return CB_OK;
}

// Split count for a decode GEMM (M <= 128 rows, 1-CTA 128-wide tiles): about one work
// unit per SM, every split non-empty.
static int decode_splits(int N, int K, const DeviceInfo& di) {
  static const int cap = [] {  // CB_DECODE_MAX_SPLITS: a lower cap, for sweeps
    const char* e = getenv("CB_DECODE_MAX_SPLITS");
    return e ? std::max(1, std::min(DEC_MAX_SPLITS, atoi(e))) : DEC_MAX_SPLITS;
  }();
  const int tiles = (N + 127) / 128, kb = (K + GEMM_BK - 1) / GEMM_BK;
  int s = std::max(1, std::min(cap, (di.sms + tiles / 2) / tiles));
  s = std::min(s, kb);
  const int per = (kb + s - 1) / s;
  return (kb + per - 1) / per;
}

static cudaError_t enqueue_decode_step(cb_ctx* c, int B, float softcap, cudaStream_t st) {
  DecodeState* s = c->decode;
  const cb_model_config& cfg = c->cfg;
  const int S = cfg.seq, d = cfg.dim, hid = c->hidden_l, V = cfg.vocab, L = cfg.nlayers;
  const int H = c->heads_l, Hk = c->kv_heads_l, qd = c->q_dim, nq = c->n_qkv;
  const float alpha = 1.0f / sqrtf(2.0f * (float)L);
  const DeviceInfo& di = device_info(c->device);
  const int rb = (B + ROW_WARPS - 1) / ROW_WARPS;
  cudaError_t e;
  auto gemm = [&](const CUtensorMap& ta, const CUtensorMap& tb, int N, int K, int layer,
                  float a, int* splits_out) -> cudaError_t {
    const int sp = decode_splits(N, K, di);
    *splits_out = sp;
    if ((size_t)sp * B * N > s->part_elems) return cudaErrorInvalidValue;
    EpiPartialF32 ep{s->part, N, a, (size_t)B * N};
    return launch_gemm_bn<128, EpiPartialF32>(ta, tb, B, N, K, layer, ep, c->dev_err, di.sms, sp,
                                              st, nullptr, nullptr, /*pdl=*/true);
  };
  // The GEMMs use programmatic dependent launch: their CTAs are scheduled as soon as
  // every CTA of the kernel before has started (the element-wise kernels signal it on
  // entry), set up barriers, TMEM and descriptors, and wait in pdl_enter() before their
  // first memory access. The element-wise kernels launch normally: with PDL their many
  // waiting CTAs made the 64-sequence step 25 % slower (1.75 -> 2.19 ms), while PDL on
  // the GEMMs alone took it from 1.79 to 1.75 ms (1 sequence: 1.215 -> 1.169 ms).
  float* const no_rinv = nullptr;
  if ((e = launch_k(embed_rmsnorm_kernel, dim3(rb), dim3(ROW_WARPS * 32), 0, st, false,
                    (const uint32_t*)s->tok, (const __half*)c->embed, (const float*)c->gamma,
                    s->x, s->xn, B, d, V, c->dev_err, no_rinv)) != cudaSuccess)
    return e;
  const float scale_log2 = 1.4426950408889634f / sqrtf(128.0f);
  // key splits: about two CTAs per SM over (heads, sequences, splits), each split at
  // least 64 keys of the window
  const int kv_splits = std::max(1, std::min({DEC_MAX_KV_SPLITS, S / 64,
                                              (2 * di.sms + B * H - 1) / (B * H)}));
  int sp;
  for (int l = 0; l < L; ++l) {
    __half* kc = s->kc + (size_t)l * s->layer_stride;
    __half* vc = s->vc + (size_t)l * s->layer_stride;
    if ((e = gemm(s->tm_xn, c->tm_wqkv[0], nq, d, l, 1.0f, &sp)) != cudaSuccess) return e;
    const float* part = s->part;
    const int* dpos = s->d_pos;
    if ((e = launch_k(sp <= 4 ? decode_qkv_kernel<4> : decode_qkv_kernel<DEC_MAX_SPLITS>,
                      dim3((B * nq / 2 + 255) / 256), dim3(256), 0, st, false,
                      part, sp, B, nq, H, Hk, dpos, (const float2*)s->d_cs, S, s->q, kc, vc)) !=
        cudaSuccess)
      return e;
    if ((e = launch_k(decode_attn_kernel, dim3(H, B, kv_splits), dim3(DEC_ATTN_WARPS * 32), 0, st,
                      false,
                      (const __half*)s->q, (const __half*)kc, (const __half*)vc, dpos, S, H, Hk,
                      scale_log2, s->o, s->attn_acc)) != cudaSuccess)
      return e;
    if (kv_splits > 1 &&
        (e = launch_k(decode_attn_combine_kernel, dim3((B * H + 7) / 8), dim3(256), 0, st, false,
                      (const DecAttnPart*)s->attn_acc, kv_splits, H, B * H, s->o)) != cudaSuccess)
      return e;
    if ((e = gemm(s->tm_o, c->tm_wo[0], d, qd, l, alpha, &sp)) != cudaSuccess) return e;
    if ((e = launch_k(decode_residual_norm_kernel, dim3(B), dim3(DEC_NORM_THREADS), 0, st, false,
                      part, sp, B, d, 1.0f, s->x, (const float*)(c->gamma + (size_t)l * 2 * d + d),
                      s->xn)) != cudaSuccess)
      return e;
    if ((e = gemm(s->tm_xn, c->tm_w13[0], 2 * hid, d, l, 1.0f, &sp)) != cudaSuccess) return e;
    if ((e = launch_k(sp <= 4 ? decode_swiglu_kernel<4> : decode_swiglu_kernel<DEC_MAX_SPLITS>,
                      dim3((B * hid + 255) / 256), dim3(256), 0, st, false,
                      part, sp, B, hid, s->g)) != cudaSuccess)
      return e;
    if ((e = gemm(s->tm_g, c->tm_w2[0], d, hid, l, alpha, &sp)) != cudaSuccess) return e;
    const float* gnext = l + 1 < L ? c->gamma + (size_t)(l + 1) * 2 * d : c->gamma_final;
    if ((e = launch_k(decode_residual_norm_kernel, dim3(B), dim3(DEC_NORM_THREADS), 0, st, false,
                      part, sp, B, d, 1.0f, s->x, gnext, s->xn)) != cudaSuccess)
      return e;
  }
  if ((e = gemm(s->tm_xn, c->tm_embed[0], V, d, 0, 1.0f, &sp)) != cudaSuccess) return e;
  if ((e = launch_k(sp <= 4 ? decode_logits_kernel<4> : decode_logits_kernel<DEC_MAX_SPLITS>,
                    dim3(B), dim3(1024), 0, st, false, (const float*)s->part,
                    sp, B, V, softcap, s->logits, s->next)) != cudaSuccess)
    return e;
  return launch_k(decode_set_pos_kernel, dim3(1), dim3(64), 0, st, false, s->d_pos, 1,
                  (const float2*)c->rope, S, s->d_cs);
}

extern "C" {

cb_status cb_prefill(cb_ctx* ctx, const uint32_t* tokens, int32_t batch, int32_t len,
                     float softcap, float* logits_out) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  if (!ctx->weights_ready) return fail(ctx, CB_ERR_NOT_READY, "weights are not loaded");
  if (ctx->tp_world > 1)
    return fail(ctx, CB_ERR_UNSUPPORTED, "decode on a tensor-parallel context is not supported");
  const int S = ctx->cfg.seq, V = ctx->cfg.vocab;
  if (!tokens || batch <= 0 || batch > ctx->max_batch || len <= 0 || len > S)
    return fail(ctx, CB_ERR_INVALID_ARG, "bad prefill arguments");
  for (size_t i = 0; i < (size_t)batch * len; ++i)
    if (tokens[i] >= (uint32_t)V)
      return fail(ctx, CB_ERR_INVALID_ARG, "token id out of range at position " + std::to_string(i));
  CB_CUDA(cudaSetDevice(ctx->device));
  cb_status rc = alloc_decode(ctx);
  if (rc != CB_OK) return rc;
  DecodeState* s = ctx->decode;
  // prompts padded to seq (causal attention: the padding does not reach earlier positions)
  std::vector<uint32_t> padded((size_t)batch * S, 0u);
  for (int b = 0; b < batch; ++b)
    std::memcpy(&padded[(size_t)b * S], tokens + (size_t)b * len, (size_t)len * 4);
  cudaStream_t st = ctx->stream;
  CB_CUDA(cudaMemcpyAsync(ctx->tokens, padded.data(), padded.size() * 4, cudaMemcpyHostToDevice, st));
  CB_CUDA(cudaMemsetAsync(ctx->targets, 0, padded.size() * 4, st));
  KvDest kv{s->kc, s->vc, s->layer_stride};
  cudaError_t e = enqueue_forward(ctx, batch, softcap, st, false, &kv);
  if (e != cudaSuccess) return fail(ctx, CB_ERR_CUDA, std::string("prefill: ") + cudaGetErrorString(e));
  s->pos = len;
  s->batch = batch;
  s->softcap = softcap;
  CB_CUDA(cudaMemcpyAsync(s->d_pos, &s->pos, sizeof(int), cudaMemcpyHostToDevice, st));
  decode_set_pos_kernel<<<1, 64, 0, st>>>(s->d_pos, 0, ctx->rope, S, s->d_cs);
  CB_CUDA(cudaGetLastError());
  rc = read_device_error(ctx);
  if (rc != CB_OK) return rc;
  ctx->last_batch = batch;
  ctx->last_softcap = softcap;
  ctx->x_final = ctx->x;
  if (logits_out) {
    std::vector<int32_t> rows(batch);
    for (int b = 0; b < batch; ++b) rows[b] = b * S + len - 1;
    return cb_sampled_logits(ctx, rows.data(), batch, logits_out);
  }
  return CB_OK;
}

cb_status cb_decode_step(cb_ctx* ctx, const uint32_t* tokens, int32_t batch, float* logits_out,
                         uint32_t* next_out) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  DecodeState* s = ctx->decode;
  if (!s || s->batch == 0) return fail(ctx, CB_ERR_NOT_READY, "no prefill has run");
  if (!tokens || batch != s->batch)
    return fail(ctx, CB_ERR_INVALID_ARG, "decode batch must equal the prefill batch");
  if (s->pos >= ctx->cfg.seq)
    return fail(ctx, CB_ERR_INVALID_ARG, "the sequence is full (seq tokens)");
  for (int i = 0; i < batch; ++i)
    if (tokens[i] >= (uint32_t)ctx->cfg.vocab)
      return fail(ctx, CB_ERR_INVALID_ARG, "token id out of range");
  CB_CUDA(cudaSetDevice(ctx->device));
  cudaStream_t st = ctx->stream;
  CB_CUDA(cudaMemcpyAsync(s->tok, tokens, (size_t)batch * 4, cudaMemcpyHostToDevice, st));
  uint32_t sc_bits;
  std::memcpy(&sc_bits, &s->softcap, 4);
  const auto key = std::make_pair((int)batch, sc_bits);
  auto it = s->graphs.find(key);
  if (it == s->graphs.end()) {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    CB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = enqueue_decode_step(ctx, batch, s->softcap, st);
    cudaError_t e2 = cudaStreamEndCapture(st, &graph);
    if (e != cudaSuccess || e2 != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();
      return fail(ctx, CB_ERR_CUDA, std::string("decode capture: ") +
                                        cudaGetErrorString(e != cudaSuccess ? e : e2));
    }
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess)
      return fail(ctx, CB_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    it = s->graphs.emplace(key, exec).first;
  }
  CB_CUDA(cudaGraphLaunch(it->second, st));
  const size_t n_logits = (size_t)batch * ctx->cfg.vocab;
  if (logits_out)
    CB_CUDA(cudaMemcpyAsync(s->h_logits, s->logits, n_logits * 4, cudaMemcpyDeviceToHost, st));
  if (next_out)
    CB_CUDA(cudaMemcpyAsync(s->h_next, s->next, (size_t)batch * 4, cudaMemcpyDeviceToHost, st));
  cb_status rc = read_device_error(ctx);
  if (rc != CB_OK) return rc;
  s->pos += 1;
  if (logits_out) std::memcpy(logits_out, s->h_logits, n_logits * 4);
  if (next_out) std::memcpy(next_out, s->h_next, (size_t)batch * 4);
  return CB_OK;
}

cb_status cb_decode_position(const cb_ctx* ctx, int32_t* pos) {
  if (!ctx || !pos) return CB_ERR_INVALID_ARG;
  *pos = ctx->decode ? ctx->decode->pos : 0;
  return CB_OK;
}

}  // extern "C"
