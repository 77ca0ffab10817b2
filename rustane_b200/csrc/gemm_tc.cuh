// Persistent tcgen05 GEMM for sm_100a:  C[M,N] = A[M,K] * B[N,K]^T  (both K-major fp16,
// fp32 accumulation in TMEM), with the forward pass's fusions applied in the
// epilogue while the accumulator is still in registers.
//
// Roles (320 threads, one CTA per SM; the kernel body at the end of this file):
//   warp 0, lane 0 : TMA producer. 128x64 A tile + (BN or BN/2)x64 B tile per stage,
//                    128-byte swizzle, mbarrier expect-tx completion.
//   warp 1         : allocates TMEM (2 x BN columns: double-buffered
//                    accumulator); lane 0 issues tcgen05.mma (K=16 steps)
//                    and tcgen05.commit to release smem stages / hand over
//                    finished accumulators.
//   warps 2..9     : epilogue, two groups of four that take alternate tiles.
// Tiles are visited n-fastest so CTAs running at the same time share A rows
// and the weight matrix (B) stays resident in L2.
//
// Epilogues (the reference ops they replace):
//   EpiStoreF16   plain fp16 store (tests / generic use)
//   EpiStoreF32   fp32 store with optional softcap (sampled-logit dump)
//   EpiQkvRope    Q/K/V split + RoPE on interleaved pairs, head-major store
//                 (crates/engine/src/kernels/sdpa_fwd.rs:24-60,117-150,213-221)
//   EpiScaledF16  delta = alpha * acc for the residual add (layer.rs:4471, ffn_fused.rs:144-154)
//   EpiScaledF32  the same in fp32 (tensor-parallel partials before the all-reduce)
//   EpiSwiglu     g = silu(h1) * h3 from interleaved W1/W3 columns
//                 (crates/engine/src/kernels/ffn_fused.rs:79-80,105-107)
//   EpiCrossEntropy  per-(row, N-tile) running max / sum-exp and target logit
//                 of the tied LM head, so logits never reach HBM
//                 (crates/engine/src/full_model.rs:436-471, cpu/cross_entropy.rs:58-96)
//   EpiResidualNorm  x += alpha * acc in place (the fp32 residual, read by TMA two
//                 chunks ahead), fp16(x * gamma) for the next GEMM and per-row partial
//                 sums of x^2 (layer.rs:4471 vsma + the following rmsnorm)
//   RowScaled<E>  E applied to acc * rinv[row], rinv from those partial sums: the
//                 RMSNorm's 1/rms applied after the GEMM, where it commutes
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <math_constants.h>
#include <stdint.h>

#include "ptx.cuh"

namespace cb {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_EPI_WARPS = 8;
constexpr int GEMM_THREADS = 64 + 32 * GEMM_EPI_WARPS;

// PAIR: a two-CTA cluster computes a 256 x BN tile (each CTA 128 rows, half of B).
// TMA_IN: the epilogue reads a 32 x 32 fp32 box of an input matrix per chunk (two 4 KB
// slots per epilogue warp); the operand ring then has 4 stages.
template <int BN, bool PAIR = false, bool TMA_IN = false>
struct GemmCfg {
  static_assert(BN == 128 || BN == 256, "BN must be 128 or 256");
  static_assert(!PAIR || BN == 256, "CTA pairs use 256-wide tiles");
  static constexpr int TILE_M = PAIR ? 2 * GEMM_BM : GEMM_BM;
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // rows of B each CTA loads
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = B_ROWS * GEMM_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (STAGE_BYTES <= 32768 && !TMA_IN) ? 6 : 4;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int IN_SLOT_BYTES = 4096;  // 32 rows x 32 fp32, 128-byte swizzle
  static constexpr int IN_BYTES = TMA_IN ? GEMM_EPI_WARPS * 2 * IN_SLOT_BYTES : 0;
  static constexpr int BAR_BYTES = TMA_IN ? 512 : 256;
  static constexpr int EPI_BUF_BYTES = 4096;  // per epilogue warp (32 rows x 128 B)
  static constexpr int SMEM_BYTES =
      STAGES * STAGE_BYTES + IN_BYTES + 1024 + BAR_BYTES + GEMM_EPI_WARPS * EPI_BUF_BYTES;
};

// ------------------------------------------------------------------ epilogues

// Epilogue interface:
//   begin_row(row, valid)          once per tile row
//   prefetch(row, col0, Pre&)      global loads a chunk needs, issued one chunk ahead
//   chunk(row, col0, v, Pre, out, dst)
//                                  consumes 32 accumulator columns of one row and
//                                  produces OUT_BYTES bytes of output (`out`, in 16-byte
//                                  pieces) for the contiguous destination segment `dst`
//   end_row(row, n_blk)
// OUT_BYTES = 0: the epilogue writes nothing per chunk (the cross-entropy partials are
// written in end_row). The kernel stores `out` through warp_store_rows: each warp's 32
// row segments are staged in shared memory and written back so every store instruction
// covers whole 16-byte-aligned row segments, instead of one 16-byte piece of 32
// different rows (4-8x fewer L1 wavefronts).
struct NoPre {};

template <class Epi, class = void>
struct EpiAtomic { static constexpr bool value = false; };
template <class Epi>
struct EpiAtomic<Epi, decltype(void(Epi::ATOMIC))> { static constexpr bool value = Epi::ATOMIC; };

// Epilogues with set_split(k) are told which K split a work unit covers (split-K into
// separate partial buffers).
template <class Epi, class = void>
struct EpiHasSplit { static constexpr bool value = false; };
template <class Epi>
struct EpiHasSplit<Epi, decltype(void(&Epi::set_split))> { static constexpr bool value = true; };

// Epilogues with ROW_SCALE get the accumulator values multiplied by their member rs.
template <class Epi, class = void>
struct EpiRowScale { static constexpr bool value = false; };
template <class Epi>
struct EpiRowScale<Epi, decltype(void(Epi::ROW_SCALE))> { static constexpr bool value = Epi::ROW_SCALE; };

// Epilogues with TMA_IN get, per chunk, the 32 fp32 values of their row from the
// kernel's input tensor map (tmC) at the chunk's columns, and produce a second output
// (OUT2_BYTES into out2 / dst2) besides the first.
template <class Epi, class = void>
struct EpiTmaIn { static constexpr bool value = false; };
template <class Epi>
struct EpiTmaIn<Epi, decltype(void(Epi::TMA_IN))> { static constexpr bool value = Epi::TMA_IN; };

__device__ __forceinline__ uint4 pack8_f16(const float* f) {
  uint4 w;
  w.x = pack_half2(f[0], f[1]);
  w.y = pack_half2(f[2], f[3]);
  w.z = pack_half2(f[4], f[5]);
  w.w = pack_half2(f[6], f[7]);
  return w;
}

// softcap * tanh(z / softcap) over a 32-value chunk (der: 1 - tanh^2, nullable), out of
// line: tanhf inlined 32 times into the unrolled epilogues made the LM-head GEMM's code
// large enough to stall its warps on instruction fetch (ncu: "no instruction" stalls 5.8
// per issue against 0.2 in the W1/W3 GEMM, tensor pipe 45 % against 75 % active), for a
// path that is off by default. The callers copy through a local array only when softcap
// > 0, so the default path keeps its values in registers.
__device__ __noinline__ void softcap_chunk(float* z, float softcap, float* der) {
  const float inv = 1.0f / softcap;
  for (int i = 0; i < 32; ++i) {
    const float t = tanhf(z[i] * inv);
    z[i] = softcap * t;
    if (der) der[i] = 1.0f - t * t;
  }
}

// Warp-cooperative transposed store of 32 row segments of NB bytes (32, 64 or 128):
// lane L owns row L's segment (out[0 .. NB/16)) and its address; `wbuf` is this warp's
// 32*NB-byte shared buffer. Pieces are XOR-swizzled so both phases are conflict-free.
template <int NB, bool ATOMIC_ADD = false>
__device__ __forceinline__ void warp_store_rows(uint8_t* wbuf, const uint4 (&out)[8],
                                                uint8_t* dst, bool ok) {
  constexpr int Q = NB / 16;       // 16-byte pieces per row
  constexpr int RPI = 32 / Q;      // rows covered by one store instruction
  const int lane = threadIdx.x & 31;
  const int sw = (lane / (8 / Q)) & (Q - 1);
#pragma unroll
  for (int j = 0; j < Q; ++j)
    *reinterpret_cast<uint4*>(wbuf + lane * NB + ((j ^ sw) << 4)) = out[j];
  __syncwarp();
  const unsigned long long my = reinterpret_cast<unsigned long long>(ok ? dst : nullptr);
#pragma unroll
  for (int k = 0; k < Q; ++k) {
    const int r = k * RPI + lane / Q;
    const int j = lane % Q;
    const unsigned long long base = __shfl_sync(0xffffffffu, my, r);
    const int swr = (r / (8 / Q)) & (Q - 1);
    const uint4 x = *reinterpret_cast<const uint4*>(wbuf + r * NB + ((j ^ swr) << 4));
    if (base) {
      uint8_t* p = reinterpret_cast<uint8_t*>(base) + (j << 4);
      if constexpr (ATOMIC_ADD)  // four fp32 lanes added in L2 (sm_90+ vector atomic)
        atomicAdd(reinterpret_cast<float4*>(p), *reinterpret_cast<const float4*>(&x));
      else
        *reinterpret_cast<uint4*>(p) = x;
    }
  }
  __syncwarp();
}

// The inverse of warp_store_rows, in two halves so that one chunk's loads are in flight
// while the previous chunk is processed. warp_issue_rows: the warp's loads, coalesced
// over whole row segments, into registers (src = nullptr: zeros); warp_finish_rows:
// those pieces transposed through the warp's shared buffer, so that lane L receives the
// NB-byte segment of row L in in[0 .. NB/16).
template <int NB>
__device__ __forceinline__ void warp_issue_rows(const uint8_t* src, uint4 (&x)[NB / 16]) {
  constexpr int Q = NB / 16;
  constexpr int RPI = 32 / Q;
  const int lane = threadIdx.x & 31;
  const unsigned long long my = reinterpret_cast<unsigned long long>(src);
#pragma unroll
  for (int k = 0; k < Q; ++k) {
    const int r = k * RPI + lane / Q;
    const int j = lane % Q;
    const unsigned long long base = __shfl_sync(0xffffffffu, my, r);
    x[k] = make_uint4(0u, 0u, 0u, 0u);
    if (base) x[k] = __ldg(reinterpret_cast<const uint4*>(base) + j);
  }
}

template <int NB>
__device__ __forceinline__ void warp_finish_rows(uint8_t* wbuf, const uint4 (&x)[NB / 16],
                                                 uint4 (&in)[8]) {
  constexpr int Q = NB / 16;
  constexpr int RPI = 32 / Q;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < Q; ++k) {
    const int r = k * RPI + lane / Q;
    const int j = lane % Q;
    const int swr = (r / (8 / Q)) & (Q - 1);
    *reinterpret_cast<uint4*>(wbuf + r * NB + ((j ^ swr) << 4)) = x[k];
  }
  __syncwarp();
  const int sw = (lane / (8 / Q)) & (Q - 1);
#pragma unroll
  for (int j = 0; j < Q; ++j) in[j] = *reinterpret_cast<const uint4*>(wbuf + lane * NB + ((j ^ sw) << 4));
  __syncwarp();
}

// Epilogues with IN_BYTES > 0 read a row segment per chunk: the kernel loads it (from
// in_src(row, col)) one chunk ahead with warp_issue_rows and hands it to chunk() in the
// chunk's output array.
template <class Epi, class = void>
struct EpiInBytes { static constexpr int value = 0; };
template <class Epi>
struct EpiInBytes<Epi, decltype(void(Epi::IN_BYTES))> { static constexpr int value = Epi::IN_BYTES; };

struct EpiStoreF16 {
  using Pre = NoPre;
  static constexpr int OUT_BYTES = 64;
  __half* out;
  int ldo;
  __device__ __forceinline__ void begin_row(int, bool) {}
  __device__ __forceinline__ void prefetch(int, int, Pre&) {}
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre&,
                                        uint4 (&o)[8], uint8_t*& dst) {
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = pack8_f16(v + 8 * j);
    dst = reinterpret_cast<uint8_t*>(out + (size_t)row * ldo + col0);
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

// fp16 store of the attention-output gradient dA (token-major [T, heads*128]) that also
// yields the attention backward's D[b, h, q] = sum_d dA[t, h*128+d] * O[t, h*128+d]
// (t = b*seq + q): each thread owns one row, its four 32-column chunks of a head arrive
// in order, and the dot product is taken over the fp16-rounded dA values the attention
// kernel will read. O's row segment is the chunk input (IN_BYTES). Column tiles start on
// head boundaries (BN = 256).
struct EpiStoreF16Dsum {
  using Pre = NoPre;
  static constexpr int OUT_BYTES = 64;
  static constexpr int IN_BYTES = 64;
  __half* out;
  int ldo;
  const __half* o;  // attention output, same layout as out
  float* dsum;      // [batch, heads, seq]
  int seq, heads;
  float acc;
  __device__ __forceinline__ const uint8_t* in_src(int row, int col0) const {
    return reinterpret_cast<const uint8_t*>(o + (size_t)row * ldo + col0);
  }
  __device__ __forceinline__ void begin_row(int, bool) { acc = 0.f; }
  __device__ __forceinline__ void prefetch(int, int, Pre&) {}
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre&,
                                        uint4 (&io)[8], uint8_t*& dst) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 ov = io[j];
      const uint4 gv = pack8_f16(v + 8 * j);
      const __half2* oh = reinterpret_cast<const __half2*>(&ov);
      const __half2* gh = reinterpret_cast<const __half2*>(&gv);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 a = __half22float2(oh[k]), g = __half22float2(gh[k]);
        acc = fmaf(a.x, g.x, fmaf(a.y, g.y, acc));
      }
      io[j] = gv;
    }
    if ((col0 & 127) == 96) {  // last chunk of head col0 / 128
      const int b = row / seq, q = row - b * seq;
      dsum[((size_t)b * heads + (col0 >> 7)) * seq + q] = acc;
      acc = 0.f;
    }
    dst = reinterpret_cast<uint8_t*>(out + (size_t)row * ldo + col0);
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

struct EpiStoreF32 {
  using Pre = NoPre;
  static constexpr int OUT_BYTES = 128;
  float* out;
  int ldo;
  float softcap;  // > 0: out = softcap * tanh(acc / softcap)
  __device__ __forceinline__ void begin_row(int, bool) {}
  __device__ __forceinline__ void prefetch(int, int, Pre&) {}
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre&,
                                        uint4 (&o)[8], uint8_t*& dst) {
    float z[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) z[i] = v[i];
    if (softcap > 0.f) {
      float t[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) t[i] = z[i];
      softcap_chunk(t, softcap, nullptr);
#pragma unroll
      for (int i = 0; i < 32; ++i) z[i] = t[i];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      o[j] = make_uint4(__float_as_uint(z[4 * j]), __float_as_uint(z[4 * j + 1]),
                        __float_as_uint(z[4 * j + 2]), __float_as_uint(z[4 * j + 3]));
    dst = reinterpret_cast<uint8_t*>(out + (size_t)row * ldo + col0);
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

// Columns [0, q_dim) -> Q, [q_dim, q_dim+kv_dim) -> K, rest -> V. Head dim 128.
// Output layout [batch, heads, seq, 128] (row = b*seq + s). RoPE on Q and K rotates
// pairs (2i, 2i+1) by theta = s * 10000^(-2i/128); the (cos, sin) table is
// pair-major [64][seq] so the lanes of a warp (consecutive positions) read it contiguously.
struct EpiQkvRope {
  struct Pre {
    float2 cs[16];  // (cos, sin) of the chunk's 16 frequency pairs
  };
  static constexpr int OUT_BYTES = 64;
  __half* q;
  __half* k;
  __half* v;
  const float2* rope;  // [64][seq]
  int seq;
  int heads;
  int kv_heads;
  __device__ __forceinline__ void begin_row(int, bool) {}
  __device__ __forceinline__ void prefetch(int row, int col0, Pre& p) {
    if (col0 >= (heads + kv_heads) * 128) return;  // V columns are not rotated
    const int s = row % seq;
    const float2* rs = rope + (size_t)((col0 & 127) >> 1) * seq + s;
#pragma unroll
    for (int i = 0; i < 16; ++i) p.cs[i] = __ldg(rs + (size_t)i * seq);
  }
  __device__ __forceinline__ void chunk(int row, int col0, const float (&acc)[32], const Pre& p,
                                        uint4 (&o)[8], uint8_t*& dst) {
    const int q_dim = heads * 128;
    const int kv_dim = kv_heads * 128;
    const int b = row / seq;
    const int s = row - b * seq;
    __half* base;
    int c = col0;
    bool rot = true;
    int nh;
    if (c < q_dim) {
      base = q;
      nh = heads;
    } else if (c < q_dim + kv_dim) {
      base = k;
      c -= q_dim;
      nh = kv_heads;
    } else {
      base = v;
      c -= q_dim + kv_dim;
      nh = kv_heads;
      rot = false;
    }
    const int h = c >> 7;
    const int d0 = c & 127;
    float r[32];
    if (rot) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float a = acc[2 * i], bb = acc[2 * i + 1];
        r[2 * i] = a * p.cs[i].x - bb * p.cs[i].y;
        r[2 * i + 1] = bb * p.cs[i].x + a * p.cs[i].y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = acc[i];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = pack8_f16(r + 8 * j);
    dst = reinterpret_cast<uint8_t*>(base + (((size_t)b * nh + h) * seq + s) * 128 + d0);
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

// delta[row, col] = fp16(alpha * acc): the O-proj / down-proj output handed to the
// next add_rmsnorm kernel, which adds it to the fp32 residual stream. Write-only, so
// the epilogue never waits on global loads.
struct EpiScaledF16 {
  using Pre = NoPre;
  static constexpr int OUT_BYTES = 64;
  __half* out;
  int ldo;
  float alpha;
  __device__ __forceinline__ void begin_row(int, bool) {}
  __device__ __forceinline__ void prefetch(int, int, Pre&) {}
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre&,
                                        uint4 (&o)[8], uint8_t*& dst) {
    float r[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = alpha * v[i];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = pack8_f16(r + 8 * j);
    dst = reinterpret_cast<uint8_t*>(out + (size_t)row * ldo + col0);
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

// delta[row, col] = alpha * acc in fp32: the tensor-parallel partial O / down
// projection that is all-reduced across ranks before the residual add.
struct EpiScaledF32 {
  using Pre = NoPre;
  static constexpr int OUT_BYTES = 128;
  float* out;
  int ldo;
  float alpha;
  __device__ __forceinline__ void begin_row(int, bool) {}
  __device__ __forceinline__ void prefetch(int, int, Pre&) {}
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre&,
                                        uint4 (&o)[8], uint8_t*& dst) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 w = make_float4(alpha * v[4 * j], alpha * v[4 * j + 1], alpha * v[4 * j + 2],
                                   alpha * v[4 * j + 3]);
      o[j] = *reinterpret_cast<const uint4*>(&w);
    }
    dst = reinterpret_cast<uint8_t*>(out + (size_t)row * ldo + col0);
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

// delta[row, col] += alpha * acc (fp32 vector atomics into a zeroed buffer): the
// split-K form of the O / down projection, used when the tile count alone fills the
// GPU poorly. Exactly two K halves add onto zero, so the sum is order-independent.
struct EpiScaledF32Add {
  using Pre = NoPre;
  static constexpr int OUT_BYTES = 128;
  static constexpr bool ATOMIC = true;
  float* out;
  int ldo;
  float alpha;
  __device__ __forceinline__ void begin_row(int, bool) {}
  __device__ __forceinline__ void prefetch(int, int, Pre&) {}
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre&,
                                        uint4 (&o)[8], uint8_t*& dst) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 w = make_float4(alpha * v[4 * j], alpha * v[4 * j + 1], alpha * v[4 * j + 2],
                                   alpha * v[4 * j + 3]);
      o[j] = *reinterpret_cast<const uint4*>(&w);
    }
    dst = reinterpret_cast<uint8_t*>(out + (size_t)row * ldo + col0);
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

// B rows interleave W1 and W3 columns: row 2j = W1[:, j], row 2j+1 = W3[:, j].
// g[row, j] = silu(h1_j) * h3_j, silu(z) = z / (1 + e^-z). The quotient uses the
// approximate divide (reciprocal + multiply, 2 ulp; 0 once 1 + e^-z passes 2^126, the
// limit of silu there) for a result rounded to fp16: with the IEEE divide the SwiGLU
// epilogues kept the special-function (XU) pipe ~70 % busy (ncu) and the W1/W3 GEMM
// ran 10 % slower.
struct EpiSwiglu {
  using Pre = NoPre;
  static constexpr int OUT_BYTES = 32;
  __half* g;
  int ldg;
  __device__ __forceinline__ void begin_row(int, bool) {}
  __device__ __forceinline__ void prefetch(int, int, Pre&) {}
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre&,
                                        uint4 (&o)[8], uint8_t*& dst) {
    float r[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float h1 = v[2 * j], h3 = v[2 * j + 1];
      r[j] = __fdividef(h1, 1.0f + __expf(-h1)) * h3;
    }
    o[0] = pack8_f16(r);
    o[1] = pack8_f16(r + 8);
    dst = reinterpret_cast<uint8_t*>(g + (size_t)row * ldg + (col0 >> 1));
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

// Training forward of W1/W3: g as EpiSwiglu, and the pre-activations (h1, h3
// interleaved, as the accumulator holds them) saved in fp16 for the backward pass.
struct EpiSwigluSave {
  using Pre = NoPre;
  static constexpr int OUT_BYTES = 32;
  __half* g;
  int ldg;
  __half* h13;
  int ldh;
  __device__ __forceinline__ void begin_row(int, bool) {}
  __device__ __forceinline__ void prefetch(int, int, Pre&) {}
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre&,
                                        uint4 (&o)[8], uint8_t*& dst) {
    float r[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float h1 = v[2 * j], h3 = v[2 * j + 1];
      r[j] = __fdividef(h1, 1.0f + __expf(-h1)) * h3;
    }
    uint4* hs = reinterpret_cast<uint4*>(h13 + (size_t)row * ldh + col0);
#pragma unroll
    for (int j = 0; j < 4; ++j) hs[j] = pack8_f16(v + 8 * j);
    o[0] = pack8_f16(r);
    o[1] = pack8_f16(r + 8);
    dst = reinterpret_cast<uint8_t*>(g + (size_t)row * ldg + (col0 >> 1));
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

// Backward of the SwiGLU gate, fused into dG = (alpha dY) W2 (layer.rs:6760-6771):
// for hidden column j, sig = 1/(1 + e^-h1), dh3 = dG h1 sig, dh1 = dG h3 sig (1 +
// h1 (1 - sig)). Writes dh1, dh3 interleaved like the W1/W3 storage rows, the layout
// the next GEMMs (dX = dH13 W13, dW13 = dH13^T X2n) read. The row's saved (h1, h3)
// pairs of the chunk (128 B) arrive in o[] (IN_BYTES: loaded by the kernel, coalesced).
struct EpiSwigluBwd {
  using Pre = NoPre;
  static constexpr int OUT_BYTES = 128;
  static constexpr int IN_BYTES = 128;
  __half* dh13;
  const __half* h13;
  int ld;  // 2 * hidden
  __device__ __forceinline__ const uint8_t* in_src(int row, int col0) const {
    return reinterpret_cast<const uint8_t*>(h13 + (size_t)row * ld + 2 * col0);
  }
  __device__ __forceinline__ void begin_row(int, bool) {}
  __device__ __forceinline__ void prefetch(int, int, Pre&) {}
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre&,
                                        uint4 (&o)[8], uint8_t*& dst) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 hv = o[i];
      const __half2* hh = reinterpret_cast<const __half2*>(&hv);
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 h = __half22float2(hh[k]);  // (h1, h3) of column 4i + k
        const float dg = v[4 * i + k];
        const float sig = __fdividef(1.0f, 1.0f + __expf(-h.x));
        const float dh3 = dg * h.x * sig;
        const float dh1 = dg * h.y * sig * (1.0f + h.x * (1.0f - sig));
        w[k] = pack_half2(dh1, dh3);
      }
      o[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    dst = reinterpret_cast<uint8_t*>(dh13 + (size_t)row * ld + 2 * col0);
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

// Gradient of the loss w.r.t. the logits, recomputed from the saved per-token
// log-sum-exp (tok_loss + target logit): dl = softmax(z) - onehot(target), times the
// softcap derivative 1 - tanh^2 when softcap > 0 (cross_entropy.rs:58-96,
// full_model.rs:600-611). fp16 output, unscaled (the 1/seq and loss scale are applied
// by the GEMMs that consume it, where the values are fp32).
struct EpiCeBwd {
  using Pre = NoPre;
  static constexpr int OUT_BYTES = 64;
  __half* dl;
  int ldo;
  const uint32_t* targets;
  const float* tok_loss;
  const float* tgt_logit;
  float softcap;
  float lse;
  int tgt;
  __device__ __forceinline__ void begin_row(int row, bool valid) {
    tgt = valid ? (int)targets[row] : -1;
    lse = valid ? tok_loss[row] + tgt_logit[row] : 0.f;
  }
  __device__ __forceinline__ void prefetch(int, int, Pre&) {}
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre&,
                                        uint4 (&o)[8], uint8_t*& dst) {
    float z[32], der[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      z[i] = v[i];
      der[i] = 1.0f;
    }
    if (softcap > 0.f) {
      float t[32], dt[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) t[i] = z[i];
      softcap_chunk(t, softcap, dt);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        z[i] = t[i];
        der[i] = dt[i];
      }
    }
    float r[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float g = __expf(z[i] - lse);
      if (col0 + i == tgt) g -= 1.0f;
      r[i] = g * der[i];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = pack8_f16(r + 8 * j);
    dst = reinterpret_cast<uint8_t*>(dl + (size_t)row * ldo + col0);
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

// alpha * acc into slice `split` of a [splits][M][ldo] fp32 partial buffer: split-K of
// the weight-gradient GEMMs (K = tokens), reduced afterwards in a fixed order.
struct EpiPartialF32 {
  using Pre = NoPre;
  static constexpr int OUT_BYTES = 128;
  float* out;
  int ldo;
  float alpha;
  size_t split_stride;
  __device__ __forceinline__ void set_split(int s) { out += (size_t)s * split_stride; }
  __device__ __forceinline__ void begin_row(int, bool) {}
  __device__ __forceinline__ void prefetch(int, int, Pre&) {}
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre&,
                                        uint4 (&o)[8], uint8_t*& dst) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 w = make_float4(alpha * v[4 * j], alpha * v[4 * j + 1], alpha * v[4 * j + 2],
                                   alpha * v[4 * j + 3]);
      o[j] = *reinterpret_cast<const uint4*>(&w);
    }
    dst = reinterpret_cast<uint8_t*>(out + (size_t)row * ldo + col0);
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

// Fused LM head + cross-entropy partials. For each row and N-tile writes
// (max_z, sum exp(z - max_z)) over the tile's logits z (softcapped if
// softcap > 0) and, for the tile holding targets[row], that logit.
struct EpiCrossEntropy {
  using Pre = NoPre;
  static constexpr int OUT_BYTES = 0;
  float2* part;      // [M, nparts]
  int nparts;
  const uint32_t* targets;
  float* tgt_logit;  // [M]
  float softcap;
  // per-thread running state
  float m, s;
  int tgt;
  __device__ __forceinline__ void begin_row(int row, bool valid) {
    m = -CUDART_INF_F;
    s = 0.f;
    tgt = valid ? (int)targets[row] : -1;
  }
  __device__ __forceinline__ void prefetch(int, int, Pre&) {}
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre&,
                                        uint4 (&)[8], uint8_t*&) {
    float z[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) z[i] = v[i];
    if (softcap > 0.f) {
      float t[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) t[i] = z[i];
      softcap_chunk(t, softcap, nullptr);
#pragma unroll
      for (int i = 0; i < 32; ++i) z[i] = t[i];
    }
    float cm = -CUDART_INF_F;
#pragma unroll
    for (int i = 0; i < 32; ++i) cm = fmaxf(cm, z[i]);
    const unsigned rel = (unsigned)(tgt - col0);
    if (rel < 32u) {
      float zt = z[0];
#pragma unroll
      for (int i = 1; i < 32; ++i) zt = (rel == (unsigned)i) ? z[i] : zt;
      tgt_logit[row] = zt;
    }
    const float L2E = 1.4426950408889634f;
    if (cm > m) {
      s *= exp2_mufu((m - cm) * L2E);
      m = cm;
    }
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) acc += exp2_mufu((z[i] - m) * L2E);
    s += acc;
  }
  __device__ __forceinline__ void end_row(int row, int n_blk) {
    part[(size_t)row * nparts + n_blk] = make_float2(m, s);
  }
};

// Residual update + the first half of the next RMSNorm, fused into the O and down
// projections: x = x + alpha * acc (fp32, in place), xh = fp16(x * gamma) as the next
// GEMM's A operand, and per row the sum of x^2 over each 128-column group into
// ss_part[row][col / 128] (fixed-order partials: the consumer adds them in order, so the
// loss stays bit-reproducible). The 1/rms factor is applied by the consumer GEMM
// (RowScaled), since rmsnorm(x) W^T = rinv * ((x o gamma) W^T).
// Data movement is all TMA (TMA_IN): the kernel loads each 32 x 32 box of the old x into
// shared memory two chunks ahead (tmC), chunk_tma overwrites it in place with the new x
// and writes fp16(x * gamma) into a 32 x 32 staging box, and the kernel stores both
// boxes with TMA (tmC, tmD).
struct EpiResidualNorm {
  struct Pre {
    float4 g[8];  // gamma of the chunk's 32 columns, loaded one chunk ahead
  };
  static constexpr bool TMA_IN = true;
  static constexpr int OUT_BYTES = 0;
  const float* gamma;
  float* ss_part;
  int n_part;  // d / 128
  float alpha;
  float ss;
  __device__ __forceinline__ void begin_row(int, bool) { ss = 0.f; }
  __device__ __forceinline__ void prefetch(int, int col0, Pre& p) {
    const float4* g4 = reinterpret_cast<const float4*>(gamma + col0);  // same for all lanes
#pragma unroll
    for (int j = 0; j < 8; ++j) p.g[j] = __ldg(g4 + j);
  }
  // xrow: this row's 128 bytes of x in the 128-byte-swizzled box (16-byte piece k at
  // xrow + ((k ^ sw128) << 4)); hrow: its 64 bytes in the 64-byte-swizzled fp16 box
  // (piece k at hrow + ((k ^ sw64) << 4)).
  __device__ __forceinline__ void chunk_tma(int row, int col0, const float (&v)[32],
                                            const Pre& p, uint8_t* xrow, int sw128,
                                            uint8_t* hrow, int sw64) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
    float4 a[8];  // loads of a half first: the in-place stores would otherwise order them
#pragma unroll
    for (int j = 4 * hh; j < 4 * hh + 4; ++j)
      a[j] = *reinterpret_cast<const float4*>(xrow + ((j ^ sw128) << 4));
#pragma unroll
    for (int j = 4 * hh; j < 4 * hh + 4; ++j) {
      const float4 g = p.g[j];
      float4 n;
      n.x = fmaf(alpha, v[4 * j], a[j].x);
      n.y = fmaf(alpha, v[4 * j + 1], a[j].y);
      n.z = fmaf(alpha, v[4 * j + 2], a[j].z);
      n.w = fmaf(alpha, v[4 * j + 3], a[j].w);
      *reinterpret_cast<float4*>(xrow + ((j ^ sw128) << 4)) = n;
      ss = fmaf(n.x, n.x, fmaf(n.y, n.y, fmaf(n.z, n.z, fmaf(n.w, n.w, ss))));
      const uint2 h = make_uint2(pack_half2(n.x * g.x, n.y * g.y), pack_half2(n.z * g.z, n.w * g.w));
      *reinterpret_cast<uint2*>(hrow + (((j >> 1) ^ sw64) << 4) + (j & 1) * 8) = h;
    }
    }
    if ((col0 & 127) == 96) {  // last chunk of a 128-column group
      ss_part[(size_t)row * n_part + (col0 >> 7)] = ss;
      ss = 0.f;
    }
  }
  __device__ __forceinline__ void end_row(int, int) {}
};

// The inner epilogue applied to acc * rinv[row], rinv = 1 / sqrt(sum(ss_part[row]) / d +
// eps) from the partial sums EpiResidualNorm wrote (the RMSNorm of the row whose fp16
// x * gamma is this GEMM's A operand).
// (The kernel multiplies the accumulator values by rs as it reads them: ROW_SCALE.)
template <class Inner>
struct RowScaled {
  using Pre = typename Inner::Pre;
  static constexpr int OUT_BYTES = Inner::OUT_BYTES;
  static constexpr bool ROW_SCALE = true;
  Inner in;
  const float* ss_part;
  int n_part;
  float dim;  // the row length d
  float eps;
  float rs;
  __device__ __forceinline__ void begin_row(int row, bool valid) {
    rs = 1.f;
    if (valid) {
      const float* p = ss_part + (size_t)row * n_part;
      float t = 0.f;
      if ((n_part & 3) == 0 && n_part <= 16) {  // up to 4 independent 16-byte loads, summed in order
        float4 q[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (4 * i < n_part) q[i] = __ldg(reinterpret_cast<const float4*>(p) + i);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (4 * i < n_part) t = (((t + q[i].x) + q[i].y) + q[i].z) + q[i].w;
      } else {
        for (int i = 0; i < n_part; ++i) t += p[i];
      }
      rs = 1.0f / sqrtf(t / dim + eps);
    }
    in.begin_row(row, valid);
  }
  __device__ __forceinline__ void prefetch(int row, int col0, Pre& p) { in.prefetch(row, col0, p); }
  __device__ __forceinline__ void chunk(int row, int col0, const float (&v)[32], const Pre& p,
                                        uint4 (&o)[8], uint8_t*& dst) {
    in.chunk(row, col0, v, p, o, dst);  // v already scaled by rs
  }
  __device__ __forceinline__ void end_row(int row, int n_blk) { in.end_row(row, n_blk); }
};

// Split-K with a last-arrival reduction, for the fused epilogues that need whole sums
// (residual + norm, RoPE, SwiGLU, cross-entropy) when a GEMM has too few tiles to fill
// the GPU. Work unit = (tile, K split). Every unit writes its fp32 partial accumulator to
// `ws` (slab [tile][rank][split], laid out [chunk][float4 column group][row] so that each
// warp store and load covers 512 contiguous bytes), then adds 1 to the tile's counter in
// `cnt`. The unit that brings the counter to `splits` adds the partials in split order
// (0, 1, ..., its own taken from TMEM) and runs the epilogue; it also resets the counter
// for the next launch. No unit ever waits for another, and the summation order is fixed,
// so results are bit-reproducible. ws = nullptr: plain (unsplit or accumulating) units.
struct SplitFix {
  float4* ws;
  int* cnt;
};

// Split-K helpers (only the FIX instantiations of the kernel contain them).
// splitfix_write: the thread's row of the first n_chunks 32-column chunks of the TMEM
// accumulator at t_row into its slab (dst = slab + row; float4 group j of chunk c at
// dst[(c * 8 + j) * 128]). Rows past M (row_ok false) take part in the warp's TMEM loads
// but store nothing: their sums are never used.
__device__ __forceinline__ void splitfix_write(uint32_t t_row, int n_chunks, float4* dst,
                                               bool row_ok) {
#pragma unroll 1
  for (int c = 0; c < n_chunks; ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + c * 32, r);
    tmem_ld_wait_regs(r);
    if (row_ok) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        __stcg(dst + ((size_t)c * 8 + j) * 128,
               make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                           __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
    }
  }
}

// splitfix_reduce: the accumulator's first n_chunks chunks replaced by the sum of all
// splits' partials in split order (slab s at slab0 + s * slab_f4 float4s; this unit's own,
// my_split, read from TMEM), in 16-column halves. The other splits' pieces of a half are
// loaded in batches of FIX_BATCH splits, all loads of a batch in flight before its adds
// (one L2 round trip per batch and half, not one per split: with one split's loads in
// flight the reduction ran at a few GB/s per CTA). Rows past M (row_ok false) load nothing.
constexpr int FIX_BATCH = 4;
__device__ __forceinline__ void splitfix_reduce(uint32_t t_row, int n_chunks, const float4* slab0,
                                             int slab_f4, int splits, int my_split, int rr,
                                             bool row_ok) {
#pragma unroll 1
  for (int h = 0; h < 2 * n_chunks; ++h) {
    const int c = h >> 1;
    uint32_t r[16];
    tmem_ld_32x32b_x16(t_row + h * 16, r);
    const float4* base = slab0 + ((size_t)c * 8 + (h & 1) * 4) * 128 + rr;
    float acc[16];
#pragma unroll 1
    for (int sp0 = 0; sp0 < splits; sp0 += FIX_BATCH) {
      float4 buf[FIX_BATCH][4];
#pragma unroll
      for (int i = 0; i < FIX_BATCH; ++i) {
        const int sp = sp0 + i;
        const bool ld = row_ok && sp < splits && sp != my_split;
        const float4* src = base + (size_t)sp * slab_f4;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          buf[i][j] = ld ? __ldcg(src + j * 128) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      if (sp0 == 0) tmem_ld_wait_regs16(r);
#pragma unroll
      for (int i = 0; i < FIX_BATCH; ++i) {
        const int sp = sp0 + i;
        if (sp >= splits) break;
        float t[16];
        if (sp == my_split) {
#pragma unroll
          for (int q = 0; q < 16; ++q) t[q] = __uint_as_float(r[q]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            t[4 * j] = buf[i][j].x;
            t[4 * j + 1] = buf[i][j].y;
            t[4 * j + 2] = buf[i][j].z;
            t[4 * j + 3] = buf[i][j].w;
          }
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) acc[q] = (sp == 0) ? t[q] : acc[q] + t[q];
      }
    }
#pragma unroll
    for (int q = 0; q < 16; ++q) r[q] = __float_as_uint(acc[q]);
    tmem_st_32x32b_x16(t_row + h * 16, r);
  }
}

template <class Epi>
struct EpiCanFix {
  static constexpr bool value =
      !EpiAtomic<Epi>::value && !EpiHasSplit<Epi>::value && EpiInBytes<Epi>::value == 0;
};

// ------------------------------------------------------------------ kernel
//
// One body, two modes:
//   PAIR = false : one CTA computes a 128 x BN tile (tcgen05.mma.cta_group::1, M = 128).
//   PAIR = true  : a cluster of two CTAs computes a 256 x 256 tile with
//                  tcgen05.mma.cta_group::2 (M = 256) issued by the even CTA. Each CTA
//                  loads its own 128 rows of A and its own 128 rows of B (no multicast);
//                  both loads count on the even CTA's `full` barrier; the even CTA's
//                  commits release both CTAs' stages and accumulators (multicast commit).
//                  Per SM this moves 32 KB of operands per 4.2 MFLOP instead of 48 KB.
// Epilogue: warps 2..9 form two groups of four; group g drains accumulator buffer g,
// so consecutive tiles' epilogues overlap. In each group warp w reads TMEM lanes
// 32*(w%4)..+31: one thread per output row, BN columns in chunks of 32, the next
// chunk's TMEM load in flight while the current one is processed.

// Operand layouts (the LAYOUT template argument): bit 0 set = A is MN-major (stored
// [K][M], M contiguous: A = X^T of a row-major X), bit 1 = B is MN-major ([K][N]).
// Backward GEMMs use them: dX = dY * W reads W as stored (B MN-major) and
// dW = dY^T * X reads both activations as stored (A and B MN-major).
// An MN-major operand is loaded as 64 (MN) x 64 (K) boxes, 8 KB each, laid side by
// side along MN; its UMMA descriptor uses LBO = 8 KB between MN blocks and SBO =
// 1 KB between 8-row K groups, and each K = 16 step advances 2 KB.
constexpr int GEMM_A_MN = 1;
constexpr int GEMM_B_MN = 2;
constexpr int MN_BOX_BYTES = 64 * 64 * 2;

template <int BN, bool PAIR, class Epi, int LAYOUT = 0, bool FIX = false>
__device__ __forceinline__ void gemm_tn_body(const CUtensorMap* tmA, const CUtensorMap* tmB,
                                             const CUtensorMap* tmC, const CUtensorMap* tmD,
                                             int M, int N, int K, int b_z, int splits,
                                             const Epi& epi, SplitFix fix, int* err) {
  constexpr bool TIN = EpiTmaIn<Epi>::value;
  using Cfg = GemmCfg<BN, PAIR, TIN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int TILE_M = Cfg::TILE_M;
  constexpr int NC = BN / 32;  // TMEM chunks per row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* in_slots = smem + STAGES * Cfg::STAGE_BYTES;  // TMA_IN boxes (1024-aligned)
  uint8_t* bar_base = in_slots + Cfg::IN_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_base);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  static_assert((2 * STAGES + 5) * 8 + 4 <= 160, "barriers overlap the split-K flags");
  uint64_t* in_bar = reinterpret_cast<uint64_t*>(bar_base + 256);  // TMA_IN: 2 per epilogue warp
  uint8_t* epi_bufs = bar_base + Cfg::BAR_BYTES;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int n_units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int m_tiles = (M + TILE_M - 1) / TILE_M;
  const int n_tiles = (N + BN - 1) / BN;
  // Work unit = (tile, K split): unit u covers tile u / splits and k-blocks
  // [split * kb_per, ...) of it. splits > 1 only with an accumulating, partial-buffer or
  // SplitFix epilogue; the host keeps splits <= ceil(kb / kb_per), so no unit is empty.
  const int num_tiles = m_tiles * n_tiles * splits;
  const int kb_total = (K + GEMM_BK - 1) / GEMM_BK;
  const int kb_per = (kb_total + splits - 1) / splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], (PAIR ? 2 : 1) * 4);
    }
    mbar_init(drain, 1);
    if constexpr (FIX) {  // split-K hand-offs of the two epilogue groups
      uint64_t* fb = reinterpret_cast<uint64_t*>(bar_base + 176);
      mbar_init(&fb[0], 4);
      mbar_init(&fb[1], 4);
      mbar_init(&fb[2], 1);
      mbar_init(&fb[3], 1);
    }
    if constexpr (TIN) {
      for (int i = 0; i < 2 * GEMM_EPI_WARPS; ++i) mbar_init(&in_bar[i], 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(tmA);
    tma_prefetch_desc(tmB);
    if constexpr (TIN) {
      tma_prefetch_desc(tmC);
      tma_prefetch_desc(tmD);
    }
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_enter();  // the setup above overlaps the previous kernel under PDL

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs of a pair)
      // Both operands are re-read by other tiles (A by every n-tile of its row block, B
      // by every m-block): keep both in L2. Evict-first on A let the streaming outputs
      // push A out before its last n-tile (A read ~2.2x from DRAM, 1.6 % slower).
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = policy_evict_last();
      uint32_t it = 0;
      bool ok = true;
      for (int u = unit; u < num_tiles && ok; u += n_units) {
        const int tile = u / splits;
        const int kb0 = (u % splits) * kb_per;
        const int kb1 = min(kb0 + kb_per, kb_total);
        const int m0 = (tile / n_tiles) * TILE_M + (int)rank * GEMM_BM;
        const int n0 = (tile % n_tiles) * BN + (int)rank * Cfg::B_ROWS;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, err)) { ok = false; break; }
          uint8_t* a_dst = sA + s * Cfg::A_BYTES;
          uint8_t* b_dst = sB + s * Cfg::B_BYTES;
          const int k0 = kb * GEMM_BK;
          if (PAIR) {
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * Cfg::STAGE_BYTES);
            const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
            if constexpr (LAYOUT & GEMM_A_MN) {
#pragma unroll
              for (int j = 0; j < GEMM_BM / 64; ++j)
                tma_load_3d_pair(a_dst + j * MN_BOX_BYTES, tmA, bar, m0 + 64 * j, k0, 0, pol_a);
            } else {
              tma_load_3d_pair(a_dst, tmA, bar, k0, m0, 0, pol_a);
            }
            if constexpr (LAYOUT & GEMM_B_MN) {
#pragma unroll
              for (int j = 0; j < Cfg::B_ROWS / 64; ++j)
                tma_load_3d_pair(b_dst + j * MN_BOX_BYTES, tmB, bar, n0 + 64 * j, k0, b_z, pol_b);
            } else {
              tma_load_3d_pair(b_dst, tmB, bar, k0, n0, b_z, pol_b);
            }
          } else {
            mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
            if constexpr (LAYOUT & GEMM_A_MN) {
#pragma unroll
              for (int j = 0; j < GEMM_BM / 64; ++j)
                tma_load_3d(a_dst + j * MN_BOX_BYTES, tmA, &full[s], m0 + 64 * j, k0, 0, pol_a);
            } else {
              tma_load_3d(a_dst, tmA, &full[s], k0, m0, 0, pol_a);
            }
            if constexpr (LAYOUT & GEMM_B_MN) {
#pragma unroll
              for (int j = 0; j < Cfg::B_ROWS / 64; ++j)
                tma_load_3d(b_dst + j * MN_BOX_BYTES, tmB, &full[s], n0 + 64 * j, k0, b_z, pol_b);
            } else {
              tma_load_3d(b_dst, tmB, &full[s], k0, n0, b_z, pol_b);
            }
          }
        }
      }
      // Drain: wait (bounded) for copies still in flight. The even CTA's full
      // barriers count both CTAs' bytes, so it drains for the pair.
      if (rank == 0) {
        uint32_t first = it > (uint32_t)STAGES ? it - STAGES : 0u;
        for (uint32_t j = first; j < it; ++j)
          mbar_wait(&full[j % STAGES], (j / STAGES) & 1u, err);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (the even CTA of a pair)
      constexpr uint32_t idesc = umma_idesc_f16(TILE_M, BN) |
                                 ((LAYOUT & GEMM_A_MN) ? (1u << 15) : 0u) |
                                 ((LAYOUT & GEMM_B_MN) ? (1u << 16) : 0u);
      uint32_t it = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      bool ok = true;
      for (int u = unit; u < num_tiles && ok; u += n_units) {
        const int kb0 = (u % splits) * kb_per;
        const int kb1 = min(kb0 + kb_per, kb_total);
        if (!mbar_wait(&tempty[acc], acc_ph ^ 1u, err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&full[s], ph, err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * Cfg::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + s * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k) {
            const uint64_t ad = (LAYOUT & GEMM_A_MN)
                                    ? sw128_mnmajor_desc(a_addr + k * 2048, MN_BOX_BYTES)
                                    : sw128_kmajor_desc(a_addr + k * 32);
            const uint64_t bd = (LAYOUT & GEMM_B_MN)
                                    ? sw128_mnmajor_desc(b_addr + k * 2048, MN_BOX_BYTES)
                                    : sw128_kmajor_desc(b_addr + k * 32);
            const uint32_t accum = (kb != kb0) || (k != 0);
            if (PAIR) umma_f16_ss_pair(d_tmem, ad, bd, idesc, accum);
            else umma_f16_ss(d_tmem, ad, bd, idesc, accum);
          }
          if (PAIR) umma_commit_pair_mc(&empty[s], 0x3);
          else umma_commit(&empty[s]);
        }
        if (!ok) break;
        if (PAIR) umma_commit_pair_mc(&tfull[acc], 0x3);
        else umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1u;
      }
      // Drain: every MMA issued here completes before TMEM (and the peer's smem) is released.
      if (PAIR) umma_commit_pair_mc(drain, 0x1);
      else umma_commit(drain);
      mbar_wait(drain, 0, err);
    }
  } else {
    // ---------------- epilogue: warps 2..5 drain accumulator 0, warps 6..9 accumulator 1
    const int group = (warp - 2) >> 2;
    const int quad = warp & 3;
    const uint32_t tempty_addr =
        PAIR ? mapa_shared(smem_u32(&tempty[group]), 0) : smem_u32(&tempty[group]);
    uint32_t ph = 0;
    int it = 0;
    // TMA_IN: this warp's two input slots; loads are issued two chunks ahead (the first
    // two of a tile before its accumulator is ready) and consumed in order.
    uint64_t* my_in_bar = in_bar + (warp - 2) * 2;
    uint8_t* my_in = in_slots + (warp - 2) * 2 * Cfg::IN_SLOT_BYTES;
    uint32_t in_issued = 0, in_used = 0;
    // Split-K reduction (SplitFix), in the barrier area after the barriers and the TMEM
    // slot (which end below byte 160): each group's "this unit arrived last" flag, and
    // its two hand-off barriers (four warps' partials written -> flag decided).
    volatile int* fix_last = reinterpret_cast<volatile int*>(bar_base + 160);
    uint64_t* fix_written = reinterpret_cast<uint64_t*>(bar_base + 176) + group;
    uint64_t* fix_decided = reinterpret_cast<uint64_t*>(bar_base + 192) + group;
    uint32_t fix_ph = 0;
    // FIX: the instantiation for split units with the last-arrival reduction; the
    // others are compiled without it (no register cost on the unsplit paths).
    constexpr bool CAN_FIX = FIX && EpiCanFix<Epi>::value;
    const bool fixing = CAN_FIX && fix.ws != nullptr && splits > 1;
    const int rr = quad * 32 + lane;  // the row this thread owns within the CTA's 128
    for (int u = unit; u < num_tiles; u += n_units, ++it) {
      if ((it & 1) != group) continue;
      const int tile = u / splits;
      const int my_split = u % splits;
      const int m_blk = tile / n_tiles;
      const int n_blk = tile % n_tiles;
      const int row0w = m_blk * TILE_M + (int)rank * GEMM_BM + quad * 32;
      const int slab_tile = tile * (PAIR ? 2 : 1) + (int)rank;
      // slab s of this tile: 128 rows x BN fp32 as [chunk][8 float4 groups][128 rows]
      auto slab = [&](int s) -> float4* {
        return fix.ws + ((size_t)slab_tile * splits + s) * (size_t)(GEMM_BM * BN / 4);
      };
      auto in_issue = [&](int c) {
        if constexpr (TIN) {
          const int col = n_blk * BN + c * 32;
          if (c < NC && col < N) {
            const int slot = (int)(in_issued & 1u);
            if (lane == 0) {
              bulk_wait_read<0>();  // the slot's last store (chunk c - 2) has read it
              mbar_arrive_expect_tx(&my_in_bar[slot], Cfg::IN_SLOT_BYTES);
              tma_load_2d(my_in + slot * Cfg::IN_SLOT_BYTES, tmC, &my_in_bar[slot], col, row0w);
            }
            ++in_issued;
          }
        }
      };
      if (!fixing) {  // a split unit learns only after its accumulator whether it reduces
        in_issue(0);
        in_issue(1);
      }
      // Per-row setup and the first chunk's global loads go out before the accumulator
      // is ready, so their latency hides behind the wait.
      const int row = m_blk * TILE_M + (int)rank * GEMM_BM + quad * 32 + lane;
      const bool row_ok = row < M;
      Epi e = epi;
      if constexpr (EpiHasSplit<Epi>::value) e.set_split(u % splits);
      e.begin_row(row, row_ok);
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(group * BN);
      typename Epi::Pre pa, pb;
      uint8_t* wbuf = epi_bufs + (warp - 2) * Cfg::EPI_BUF_BYTES;
      constexpr int IN_NB = EpiInBytes<Epi>::value > 0 ? EpiInBytes<Epi>::value : 16;
      uint4 in_next[IN_NB / 16];  // the next chunk's input pieces, loads in flight
      auto issue_in = [&](int col) {
        if constexpr (EpiInBytes<Epi>::value > 0)
          warp_issue_rows<IN_NB>(row_ok && col < N ? e.in_src(row, col) : nullptr, in_next);
      };
      // One chunk: TMEM -> registers, epilogue math, warp-cooperative store. Global
      // operands (Pre) are loaded one chunk ahead; the TMEM load latency is covered by
      // the other epilogue group. col < N is warp-uniform.
      auto do_chunk = [&](int c, const typename Epi::Pre& pre) {
        const int col = n_blk * BN + c * 32;
        if (col >= N) return;
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait_regs(r);
        uint4 outv[8];
        uint8_t* dst = nullptr;
        if constexpr (TIN) {
          const int slot = (int)(in_used & 1u);
          const bool in_ok = mbar_wait(&my_in_bar[slot], (in_used >> 1) & 1u, err);
          ++in_used;
          uint8_t* xbox = my_in + slot * Cfg::IN_SLOT_BYTES;
          uint8_t* hbox = wbuf + slot * 2048;  // fp16 staging box, 32 rows x 64 B
          if (lane == 0) bulk_wait_read<1>();  // chunk c - 2's store of hbox has read it
          __syncwarp();
          if (row_ok && in_ok) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
            e.chunk_tma(row, col, v, pre, xbox + lane * 128, lane & 7, hbox + lane * 64,
                        (lane >> 1) & 3);
          }
          fence_proxy_async_smem();  // generic writes -> visible to the TMA stores
          __syncwarp();
          if (lane == 0 && in_ok) {
            tma_store_2d(tmC, xbox, col, row0w);  // rows past M are not written
            tma_store_2d(tmD, hbox, col, row0w);
            bulk_commit_group();
          }
          in_issue(c + 2);
        } else {
          if constexpr (EpiInBytes<Epi>::value > 0) {
            warp_finish_rows<IN_NB>(wbuf, in_next, outv);
            if (c + 1 < NC) issue_in(col + 32);
          }
          if (row_ok) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              v[i] = __uint_as_float(r[i]);
              if constexpr (EpiRowScale<Epi>::value) v[i] *= e.rs;
            }
            e.chunk(row, col, v, pre, outv, dst);
          }
          if constexpr (Epi::OUT_BYTES > 0)
            warp_store_rows<(Epi::OUT_BYTES > 0 ? Epi::OUT_BYTES : 16), EpiAtomic<Epi>::value>(
                wbuf, outv, dst, row_ok);
        }
      };
      const int col_base = n_blk * BN;
      if (!fixing && row_ok && col_base < N) e.prefetch(row, col_base, pa);
      issue_in(col_base);
      if (!mbar_wait(&tfull[group], ph, err)) break;
      ph ^= 1u;
      tc_fence_after();
      if constexpr (CAN_FIX) {
        if (fixing) {
          // this unit's partial out to its slab (raw accumulator: the row scale and the
          // epilogue apply to the sum)
          const int n_chunks = min(NC, (N - col_base + 31) / 32);
          splitfix_write(t_row, n_chunks, slab(my_split) + rr, row_ok);
          __threadfence();  // the partial is visible device-wide before the arrival
          // The group's four warps hand over through mbarriers with bounded waits (a warp
          // that gives up on an error never leaves the others waiting without a limit).
          __syncwarp();
          if (lane == 0) mbar_arrive(fix_written);
          if (quad == 0 && lane == 0) {
            int last = -1;  // -1: the hand-off failed (an expired wait)
            if (mbar_wait(fix_written, fix_ph, err)) {
              const int old = atomicAdd(&fix.cnt[slab_tile], 1);
              last = old == splits - 1;
              if (last) fix.cnt[slab_tile] = 0;  // all splits arrived: zero for the next launch
            }
            fix_last[group] = last;
            mbar_arrive(fix_decided);
          }
          const bool decided = mbar_wait(fix_decided, fix_ph, err);
          fix_ph ^= 1u;
          const int last_flag = decided ? fix_last[group] : -1;
          if (last_flag < 0) break;
          if (!last_flag) {  // another split reduces this tile: hand the TMEM back
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if (PAIR) mbar_arrive_cluster(tempty_addr);
              else mbar_arrive(&tempty[group]);
            }
            continue;
          }
          __threadfence();  // the other splits' partials, published before their arrivals
          // Sum of all splits' partials in split order, this unit's own taken from TMEM,
          // written back over the accumulator: the epilogue below then runs unchanged.
          // The next split's loads are issued before the current one's adds.
          splitfix_reduce(t_row, n_chunks, slab(0), GEMM_BM * BN / 4, splits, my_split, rr,
                          row_ok);
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          tc_fence_after();
          in_issue(0);
          in_issue(1);
          if (row_ok && col_base < N) e.prefetch(row, col_base, pa);
        }
      }
#pragma unroll 1
      for (int c = 0; c < NC; c += 2) {
        const int col_b = col_base + (c + 1) * 32;
        if (row_ok && col_b < N) e.prefetch(row, col_b, pb);
        do_chunk(c, pa);
        if (c + 2 < NC && row_ok && col_b + 32 < N) e.prefetch(row, col_b + 32, pa);
        do_chunk(c + 1, pb);
      }
      if (row_ok) e.end_row(row, n_blk);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR) mbar_arrive_cluster(tempty_addr);
        else mbar_arrive(&tempty[group]);
      }
    }
    // Error exit: input loads still in flight complete before the CTA exits (bounded);
    // the epilogue's TMA stores finish before the CTA's shared memory goes away.
    for (; in_used < in_issued; ++in_used)
      mbar_wait(&my_in_bar[in_used & 1u], (in_used >> 1) & 1u, err);
    if constexpr (TIN) {
      if (lane == 0) bulk_wait_all();
    }
  }

  tc_fence_before();
  __syncthreads();
  __syncwarp();
  if (PAIR) cluster_sync();  // the peer's smem and barriers stay alive until both are done
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// tmC, tmD: the TMA_IN epilogue's in/out matrix and its second output (unused otherwise).
template <int BN, class Epi, int LAYOUT = 0, bool FIX = false>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                   int M, int N, int K, int b_z, int splits, Epi epi, SplitFix fix, int* err) {
  gemm_tn_body<BN, false, Epi, LAYOUT, FIX>(&tmA, &tmB, &tmC, &tmD, M, N, K, b_z, splits, epi,
                                            fix, err);
}

template <class Epi, int LAYOUT = 0, bool FIX = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    gemm_tn_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC,
                        const __grid_constant__ CUtensorMap tmD, int M, int N, int K, int b_z,
                        int splits, Epi epi, SplitFix fix, int* err) {
  gemm_tn_body<256, true, Epi, LAYOUT, FIX>(&tmA, &tmB, &tmC, &tmD, M, N, K, b_z, splits, epi,
                                            fix, err);
}

}  // namespace cb
