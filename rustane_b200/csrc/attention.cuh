// Causal self-attention forward, head_dim 128, online softmax (flash style).
//
// Math follows the reference sdpaFwd graph (crates/engine/src/kernels/sdpa_fwd.rs:
// scores * 1/sqrt(hd) at :70,:223-233; additive causal mask -65504 above the
// diagonal at :41-51,:245; softmax at :246; P*V at :247). Masked keys are skipped
// here instead of adding -65504, which gives the same softmax in fp32.
//
// Layout: q, k, v are [batch, heads, seq, 128] fp16 (written by the QKV GEMM
// epilogue); out is [batch*seq, heads*128] fp16, the A operand of the O-proj GEMM.
//
// One CTA = 64 queries of one (batch, head); 4 warps x 16 query rows. K/V tiles
// of 64 keys are double-buffered in shared memory with cp.async; scores and P*V
// use m16n8k16 warp MMAs with fp32 accumulation. Only key tiles at or below the
// diagonal are visited (causal tile skipping); heavy query tiles launch first.
#pragma once
#include <cuda_fp16.h>
#include <math_constants.h>
#include <stdint.h>

#include "ptx.cuh"

namespace cb {

constexpr int ATT_BQ = 64;
constexpr int ATT_BKV = 64;
constexpr int ATT_D = 128;
constexpr int ATT_THREADS = 128;
constexpr int ATT_SMEM = (ATT_BQ + 4 * ATT_BKV) * ATT_D * 2;  // Q + 2x(K,V) = 80 KB

// Byte offset of 16-byte chunk `c` (0..15) of row `r` in a [rows][128] fp16 tile,
// XOR-swizzled so ldmatrix row groups hit distinct banks.
__device__ __forceinline__ uint32_t att_off(int r, int c) {
  return (uint32_t)(r * 256 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void att_load_tile(uint32_t s_base, const __half* g, int rows) {
  // rows x 16 chunks, 128 threads
  for (int i = threadIdx.x; i < rows * 16; i += ATT_THREADS) {
    int r = i >> 4, c = i & 15;
    cp_async_16(s_base + att_off(r, c), g + (size_t)r * ATT_D + c * 8);
  }
}

__global__ void __launch_bounds__(ATT_THREADS)
    attn_fwd_causal_kernel(const __half* __restrict__ q, const __half* __restrict__ k,
                           const __half* __restrict__ v, __half* __restrict__ out, int seq,
                           int heads, int kv_heads, float scale_log2, float* __restrict__ lse) {
  extern __shared__ __align__(128) uint8_t att_smem[];
  const uint32_t sQ = smem_u32(att_smem);
  const uint32_t sK0 = sQ + ATT_BQ * 256;
  const uint32_t sV0 = sK0 + 2 * ATT_BKV * 256;
  const uint32_t KV_BUF = ATT_BKV * 256;

  const int qt = gridDim.x - 1 - blockIdx.x;  // heavy (late) query tiles first
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hk = h / (heads / kv_heads);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;

  const __half* Qg = q + (((size_t)b * heads + h) * seq + (size_t)qt * ATT_BQ) * ATT_D;
  const __half* Kg = k + ((size_t)b * kv_heads + hk) * seq * ATT_D;
  const __half* Vg = v + ((size_t)b * kv_heads + hk) * seq * ATT_D;
  const int n_kv = (qt * ATT_BQ + ATT_BQ + ATT_BKV - 1) / ATT_BKV;

  att_load_tile(sQ, Qg, ATT_BQ);
  att_load_tile(sK0, Kg, ATT_BKV);
  att_load_tile(sV0, Vg, ATT_BKV);
  cp_async_commit();

  uint32_t qf[8][4];
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-CUDART_INF_F, -CUDART_INF_F};
  float l_run[2] = {0.f, 0.f};

  for (int j = 0; j < n_kv; ++j) {
    const int buf = j & 1;
    if (j + 1 < n_kv) {
      att_load_tile(sK0 + (buf ^ 1) * KV_BUF, Kg + (size_t)(j + 1) * ATT_BKV * ATT_D, ATT_BKV);
      att_load_tile(sV0 + (buf ^ 1) * KV_BUF, Vg + (size_t)(j + 1) * ATT_BKV * ATT_D, ATT_BKV);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    if (j == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        int mi = lane >> 3;
        int r = warp * 16 + (mi & 1) * 8 + (lane & 7);
        int c = ks * 2 + (mi >> 1);
        ldmatrix_x4(qf[ks], sQ + att_off(r, c));
      }
    }

    // ---- S = Q K^T  (16 x 64 per warp)
    const uint32_t sK = sK0 + buf * KV_BUF;
    const uint32_t sV = sV0 + buf * KV_BUF;
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of 8-key n-tiles
        uint32_t kb[4];
        int mi = lane >> 3;
        int r = np * 16 + (mi >> 1) * 8 + (lane & 7);
        int c = ks * 2 + (mi & 1);
        ldmatrix_x4(kb, sK + att_off(r, c));
        mma_16816(s[2 * np], qf[ks], kb[0], kb[1]);
        mma_16816(s[2 * np + 1], qf[ks], kb[2], kb[3]);
      }
    }

    // ---- causal mask on the diagonal tile
    const int q_lo = qt * ATT_BQ + warp * 16 + g;  // rows q_lo and q_lo + 8
    const int k_base = j * ATT_BKV;
    if (k_base + ATT_BKV - 1 > qt * ATT_BQ + warp * 16) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        int kk = k_base + nt * 8 + 2 * tig;
        if (kk > q_lo) s[nt][0] = -CUDART_INF_F;
        if (kk + 1 > q_lo) s[nt][1] = -CUDART_INF_F;
        if (kk > q_lo + 8) s[nt][2] = -CUDART_INF_F;
        if (kk + 1 > q_lo + 8) s[nt][3] = -CUDART_INF_F;
      }
    }

    // ---- online softmax (base 2; scale_log2 = log2(e)/sqrt(128))
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float mx = -CUDART_INF_F;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) mx = fmaxf(mx, fmaxf(s[nt][2 * r], s[nt][2 * r + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      float m_new = fmaxf(m_run[r], mx * scale_log2);
      float corr = exp2f(m_run[r] - m_new);
      m_run[r] = m_new;
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        float p0 = exp2f(s[nt][2 * r] * scale_log2 - m_new);
        float p1 = exp2f(s[nt][2 * r + 1] * scale_log2 - m_new);
        s[nt][2 * r] = p0;
        s[nt][2 * r + 1] = p1;
        sum += p0 + p1;
      }
      l_run[r] = l_run[r] * corr + sum;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        o[dt][2 * r] *= corr;
        o[dt][2 * r + 1] *= corr;
      }
    }

    // ---- O += P V
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {  // 16 keys per step
      uint32_t pa[4];
      pa[0] = pack_half2(s[2 * ks][0], s[2 * ks][1]);
      pa[1] = pack_half2(s[2 * ks][2], s[2 * ks][3]);
      pa[2] = pack_half2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
      pa[3] = pack_half2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {  // pairs of 8-dim n-tiles
        uint32_t vb[4];
        int mi = lane >> 3;
        int r = ks * 16 + (mi & 1) * 8 + (lane & 7);
        int c = dp * 2 + (mi >> 1);
        ldmatrix_x4_trans(vb, sV + att_off(r, c));
        mma_16816(o[2 * dp], pa, vb[0], vb[1]);
        mma_16816(o[2 * dp + 1], pa, vb[2], vb[3]);
      }
    }
    __syncthreads();  // buffer `buf` is refilled two iterations later
  }

  // ---- normalise and store
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_run[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (lse && tig == 0)  // base-2 log-sum-exp of the scaled scores, for the backward pass
      lse[((size_t)b * heads + h) * seq + qt * ATT_BQ + warp * 16 + g + 8 * r] =
          m_run[r] + log2f(l);
    l_run[r] = 1.0f / l;
  }
  const int q_row = qt * ATT_BQ + warp * 16 + g;
  __half* out0 = out + ((size_t)b * seq + q_row) * ((size_t)heads * ATT_D) + h * ATT_D;
  __half* out1 = out0 + (size_t)8 * heads * ATT_D;
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    int col = dt * 8 + 2 * tig;
    *reinterpret_cast<uint32_t*>(out0 + col) = pack_half2(o[dt][0] * l_run[0], o[dt][1] * l_run[0]);
    *reinterpret_cast<uint32_t*>(out1 + col) = pack_half2(o[dt][2] * l_run[1], o[dt][3] * l_run[1]);
  }
}

}  // namespace cb
