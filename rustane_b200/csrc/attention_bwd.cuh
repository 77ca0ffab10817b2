// Causal self-attention backward, head_dim 128 (flash-attention-2 style: scores are
// recomputed from Q, K and the saved log-sum-exp, nothing of size seq x seq is stored).
//
// Math (the derivative of sdpaFwd, crates/engine/src/kernels/sdpa_fwd.rs:223-258, the
// reference's ANE backward being sdpa_bwd.rs; layer.rs:6900-6990 drives it):
//   S = Q K^T / sqrt(128), P = softmax_causal(S), O = P V
//   dV = P^T dO
//   dP = dO V^T, D_q = sum_d dO[q,d] O[q,d], dS = P o (dP - D)
//   dQ = dS K / sqrt(128),  dK = dS^T Q / sqrt(128)
// and RoPE is undone on dQ and dK (rope_backward_inplace, layer.rs:7391-7408: the
// rotation by -theta), since Q and K were saved after rotation.
//
// Layout: q, k, v [batch, heads, seq, 128] fp16 (as the forward's QKV epilogue wrote
// them); o and dO [batch*seq, heads*128] fp16 (token-major, as the O projection reads
// and writes them); lse2 [batch, heads, seq] (base-2 log-sum-exp of the scaled scores,
// from the forward); dsum [batch, heads, seq] = D. Outputs: dK and dV as fp16 straight
// into the token-major dQKV buffer [batch*seq, q_dim + 2 kv_dim] (the A operand of the
// QKV backward GEMMs); dQ accumulated in fp32 into dq32 [batch*seq, q_dim] with atomics
// (several key blocks add to each query row), finished by attn_bwd_dq_kernel.
//
// One CTA = 64 keys of one (batch, kv head), looping over the query heads of its group
// and over the query blocks at or after it; 4 warps x 16 keys; m16n8k16 warp MMAs
// with fp32 accumulation, tiles staged with cp.async.
#pragma once
#include <cuda_fp16.h>
#include <math_constants.h>
#include <stdint.h>

#include "attention.cuh"
#include "ptx.cuh"

namespace cb {

constexpr int AB_BK = 64;  // keys per CTA
constexpr int AB_BQ = 64;  // queries per step
constexpr int AB_THREADS = 128;
// K, V, Q, dO tiles (16 KB each) + dS^T (64 x 64 fp16, 8 KB)
constexpr int AB_SMEM = 4 * 64 * 256 + 64 * 128;

// D[b, h, q] = sum_d dO[t, h*128 + d] * O[t, h*128 + d]; 16 lanes per (token, head),
// 16-byte loads.
__global__ void attn_bwd_dsum_kernel(const __half* __restrict__ o, const __half* __restrict__ dout,
                                     float* __restrict__ dsum, int T, int seq, int heads) {
  const int w = blockIdx.x * (blockDim.x >> 4) + (threadIdx.x >> 4);
  const int sub = threadIdx.x & 15;
  const bool ok = w < T * heads;
  float v = 0.f;
  int t = 0, h = 0;
  if (ok) {
    t = w / heads;
    h = w % heads;
    const size_t off = (size_t)t * heads * 128 + h * 128 + sub * 8;
    const uint4 a = *reinterpret_cast<const uint4*>(o + off);
    const uint4 g = *reinterpret_cast<const uint4*>(dout + off);
    const __half2* ah = reinterpret_cast<const __half2*>(&a);
    const __half2* gh = reinterpret_cast<const __half2*>(&g);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 x = __half22float2(ah[k]), y = __half22float2(gh[k]);
      v = fmaf(x.x, y.x, fmaf(x.y, y.y, v));
    }
  }
#pragma unroll
  for (int m = 8; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  if (ok && sub == 0) {
    const int b = t / seq, q = t % seq;
    dsum[((size_t)b * heads + h) * seq + q] = v;
  }
}

// 64 token-major rows (row stride `ld` halfs) x 128 columns into a swizzled tile.
__device__ __forceinline__ void ab_load_rows(uint32_t s_base, const __half* g, size_t ld) {
  for (int i = threadIdx.x; i < 64 * 16; i += AB_THREADS) {
    const int r = i >> 4, c = i & 15;
    cp_async_16(s_base + att_off(r, c), g + (size_t)r * ld + c * 8);
  }
}

// Inverse RoPE of one (even, odd) pair at position p, pair index i:
// (d0, d1) -> (c d0 + s d1, -s d0 + c d1).
__device__ __forceinline__ void rope_back(float& d0, float& d1, const float2* rope, int seq,
                                          int i, int p) {
  const float2 cs = rope[(size_t)i * seq + p];
  const float a = d0, b = d1;
  d0 = cs.x * a + cs.y * b;
  d1 = -cs.y * a + cs.x * b;
}

__global__ void __launch_bounds__(AB_THREADS)
    attn_bwd_kernel(const __half* __restrict__ q, const __half* __restrict__ k,
                    const __half* __restrict__ v, const __half* __restrict__ dout,
                    const float* __restrict__ lse2, const float* __restrict__ dsum,
                    const float2* __restrict__ rope, float* __restrict__ dq32,
                    __half* __restrict__ dqkv, int seq, int heads, int kv_heads,
                    float scale_log2, float scale) {
  extern __shared__ __align__(128) uint8_t ab_smem[];
  const uint32_t sK = smem_u32(ab_smem);
  const uint32_t sV = sK + 64 * 256;
  const uint32_t sQ = sV + 64 * 256;
  const uint32_t sO = sQ + 64 * 256;  // dO tile
  const uint32_t sDS = sO + 64 * 256;  // dS^T [64 keys][64 queries] fp16, 128-byte rows

  const int kt = blockIdx.x;  // key block (early blocks see the most queries: launched first)
  const int hk = blockIdx.y;
  const int b = blockIdx.z;
  const int group = heads / kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int q_dim = heads * 128, n_qkv = q_dim + 2 * kv_heads * 128;

  const __half* Kg = k + (((size_t)b * kv_heads + hk) * seq + (size_t)kt * AB_BK) * 128;
  const __half* Vg = v + (((size_t)b * kv_heads + hk) * seq + (size_t)kt * AB_BK) * 128;
  ab_load_rows(sK, Kg, 128);
  ab_load_rows(sV, Vg, 128);
  cp_async_commit();

  float dk[16][4], dv[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) dk[i][j] = dv[i][j] = 0.f;

  const int key_lo = kt * AB_BK + warp * 16 + g;  // this thread's key rows: key_lo, key_lo + 8
  const int n_qb = seq / AB_BQ;

  for (int hh = 0; hh < group; ++hh) {
    const int h = hk * group + hh;
    const __half* Qg = q + ((size_t)b * heads + h) * seq * 128;
    const __half* dOg = dout + (size_t)b * seq * q_dim + (size_t)h * 128;
    const float* lse_h = lse2 + ((size_t)b * heads + h) * seq;
    const float* d_h = dsum + ((size_t)b * heads + h) * seq;
    for (int qb = kt; qb < n_qb; ++qb) {
      __syncthreads();  // the previous step's Q / dO / dS tiles are no longer read
      ab_load_rows(sQ, Qg + (size_t)qb * AB_BQ * 128, 128);
      ab_load_rows(sO, dOg + (size_t)qb * AB_BQ * q_dim, q_dim);
      cp_async_commit();
      cp_async_wait<0>();
      __syncthreads();

      // ---- S^T = K Q^T and dP^T = V dO^T (16 keys x 64 queries per warp)
      float st[8][4], dpt[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) st[i][j] = dpt[i][j] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t ka[4], va[4];
        {
          const int mi = lane >> 3;
          const int r = warp * 16 + (mi & 1) * 8 + (lane & 7);
          const int c = ks * 2 + (mi >> 1);
          ldmatrix_x4(ka, sK + att_off(r, c));
          ldmatrix_x4(va, sV + att_off(r, c));
        }
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t qb4[4], ob4[4];
          const int mi = lane >> 3;
          const int r = np * 16 + (mi >> 1) * 8 + (lane & 7);
          const int c = ks * 2 + (mi & 1);
          ldmatrix_x4(qb4, sQ + att_off(r, c));
          ldmatrix_x4(ob4, sO + att_off(r, c));
          mma_16816(st[2 * np], ka, qb4[0], qb4[1]);
          mma_16816(st[2 * np + 1], ka, qb4[2], qb4[3]);
          mma_16816(dpt[2 * np], va, ob4[0], ob4[1]);
          mma_16816(dpt[2 * np + 1], va, ob4[2], ob4[3]);
        }
      }

      // ---- P^T = 2^(S^T c - lse2[q]) (causal: keys after the query are 0),
      //      dS^T = P^T o (dP^T - D[q])
      const bool diag = (qb == kt);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int q0 = qb * AB_BQ + nt * 8 + 2 * tig;
        const float l0 = lse_h[q0], l1 = lse_h[q0 + 1];
        const float d0 = d_h[q0], d1 = d_h[q0 + 1];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key_lo + (e >> 1) * 8;
          const int qq = q0 + (e & 1);
          float p = exp2f(st[nt][e] * scale_log2 - ((e & 1) ? l1 : l0));
          if (diag && key > qq) p = 0.f;
          st[nt][e] = p;
          dpt[nt][e] = p * (dpt[nt][e] - ((e & 1) ? d1 : d0));
        }
      }

      // ---- dV += P^T dO, dK += dS^T Q (A operands straight from the accumulators)
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {  // 16 queries per step
        uint32_t pa[4], sa[4];
        pa[0] = pack_half2(st[2 * ks][0], st[2 * ks][1]);
        pa[1] = pack_half2(st[2 * ks][2], st[2 * ks][3]);
        pa[2] = pack_half2(st[2 * ks + 1][0], st[2 * ks + 1][1]);
        pa[3] = pack_half2(st[2 * ks + 1][2], st[2 * ks + 1][3]);
        sa[0] = pack_half2(dpt[2 * ks][0], dpt[2 * ks][1]);
        sa[1] = pack_half2(dpt[2 * ks][2], dpt[2 * ks][3]);
        sa[2] = pack_half2(dpt[2 * ks + 1][0], dpt[2 * ks + 1][1]);
        sa[3] = pack_half2(dpt[2 * ks + 1][2], dpt[2 * ks + 1][3]);
#pragma unroll
        for (int dp = 0; dp < 8; ++dp) {  // pairs of 8-dim n-tiles
          uint32_t ob4[4], qb4[4];
          const int mi = lane >> 3;
          const int r = ks * 16 + (mi & 1) * 8 + (lane & 7);
          const int c = dp * 2 + (mi >> 1);
          ldmatrix_x4_trans(ob4, sO + att_off(r, c));
          ldmatrix_x4_trans(qb4, sQ + att_off(r, c));
          mma_16816(dv[2 * dp], pa, ob4[0], ob4[1]);
          mma_16816(dv[2 * dp + 1], pa, ob4[2], ob4[3]);
          mma_16816(dk[2 * dp], sa, qb4[0], qb4[1]);
          mma_16816(dk[2 * dp + 1], sa, qb4[2], qb4[3]);
        }
      }

      // ---- dS^T to shared memory (fp16), then dQ_blk = dS K for this block's keys
      {
        const int r0 = warp * 16 + g;  // local key rows r0, r0 + 8
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int col = nt * 8 + 2 * tig;  // local query column
          const int chunk = col >> 3, within = (col & 7) * 2;
          const uint32_t a0 = sDS + r0 * 128 + (((chunk ^ (r0 & 7)) << 4) | within);
          const uint32_t a1 = sDS + (r0 + 8) * 128 + (((chunk ^ ((r0 + 8) & 7)) << 4) | within);
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(a0), "r"(pack_half2(dpt[nt][0], dpt[nt][1])));
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(a1), "r"(pack_half2(dpt[nt][2], dpt[nt][3])));
        }
      }
      __syncthreads();
      {
        // warp w: queries w*16 .. +15 of this block, all 128 dims; A = dS (queries x
        // keys) read transposed out of dS^T, B = K (keys x dims).
        float acc[16][4];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {  // 16 keys per step
          uint32_t a[4];
          {
            const int mi = lane >> 3;
            const int key = ks * 16 + (mi >> 1) * 8 + (lane & 7);  // dS^T row
            const int chunk = (warp * 16 + (mi & 1) * 8) >> 3;     // query chunk
            ldmatrix_x4_trans(a, sDS + key * 128 + ((chunk ^ (key & 7)) << 4));
          }
#pragma unroll
          for (int dp = 0; dp < 8; ++dp) {
            uint32_t kb4[4];
            const int mi = lane >> 3;
            const int r = ks * 16 + (mi & 1) * 8 + (lane & 7);
            const int c = dp * 2 + (mi >> 1);
            ldmatrix_x4_trans(kb4, sK + att_off(r, c));
            mma_16816(acc[2 * dp], a, kb4[0], kb4[1]);
            mma_16816(acc[2 * dp + 1], a, kb4[2], kb4[3]);
          }
        }
        const int qrow = qb * AB_BQ + warp * 16 + g;  // and qrow + 8
        float* d0 = dq32 + ((size_t)b * seq + qrow) * q_dim + (size_t)h * 128;
        float* d1 = d0 + (size_t)8 * q_dim;
#pragma unroll
        for (int dt = 0; dt < 16; ++dt) {
          const int col = dt * 8 + 2 * tig;
          atomicAdd(reinterpret_cast<float2*>(d0 + col), make_float2(acc[dt][0], acc[dt][1]));
          atomicAdd(reinterpret_cast<float2*>(d1 + col), make_float2(acc[dt][2], acc[dt][3]));
        }
      }
    }
  }

  // ---- dK (scaled, RoPE undone) and dV into the token-major dQKV buffer
  const int p0 = key_lo, p1 = key_lo + 8;  // positions
  __half* rk0 = dqkv + ((size_t)b * seq + p0) * n_qkv + q_dim + (size_t)hk * 128;
  __half* rk1 = rk0 + (size_t)8 * n_qkv;
  __half* rv0 = rk0 + (size_t)kv_heads * 128;
  __half* rv1 = rk1 + (size_t)kv_heads * 128;
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int col = dt * 8 + 2 * tig;
    const int pair = col >> 1;
    float a0 = dk[dt][0] * scale, a1 = dk[dt][1] * scale;
    float c0 = dk[dt][2] * scale, c1 = dk[dt][3] * scale;
    rope_back(a0, a1, rope, seq, pair, p0);
    rope_back(c0, c1, rope, seq, pair, p1);
    *reinterpret_cast<uint32_t*>(rk0 + col) = pack_half2(a0, a1);
    *reinterpret_cast<uint32_t*>(rk1 + col) = pack_half2(c0, c1);
    *reinterpret_cast<uint32_t*>(rv0 + col) = pack_half2(dv[dt][0], dv[dt][1]);
    *reinterpret_cast<uint32_t*>(rv1 + col) = pack_half2(dv[dt][2], dv[dt][3]);
  }
}

// dQ = dq32 * scale with RoPE undone, into the q columns of dQKV (fp16).
// One thread per (token, 8 consecutive dims of one head): two 16-byte loads of dq32, two
// of rope_pm (the (cos, sin) table in position-major order [seq][64]) and one 16-byte
// store.
__global__ void attn_bwd_dq_kernel(const float* __restrict__ dq32,
                                   const float2* __restrict__ rope_pm,
                                   __half* __restrict__ dqkv, int T, int seq, int heads,
                                   int n_qkv, float scale) {
  const int q8 = heads * 16;  // 8-dim groups per token
  const size_t n = (size_t)T * q8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / q8);
    const int g = (int)(i - (size_t)t * q8);
    const float4* src = reinterpret_cast<const float4*>(dq32) + 2 * i;
    const float4 d0 = src[0], d1 = src[1];
    const float4* rp =
        reinterpret_cast<const float4*>(rope_pm + (size_t)(t % seq) * 64 + (g & 15) * 4);
    const float4 r0 = rp[0], r1 = rp[1];  // (cos, sin) of pairs 4(g%16) .. +3
    const float a[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
    const float cs[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
    uint32_t w[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float x = a[2 * p] * scale, y = a[2 * p + 1] * scale;
      const float c = cs[2 * p], sn = cs[2 * p + 1];
      w[p] = pack_half2(c * x + sn * y, -sn * x + c * y);
    }
    *reinterpret_cast<uint4*>(dqkv + (size_t)t * n_qkv + (size_t)g * 8) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace cb
