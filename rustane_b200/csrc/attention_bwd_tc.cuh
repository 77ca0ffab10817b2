// Causal self-attention backward on the 5th-generation tensor cores (tcgen05/TMEM),
// head_dim 128. Same math as attention_bwd.cuh (the m16n8k16 version, kept for
// seq % 128 != 0):
//   S = Q K^T / sqrt(128), P = 2^(S log2(e) - lse2), dV = P^T dO,
//   dP = dO V^T, dS = P o (dP - D), dQ = dS K / sqrt(128), dK = dS^T Q / sqrt(128),
// RoPE undone on dQ and dK.
//
// One CTA = 128 keys of one (batch, kv head), looping over the query heads of its group
// and the 64-query blocks at or after its keys. Keys are the M = 128 rows of every
// product, so dK and dV accumulate in TMEM over the whole loop. TMEM (512 columns):
//   dK [0,128)  dV [128,256)  S^T [256,320)  dP^T [320,384)  dQ^T [384,448)
// Per query block (64 queries):
//   S^T  = K Q^T        (M=128 keys,  N=64, K=128 dims; A=K, B=Q, both K-major)
//   dP^T = V dO^T       (M=128 keys,  N=64, K=128)
//   softmax warps (thread = key row): P^T and dS^T in fp16 into shared memory
//   dV  += P^T dO       (M=128, N=128 dims, K=64 queries; B=dO MN-major)
//   dK  += dS^T Q       (M=128, N=128, K=64; B=Q MN-major)
//   dQ^T = K^T dS^T     (M=128 dims, N=64, K=128 keys; A=K MN-major, B=dS^T MN-major)
//   dQ warps (thread = dim): dQ^T from TMEM into a [64 queries][128 dims] fp32 tile in
//   shared memory, added into dq32 by one TMA reduce-add.
// The block's log-sum-exp and D values (64 floats each) arrive with Q and dO by bulk copy.
// At the end the softmax warps write dK (scaled, RoPE undone) and dV into the K / V tiles'
// shared memory and store them to dQKV with TMA.
// 320 threads: warp 0 TMA producer (K, V once; Q and dO double-buffered), warp 1 TMEM
// owner + MMA issuer, warps 2-5 softmax, warps 6-9 dQ. Every mbarrier wait is bounded.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <math_constants.h>
#include <stdint.h>

#include "attention_bwd.cuh"
#include "ptx.cuh"

namespace cb {

constexpr int AT_BK = 128;  // keys per CTA
constexpr int AT_BQ = 64;   // queries per step
constexpr int AT_THREADS = 320;
// shared memory map (bytes from the 1024-aligned base)
constexpr int AT_K_OFF = 0;           // 2 x 16 KB: dims 0-63 | 64-127, [128 keys][128 B]
constexpr int AT_V_OFF = 32768;       // same
constexpr int AT_Q_OFF = 65536;       // 2 buffers x (2 x 8 KB): [64 queries][128 B] halves
constexpr int AT_O_OFF = 98304;       // dO, same layout as Q
constexpr int AT_P_OFF = 131072;      // P^T  [128 keys][64 queries] fp16, 128-byte swizzle
constexpr int AT_DS_OFF = 147456;     // dS^T same
constexpr int AT_LSE_OFF = 163840;    // 2 buffers x (lse 256 B, D 256 B)
constexpr int AT_DQ_OFF = 164864;     // dQ staging [64 queries][128 dims] fp32, 32 KB
constexpr int AT_BAR_OFF = 197632;
constexpr int AT_SMEM = AT_BAR_OFF + 256 + 1024;
constexpr uint32_t AT_TMEM_COLS = 512;

__global__ void __launch_bounds__(AT_THREADS, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmDQ,
                       const __grid_constant__ CUtensorMap tmDKV,
                       const float* __restrict__ lse2, const float* __restrict__ dsum,
                       const float2* __restrict__ rope, float* __restrict__ dq32,
                       int seq, int heads, int kv_heads,
                       float scale_log2, float scale, int* err) {
  extern __shared__ uint8_t at_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(at_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AT_BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;   // [2]
  uint64_t* q_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 6;
  uint64_t* p_full = bars + 7;
  uint64_t* p_free = bars + 8;
  uint64_t* dq_full = bars + 9;
  uint64_t* dq_free = bars + 10;
  uint64_t* done = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x;  // key block: early blocks see the most queries, launched first
  const int hk = blockIdx.y, b = blockIdx.z;
  const int group = heads / kv_heads;
  const int q_dim = heads * 128;
  const int k0 = kt * AT_BK;
  const int qb0 = k0 / AT_BQ, n_qb = seq / AT_BQ - qb0;  // query blocks at or after the keys
  const int n_steps = group * n_qb;
  const int kv_row0 = (b * kv_heads + hk) * seq + k0;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(&q_full[0], 1);
    mbar_init(&q_full[1], 1);
    mbar_init(&q_empty[0], 1);
    mbar_init(&q_empty[1], 1);
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(p_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 4);
    mbar_init(done, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
    tma_prefetch_desc(&tmDQ);
    tma_prefetch_desc(&tmDKV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, AT_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_dk = tmem, t_dv = tmem + 128, t_s = tmem + 256, t_dp = tmem + 320,
                 t_dq = tmem + 384;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer
      mbar_arrive_expect_tx(kv_full, 65536);
      tma_load_2d(smem + AT_K_OFF, &tmK, kv_full, 0, kv_row0);
      tma_load_2d(smem + AT_K_OFF + 16384, &tmK, kv_full, 64, kv_row0);
      tma_load_2d(smem + AT_V_OFF, &tmV, kv_full, 0, kv_row0);
      tma_load_2d(smem + AT_V_OFF + 16384, &tmV, kv_full, 64, kv_row0);
      for (int n = 0; n < n_steps; ++n) {
        const int qbuf = n & 1;
        if (!mbar_wait(&q_empty[qbuf], ((n >> 1) & 1) ^ 1u, err)) break;
        const int h = hk * group + n / n_qb;
        const int q0 = (qb0 + n % n_qb) * AT_BQ;
        mbar_arrive_expect_tx(&q_full[qbuf], 32768 + 512);
        uint8_t* qd = smem + AT_Q_OFF + qbuf * 16384;
        uint8_t* od = smem + AT_O_OFF + qbuf * 16384;
        const int q_row = (b * heads + h) * seq + q0;
        tma_load_2d(qd, &tmQ, &q_full[qbuf], 0, q_row);
        tma_load_2d(qd + 8192, &tmQ, &q_full[qbuf], 64, q_row);
        const int o_row = b * seq + q0;
        tma_load_2d(od, &tmDO, &q_full[qbuf], h * 128, o_row);
        tma_load_2d(od + 8192, &tmDO, &q_full[qbuf], h * 128 + 64, o_row);
        uint8_t* ld = smem + AT_LSE_OFF + qbuf * 512;
        const size_t lrow = ((size_t)b * heads + h) * seq + q0;
        bulk_load(ld, lse2 + lrow, 256, &q_full[qbuf]);
        bulk_load(ld + 256, dsum + lrow, 256, &q_full[qbuf]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc_s = umma_idesc_f16(AT_BK, AT_BQ);           // K-major A, B
      constexpr uint32_t idesc_acc = umma_idesc_f16_bmn(AT_BK, 128);       // B MN-major
      constexpr uint32_t idesc_dq = umma_idesc_f16(128, AT_BQ) | (1u << 15) | (1u << 16);
      const uint32_t k_addr = smem_u32(smem + AT_K_OFF);
      const uint32_t v_addr = smem_u32(smem + AT_V_OFF);
      const uint32_t p_addr = smem_u32(smem + AT_P_OFF);
      const uint32_t ds_addr = smem_u32(smem + AT_DS_OFF);
      // S^T and dP^T of step n+1 are issued as soon as the softmax warps have read step
      // n's (s_free), ahead of step n's dV / dK / dQ, so the tensor pipe computes them
      // while the softmax of step n runs.
      auto issue_sd = [&](int n) -> bool {
        const int qbuf = n & 1;
        const uint32_t q_addr = smem_u32(smem + AT_Q_OFF + qbuf * 16384);
        const uint32_t o_addr = smem_u32(smem + AT_O_OFF + qbuf * 16384);
        if (!mbar_wait(&q_full[qbuf], (n >> 1) & 1, err)) return false;
        if (!mbar_wait(s_free, (n & 1) ^ 1u, err)) return false;  // step n-1's S^T / dP^T read
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // head dims in steps of 16
          const uint32_t ka = (uint32_t)((k >> 2) * 16384 + (k & 3) * 32);
          const uint32_t qa = (uint32_t)((k >> 2) * 8192 + (k & 3) * 32);
          umma_f16_ss(t_s, sw128_kmajor_desc(k_addr + ka), sw128_kmajor_desc(q_addr + qa),
                      idesc_s, k != 0);
          umma_f16_ss(t_dp, sw128_kmajor_desc(v_addr + ka), sw128_kmajor_desc(o_addr + qa),
                      idesc_s, k != 0);
        }
        umma_commit(s_full);
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, err) && (n_steps == 0 || issue_sd(0));
      for (int n = 0; n < n_steps && ok; ++n) {
        const int qbuf = n & 1;
        const uint32_t q_addr = smem_u32(smem + AT_Q_OFF + qbuf * 16384);
        const uint32_t o_addr = smem_u32(smem + AT_O_OFF + qbuf * 16384);
        if (n + 1 < n_steps && !issue_sd(n + 1)) break;
        if (!mbar_wait(p_full, n & 1, err)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < AT_BQ / 16; ++k) {  // queries in steps of 16
          const uint64_t pa = sw128_kmajor_desc(p_addr + k * 32);
          const uint64_t da = sw128_kmajor_desc(ds_addr + k * 32);
          const uint32_t acc = (n != 0) || (k != 0);
          umma_f16_ss(t_dv, pa, sw128_mnmajor_desc(o_addr + k * 2048, 8192), idesc_acc, acc);
          umma_f16_ss(t_dk, da, sw128_mnmajor_desc(q_addr + k * 2048, 8192), idesc_acc, acc);
        }
        if (!mbar_wait(dq_free, (n & 1) ^ 1u, err)) break;  // dQ^T of step n-1 read
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < AT_BK / 16; ++k) {  // keys in steps of 16
          umma_f16_ss(t_dq, sw128_mnmajor_desc(k_addr + k * 2048, 16384),
                      sw128_mnmajor_desc(ds_addr + k * 2048, 8192), idesc_dq, k != 0);
        }
        umma_commit(dq_full);
        umma_commit(&q_empty[qbuf]);
        umma_commit(p_free);
      }
      umma_commit(done);
      mbar_wait(done, 0, err);
    }
  } else if (warp < 6) {
    // ---------------- softmax warps: thread = key row r (TMEM lane r)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int key = k0 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    uint8_t* prow = smem + AT_P_OFF + r * 128;
    uint8_t* drow = smem + AT_DS_OFF + r * 128;
    bool ok = true;
    for (int n = 0; n < n_steps; ++n) {
      const int h = hk * group + n / n_qb;
      const int q0 = (qb0 + n % n_qb) * AT_BQ;
      (void)h;
      // this step's lse and D (landed with Q and dO; S^T is issued only after that)
      const float* lse_h = reinterpret_cast<const float*>(smem + AT_LSE_OFF + (n & 1) * 512);
      const float* d_h = lse_h + 64;
      if (!mbar_wait(s_full, n & 1, err)) { ok = false; break; }
      // lse / D were bulk-copied with Q: observe that copy's barrier too (already
      // complete; it cannot move on before this step's MMAs, which wait for p_full)
      if (!mbar_wait(&q_full[n & 1], (n >> 1) & 1, err)) { ok = false; break; }
      tc_fence_after();
      uint32_t sv[2][32], dv[2][32];
      tmem_ld_32x32b_x32(t_s + lane_off, sv[0]);
      tmem_ld_32x32b_x32(t_s + lane_off + 32, sv[1]);
      tmem_ld_32x32b_x32(t_dp + lane_off, dv[0]);
      tmem_ld_32x32b_x32(t_dp + lane_off + 32, dv[1]);
      tmem_ld_wait_regs(sv[0]);
      tmem_ld_wait_regs(sv[1]);
      tmem_ld_wait_regs(dv[0]);
      tmem_ld_wait_regs(dv[1]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      uint32_t pw[32], dw[32];  // P^T and dS^T of this row, fp16 pairs
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float pp[2], dd[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int jj = i * 2 + e;       // column within this half
            const int qi = half * 32 + jj;  // query index within the block
            float p = exp2_mufu(__uint_as_float(sv[half][jj]) * scale_log2 - lse_h[qi]);
            if (key > q0 + qi) p = 0.f;     // causal mask
            pp[e] = p;
            dd[e] = p * (__uint_as_float(dv[half][jj]) - d_h[qi]);
          }
          pw[half * 16 + i] = pack_half2(pp[0], pp[1]);
          dw[half * 16 + i] = pack_half2(dd[0], dd[1]);
        }
      }
      if (!mbar_wait(p_free, (n & 1) ^ 1u, err)) { ok = false; break; }  // step n-1's P, dS used
#pragma unroll
      for (int chunk = 0; chunk < 8; ++chunk) {  // 16-byte chunks of 8 queries
        const int phys = (chunk ^ (r & 7)) << 4;
        *reinterpret_cast<uint4*>(prow + phys) =
            make_uint4(pw[4 * chunk], pw[4 * chunk + 1], pw[4 * chunk + 2], pw[4 * chunk + 3]);
        *reinterpret_cast<uint4*>(drow + phys) =
            make_uint4(dw[4 * chunk], dw[4 * chunk + 1], dw[4 * chunk + 2], dw[4 * chunk + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // ---------------- dK (scaled, RoPE undone) and dV of this CTA's keys into dQKV: each
    // thread writes its key row into the K / V tiles' shared memory (free once every MMA
    // is done), 128-byte swizzled like the tensor map tmDKV, then two TMA stores per tile.
    const bool fin = ok && mbar_wait(done, 0, err);
    if (fin) {
      tc_fence_after();
      uint8_t* krow = smem + AT_K_OFF + r * 128;
      uint8_t* vrow = smem + AT_V_OFF + r * 128;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t kw[32], vw[32];
        tmem_ld_32x32b_x32(t_dk + lane_off + c * 32, kw);
        tmem_ld_32x32b_x32(t_dv + lane_off + c * 32, vw);
        tmem_ld_wait_regs(kw);
        tmem_ld_wait_regs(vw);
        const int hoff = (c >> 1) * 16384;  // dims 0-63 | 64-127
#pragma unroll
        for (int g4 = 0; g4 < 4; ++g4) {
          uint32_t kp[4], vp[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int col = g4 * 8 + i * 2;
            float a0 = __uint_as_float(kw[col]) * scale, a1 = __uint_as_float(kw[col + 1]) * scale;
            rope_back(a0, a1, rope, seq, (c * 32 + col) >> 1, key);
            kp[i] = pack_half2(a0, a1);
            vp[i] = pack_half2(__uint_as_float(vw[col]), __uint_as_float(vw[col + 1]));
          }
          const int chunk = (c & 1) * 4 + g4;  // 16-byte chunk within the 128-byte row
          const int off = hoff + ((chunk ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(krow + off) = make_uint4(kp[0], kp[1], kp[2], kp[3]);
          *reinterpret_cast<uint4*>(vrow + off) = make_uint4(vp[0], vp[1], vp[2], vp[3]);
        }
      }
    }
    fence_proxy_async_smem();
    named_barrier_sync(2, 128);  // the four softmax warps
    if (threadIdx.x == 2 * 32 && fin) {
      const int row = b * seq + k0;
      const int ck = q_dim + hk * 128, cv = q_dim + kv_heads * 128 + hk * 128;
      tma_store_2d(&tmDKV, smem + AT_K_OFF, ck, row);
      tma_store_2d(&tmDKV, smem + AT_K_OFF + 16384, ck + 64, row);
      tma_store_2d(&tmDKV, smem + AT_V_OFF, cv, row);
      tma_store_2d(&tmDKV, smem + AT_V_OFF + 16384, cv + 64, row);
      bulk_commit_group();
      bulk_wait_read<0>();  // shared memory stays valid until the stores have read it
    }
  } else {
    // ---------------- dQ warps: thread = head dim (TMEM lane), adds dQ^T into dq32
    const int quad = warp & 3;
    const int dim = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    for (int n = 0; n < n_steps; ++n) {
      const int h = hk * group + n / n_qb;
      const int q0 = (qb0 + n % n_qb) * AT_BQ;
      if (!mbar_wait(dq_full, n & 1, err)) break;
      tc_fence_after();
      uint32_t w[2][32];
      tmem_ld_32x32b_x32(t_dq + lane_off, w[0]);
      tmem_ld_32x32b_x32(t_dq + lane_off + 32, w[1]);
      tmem_ld_wait_regs(w[0]);
      tmem_ld_wait_regs(w[1]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
      // the previous step's reduction must have read the staging tile
      if (threadIdx.x == 6 * 32) bulk_wait_read_all();
      named_barrier_sync(1, 128);
      float* stage = reinterpret_cast<float*>(smem + AT_DQ_OFF);
#pragma unroll
      for (int half = 0; half < 2; ++half)
#pragma unroll
        for (int j = 0; j < 32; ++j)  // lanes write 32 consecutive dims of one query row
          stage[(half * 32 + j) * 128 + dim] = __uint_as_float(w[half][j]);
      fence_proxy_async_smem();
      named_barrier_sync(1, 128);
      if (threadIdx.x == 6 * 32) {
        tma_reduce_add_2d(&tmDQ, stage, h * 128, b * seq + q0);
        bulk_commit_group();
      }
    }
    if (threadIdx.x == 6 * 32) bulk_wait_all();  // reductions complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, AT_TMEM_COLS);
  }
}

}  // namespace cb
