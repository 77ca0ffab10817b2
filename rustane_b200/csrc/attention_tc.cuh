// Causal self-attention forward on the 5th-generation tensor cores (tcgen05/TMEM),
// head_dim 128, online softmax. Same math as attention.cuh (the reference sdpaFwd
// graph, crates/engine/src/kernels/sdpa_fwd.rs:223-258: scores * 1/sqrt(hd), causal
// mask, softmax, P*V); masked keys are skipped, not added as -65504.
//
// One CTA = 128 queries of one (batch, head); 96 KB of shared memory and 256 TMEM
// columns, so two CTAs share an SM. 192 threads:
//   warp 0 lane 0 : TMA producer. Q tile once (128 x 128), then per 64-key tile j:
//                   K_j (double-buffered) and V_j (single buffer), 128-byte swizzle.
//   warp 1        : TMEM owner; lane 0 issues the UMMAs:
//                     S_j = Q K_j^T   (M=128, N=64, K=128; A and B K-major) into one of
//                                      two TMEM S buffers, S_{j+1} issued before P_j is
//                                      ready so it overlaps the softmax of tile j
//                     O  += P_j V_j   (M=128, N=128, K=64; P K-major from smem,
//                                      V MN-major straight from its TMA tile)
//   warps 2..5    : softmax, one thread per query row (TMEM lane): reads its 64 scores,
//                   applies the causal mask on the diagonal tiles, updates the running
//                   max / sum in base 2, rescales its O row in TMEM when the max grows,
//                   writes P (fp16) into the swizzled A-operand tile, and at the end
//                   divides O by the row sum and stores the output row.
// Layout: q, k, v are [batch, heads, seq, 128] fp16 (rows of a [batch*heads*seq, 128]
// matrix for the tensor maps); out is [batch*seq, heads*128] fp16. seq % 128 == 0.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <math_constants.h>
#include <stdint.h>

#include "ptx.cuh"

namespace cb {

constexpr int FA_BQ = 128;
constexpr int FA_BKV = 64;
constexpr int FA_THREADS = 192;
// shared memory map (bytes from the 1024-aligned base)
constexpr int FA_Q_OFF = 0;             // 2 x 16 KB: head dims 0-63 | 64-127, [128 rows][128 B]
constexpr int FA_K_OFF = 32768;         // 2 buffers x (2 x 8 KB), [64 keys][128 B]
constexpr int FA_V_OFF = 65536;         // 2 x 8 KB: head dims 0-63 | 64-127, [64 keys][128 B]
constexpr int FA_P_OFF = 81920;         // 16 KB: [128 rows][64 keys] fp16
constexpr int FA_BAR_OFF = 98304;
constexpr int FA_SMEM = FA_BAR_OFF + 256 + 1024;
constexpr uint32_t FA_TMEM_COLS = 256;  // S0 [0,64) S1 [64,128) O [128,256)

__global__ void __launch_bounds__(FA_THREADS, 2)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, __half* __restrict__ out, int seq,
                       int heads, int kv_heads, float scale_log2, int* err) {
  extern __shared__ uint8_t fa_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FA_BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 6;
  uint64_t* s_full = bars + 7;   // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* pv_done = bars + 10;
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // heavy (late) query tiles first
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hk = h / (heads / kv_heads);
  const int q_row0 = ((b * heads + h) * seq) + qt * FA_BQ;
  const int kv_row0 = (b * kv_heads + hk) * seq;
  const int n_kv = (qt + 1) * (FA_BQ / FA_BKV);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(&k_full[0], 1);
    mbar_init(&k_full[1], 1);
    mbar_init(&k_empty[0], 1);
    mbar_init(&k_empty[1], 1);
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, FA_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s0 = tmem, t_o = tmem + 128;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: Q, then K one tile ahead of V
      mbar_arrive_expect_tx(q_full, 32768);
      tma_load_2d(smem + FA_Q_OFF, &tmQ, q_full, 0, q_row0);
      tma_load_2d(smem + FA_Q_OFF + 16384, &tmQ, q_full, 64, q_row0);
      auto load_k = [&](int j) -> bool {
        const int kb = j & 1;
        if (!mbar_wait(&k_empty[kb], ((j >> 1) & 1) ^ 1u, err)) return false;
        mbar_arrive_expect_tx(&k_full[kb], 16384);
        uint8_t* dst = smem + FA_K_OFF + kb * 16384;
        tma_load_2d(dst, &tmK, &k_full[kb], 0, kv_row0 + j * FA_BKV);
        tma_load_2d(dst + 8192, &tmK, &k_full[kb], 64, kv_row0 + j * FA_BKV);
        return true;
      };
      bool ok = load_k(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv && !load_k(j + 1)) break;
        if (!mbar_wait(v_empty, (j & 1) ^ 1u, err)) break;
        mbar_arrive_expect_tx(v_full, 16384);
        tma_load_2d(smem + FA_V_OFF, &tmV, v_full, 0, kv_row0 + j * FA_BKV);
        tma_load_2d(smem + FA_V_OFF + 8192, &tmV, v_full, 64, kv_row0 + j * FA_BKV);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc_s = umma_idesc_f16(FA_BQ, FA_BKV);
      constexpr uint32_t idesc_pv = umma_idesc_f16_bmn(FA_BQ, 128);
      const uint32_t q_addr = smem_u32(smem + FA_Q_OFF);
      const uint32_t k_addr = smem_u32(smem + FA_K_OFF);
      const uint32_t v_addr = smem_u32(smem + FA_V_OFF);
      const uint32_t p_addr = smem_u32(smem + FA_P_OFF);
      auto issue_s = [&](int j) -> bool {
        const int kb = j & 1;
        if (!mbar_wait(&k_full[kb], (j >> 1) & 1, err)) return false;
        tc_fence_after();
        const uint32_t d = t_s0 + (uint32_t)(kb * FA_BKV);
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // head dim in steps of 16
          const uint32_t off = (uint32_t)((k >> 2) * 16384 + (k & 3) * 32);
          const uint32_t koff = (uint32_t)(kb * 16384 + (k >> 2) * 8192 + (k & 3) * 32);
          umma_f16_ss(d, sw128_kmajor_desc(q_addr + off), sw128_kmajor_desc(k_addr + koff),
                      idesc_s, k != 0);
        }
        umma_commit(&k_empty[kb]);
        umma_commit(&s_full[kb]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, err) && issue_s(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) break;
        if (!mbar_wait(p_full, j & 1, err)) break;
        if (!mbar_wait(v_full, j & 1, err)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < FA_BKV / 16; ++k) {  // keys in steps of 16
          umma_f16_ss(t_o, sw128_kmajor_desc(p_addr + k * 32),
                      sw128_mnmajor_desc(v_addr + k * 2048, 8192), idesc_pv, (j | k) != 0);
        }
        umma_commit(v_empty);
        umma_commit(pv_done);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, err);
    }
  } else {
    // ---------------- softmax warps: thread = query row r (TMEM lane r)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int q_idx = qt * FA_BQ + r;
    uint8_t* p_row = smem + FA_P_OFF + r * 128;
    float m_run = -CUDART_INF_F, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int kb = j & 1;
      if (!mbar_wait(&s_full[kb], (j >> 1) & 1, err)) { ok = false; break; }
      tc_fence_after();
      uint32_t sa[32], sb[32];
      tmem_ld_32x32b_x32(t_s0 + lane_off + (uint32_t)(kb * FA_BKV), sa);
      tmem_ld_32x32b_x32(t_s0 + lane_off + (uint32_t)(kb * FA_BKV + 32), sb);
      tmem_ld_wait_regs(sa);
      tmem_ld_wait_regs(sb);
      float s[64];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        s[i] = __uint_as_float(sa[i]) * scale_log2;
        s[32 + i] = __uint_as_float(sb[i]) * scale_log2;
      }
      const int key0 = j * FA_BKV;
      if (key0 + FA_BKV - 1 > q_idx) {  // diagonal tile: mask keys after the query
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (key0 + i > q_idx) s[i] = -CUDART_INF_F;
      }
      float mx = s[0];
#pragma unroll
      for (int i = 1; i < 64; ++i) mx = fmaxf(mx, s[i]);
      const float m_new = fmaxf(m_run, mx);
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        s[i] = exp2f(s[i] - m_new);
        sum += s[i];
      }
      const float corr = exp2f(m_run - m_new);
      l_run = l_run * corr + sum;
      m_run = m_new;
      if (j > 0) {
        // P_{j-1} has been consumed and O holds P_{0..j-1} V: rescale it if needed.
        if (!mbar_wait(pv_done, (j - 1) & 1, err)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, corr != 1.0f)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(t_o + lane_off + c * 32, o);
            tmem_ld_wait_regs(o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
            tmem_st_32x32b_x32(t_o + lane_off + c * 32, o);
          }
          tmem_st_wait();
        }
      }
      // P row -> swizzled K-major A tile (16-byte chunk c of row r at c ^ (r & 7)).
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 w;
        w.x = pack_half2(s[8 * c + 0], s[8 * c + 1]);
        w.y = pack_half2(s[8 * c + 2], s[8 * c + 3]);
        w.z = pack_half2(s[8 * c + 4], s[8 * c + 5]);
        w.w = pack_half2(s[8 * c + 6], s[8 * c + 7]);
        *reinterpret_cast<uint4*>(p_row + ((c ^ (r & 7)) << 4)) = w;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && mbar_wait(pv_done, (n_kv - 1) & 1, err)) {
      tc_fence_after();
      const float inv = 1.0f / l_run;
      __half* dst = out + ((size_t)b * seq + q_idx) * ((size_t)heads * 128) + h * 128;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(t_o + lane_off + c * 32, o);
        tmem_ld_wait_regs(o);
        uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint4 w;
          w.x = pack_half2(__uint_as_float(o[8 * k + 0]) * inv, __uint_as_float(o[8 * k + 1]) * inv);
          w.y = pack_half2(__uint_as_float(o[8 * k + 2]) * inv, __uint_as_float(o[8 * k + 3]) * inv);
          w.z = pack_half2(__uint_as_float(o[8 * k + 4]) * inv, __uint_as_float(o[8 * k + 5]) * inv);
          w.w = pack_half2(__uint_as_float(o[8 * k + 6]) * inv, __uint_as_float(o[8 * k + 7]) * inv);
          d4[k] = w;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, FA_TMEM_COLS);
  }
}

}  // namespace cb
