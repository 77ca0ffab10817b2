// Causal self-attention forward on the 5th-generation tensor cores (tcgen05/TMEM),
// head_dim 128, online softmax. Same math as attention.cuh (the reference sdpaFwd
// graph, crates/engine/src/kernels/sdpa_fwd.rs:223-258: scores * 1/sqrt(hd), causal
// mask, softmax, P*V); masked keys are skipped, not added as -65504.
//
// One CTA = two 128-query tiles of one (batch, head), the heavy (late) one first and a
// light one after it (query tiles n-1-p and p: every CTA does the same number of key
// steps); the second tile's Q is loaded as soon as the first tile's last S is done, and
// the first tile's output is staged in the V buffers, so the second tile's first Q K^T
// runs while it is stored. 96 KB of shared memory and 256 TMEM columns, so two CTAs
// share an SM. 192 threads:
//   warp 0 lane 0 : TMA producer. Q tile once (128 x 128), then per 64-key tile j:
//                   K_j and V_j (both double-buffered), 128-byte swizzle.
//   warp 1        : TMEM owner; lane 0 issues the UMMAs:
//                     S_j = Q K_j^T   (M=128, N=64, K=128; A and B K-major) into one of
//                                      two TMEM S buffers, S_{j+1} issued before P_j is
//                                      ready so it overlaps the softmax of tile j
//                     O  += P_j V_j   (M=128, N=128, K=64; P read from TMEM, where it
//                                      overwrites S_j, V MN-major from its TMA tile)
//   warps 2..5    : softmax, one thread per query row (TMEM lane): reads its 64 scores,
//                   applies the causal mask on the diagonal tiles, updates the running
//                   max / sum in base 2 (exponentials on the MUFU), rescales its O row in
//                   TMEM only when the max grows past the reference max by 2^8, writes P
//                   (fp16, packed in pairs) over its S row in TMEM, and at the end of a
//                   tile divides O by the row sum into the V tiles' shared memory, from
//                   where one TMA store writes the 128 x 128 output tile.
// Layout: q, k, v are [batch, heads, seq, 128] fp16 (rows of a [batch*heads*seq, 128]
// matrix for the tensor maps); the output (tensor map tmO) is [batch*seq, heads*128]
// fp16. seq % 128 == 0.
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
constexpr int FA_V_OFF = 65536;         // 2 buffers x (2 x 8 KB): head dims 0-63 | 64-127
constexpr int FA_BAR_OFF = 98304;
constexpr int FA_SMEM = FA_BAR_OFF + 256 + 1024;
constexpr uint32_t FA_TMEM_COLS = 256;  // S0/P0 [0,64) S1/P1 [64,128) O [128,256)

// The O accumulator and row sum keep a stale reference max until the running max
// exceeds it by this much (base-2 log): P values stay <= 2^8, and most tiles skip
// the TMEM read-scale-write of O.
constexpr float FA_RESCALE_THRESHOLD = 8.0f;

__global__ void __launch_bounds__(FA_THREADS, 2)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmO, int seq, int heads,
                       int kv_heads, float scale_log2, float* __restrict__ lse, int* err) {
  extern __shared__ uint8_t fa_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FA_BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* pv_done = bars + 12;
  uint64_t* drain = bars + 13;
  uint64_t* q_empty = bars + 14;  // tile 0's last S is done: the Q buffer takes tile 1's Q
  uint64_t* o_done = bars + 15;   // tile 0's output has left the V buffers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Two query tiles of one (batch, head) per CTA, the heavy one first: tiles n_qt-1-p
  // and p (2 (n_qt-p) and 2 (p+1) key steps: every CTA does 2 (n_qt+1) steps). The middle
  // tile of an odd count runs alone.
  const int n_qt = seq / FA_BQ;
  const int pr = blockIdx.x;
  const int qt_a = n_qt - 1 - pr;
  const int n_tiles = (qt_a == pr) ? 1 : 2;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hk = h / (heads / kv_heads);
  const int kv_row0 = (b * kv_heads + hk) * seq;
  constexpr int SPT = FA_BQ / FA_BKV;  // key steps per query tile
  const int n0 = (qt_a + 1) * SPT;     // steps of tile 0
  const int n_total = n0 + (n_tiles == 2 ? (pr + 1) * SPT : 0);
  auto tile_qt = [&](int t) { return t == 0 ? qt_a : pr; };
  auto q_row_of = [&](int t) { return (b * heads + h) * seq + tile_qt(t) * FA_BQ; };
  // global step g (both tiles in sequence) -> key tile within its query tile
  auto step_kt = [&](int g) { return g < n0 ? g : g - n0; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(&k_full[0], 1);
    mbar_init(&k_full[1], 1);
    mbar_init(&k_empty[0], 1);
    mbar_init(&k_empty[1], 1);
    mbar_init(&v_full[0], 1);
    mbar_init(&v_full[1], 1);
    mbar_init(&v_empty[0], 1);
    mbar_init(&v_empty[1], 1);
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    mbar_init(q_empty, 1);
    mbar_init(o_done, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
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
  pdl_enter();  // lets the next GEMM (launched with PDL) schedule its CTAs early

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: Q, then K one step ahead of V; tile 1's Q as soon as
      // tile 0's last S is done, tile 1's first V once tile 0's output left the V buffers
      auto load_q = [&](int t) {
        mbar_arrive_expect_tx(q_full, 32768);
        tma_load_2d(smem + FA_Q_OFF, &tmQ, q_full, 0, q_row_of(t));
        tma_load_2d(smem + FA_Q_OFF + 16384, &tmQ, q_full, 64, q_row_of(t));
      };
      auto load_k = [&](int g) -> bool {
        const int kb = g & 1;
        if (!mbar_wait(&k_empty[kb], ((g >> 1) & 1) ^ 1u, err)) return false;
        mbar_arrive_expect_tx(&k_full[kb], 16384);
        uint8_t* dst = smem + FA_K_OFF + kb * 16384;
        tma_load_2d(dst, &tmK, &k_full[kb], 0, kv_row0 + step_kt(g) * FA_BKV);
        tma_load_2d(dst + 8192, &tmK, &k_full[kb], 64, kv_row0 + step_kt(g) * FA_BKV);
        return true;
      };
      load_q(0);
      bool ok = load_k(0);
      for (int g = 0; g < n_total && ok; ++g) {
        if (g + 1 < n_total) {
          if (g + 1 == n0) {  // tile 1's Q into the Q buffer
            if (!mbar_wait(q_empty, 0, err)) break;
            load_q(1);
          }
          if (!load_k(g + 1)) break;
        }
        const int vb = g & 1;
        if (!mbar_wait(&v_empty[vb], ((g >> 1) & 1) ^ 1u, err)) break;
        if (g == n0 && !mbar_wait(o_done, 0, err)) break;
        mbar_arrive_expect_tx(&v_full[vb], 16384);
        uint8_t* vdst = smem + FA_V_OFF + vb * 16384;
        tma_load_2d(vdst, &tmV, &v_full[vb], 0, kv_row0 + step_kt(g) * FA_BKV);
        tma_load_2d(vdst + 8192, &tmV, &v_full[vb], 64, kv_row0 + step_kt(g) * FA_BKV);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer (the steps of both tiles in one sequence)
      constexpr uint32_t idesc_s = umma_idesc_f16(FA_BQ, FA_BKV);
      constexpr uint32_t idesc_pv = umma_idesc_f16_bmn(FA_BQ, 128);
      const uint32_t q_addr = smem_u32(smem + FA_Q_OFF);
      const uint32_t k_addr = smem_u32(smem + FA_K_OFF);
      const uint32_t v_addr = smem_u32(smem + FA_V_OFF);
      auto issue_s = [&](int g) -> bool {
        const int kb = g & 1;
        if (step_kt(g) == 0 && !mbar_wait(q_full, g == 0 ? 0u : 1u, err)) return false;
        if (!mbar_wait(&k_full[kb], (g >> 1) & 1, err)) return false;
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
        if (n_tiles == 2 && g == n0 - 1) umma_commit(q_empty);
        return true;
      };
      bool ok = issue_s(0);
      for (int g = 0; g < n_total && ok; ++g) {
        if (g + 1 < n_total && !issue_s(g + 1)) break;
        const int vb = g & 1;
        if (!mbar_wait(p_full, g & 1, err)) break;
        if (!mbar_wait(&v_full[vb], (g >> 1) & 1, err)) break;
        tc_fence_after();
        const uint32_t p_tmem = t_s0 + (uint32_t)(vb * FA_BKV);  // P over S's columns
        const int kt = step_kt(g);
#pragma unroll
        for (int k = 0; k < FA_BKV / 16; ++k) {  // keys in steps of 16 (8 packed columns)
          umma_f16_ts(t_o, p_tmem + k * 8,
                      sw128_mnmajor_desc(v_addr + vb * 16384 + k * 2048, 8192), idesc_pv,
                      (kt | k) != 0);
        }
        umma_commit(&v_empty[vb]);
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
    bool ok = true;
    for (int t = 0; t < n_tiles; ++t) {
      const int qt = tile_qt(t);
      const int q_idx = qt * FA_BQ + r;
      const int n_kv = (qt + 1) * SPT;
      const int g0 = t == 0 ? 0 : n0;
      float m_run = -CUDART_INF_F, l_run = 0.f;
      for (int jt = 0; jt < n_kv && ok; ++jt) {
        const int g = g0 + jt;
        const int kb = g & 1;
        if (!mbar_wait(&s_full[kb], (g >> 1) & 1, err)) { ok = false; break; }
        tc_fence_after();
        uint32_t sa[32], sb[32];
        tmem_ld_32x32b_x32(t_s0 + lane_off + (uint32_t)(kb * FA_BKV), sa);
        tmem_ld_32x32b_x32(t_s0 + lane_off + (uint32_t)(kb * FA_BKV + 32), sb);
        tmem_ld_wait_regs(sa);
        tmem_ld_wait_regs(sb);
        // Raw scores; the scale (> 0) commutes with max, so it is folded into the
        // exponent argument. Reductions use 8 independent accumulators (short chains).
        float s[64];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = __uint_as_float(sa[i]);
          s[32 + i] = __uint_as_float(sb[i]);
        }
        const int key0 = jt * FA_BKV;
        if (key0 + FA_BKV - 1 > q_idx) {  // diagonal tile: mask keys after the query
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (key0 + i > q_idx) s[i] = -CUDART_INF_F;
        }
        float m8[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) m8[a] = s[a];
#pragma unroll
        for (int i = 8; i < 64; ++i) m8[i & 7] = fmaxf(m8[i & 7], s[i]);
        const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                               fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * scale_log2;
        // Lazy rescaling: move the reference max only when it is exceeded by the threshold.
        float corr = 1.0f;
        bool need = false;
        if (jt == 0) {
          m_run = mx;  // key tile 0 always holds key 0 <= every query, so mx is finite
        } else if (mx > m_run + FA_RESCALE_THRESHOLD) {
          need = true;
          corr = exp2_mufu(m_run - mx);
          m_run = mx;
          l_run *= corr;
        }
        const float neg_m = -m_run;
        float l8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        // All exponentials on the MUFU (ex2.approx): measured faster than sending half of
        // them to an FMA-pipe polynomial (3.45-3.50 against 3.73 ms of attention per
        // 600m-A forward), the MUFU not being the limit here.
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
          s[i] = exp2_mufu(fmaf(s[i], scale_log2, neg_m));
          s[i + 1] = exp2_mufu(fmaf(s[i + 1], scale_log2, neg_m));
          l8[(i >> 1) & 7] += s[i] + s[i + 1];
        }
        const float sum = ((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7]));
        l_run += sum;
        // P (fp16 pairs) over the first 32 columns of this row of S. The PV of two steps
        // back read this buffer and completed before this S was computed.
        {
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) pk[i] = pack_half2(s[2 * i], s[2 * i + 1]);
          tmem_st_32x32b_x32(t_s0 + lane_off + (uint32_t)(kb * FA_BKV), pk);
        }
        if (jt > 0) {
          // O holds this tile's P V of the steps before once the previous PV is done:
          // rescale it if needed.
          if (!mbar_wait(pv_done, (g - 1) & 1, err)) { ok = false; break; }
          tc_fence_after();
          if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              uint32_t o[32];
              tmem_ld_32x32b_x32(t_o + lane_off + c * 32, o);
              tmem_ld_wait_regs(o);
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
              tmem_st_32x32b_x32(t_o + lane_off + c * 32, o);
            }
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
      }
      // ---------------- this tile's output: O / l in fp16 into the V buffers (free once
      // the tile's last PV is done), 128-byte swizzled like the output tensor map (two
      // 64-column halves of [128 rows][128 B]), then one TMA store of the 128 x 128 tile.
      const bool fin = ok && mbar_wait(pv_done, (g0 + n_kv - 1) & 1, err);
      if (fin) {
        tc_fence_after();
        const float inv = 1.0f / l_run;
        // Log-sum-exp of the scaled scores in base 2 (lse2 = log2 sum_k 2^(s_k c)), kept
        // for the backward pass: P = 2^(s c - lse2).
        if (lse) lse[q_row_of(t) + r] = m_run + log2f(l_run);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(t_o + lane_off + c * 32, o);
          tmem_ld_wait_regs(o);
          uint8_t* half_tile = smem + FA_V_OFF + (c >> 1) * 16384 + r * 128;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint4 w;
            w.x = pack_half2(__uint_as_float(o[8 * k + 0]) * inv, __uint_as_float(o[8 * k + 1]) * inv);
            w.y = pack_half2(__uint_as_float(o[8 * k + 2]) * inv, __uint_as_float(o[8 * k + 3]) * inv);
            w.z = pack_half2(__uint_as_float(o[8 * k + 4]) * inv, __uint_as_float(o[8 * k + 5]) * inv);
            w.w = pack_half2(__uint_as_float(o[8 * k + 6]) * inv, __uint_as_float(o[8 * k + 7]) * inv);
            const int chunk = (c & 1) * 4 + k;  // 16-byte chunk within the 128-byte row
            *reinterpret_cast<uint4*>(half_tile + ((chunk ^ (r & 7)) << 4)) = w;
          }
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      named_barrier_sync(1, 128);  // the four softmax warps
      if (threadIdx.x == 64) {
        if (fin) {
          const int o_row = b * seq + qt * FA_BQ;
          tma_store_2d(&tmO, smem + FA_V_OFF, h * 128, o_row);
          tma_store_2d(&tmO, smem + FA_V_OFF + 16384, h * 128 + 64, o_row);
          bulk_commit_group();
          bulk_wait_read<0>();  // the V buffers stay untouched until the store has read them
        }
        if (t == 0 && n_tiles == 2) mbar_arrive(o_done);  // the producer may load V again
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
