// Causal self-attention forward on the 5th-generation tensor cores (tcgen05/TMEM),
// head_dim 128, online softmax. Same math as attention.cuh (the reference sdpaFwd
// graph, crates/engine/src/kernels/sdpa_fwd.rs:223-258: scores * 1/sqrt(hd), causal
// mask, softmax, P*V); masked keys are skipped, not added as -65504.
//
// One CTA = one block of 256 query rows of one (batch, head): two 128-row query tiles
// Q0, Q1 (tiles 2m and 2m+1) worked on at the same time by two softmax warpgroups and
// fed by one stream of 128-key blocks K_j, V_j shared by both (a block of seq % 256 ==
// 128 rows at the end of a sequence has tile 0 only). Tile t needs key blocks 0..qt_t;
// the last block of each tile is its diagonal. The MMAs of the two tiles interleave so
// that one tile's softmax always runs while the tensor cores work on the other tile:
//   S0_0, S1_0, [P0_0] PV0_0, S0_1, [P1_0] PV1_0, S1_1, [P0_1] PV0_1, S0_2, ...
// (S_t(j+1) reuses the TMEM columns of P_t(j); tcgen05 MMAs of one thread run in
// order, so it is issued right after PV_t(j), which reads them.)
//
// 320 threads, one CTA per SM (192 KB of shared memory, all 512 TMEM columns):
//   warp 0 lane 0 : TMA producer: Q0, Q1 once, then per key block j: K_j and V_j into
//                   two-deep rings, 128-byte swizzle.
//   warp 1        : TMEM owner; lane 0 issues the UMMAs:
//                     S_t = Q_t K_j^T   (M=128, N=128 keys, K=128; A and B K-major)
//                     O_t += P_t V_j    (M=128, N=128, K=128 keys; P from TMEM where it
//                                        overwrote S_t, V MN-major from its TMA tile)
//   warps 2..5    : softmax of tile 0, warps 6..9 : softmax of tile 1; one thread per
//                   query row (TMEM lane). Per key block: a first pass over the 128
//                   scores for the row max (TMEM loads, two chunks in flight), then a
//                   second pass computing P = 2^(s c - m) in base 2 on the MUFU, the row
//                   sum, and P (fp16 pairs) written over the scores. The O row in TMEM is
//                   rescaled only when the running max passes the reference max by 2^8
//                   (lazy rescaling); by the time S_t(j) is complete, PV_t(j-1) is too (it
//                   was issued before), so O is stable when it is rescaled. At the end of
//                   a tile, O / l in fp16 goes into the tile's Q buffer (no longer read)
//                   and one TMA store writes the 128 x 128 output tile.
// Layout: q, k, v are [batch, heads, seq, 128] fp16 (rows of a [batch*heads*seq, 128]
// matrix for the tensor maps, K and V in 128-row boxes); the output (tensor map tmO) is
// [batch*seq, heads*128] fp16. seq % 128 == 0. The grid is one-dimensional with the
// heaviest blocks (the latest query rows, which need the most key blocks) first.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <math_constants.h>
#include <stdint.h>

#include "ptx.cuh"

namespace cb {

constexpr int FA_BQ = 128;   // query rows per tile
constexpr int FA_BKV = 128;  // keys per block (rows of the K and V tensor-map boxes)
constexpr int FA_THREADS = 320;
// shared memory map (bytes from the 1024-aligned base)
constexpr int FA_Q_OFF = 0;        // 2 tiles x 32 KB: head dims 0-63 | 64-127, [128 rows][128 B]
constexpr int FA_K_OFF = 65536;    // 2 slots x 32 KB: dims 0-63 | 64-127, [128 keys][128 B]
constexpr int FA_V_OFF = 131072;   // 2 slots x 32 KB, same layout (read MN-major)
constexpr int FA_BAR_OFF = 196608;
constexpr int FA_SMEM = FA_BAR_OFF + 256 + 1024;
constexpr uint32_t FA_TMEM_COLS = 512;  // S0/P0 [0,128) S1/P1 [128,256) O0 [256,384) O1 [384,512)

// The O accumulator and row sum keep a stale reference max until the running max
// exceeds it by this much (base-2 log): P values stay <= 2^8, and most blocks skip
// the TMEM read-scale-write of O.
constexpr float FA_RESCALE_THRESHOLD = 8.0f;

// Blocks of 256 query rows per sequence.
__host__ __device__ constexpr int fa_blocks(int seq) { return (seq / FA_BQ + 1) / 2; }

__global__ void __launch_bounds__(FA_THREADS, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmO, int seq, int heads,
                       int kv_heads, int batch, float scale_log2, float* __restrict__ lse,
                       int* err) {
  extern __shared__ uint8_t fa_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FA_BAR_OFF);
  uint64_t* q_full = bars + 0;    // [2] per tile
  uint64_t* k_full = bars + 2;    // [2] per slot
  uint64_t* k_empty = bars + 4;   // [2]
  uint64_t* v_full = bars + 6;    // [2]
  uint64_t* v_empty = bars + 8;   // [2]
  uint64_t* s_full = bars + 10;   // [2] per tile
  uint64_t* p_full = bars + 12;   // [2] per tile (one arrival per softmax warp)
  uint64_t* o_final = bars + 14;  // [2] per tile: its last PV is done
  uint64_t* drain = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // work item: heaviest blocks first
  const int n_blk = fa_blocks(seq);
  const int n_qt = seq / FA_BQ;
  const int hb_count = heads * batch;
  const int mb = n_blk - 1 - (int)blockIdx.x / hb_count;
  const int hb = (int)blockIdx.x % hb_count;
  const int b = hb / heads;
  const int h = hb - b * heads;
  const int hk = h / (heads / kv_heads);
  const int kv_row0 = (b * kv_heads + hk) * seq;
  const int n_t = (2 * mb + 1 < n_qt) ? 2 : 1;  // query tiles in this block
  const int n_steps = 2 * mb + n_t;              // key blocks (tile n_t - 1 needs them all)
  auto qt_of = [&](int t) { return 2 * mb + t; };
  auto q_row_of = [&](int t) { return (b * heads + h) * seq + qt_of(t) * FA_BQ; };
  // tile t needs key block j; the last tile needs every block
  auto active = [&](int t, int j) { return t < n_t && j <= qt_of(t); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_final[i], 1);
    }
    mbar_init(drain, 1);
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
  pdl_enter();  // lets the next GEMM (launched with PDL) schedule its CTAs early

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: both Q tiles, then K_j and V_j one block ahead
      for (int t = 0; t < n_t; ++t) {
        uint8_t* dst = smem + FA_Q_OFF + t * 32768;
        mbar_arrive_expect_tx(&q_full[t], 32768);
        tma_load_2d(dst, &tmQ, &q_full[t], 0, q_row_of(t));
        tma_load_2d(dst + 16384, &tmQ, &q_full[t], 64, q_row_of(t));
      }
      for (int j = 0; j < n_steps; ++j) {
        const int sl = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1u;
        const int row = kv_row0 + j * FA_BKV;
        if (!mbar_wait(&k_empty[sl], ph, err)) break;
        mbar_arrive_expect_tx(&k_full[sl], 32768);
        uint8_t* kd = smem + FA_K_OFF + sl * 32768;
        tma_load_2d(kd, &tmK, &k_full[sl], 0, row);
        tma_load_2d(kd + 16384, &tmK, &k_full[sl], 64, row);
        if (!mbar_wait(&v_empty[sl], ph, err)) break;
        mbar_arrive_expect_tx(&v_full[sl], 32768);
        uint8_t* vd = smem + FA_V_OFF + sl * 32768;
        tma_load_2d(vd, &tmV, &v_full[sl], 0, row);
        tma_load_2d(vd + 16384, &tmV, &v_full[sl], 64, row);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc_s = umma_idesc_f16(FA_BQ, FA_BKV);
      constexpr uint32_t idesc_pv = umma_idesc_f16_bmn(FA_BQ, 128);
      const int last_t = n_t - 1;  // the tile that uses every key block last
      auto issue_s = [&](int t, int j) -> bool {
        if (j == 0 && !mbar_wait(&q_full[t], 0, err)) return false;
        if (!mbar_wait(&k_full[j & 1], (j >> 1) & 1, err)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + FA_Q_OFF + t * 32768);
        const uint32_t k_addr = smem_u32(smem + FA_K_OFF + (j & 1) * 32768);
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // head dim in steps of 16
          const uint32_t off = (uint32_t)((k >> 2) * 16384 + (k & 3) * 32);
          umma_f16_ss(tmem + (uint32_t)(t * 128), sw128_kmajor_desc(q_addr + off),
                      sw128_kmajor_desc(k_addr + off), idesc_s, k != 0);
        }
        umma_commit(&s_full[t]);
        if (t == last_t) umma_commit(&k_empty[j & 1]);  // both tiles' S of block j issued
        return true;
      };
      auto issue_pv = [&](int t, int j) -> bool {
        if (!mbar_wait(&p_full[t], j & 1, err)) return false;
        if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1, err)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + FA_V_OFF + (j & 1) * 32768);
        const uint32_t p_tmem = tmem + (uint32_t)(t * 128);  // P over S_t's columns
#pragma unroll
        for (int k = 0; k < FA_BKV / 16; ++k)  // keys in steps of 16 (8 packed columns)
          umma_f16_ts(tmem + 256u + (uint32_t)(t * 128), p_tmem + k * 8,
                      sw128_mnmajor_desc(v_addr + k * 2048, 16384), idesc_pv, (j | k) != 0);
        if (t == last_t) umma_commit(&v_empty[j & 1]);
        if (j == qt_of(t)) umma_commit(&o_final[t]);
        return true;
      };
      bool ok = true;
      for (int t = 0; t < n_t && ok; ++t) ok = issue_s(t, 0);
      for (int j = 0; j < n_steps && ok; ++j) {
        for (int t = 0; t < 2 && ok; ++t) {
          if (!active(t, j)) continue;
          ok = issue_pv(t, j);
          if (ok && active(t, j + 1)) ok = issue_s(t, j + 1);
        }
      }
      // Drain: every MMA issued here completes before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, err);
    }
  } else {
    // ---------------- softmax warpgroups: thread = query row r (TMEM lane r) of tile t
    const int t = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t t_s = tmem + lane_off + (uint32_t)(t * 128);
    const uint32_t t_o = tmem + lane_off + 256u + (uint32_t)(t * 128);
    bool ok = t < n_t;
    const int qt = qt_of(t);
    float m_run = -CUDART_INF_F, l_run = 0.f;
    for (int j = 0; ok && j <= qt; ++j) {
      if (!mbar_wait(&s_full[t], j & 1, err)) { ok = false; break; }
      tc_fence_after();
      const bool diag = j == qt;  // keys 128 j + i with i > r are masked
      // pass 1: the row max of the raw scores (the scale > 0 commutes with max)
      float m8[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) m8[a] = -CUDART_INF_F;
#pragma unroll
      for (int c = 0; c < 4; c += 2) {
        uint32_t sa[32], sb[32];
        tmem_ld_32x32b_x32(t_s + c * 32, sa);
        tmem_ld_32x32b_x32(t_s + c * 32 + 32, sb);
        tmem_ld_wait_regs(sa);
        tmem_ld_wait_regs(sb);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float xa = (diag && c * 32 + i > r) ? -CUDART_INF_F : __uint_as_float(sa[i]);
          const float xb = (diag && c * 32 + 32 + i > r) ? -CUDART_INF_F : __uint_as_float(sb[i]);
          m8[i & 7] = fmaxf(m8[i & 7], fmaxf(xa, xb));
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * scale_log2;
      // Lazy rescaling: move the reference max only when it is exceeded by the threshold.
      float corr = 1.0f;
      bool need = false;
      if (j == 0) {
        m_run = mx;  // key block 0 holds key 0 <= every query, so mx is finite
      } else if (mx > m_run + FA_RESCALE_THRESHOLD) {
        need = true;
        corr = exp2_mufu(m_run - mx);
        m_run = mx;
        l_run *= corr;
      }
      const float neg_m = -m_run;
      // pass 2: P = 2^(s c - m) chunk by chunk (the next chunk's scores in flight), row
      // sum, P as fp16 pairs over the scores already read (chunk c -> columns 16c..16c+15)
      float l8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint32_t cur[32], nxt[32];
      tmem_ld_32x32b_x32(t_s, cur);
      tmem_ld_wait_regs(cur);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c + 1 < 4) tmem_ld_32x32b_x32(t_s + (c + 1) * 32, nxt);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float s0 = (diag && c * 32 + i > r) ? -CUDART_INF_F : __uint_as_float(cur[i]);
          const float s1 = (diag && c * 32 + i + 1 > r) ? -CUDART_INF_F : __uint_as_float(cur[i + 1]);
          const float p0 = exp2_mufu(fmaf(s0, scale_log2, neg_m));
          const float p1 = exp2_mufu(fmaf(s1, scale_log2, neg_m));
          l8[(i >> 1) & 7] += p0 + p1;
          pk[i >> 1] = pack_half2(p0, p1);
        }
        tmem_st_32x32b_x16(t_s + c * 16, pk);
        if (c + 1 < 4) {
          tmem_ld_wait_regs(nxt);
#pragma unroll
          for (int i = 0; i < 32; ++i) cur[i] = nxt[i];
        }
      }
      l_run += ((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7]));
      // O holds this tile's P V of the blocks before (PV_t(j-1) was issued before S_t(j)
      // and is complete): rescale it if any row of the warp needs it.
      if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(t_o + c * 32, o);
          tmem_ld_wait_regs(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
          tmem_st_32x32b_x32(t_o + c * 32, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    // ---------------- the tile's output: O / l in fp16 into its Q buffer (every S of the
    // tile completed before its last PV), 128-byte swizzled like the output tensor map
    // (two 64-column halves of [128 rows][128 B]), then one TMA store of the tile.
    const bool fin = ok && mbar_wait(&o_final[t], 0, err);
    uint8_t* obuf = smem + FA_Q_OFF + t * 32768;
    if (fin) {
      tc_fence_after();
      const float inv = 1.0f / l_run;
      // Log-sum-exp of the scaled scores in base 2 (lse2 = log2 sum_k 2^(s_k c)), kept
      // for the backward pass: P = 2^(s c - lse2).
      if (lse) lse[q_row_of(t) + r] = m_run + log2f(l_run);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(t_o + c * 32, o);
        tmem_ld_wait_regs(o);
        uint8_t* half_tile = obuf + (c >> 1) * 16384 + r * 128;
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
    // the four warps of this tile (every warp of the group reaches it, done or not)
    if (t == 0) named_barrier_sync_c<1>(128);
    else named_barrier_sync_c<2>(128);
    if (fin && quad == 2 && lane == 0) {  // the group's first warp (warp 2 or 6)
      const int o_row = b * seq + qt * FA_BQ;
      tma_store_2d(&tmO, obuf, h * 128, o_row);
      tma_store_2d(&tmO, obuf + 16384, h * 128 + 64, o_row);
      bulk_commit_group();
      bulk_wait_all();  // shared memory stays alive until the store has completed
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
