// Causal self-attention forward on the 5th-generation tensor cores (tcgen05/TMEM),
// head_dim 128, online softmax. Same math as attention.cuh (the reference sdpaFwd
// graph, crates/engine/src/kernels/sdpa_fwd.rs:223-258: scores * 1/sqrt(hd), causal
// mask, softmax, P*V); masked keys are skipped, not added as -65504.
//
// Persistent: the work items are single 128-query tiles of one (batch, head). The host
// gives every CTA a list of tiles (a schedule table, see attn_schedule in bridge.cu):
// tiles are taken in chunks of heads whose K and V fit in L2 together, the latest (most
// key steps) tiles of a chunk first, each assigned to the CTA with the least work so far,
// so the CTAs finish within about one small tile of each other and the tiles that run at
// the same time share their K and V through L2 (a CTA per pair of tiles left up to a
// third of the SMs idle in the last wave at 8-64 sequences of 512; heaviest-first over
// all heads at once re-read K and V from HBM for every tile). One tile's output is
// written while the next tile's first Q K^T runs: the next Q is loaded as soon as the
// tile's last S is done, the output is staged in the V buffers (the next tile's first V
// waits for the store to have read them). 96 KB of shared memory and 256 TMEM columns,
// so two CTAs share an SM (grid = min(tiles, 2 x SMs)).
// 192 threads:
//   warp 0 lane 0 : TMA producer. Per tile its Q (128 x 128), then per 64-key step j:
//                   K_j one step ahead of V_j (both double-buffered), 128-byte swizzle.
//   warp 1        : TMEM owner; lane 0 issues the UMMAs:
//                     S_j = Q K_j^T   (M=128, N=64, K=128; A and B K-major) into one of
//                                      two TMEM S buffers, S_{j+1} issued before P_j is
//                                      ready so it overlaps the softmax of step j (at a
//                                      tile boundary the tile's last PV goes first: the
//                                      next tile's S needs its Q, loaded only then)
//                     O  += P_j V_j   (M=128, N=128, K=64; P read from TMEM, where it
//                                      overwrites S_j, V MN-major from its TMA tile)
//   warps 2..5    : softmax, one thread per query row (TMEM lane): reads its 64 scores,
//                   applies the causal mask on the diagonal steps, updates the running
//                   max / sum in base 2 (exponentials on the MUFU), rescales its O row in
//                   TMEM only when the max grows past the reference max by 2^8, writes P
//                   (fp16, packed in pairs) over its S row in TMEM, and at the end of a
//                   tile divides O by the row sum into the V buffers' shared memory, from
//                   where one TMA store per 64 columns writes the 128 x 128 output tile.
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

// The sequence of 64-key steps one CTA works through: its tiles (see above) one after
// the other. Every role keeps its own cursor and advances it in the same order.
// The 64-key steps one CTA works through: the tiles of its list in the schedule table
// (sched: [gridDim.x + 1] offsets into the items that follow them; an item is
// (batch * heads + head) * n_qt + query tile), one after the other. Every role keeps its
// own cursor and advances it in the same order.
struct FaCursor {
  const int* p;    // current item
  const int* end;  // end of this CTA's list
  int n_qt, heads;
  int ord;  // tiles of this CTA before the current one
  int qt, b, h, kt, n_kt;
  __device__ FaCursor(const int* __restrict__ sched, int seq, int heads_)
      : n_qt(seq / 128), heads(heads_), ord(0) {
    const int* items = sched + gridDim.x + 1;
    p = items + __ldg(sched + blockIdx.x);
    end = items + __ldg(sched + blockIdx.x + 1);
    pick();
  }
  __device__ void pick() {
    if (p < end) {
      const int w = __ldg(p);
      const int hb = w / n_qt;
      qt = w - hb * n_qt;
      b = hb / heads;
      h = hb - b * heads;
      kt = 0;
      n_kt = (qt + 1) * (128 / 64);
    }
  }
  __device__ bool valid() const { return p < end; }
  __device__ bool last_step() const { return kt == n_kt - 1; }
  __device__ void next_tile() {
    ++p;
    ++ord;
    pick();
  }
  __device__ void next() {
    if (++kt == n_kt) next_tile();
  }
};

__global__ void __launch_bounds__(FA_THREADS, 2)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmO, int seq, int heads,
                       int kv_heads, const int* __restrict__ sched, float scale_log2,
                       float* __restrict__ lse, int* err) {
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
  uint64_t* q_empty = bars + 14;  // a tile's last S is done: the Q buffer takes the next Q
  uint64_t* o_done = bars + 15;   // a tile's output has left the V buffers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int group = heads / kv_heads;

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
      // ---------------- producer: per tile its Q (once the previous tile's last S is
      // done), K one step ahead of V; a tile's first V once the previous tile's output has
      // left the V buffers
      FaCursor kc(sched, seq, heads), vc(sched, seq, heads);
      uint32_t gk = 0, gv = 0;  // steps loaded (ring positions)
      auto load_k = [&]() -> bool {
        if (kc.kt == 0) {  // the tile's Q first
          if (kc.ord > 0 && !mbar_wait(q_empty, (kc.ord - 1) & 1, err)) return false;
          const int q_row = (kc.b * heads + kc.h) * seq + kc.qt * FA_BQ;
          mbar_arrive_expect_tx(q_full, 32768);
          tma_load_2d(smem + FA_Q_OFF, &tmQ, q_full, 0, q_row);
          tma_load_2d(smem + FA_Q_OFF + 16384, &tmQ, q_full, 64, q_row);
        }
        const int kb = gk & 1;
        if (!mbar_wait(&k_empty[kb], ((gk >> 1) & 1) ^ 1u, err)) return false;
        const int row = (kc.b * kv_heads + kc.h / group) * seq + kc.kt * FA_BKV;
        mbar_arrive_expect_tx(&k_full[kb], 16384);
        uint8_t* dst = smem + FA_K_OFF + kb * 16384;
        tma_load_2d(dst, &tmK, &k_full[kb], 0, row);
        tma_load_2d(dst + 8192, &tmK, &k_full[kb], 64, row);
        kc.next();
        ++gk;
        return true;
      };
      bool ok = !kc.valid() || load_k();
      while (ok && vc.valid()) {
        if (kc.valid() && !load_k()) break;
        const int vb = gv & 1;
        if (!mbar_wait(&v_empty[vb], ((gv >> 1) & 1) ^ 1u, err)) break;
        if (vc.kt == 0 && vc.ord > 0 && !mbar_wait(o_done, (vc.ord - 1) & 1, err)) break;
        const int row = (vc.b * kv_heads + vc.h / group) * seq + vc.kt * FA_BKV;
        mbar_arrive_expect_tx(&v_full[vb], 16384);
        uint8_t* vdst = smem + FA_V_OFF + vb * 16384;
        tma_load_2d(vdst, &tmV, &v_full[vb], 0, row);
        tma_load_2d(vdst + 8192, &tmV, &v_full[vb], 64, row);
        vc.next();
        ++gv;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer: S one step ahead of PV within a tile; at a tile
      // boundary the tile's last PV first (the next tile's first S waits for its Q)
      constexpr uint32_t idesc_s = umma_idesc_f16(FA_BQ, FA_BKV);
      constexpr uint32_t idesc_pv = umma_idesc_f16_bmn(FA_BQ, 128);
      const uint32_t q_addr = smem_u32(smem + FA_Q_OFF);
      const uint32_t k_addr = smem_u32(smem + FA_K_OFF);
      const uint32_t v_addr = smem_u32(smem + FA_V_OFF);
      FaCursor sc(sched, seq, heads), pc(sched, seq, heads);
      uint32_t gs = 0, gp = 0;  // steps issued
      auto issue_s = [&]() -> bool {
        const int kb = gs & 1;
        if (sc.kt == 0 && !mbar_wait(q_full, sc.ord & 1, err)) return false;
        if (!mbar_wait(&k_full[kb], (gs >> 1) & 1, err)) return false;
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
        if (sc.last_step()) umma_commit(q_empty);
        sc.next();
        ++gs;
        return true;
      };
      auto issue_pv = [&]() -> bool {
        const int vb = gp & 1;
        if (!mbar_wait(p_full, gp & 1, err)) return false;
        if (!mbar_wait(&v_full[vb], (gp >> 1) & 1, err)) return false;
        tc_fence_after();
        const uint32_t p_tmem = t_s0 + (uint32_t)(vb * FA_BKV);  // P over S's columns
#pragma unroll
        for (int k = 0; k < FA_BKV / 16; ++k) {  // keys in steps of 16 (8 packed columns)
          umma_f16_ts(t_o, p_tmem + k * 8,
                      sw128_mnmajor_desc(v_addr + vb * 16384 + k * 2048, 8192), idesc_pv,
                      (pc.kt | k) != 0);
        }
        umma_commit(&v_empty[vb]);
        umma_commit(pv_done);
        pc.next();
        ++gp;
        return true;
      };
      bool ok = !sc.valid() || issue_s();
      while (ok && pc.valid()) {
        // S of the step after the one whose PV is next, unless that step opens a new tile
        const bool s_first = sc.valid() && sc.kt != 0;
        if (s_first && !issue_s()) break;
        if (!issue_pv()) break;
        if (!s_first && sc.valid() && !issue_s()) break;
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
    // Every warp walks every tile and reaches the named barrier of every tile whether or
    // not an earlier wait failed (a failed wait only skips the remaining work).
    FaCursor cur(sched, seq, heads);
    uint32_t g0 = 0;  // steps of the tiles before
    for (; cur.valid(); g0 += (uint32_t)cur.n_kt, cur.next_tile()) {
      const int qt = cur.qt;
      const int q_idx = qt * FA_BQ + r;
      const int n_kv = cur.n_kt;
      float m_run = -CUDART_INF_F, l_run = 0.f;
      for (int jt = 0; jt < n_kv && ok; ++jt) {
        const uint32_t g = g0 + (uint32_t)jt;
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
        const float inv = __fdividef(1.0f, l_run);  // l_run >= 1: the max term is 2^0
        // Log-sum-exp of the scaled scores in base 2 (lse2 = log2 sum_k 2^(s_k c)), kept
        // for the backward pass: P = 2^(s c - lse2).
        if (lse) lse[(cur.b * heads + cur.h) * seq + qt * FA_BQ + r] = m_run + __log2f(l_run);
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
          const int o_row = cur.b * seq + qt * FA_BQ;
          tma_store_2d(&tmO, smem + FA_V_OFF, cur.h * 128, o_row);
          tma_store_2d(&tmO, smem + FA_V_OFF + 16384, cur.h * 128 + 64, o_row);
          bulk_commit_group();
          bulk_wait_read<0>();  // the V buffers stay untouched until the store has read them
        }
        mbar_arrive(o_done);  // the producer may load V again
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
