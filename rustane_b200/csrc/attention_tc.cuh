// Causal self-attention forward on the 5th-generation tensor cores (tcgen05/TMEM),
// head_dim 128, online softmax. Same math as attention.cuh (the reference sdpaFwd
// graph, crates/engine/src/kernels/sdpa_fwd.rs:223-258: scores * 1/sqrt(hd), causal
// mask, softmax, P*V); masked keys are skipped, not added as -65504.
//
// Work item = one block of 256 query rows of one (batch, head): two 128-row query tiles
// Q0, Q1 (tiles 2m and 2m+1), worked on at the same time by two softmax warpgroups and
// fed by one stream of 128-key blocks K_j, V_j shared by both (a block of seq % 256 ==
// 128 rows at the end of a sequence has tile 0 only). Tile t needs key blocks 0..qt_t;
// the last block of each tile is its diagonal. The MMAs of the two tiles interleave so
// that one tile's softmax always runs while the tensor cores work on the other tile:
//   S0_0, S1_0, [P0_0] PV0_0, S0_1, [P1_0] PV1_0, S1_1, [P0_1] PV0_1, S0_2, ...
// (S_t(j+1) reuses the TMEM columns of P_t(j); tcgen05 MMAs of one thread run in
// order, so it is issued right after PV_t(j), which reads them.)
//
// Persistent: one CTA per SM takes items i, i + grid, i + 2 grid, ... (heaviest items,
// the latest query rows, first). TMEM and the barriers are set up once; the next item's
// Q tile is loaded as soon as the current item's last S of that tile has completed, and
// its K/V blocks stream through the same rings, so one item's tail overlaps the next
// item's start. (A CTA per item spent longer in set-up, cold loads and drain than in its
// few key blocks at seq 512.)
//
// 384 threads (three warpgroups), one CTA per SM (224 KB of shared memory, all 512 TMEM
// columns):
//   warps 0..3    : softmax of tile 0, warps 4..7 : softmax of tile 1 (224 registers a
//                   thread, setmaxnreg); one thread per query row (TMEM lane). Per key
//                   block: all 128 scores of the row loaded from TMEM at once, the row
//                   max, P = 2^(s c - m) in base 2 on the MUFU, the row sum, and P (fp16
//                   pairs) written over the scores. Only the diagonal block takes the
//                   causal mask (a uniform branch). The O row in TMEM is rescaled only
//                   when the running max passes the reference max by 2^8 (lazy
//                   rescaling); by the time S_t(j) is complete, PV_t(j-1) is too (it was
//                   issued before), so O is stable when it is rescaled. At the end of a
//                   tile, O / l in fp16 goes through the warpgroup's 16 KB staging buffer
//                   in two 64-column halves, each written by one TMA store.
//   warp 8 lane 0 : TMA producer: per item Q0, Q1, then per key block j: K_j and V_j into
//                   two-deep rings, 128-byte swizzle.
//   warp 9        : TMEM owner; lane 0 issues the UMMAs:
//                     S_t = Q_t K_j^T   (M=128, N=128 keys, K=128; A and B K-major)
//                     O_t += P_t V_j    (M=128, N=128, K=128 keys; P from TMEM where it
//                                        overwrote S_t, V MN-major from its TMA tile)
//   warps 8..11 run with 56 registers a thread (warps 10 and 11 have no role).
// Every role walks the same item sequence and counts its own barrier phases.
// Layout: q, k, v are [batch, heads, seq, 128] fp16 (rows of a [batch*heads*seq, 128]
// matrix for the tensor maps, K and V in 128-row boxes); the output (tensor map tmO,
// 64-column x 128-row boxes) is [batch*seq, heads*128] fp16. seq % 128 == 0.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <math_constants.h>
#include <stdint.h>

#include <type_traits>

#include "ptx.cuh"

namespace cb {

constexpr int FA_BQ = 128;   // query rows per tile
constexpr int FA_BKV = 128;  // keys per block (rows of the K and V tensor-map boxes)
constexpr int FA_THREADS = 384;
// setmaxnreg budget: 2 x 128 x 224 + 128 x 56 = 64512 = 384 x 168 registers at launch
constexpr int FA_SOFTMAX_REGS = 224;
constexpr int FA_CONTROL_REGS = 56;
// shared memory map (bytes from the 1024-aligned base)
constexpr int FA_Q_OFF = 0;        // 2 tiles x 32 KB: head dims 0-63 | 64-127, [128 rows][128 B]
constexpr int FA_K_OFF = 65536;    // 2 slots x 32 KB: dims 0-63 | 64-127, [128 keys][128 B]
constexpr int FA_V_OFF = 131072;   // 2 slots x 32 KB, same layout (read MN-major)
constexpr int FA_STAGE_OFF = 196608;  // 2 x 16 KB output staging, one per softmax warpgroup
constexpr int FA_BAR_OFF = 229376;
constexpr int FA_SMEM = FA_BAR_OFF + 256 + 1024;
constexpr uint32_t FA_TMEM_COLS = 512;  // S0/P0 [0,128) S1/P1 [128,256) O0 [256,384) O1 [384,512)

// The O accumulator and row sum keep a stale reference max until the running max
// exceeds it by this much (base-2 log): P values stay <= 2^8, and most blocks skip
// the TMEM read-scale-write of O.
constexpr float FA_RESCALE_THRESHOLD = 8.0f;

// Blocks of 256 query rows per sequence.
__host__ __device__ constexpr int fa_blocks(int seq) { return (seq / FA_BQ + 1) / 2; }

// One work item: block mb of (batch b, head h); heaviest (largest mb) first.
struct FaItem {
  int mb, b, h, n_t, n_steps;
  __device__ FaItem(int w, int seq, int heads, int batch) {
    const int n_blk = fa_blocks(seq);
    const int hb_count = heads * batch;
    mb = n_blk - 1 - w / hb_count;
    const int hb = w % hb_count;
    b = hb / heads;
    h = hb - b * heads;
    n_t = (2 * mb + 1 < seq / FA_BQ) ? 2 : 1;  // query tiles in this block
    n_steps = 2 * mb + n_t;                    // key blocks (tile n_t - 1 needs them all)
  }
  __device__ int qt(int t) const { return 2 * mb + t; }
  __device__ bool active(int t, int j) const { return t < n_t && j <= qt(t); }
};

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
  uint64_t* q_full = bars + 0;    // [2] per tile: Q_t loaded
  uint64_t* q_free = bars + 2;    // [2] per tile: the item's S_t MMAs done (Q_t reusable)
  uint64_t* k_full = bars + 4;    // [2] per slot
  uint64_t* k_empty = bars + 6;   // [2]
  uint64_t* v_full = bars + 8;    // [2]
  uint64_t* v_empty = bars + 10;  // [2]
  uint64_t* s_full = bars + 12;   // [2] per tile
  uint64_t* p_full = bars + 14;   // [2] per tile (one arrival per softmax warp)
  uint64_t* o_final = bars + 16;  // [2] per tile: the item's last PV_t is done
  uint64_t* drain = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_items = fa_blocks(seq) * heads * batch;
  const int group = heads / kv_heads;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_free[i], 1);
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
  if (warp == 9) {
    tmem_alloc(tmem_slot, FA_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_enter();  // lets the next GEMM (launched with PDL) schedule its CTAs early

  if (warp >= 8) {
    regs_dec<FA_CONTROL_REGS>();  // the whole warpgroup 8..11
    if (warp == 8 && lane == 0) {
      // ---------------- producer: per item Q0, Q1 (each once the previous item's S MMAs of
      // that tile are done), then K_j and V_j one block ahead through the rings
      uint32_t g = 0;        // key blocks loaded so far (ring position)
      uint32_t q_loads = 0;  // Q tiles loaded so far: tile 0 in bits 0..15, tile 1 in 16..31
      bool ok = true;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
        const FaItem it(w, seq, heads, batch);
        const int q_row0 = (it.b * heads + it.h) * seq;
        const int kv_row0 = (it.b * kv_heads + it.h / group) * seq;
        for (int t = 0; t < it.n_t && ok; ++t) {
          const uint32_t nq = (q_loads >> (16 * t)) & 0xffffu;
          if (nq > 0 && !mbar_wait(&q_free[t], (nq - 1) & 1, err)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + FA_Q_OFF + t * 32768;
          mbar_arrive_expect_tx(&q_full[t], 32768);
          tma_load_2d(dst, &tmQ, &q_full[t], 0, q_row0 + it.qt(t) * FA_BQ);
          tma_load_2d(dst + 16384, &tmQ, &q_full[t], 64, q_row0 + it.qt(t) * FA_BQ);
          q_loads += 1u << (16 * t);
        }
        for (int j = 0; j < it.n_steps && ok; ++j, ++g) {
          const int sl = g & 1;
          const uint32_t ph = ((g >> 1) & 1) ^ 1u;
          const int row = kv_row0 + j * FA_BKV;
          if (!mbar_wait(&k_empty[sl], ph, err)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[sl], 32768);
          uint8_t* kd = smem + FA_K_OFF + sl * 32768;
          tma_load_2d(kd, &tmK, &k_full[sl], 0, row);
          tma_load_2d(kd + 16384, &tmK, &k_full[sl], 64, row);
          if (!mbar_wait(&v_empty[sl], ph, err)) { ok = false; break; }
          mbar_arrive_expect_tx(&v_full[sl], 32768);
          uint8_t* vd = smem + FA_V_OFF + sl * 32768;
          tma_load_2d(vd, &tmV, &v_full[sl], 0, row);
          tma_load_2d(vd + 16384, &tmV, &v_full[sl], 64, row);
        }
      }
    } else if (warp == 9 && lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc_s = umma_idesc_f16(FA_BQ, FA_BKV);
      constexpr uint32_t idesc_pv = umma_idesc_f16_bmn(FA_BQ, 128);
      uint32_t g = 0;       // key blocks of earlier items (ring position)
      uint32_t q_uses = 0;  // Q tiles consumed so far, one bit of parity per tile (bit t)
      uint32_t steps = 0;   // key blocks of each tile so far, parity per tile (p_full phase)
      bool ok = true;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
        const FaItem it(w, seq, heads, batch);
        const int last_t = it.n_t - 1;  // the tile that uses every key block last
        auto issue_s = [&](int t, int j) -> bool {
          const uint32_t gj = g + (uint32_t)j;
          if (j == 0) {
            if (!mbar_wait(&q_full[t], (q_uses >> t) & 1u, err)) return false;
            q_uses ^= 1u << t;
          }
          if (!mbar_wait(&k_full[gj & 1], (gj >> 1) & 1, err)) return false;
          tc_fence_after();
          const uint32_t q_addr = smem_u32(smem + FA_Q_OFF + t * 32768);
          const uint32_t k_addr = smem_u32(smem + FA_K_OFF + (gj & 1) * 32768);
#pragma unroll
          for (int k = 0; k < 8; ++k) {  // head dim in steps of 16
            const uint32_t off = (uint32_t)((k >> 2) * 16384 + (k & 3) * 32);
            umma_f16_ss(tmem + (uint32_t)(t * 128), sw128_kmajor_desc(q_addr + off),
                        sw128_kmajor_desc(k_addr + off), idesc_s, k != 0);
          }
          umma_commit(&s_full[t]);
          if (t == last_t) umma_commit(&k_empty[gj & 1]);  // both tiles' S of block j issued
          if (j == it.qt(t)) umma_commit(&q_free[t]);      // the item's last S of tile t
          return true;
        };
        auto issue_pv = [&](int t, int j) -> bool {
          const uint32_t gj = g + (uint32_t)j;
          if (!mbar_wait(&p_full[t], (steps >> t) & 1u, err)) return false;
          steps ^= 1u << t;
          if (!mbar_wait(&v_full[gj & 1], (gj >> 1) & 1, err)) return false;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + FA_V_OFF + (gj & 1) * 32768);
          const uint32_t p_tmem = tmem + (uint32_t)(t * 128);  // P over S_t's columns
#pragma unroll
          for (int k = 0; k < FA_BKV / 16; ++k)  // keys in steps of 16 (8 packed columns)
            umma_f16_ts(tmem + 256u + (uint32_t)(t * 128), p_tmem + k * 8,
                        sw128_mnmajor_desc(v_addr + k * 2048, 16384), idesc_pv, (j | k) != 0);
          if (t == last_t) umma_commit(&v_empty[gj & 1]);
          if (j == it.qt(t)) umma_commit(&o_final[t]);
          return true;
        };
        for (int t = 0; t < it.n_t && ok; ++t) ok = issue_s(t, 0);
        for (int j = 0; j < it.n_steps && ok; ++j) {
          for (int t = 0; t < 2 && ok; ++t) {
            if (!it.active(t, j)) continue;
            ok = issue_pv(t, j);
            if (ok && it.active(t, j + 1)) ok = issue_s(t, j + 1);
          }
        }
        g += (uint32_t)it.n_steps;
      }
      // Drain: every MMA issued here completes before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, err);
    }
  } else {
    regs_inc<FA_SOFTMAX_REGS>();
    // ---------------- softmax warpgroups: thread = query row r (TMEM lane r) of tile t
    const int t = warp >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t t_s = tmem + lane_off + (uint32_t)(t * 128);
    const uint32_t t_o = tmem + lane_off + 256u + (uint32_t)(t * 128);
    uint8_t* stage = smem + FA_STAGE_OFF + t * 16384;  // [128 rows][128 B], 128-byte swizzle
    uint32_t steps = 0, tiles = 0;  // s_full and o_final phases
    bool ok = true;
    // Every warp of the group walks every item and reaches every named barrier whether or
    // not an earlier wait failed (a failed wait only skips the work), so no warp is ever
    // left waiting at a barrier for a warp that stopped.
    for (int w = blockIdx.x; w < n_items; w += gridDim.x) {
      const FaItem it(w, seq, heads, batch);
      if (t >= it.n_t) continue;
      const int qt = it.qt(t);
      float m_run = -CUDART_INF_F, l_run = 0.f;
      int j = 0;
      float corr = 1.0f;
      bool need = false;
      // One key block: all 128 scores of the row from TMEM (four loads in flight, one
      // wait), the row max of the raw scores (the scale > 0 commutes with max), the lazy
      // rescale decision, then P = 2^(s c - m) on the MUFU, the row sum and P as fp16
      // pairs over the scores (chunk c -> columns 16c..16c+15). Scores and exponent
      // arguments go two lanes per instruction (f32x2) where the math allows.
      auto softmax_block = [&](auto masked) {
        constexpr bool MASK = decltype(masked)::value;
        uint32_t sv[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(t_s + c * 32, sv[c]);
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_wait_regs(sv[c]);
        if constexpr (MASK) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c * 32 + i > r) sv[c][i] = __float_as_uint(-CUDART_INF_F);
        }
        float m4[4] = {-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F};
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; i += 2)
            m4[(i >> 1) & 3] = fmax3(m4[(i >> 1) & 3], __uint_as_float(sv[c][i]),
                                     __uint_as_float(sv[c][i + 1]));
        const float mx = fmax3(m4[0], m4[1], fmaxf(m4[2], m4[3])) * scale_log2;
        // Lazy rescaling: move the reference max only when it is exceeded by the threshold.
        corr = 1.0f;
        need = false;
        if (j == 0) {
          m_run = mx;  // key block 0 holds key 0 <= every query, so mx is finite
        } else if (mx > m_run + FA_RESCALE_THRESHOLD) {
          need = true;
          corr = exp2_mufu(m_run - mx);
          m_run = mx;
          l_run *= corr;
        }
        const float2 sc2 = make_float2(scale_log2, scale_log2);
        const float2 nm2 = make_float2(-m_run, -m_run);
        float2 l4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                        make_float2(0.f, 0.f)};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 x = ffma2(
                make_float2(__uint_as_float(sv[c][i]), __uint_as_float(sv[c][i + 1])), sc2, nm2);
            const float2 pp = make_float2(exp2_mufu(x.x), exp2_mufu(x.y));
            l4[(i >> 1) & 3] = fadd2(l4[(i >> 1) & 3], pp);
            pk[i >> 1] = pack_half2(pp.x, pp.y);
          }
          tmem_st_32x32b_x16(t_s + c * 16, pk);
        }
        const float2 la = fadd2(l4[0], l4[1]), lb = fadd2(l4[2], l4[3]);
        l_run += (la.x + la.y) + (lb.x + lb.y);
      };
      for (; ok && j <= qt; ++j) {
        if (!mbar_wait(&s_full[t], steps++ & 1, err)) { ok = false; break; }
        tc_fence_after();
        // The diagonal block (j == qt) masks keys 128 j + i with i > r; every other block
        // takes the variant without the mask (a uniform branch: no per-element selects).
        if (j == qt) softmax_block(std::true_type{});
        else softmax_block(std::false_type{});
        // O holds this tile's P V of the blocks before (PV_t(j-1) was issued before
        // S_t(j) and is complete): rescale it if any row of the warp needs it.
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
      // ---------------- the tile's output: O / l in fp16, 64 columns at a time through
      // the 16 KB staging buffer (128-byte swizzled like the output tensor map), each
      // half written by one TMA store. O is read completely before the next item's first
      // P of this tile is handed over, which is when its first PV may overwrite O.
      const bool fin = ok && mbar_wait(&o_final[t], tiles++ & 1, err);
      ok = ok && fin;
      const int o_row = it.b * seq + qt * FA_BQ;
      if (fin) {
        tc_fence_after();
        if (lse) lse[(it.b * heads + it.h) * seq + qt * FA_BQ + r] = m_run + log2f(l_run);
      }
      const float inv = 1.0f / l_run;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t o[2][32];
        if (fin) {
          tmem_ld_32x32b_x32(t_o + half * 64, o[0]);
          tmem_ld_32x32b_x32(t_o + half * 64 + 32, o[1]);
          tmem_ld_wait_regs(o[0]);
          tmem_ld_wait_regs(o[1]);
          // the staging buffer's previous store (if any) has finished reading it
          if (quad == 0 && lane == 0) bulk_wait_read<0>();
        }
        // the four warps of this tile (every warp of the group reaches both barriers,
        // done or not)
        if (t == 0) named_barrier_sync_c<1>(128);
        else named_barrier_sync_c<2>(128);
        if (fin) {
          uint8_t* row_p = stage + r * 128;
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t* q = o[c] + 8 * k;
              uint4 v4;
              v4.x = pack_half2(__uint_as_float(q[0]) * inv, __uint_as_float(q[1]) * inv);
              v4.y = pack_half2(__uint_as_float(q[2]) * inv, __uint_as_float(q[3]) * inv);
              v4.z = pack_half2(__uint_as_float(q[4]) * inv, __uint_as_float(q[5]) * inv);
              v4.w = pack_half2(__uint_as_float(q[6]) * inv, __uint_as_float(q[7]) * inv);
              const int chunk = c * 4 + k;  // 16-byte chunk within the 128-byte row
              *reinterpret_cast<uint4*>(row_p + ((chunk ^ (r & 7)) << 4)) = v4;
            }
        }
        fence_proxy_async_smem();
        if (t == 0) named_barrier_sync_c<1>(128);
        else named_barrier_sync_c<2>(128);
        if (fin && quad == 0 && lane == 0) {
          tma_store_2d(&tmO, stage, it.h * 128 + half * 64, o_row);
          bulk_commit_group();
        }
      }
    }
    if (quad == 0 && lane == 0) bulk_wait_all();  // stores complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, FA_TMEM_COLS);
  }
}

}  // namespace cb
