// Deterministic weight generators shared by the CUDA bridge and the CPU oracle.
//
// Everything here is integer arithmetic plus single correctly-rounded float
// operations, so host (gcc) and device (nvcc) builds produce bit-identical
// fp16 weights from the same (seed, tensor, index) triple. Weights are never
// shipped between the two sides: each side regenerates them.
//
// Two schemes:
//   CB_INIT_NORMAL    : ~N(0, sigma) for every matrix (embedding, Wq/Wk/Wv/Wo,
//                       W1/W3/W2), RMSNorm gains 1.0. The normal is an
//                       Irwin-Hall sum of four 16-bit uniforms taken from one
//                       splitmix64 hash of (seed, tensor id, element index).
//   CB_INIT_REFERENCE : the reference engine's own init. Its LCG
//                       (crates/engine/src/full_model.rs:1473-1484, identical
//                       copy at crates/engine/src/layer.rs:1556-1567) seeds
//                       each tensor with 42 + len and steps
//                       s = s*6364136223846793005 + 1442695040888963407 once
//                       before every element; value = ((s>>32)/u32::MAX*2-1)*scale.
//                       Scales follow ModelWeights::random (full_model.rs:132-141,
//                       embedding 0.005) and LayerWeights::random
//                       (layer.rs:1509-1524: Wq/Wk/Wv 1/sqrt(dim), W1/W3
//                       1/sqrt(hidden), Wo = W2 = 0).
//
// Element indices are in the reference orientation (row-major):
//   embed [vocab, dim]; wq [dim, q_dim]; wk, wv [dim, kv_dim]; wo [q_dim, dim];
//   w1, w3, w2 [dim, hidden]   (crates/engine/src/layer.rs:52-63).
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define CB_HD __host__ __device__ __forceinline__
#else
#define CB_HD static inline
#endif

enum cb_tensor_kind {
  CB_T_WQ = 0, CB_T_WK = 1, CB_T_WV = 2, CB_T_WO = 3,
  CB_T_W1 = 4, CB_T_W3 = 5, CB_T_W2 = 6
};

// Tensor ids mixed into the hash. The embedding is id 1; layer tensors follow.
CB_HD uint64_t cb_tensor_id(int layer, int kind) {
  return (layer < 0) ? 1ull : (16ull + (uint64_t)layer * 8ull + (uint64_t)kind);
}

CB_HD uint64_t cb_splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

CB_HD uint32_t cb_f32_bits(float f) {
  union { float f; uint32_t u; } v; v.f = f; return v.u;
}
CB_HD float cb_bits_f32(uint32_t u) {
  union { float f; uint32_t u; } v; v.u = u; return v.f;
}

// IEEE binary32 -> binary16, round to nearest even, with subnormals, inf, nan.
CB_HD uint16_t cb_f32_to_f16_bits(float f) {
  uint32_t x = cb_f32_bits(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return (uint16_t)(sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u));
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // >= 65520 rounds to inf
  if (ax < 0x38800000u) {                                     // below 2^-14: subnormal half
    if (ax < 0x33000000u) return (uint16_t)sign;              // <= 2^-25 rounds to zero
    uint32_t e = ax >> 23;                                    // 102..112
    uint32_t mant = (ax & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126u - e;                                // 14..24
    uint32_t m = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (m & 1u))) m++;
    return (uint16_t)(sign | m);
  }
  uint32_t e = (ax >> 23) - 112u;                             // rebias 127 -> 15
  uint32_t mant = ax & 0x7FFFFFu;
  uint32_t h = (e << 10) | (mant >> 13);
  uint32_t rem = mant & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

// binary16 -> binary32 (exact).
CB_HD float cb_f16_bits_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t e = ((uint32_t)h >> 10) & 0x1Fu;
  uint32_t m = (uint32_t)h & 0x3FFu;
  if (e == 0x1Fu) return cb_bits_f32(sign | 0x7F800000u | (m << 13));
  if (e == 0) {
    if (m == 0) return cb_bits_f32(sign);
    // subnormal: normalise
    int shift = 0;
    while ((m & 0x400u) == 0) { m <<= 1; shift++; }
    m &= 0x3FFu;
    return cb_bits_f32(sign | ((uint32_t)(113 - shift) << 23) | (m << 13));
  }
  return cb_bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}

// ---- scheme CB_INIT_NORMAL -------------------------------------------------

// Standard deviation of a sum of four independent uniforms on {0..65535}.
#define CB_IRWIN_HALL4_STD 37837.22679262339
#define CB_IRWIN_HALL4_MEAN 131070

// fp16 bits of element `index` of tensor `tid`. `mul` = sigma / CB_IRWIN_HALL4_STD
// rounded to float (computed once by the caller so both sides use the same constant).
CB_HD uint16_t cb_normal_f16(uint64_t seed, uint64_t tid, uint64_t index, float mul) {
  uint64_t h = cb_splitmix64(cb_splitmix64(seed ^ (tid * 0xD1B54A32D192ED03ull)) + index);
  int32_t s = (int32_t)(h & 0xFFFFu) + (int32_t)((h >> 16) & 0xFFFFu) +
              (int32_t)((h >> 32) & 0xFFFFu) + (int32_t)((h >> 48) & 0xFFFFu);
  float c = (float)(s - CB_IRWIN_HALL4_MEAN);  // exact: |c| < 2^18
#if defined(__CUDA_ARCH__)
  float v = __fmul_rn(c, mul);
#else
  float v = c * mul;
#endif
  return cb_f32_to_f16_bits(v);
}

// ---- scheme CB_INIT_REFERENCE (the reference's LCG) -------------------------

#define CB_LCG_A 6364136223846793005ull
#define CB_LCG_C 1442695040888963407ull

// State after `k` LCG steps from `s0` (affine-map exponentiation; exact mod 2^64).
CB_HD uint64_t cb_lcg_jump(uint64_t s0, uint64_t k) {
  uint64_t acc_a = 1, acc_c = 0;           // accumulated map x -> acc_a*x + acc_c
  uint64_t cur_a = CB_LCG_A, cur_c = CB_LCG_C;
  while (k) {
    if (k & 1ull) { acc_a = acc_a * cur_a; acc_c = acc_c * cur_a + cur_c; }
    cur_c = cur_c * cur_a + cur_c;
    cur_a = cur_a * cur_a;
    k >>= 1;
  }
  return acc_a * s0 + acc_c;
}

CB_HD uint64_t cb_lcg_step(uint64_t s) { return s * CB_LCG_A + CB_LCG_C; }

// f32 value the reference produces from LCG state `s` (already advanced) and `scale`.
CB_HD float cb_lcg_value(uint64_t s, float scale) {
  uint32_t hi = (uint32_t)(s >> 32);
#if defined(__CUDA_ARCH__)
  float a = __uint2float_rn(hi);
  float r = __fadd_rn(__fmul_rn(__fdiv_rn(a, 4294967296.0f), 2.0f), -1.0f);
  return __fmul_rn(r, scale);
#else
  volatile float a = (float)hi;                // u32 -> f32, round to nearest
  volatile float b = a / 4294967296.0f;        // u32::MAX as f32 == 2^32
  volatile float r2 = b * 2.0f;
  volatile float r = r2 - 1.0f;
  return r * scale;
#endif
}

// fp16 bits of element `index` of a reference-LCG tensor of `len` elements.
CB_HD uint16_t cb_lcg_f16(uint64_t len, uint64_t index, float scale) {
  uint64_t s = cb_lcg_jump(42ull + len, index + 1ull);
  return cb_f32_to_f16_bits(cb_lcg_value(s, scale));
}
