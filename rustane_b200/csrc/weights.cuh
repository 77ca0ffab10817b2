// Device weight layout and the kernels that fill it.
//
// Storage (fp16 unless noted), every GEMM B operand K-major ([N, K] row-major):
//   embed [vocab, dim]                 gather table and tied LM-head B operand
//   wqkv  [L, q_dim + 2*kv_dim, dim]   rows: Wq^T, Wk^T, Wv^T
//   wo    [L, dim, q_dim]              Wo^T
//   w13   [L, 2*hidden, dim]           row 2j = W1[:, j], row 2j+1 = W3[:, j]
//   w2    [L, dim, hidden]             W2 as the reference stores it (used as G * W2^T)
//   gamma [L, 2, dim] fp32, gamma_final [dim] fp32
// Element (r, c) of a storage tensor maps back to one element of a reference
// tensor (orientation of crates/engine/src/layer.rs:52-63); both the on-device
// generator and the host-f32 upload use that mapping, so a tensor-parallel rank
// generates exactly its slice of the single-GPU model.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "weight_init.h"

namespace cb {

enum StoreKind : int { ST_EMBED = 0, ST_QKV = 1, ST_WO = 2, ST_W13 = 3, ST_W2 = 4 };

// Local (this rank's) and global sizes. Under tensor parallelism a rank holds
// q heads [q_off/128, +q_dim/128), kv heads [kv_off/128, +kv_dim/128) and hidden
// columns [hid_off, +hidden); single-GPU contexts have zero offsets and local == global.
struct ShapeInfo {
  int dim, hidden, q_dim, kv_dim, vocab;          // local
  int hidden_g, q_dim_g, kv_dim_g;                // global (reference tensor shapes)
  int q_off, kv_off, hid_off;                     // this rank's offsets
};

struct RefElem {
  int kind;       // cb_tensor_kind, or -1 for the embedding
  uint64_t idx;   // element index in the reference tensor
  uint64_t len;   // reference tensor length
};

__host__ __device__ __forceinline__ RefElem ref_of_storage(int st, int r, int c,
                                                           const ShapeInfo& s) {
  RefElem e;
  switch (st) {
    case ST_EMBED:
      e.kind = -1; e.idx = (uint64_t)r * s.dim + c; e.len = (uint64_t)s.vocab * s.dim;
      break;
    case ST_QKV:
      if (r < s.q_dim) {
        e.kind = CB_T_WQ; e.idx = (uint64_t)c * s.q_dim_g + s.q_off + r;
        e.len = (uint64_t)s.dim * s.q_dim_g;
      } else if (r < s.q_dim + s.kv_dim) {
        e.kind = CB_T_WK; e.idx = (uint64_t)c * s.kv_dim_g + s.kv_off + (r - s.q_dim);
        e.len = (uint64_t)s.dim * s.kv_dim_g;
      } else {
        e.kind = CB_T_WV; e.idx = (uint64_t)c * s.kv_dim_g + s.kv_off + (r - s.q_dim - s.kv_dim);
        e.len = (uint64_t)s.dim * s.kv_dim_g;
      }
      break;
    case ST_WO:  // storage (n, k) = Wo[q_off + k, n]
      e.kind = CB_T_WO; e.idx = (uint64_t)(s.q_off + c) * s.dim + r;
      e.len = (uint64_t)s.q_dim_g * s.dim;
      break;
    case ST_W13:  // row 2j / 2j+1 = W1 / W3 column hid_off + j
      e.kind = (r & 1) ? CB_T_W3 : CB_T_W1; e.idx = (uint64_t)c * s.hidden_g + s.hid_off + (r >> 1);
      e.len = (uint64_t)s.dim * s.hidden_g;
      break;
    default:  // ST_W2: storage (n, k) = W2[n, hid_off + k]
      e.kind = CB_T_W2; e.idx = (uint64_t)r * s.hidden_g + s.hid_off + c;
      e.len = (uint64_t)s.dim * s.hidden_g;
      break;
  }
  return e;
}

struct InitParams {
  uint64_t seed;
  int scheme;        // CB_INIT_NORMAL / CB_INIT_REFERENCE (values of cuda_bridge.h)
  float normal_mul;  // sigma / CB_IRWIN_HALL4_STD, rounded to f32 on the host
  float scale_embed, scale_qkv, scale_ffn;  // reference scheme scales (host-computed f32)
};

// Fill one storage tensor [rows, cols] of layer `layer` (grid-stride).
__global__ void init_weight_kernel(__half* __restrict__ out, int st, int layer, int rows, int cols,
                                   ShapeInfo s, InitParams p) {
  const uint64_t total = (uint64_t)rows * cols;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    const RefElem e = ref_of_storage(st, r, c, s);
    uint16_t bits;
    if (p.scheme == 0) {
      const uint64_t tid = cb_tensor_id(e.kind < 0 ? -1 : layer, e.kind < 0 ? 0 : e.kind);
      bits = cb_normal_f16(p.seed, tid, e.idx, p.normal_mul);
    } else {
      float scale;
      if (e.kind < 0) scale = p.scale_embed;
      else if (e.kind <= CB_T_WV) scale = p.scale_qkv;
      else if (e.kind == CB_T_W1 || e.kind == CB_T_W3) scale = p.scale_ffn;
      else scale = 0.f;  // Wo, W2: zero init (layer.rs:1515,1518)
      bits = (scale == 0.f) ? (uint16_t)0 : cb_lcg_f16(e.len, e.idx, scale);
    }
    out[i] = __ushort_as_half(bits);
  }
}

// Convert one reference-orientation f32 tensor `src` into its storage slots.
// `sub` selects which reference tensor of a fused storage tensor src holds
// (cb_tensor_kind, or -1 for the embedding).
__global__ void load_weight_kernel(__half* __restrict__ out, int st, int rows, int cols,
                                   ShapeInfo s, int sub, const float* __restrict__ src) {
  const uint64_t total = (uint64_t)rows * cols;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    const RefElem e = ref_of_storage(st, r, c, s);
    if (e.kind != sub) continue;
    out[i] = __ushort_as_half(cb_f32_to_f16_bits(src[e.idx]));
  }
}

__global__ void fill_f32_kernel(float* __restrict__ out, size_t n, float v) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = v;
}

}  // namespace cb
