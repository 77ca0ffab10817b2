// Memory-bound row kernels of the forward pass: one warp per token row,
// 128-bit vector loads/stores, warp-shuffle reductions.
//
//   embed_rmsnorm_kernel : X[t,:] = E[tok[t],:] (fp32 residual) and the layer-0
//                          RMSNorm output Xn = X * rinv * gamma in fp16
//                          (crates/engine/src/cpu/embedding.rs:8-17,
//                           cpu/rmsnorm.rs:149-183, EPS = 1e-5 at :10)
//   add_rmsnorm_kernel   : X += delta (the scaled O / down projection), then the norm
//   ce_finalize_kernel   : per-token loss from the LM-head epilogue partials,
//                          loss_t = log(sum_v e^{z_v - m}) + m - z_tgt
//                          (crates/engine/src/cpu/cross_entropy.rs:58-96)
//   loss_mean_kernel     : fixed-order mean over tokens (deterministic)
#pragma once
#include <cuda_fp16.h>
#include <math_constants.h>
#include <stdint.h>

#include "ptx.cuh"

namespace cb {

constexpr float RMS_EPS = 1e-5f;
constexpr int ROW_WARPS = 8;  // warps per block for the row kernels

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void h8_to_f8(uint4 u, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 f8_to_h8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_half2(f[0], f[1]);
  u.y = pack_half2(f[2], f[3]);
  u.z = pack_half2(f[4], f[5]);
  u.w = pack_half2(f[6], f[7]);
  return u;
}

// dim must be a multiple of 256 (8 elements per lane per step).
__global__ void embed_rmsnorm_kernel(const uint32_t* __restrict__ tokens,
                                     const __half* __restrict__ embed,
                                     const float* __restrict__ gamma, float* __restrict__ x,
                                     __half* __restrict__ xn, int T, int dim, int vocab,
                                     int* err, float* __restrict__ rinv_out = nullptr) {
  pdl_enter();
  const int row = blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  uint32_t tok = tokens[row];
  if (tok >= (uint32_t)vocab) {  // out-of-range token id: report, use row 0
    if (lane == 0) atomicExch(err, 2);
    tok = 0;
  }
  const __half* e = embed + (size_t)tok * dim;
  float* xr = x + (size_t)row * dim;
  float ss = 0.f;
  for (int c = lane * 8; c < dim; c += 256) {
    float f[8];
    h8_to_f8(*reinterpret_cast<const uint4*>(e + c), f);
    *reinterpret_cast<float4*>(xr + c) = make_float4(f[0], f[1], f[2], f[3]);
    *reinterpret_cast<float4*>(xr + c + 4) = make_float4(f[4], f[5], f[6], f[7]);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  ss = warp_sum(ss);
  const float rinv = 1.0f / sqrtf(ss / (float)dim + RMS_EPS);
  if (rinv_out && lane == 0) rinv_out[row] = rinv;
  __half* o = xn + (size_t)row * dim;
  for (int c = lane * 8; c < dim; c += 256) {
    float f[8];
    h8_to_f8(*reinterpret_cast<const uint4*>(e + c), f);
    const float4 g0 = *reinterpret_cast<const float4*>(gamma + c);
    const float4 g1 = *reinterpret_cast<const float4*>(gamma + c + 4);
    const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = f[i] * rinv * gg[i];
    *reinterpret_cast<uint4*>(o + c) = f8_to_h8(f);
  }
}

__device__ __forceinline__ void load8(const __half* p, float (&f)[8]) {
  h8_to_f8(*reinterpret_cast<const uint4*>(p), f);
}
__device__ __forceinline__ void load8(const float* p, float (&f)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// Residual add + RMSNorm, the reference's vsma + rmsnorm pair (layer.rs:4932-4940,
// cpu/rmsnorm.rs:149-183): x = x_in + delta (projection output already scaled by alpha;
// fp16, or fp32 after a tensor-parallel all-reduce), then xn = x * rinv * gamma.
// x_in == x updates the residual in place (inference); a training forward keeps each
// layer's residual and passes a new x. rinv_out (nullable) keeps 1/rms per row.
// One warp per row; rows of up to NREG*256 elements stay in registers.
template <int NREG, typename DT>
__global__ void add_rmsnorm_kernel(const float* x_in, float* x, const DT* __restrict__ delta,
                                   const float* __restrict__ gamma, __half* __restrict__ xn,
                                   int T, int dim, float* __restrict__ rinv_out) {
  const int row = blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const float* xi = x_in + (size_t)row * dim;
  float* xr = x + (size_t)row * dim;
  const DT* dr = delta + (size_t)row * dim;
  float keep[NREG][8];
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < NREG; ++it) {
    const int c = it * 256 + lane * 8;
    if (c < dim) {
      const float4 a = *reinterpret_cast<const float4*>(xi + c);
      const float4 b = *reinterpret_cast<const float4*>(xi + c + 4);
      float dv[8];
      load8(dr + c, dv);
      float* f = keep[it];
      f[0] = a.x + dv[0]; f[1] = a.y + dv[1]; f[2] = a.z + dv[2]; f[3] = a.w + dv[3];
      f[4] = b.x + dv[4]; f[5] = b.y + dv[5]; f[6] = b.z + dv[6]; f[7] = b.w + dv[7];
      *reinterpret_cast<float4*>(xr + c) = make_float4(f[0], f[1], f[2], f[3]);
      *reinterpret_cast<float4*>(xr + c + 4) = make_float4(f[4], f[5], f[6], f[7]);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
    }
  }
  ss = warp_sum(ss);
  const float rinv = 1.0f / sqrtf(ss / (float)dim + RMS_EPS);
  if (rinv_out && lane == 0) rinv_out[row] = rinv;
  __half* o = xn + (size_t)row * dim;
#pragma unroll
  for (int it = 0; it < NREG; ++it) {
    const int c = it * 256 + lane * 8;
    if (c < dim) {
      const float4 g0 = *reinterpret_cast<const float4*>(gamma + c);
      const float4 g1 = *reinterpret_cast<const float4*>(gamma + c + 4);
      const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      float f[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = keep[it][i] * rinv * gg[i];
      *reinterpret_cast<uint4*>(o + c) = f8_to_h8(f);
    }
  }
}

// Same for rows longer than the register budget: the second pass re-reads x (L2-hot).
template <typename DT>
__global__ void add_rmsnorm_long_kernel(const float* x_in, float* x, const DT* __restrict__ delta,
                                        const float* __restrict__ gamma, __half* __restrict__ xn,
                                        int T, int dim, float* __restrict__ rinv_out) {
  const int row = blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const float* xi = x_in + (size_t)row * dim;
  float* xr = x + (size_t)row * dim;
  const DT* dr = delta + (size_t)row * dim;
  float ss = 0.f;
  for (int c = lane * 8; c < dim; c += 256) {
    const float4 a = *reinterpret_cast<const float4*>(xi + c);
    const float4 b = *reinterpret_cast<const float4*>(xi + c + 4);
    float dv[8];
    load8(dr + c, dv);
    float f[8] = {a.x + dv[0], a.y + dv[1], a.z + dv[2], a.w + dv[3],
                  b.x + dv[4], b.y + dv[5], b.z + dv[6], b.w + dv[7]};
    *reinterpret_cast<float4*>(xr + c) = make_float4(f[0], f[1], f[2], f[3]);
    *reinterpret_cast<float4*>(xr + c + 4) = make_float4(f[4], f[5], f[6], f[7]);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  ss = warp_sum(ss);
  const float rinv = 1.0f / sqrtf(ss / (float)dim + RMS_EPS);
  __half* o = xn + (size_t)row * dim;
  for (int c = lane * 8; c < dim; c += 256) {
    const float4 a = *reinterpret_cast<const float4*>(xr + c);
    const float4 b = *reinterpret_cast<const float4*>(xr + c + 4);
    const float4 g0 = *reinterpret_cast<const float4*>(gamma + c);
    const float4 g1 = *reinterpret_cast<const float4*>(gamma + c + 4);
    float f[8] = {a.x * rinv * g0.x, a.y * rinv * g0.y, a.z * rinv * g0.z, a.w * rinv * g0.w,
                  b.x * rinv * g1.x, b.y * rinv * g1.y, b.z * rinv * g1.z, b.w * rinv * g1.w};
    *reinterpret_cast<uint4*>(o + c) = f8_to_h8(f);
  }
}

// One warp per token: combine `nparts` (max, sumexp) partials, subtract the target logit.
// Writes tok_loss[t] and one partial sum per block into block_sums[blockIdx.x].
__global__ void ce_finalize_kernel(const float2* __restrict__ part, int nparts,
                                   const float* __restrict__ tgt_logit,
                                   float* __restrict__ tok_loss, float* __restrict__ block_sums,
                                   int T) {
  __shared__ float wsum[ROW_WARPS];
  const int w = threadIdx.x >> 5;
  const int row = blockIdx.x * ROW_WARPS + w;
  const int lane = threadIdx.x & 31;
  float loss = 0.f;
  if (row < T) {
    const float2* p = part + (size_t)row * nparts;
    float m = -CUDART_INF_F;
    for (int i = lane; i < nparts; i += 32) m = fmaxf(m, p[i].x);
    m = warp_max(m);
    float s = 0.f;
    for (int i = lane; i < nparts; i += 32) s += p[i].y * __expf(p[i].x - m);
    s = warp_sum(s);
    loss = logf(s) + m - tgt_logit[row];
    if (lane == 0) tok_loss[row] = loss;
  }
  if (lane == 0) wsum[w] = (row < T) ? loss : 0.f;
  __syncthreads();
  if (threadIdx.x == 0) {
    float acc = 0.f;
    for (int i = 0; i < ROW_WARPS; ++i) acc += wsum[i];
    block_sums[blockIdx.x] = acc;
  }
}

// Single block: mean over T tokens from the per-block sums (fixed order).
__global__ void loss_mean_kernel(const float* __restrict__ block_sums, int nblocks, int T,
                                 float* __restrict__ loss) {
  __shared__ double sh[256];
  double acc = 0.0;
  for (int i = threadIdx.x; i < nblocks; i += blockDim.x) acc += (double)block_sums[i];
  sh[threadIdx.x] = acc;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) loss[0] = (float)(sh[0] / (double)T);
}

// Copy selected rows of src [*, dim] fp16 into dst [n, dim] (zero rows past n up to n_pad).
// dst[r] = fp16(RMSNorm(x[rows[r]]) * gamma) for r < n, zero rows up to n_pad: the
// final-norm output of selected positions, rebuilt from the fp32 residual stream.
__global__ void gather_norm_rows_kernel(const float* __restrict__ x,
                                        const int32_t* __restrict__ rows,
                                        const float* __restrict__ gamma, int n, int n_pad,
                                        int dim, __half* __restrict__ dst) {
  const int r = blockIdx.x;
  if (r >= n_pad) return;
  __shared__ float red[32];
  __half* out = dst + (size_t)r * dim;
  if (r >= n) {
    for (int c = threadIdx.x; c < dim; c += blockDim.x) out[c] = __float2half_rn(0.f);
    return;
  }
  const float* xr = x + (size_t)rows[r] * dim;
  float ss = 0.f;
  for (int c = threadIdx.x; c < dim; c += blockDim.x) ss += xr[c] * xr[c];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
  const float rinv = 1.0f / sqrtf(tot / (float)dim + RMS_EPS);
  for (int c = threadIdx.x; c < dim; c += blockDim.x)
    out[c] = __float2half_rn(xr[c] * rinv * gamma[c]);
}

}  // namespace cb
