// C-ABI implementation of the B200 forward + loss engine (include/cuda_bridge.h).
//
// A cb_ctx owns, on one device: fp16 weights in GEMM-ready layouts (weights.cuh),
// a workspace for max_batch sequences, TMA tensor maps for every GEMM operand,
// and one CUDA graph per (batch, softcap) holding the whole forward:
//
//   embed_rmsnorm                                     full_model.rs:396-397 + rmsnorm
//   for each layer (layer.rs:4409-4624 / forward_into_pipelined :5563):
//     rmsnorm(gamma1)            [layer > 0]          cpu/rmsnorm.rs:149-183
//     GEMM Xn*Wqkv^T  -> RoPE -> Q,K,V head-major     kernels/sdpa_fwd.rs:117-150,213-221
//     causal flash attention                          kernels/sdpa_fwd.rs:223-258
//     GEMM A*Wo       -> x += alpha*o                 dyn_matmul.rs:15-75; layer.rs:4471
//     rmsnorm(gamma2)                                 layer.rs:4932-4940
//     GEMM Xn*W13^T   -> g = silu(h1)*h3              kernels/ffn_fused.rs:79-107
//     GEMM g*W2^T     -> x += alpha*ffn               kernels/ffn_fused.rs:130-154
//   rmsnorm(gamma_final)                              full_model.rs:436-444
//   GEMM Xf*E^T -> per-tile (max, sumexp), target     full_model.rs:446-461
//   ce_finalize -> per-token loss; loss_mean           cpu/cross_entropy.rs:58-96; full_model.rs:471
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <errno.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>
#include <nccl.h>

#include <cmath>
#include <cstdio>
#include <algorithm>
#include <queue>
#include <chrono>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <type_traits>
#include <utility>
#include <vector>

#include "cuda_bridge.h"
#include "attention.cuh"
#include "attention_tc.cuh"
#include "attention_bwd.cuh"
#include "attention_bwd_tc.cuh"
#include "gemm_tc.cuh"
#include "io.cuh"
#include "ptx.cuh"
#include "rowwise.cuh"
#include "weights.cuh"

using namespace cb;

#define CB_VERSION_STR "rustane_b200 cuda_bridge 0.1 (sm_100a)"

namespace {

// ------------------------------------------------------------ tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// fp16 tensor [depth][rows][k] (k contiguous) tiled as 64 x box_rows x 1 boxes, 128B swizzle.
bool make_tmap(CUtensorMap* map, const void* ptr, uint64_t k, uint64_t rows, uint64_t depth,
               uint32_t box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {k, rows, depth};
  cuuint64_t strides[2] = {k * 2, k * rows * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// MN-major fp16 operand: a row-major [depth][k][mn] array (mn contiguous) read as
// 64 (mn) x 64 (k) boxes with 128-byte swizzle (the GEMM's MN-major A or B).
bool make_tmap_mn(CUtensorMap* map, const void* ptr, uint64_t mn, uint64_t k, uint64_t depth) {
  EncodeTiledFn enc = encode_fn();
  if (!enc || mn % 8 != 0) return false;
  cuuint64_t dims[3] = {mn, k, depth};
  cuuint64_t strides[2] = {mn * 2, mn * k * 2};
  cuuint32_t box[3] = {64, 64, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// fp16 matrix [rows][cols] (row-major) tiled as 64 x box_rows boxes, 128B swizzle.
bool make_tmap_rows(CUtensorMap* map, const void* ptr, uint64_t cols, uint64_t rows,
                    uint32_t box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// fp16 matrix [rows][cols] in 32 x 32 boxes, 64-byte swizzle (the fused residual
// epilogue's fp16(x o gamma) store).
bool make_tmap_h32(CUtensorMap* map, const void* ptr, uint64_t cols, uint64_t rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// fp32 matrix [rows][cols] (row-major) tiled as box_cols x box_rows boxes, no swizzle
// (the attention backward's dQ reduce-add target) or 128-byte swizzle.
bool make_tmap_f32_rows(CUtensorMap* map, const void* ptr, uint64_t cols, uint64_t rows,
                        uint32_t box_cols, uint32_t box_rows, bool swizzle128 = false) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 4};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// fp16 matrix [rows][128] (row stride 256 B) tiled as 64 x box_rows boxes, 128B swizzle
// (Q/K/V of the tcgen05 attention).
bool make_tmap_qkv(CUtensorMap* map, const void* ptr, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {128, rows};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ------------------------------------------------------------ NCCL (loaded on demand)
// Only tensor-parallel contexts need NCCL, so the library resolves it at run time:
// $CB_NCCL_LIB, else the copy this library was built against (CB_NCCL_DEFAULT_PATH),
// else whatever libnccl.so.2 the dynamic loader finds (the one torch loaded, if any).
struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclReduceScatter) reduce_scatter = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  decltype(&ncclCommGetAsyncError) async_error = nullptr;
  std::string why;
  bool ok() const { return all_reduce != nullptr; }
};

const NcclApi& nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    std::vector<std::string> names;
    if (const char* e = getenv("CB_NCCL_LIB")) names.push_back(e);
#ifdef CB_NCCL_DEFAULT_PATH
    names.push_back(CB_NCCL_DEFAULT_PATH);
#endif
    names.push_back("libnccl.so.2");
    void* h = nullptr;
    for (const auto& n : names)
      if ((h = dlopen(n.c_str(), RTLD_NOW | RTLD_GLOBAL)) != nullptr) break;
    if (!h) {
      api.why = "libnccl.so.2 not found (set CB_NCCL_LIB)";
      return;
    }
    NcclApi a;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.init_rank = reinterpret_cast<decltype(a.init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.init_rank_config =
        reinterpret_cast<decltype(a.init_rank_config)>(dlsym(h, "ncclCommInitRankConfig"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.reduce_scatter =
        reinterpret_cast<decltype(a.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.destroy = reinterpret_cast<decltype(a.destroy)>(dlsym(h, "ncclCommDestroy"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    a.async_error = reinterpret_cast<decltype(a.async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    if (!a.get_unique_id || !a.init_rank || !a.all_reduce || !a.reduce_scatter ||
        !a.all_gather || !a.destroy ||
        !a.error_string || !a.async_error) {
      api.why = "libnccl.so.2 lacks a required symbol";
      return;
    }
    api = a;
  });
  return api;
}

// Near-even split of `n` units over `world` ranks: the first n % world ranks get one more.
void split_even(int n, int world, int rank, int* begin, int* count) {
  const int base = n / world, extra = n % world;
  *count = base + (rank < extra ? 1 : 0);
  *begin = rank * base + (rank < extra ? rank : extra);
}

// ------------------------------------------------------------ GEMM launch
// Tile modes of the tcgen05 GEMM.
enum GemmMode { GM_SINGLE128 = 0, GM_SINGLE256 = 1, GM_PAIR = 2 };

// Tensor parallelism: the forward runs in TP chunks of sequences so that one chunk's
// exchange (on its own stream, NCCL capped at tp_comm_sms(world) CTAs) overlaps the next
// chunk's GEMMs (which then use the other SMs).
constexpr int TP_MAX_CHUNKS = 8;
// NCCL's CTA cap (and the SMs the overlapped GEMMs leave it): CB_TP_COMM_SMS (4-64, read
// once per process), else 16 at two ranks and 32 from four ranks up. Measured on the ~32B
// forward: at TP = 2, 16 CTAs 1200 ms against 32 CTAs 1226 ms per step; at TP = 8, where
// the exchange is about half of the step, 16 CTAs 480 ms against 32 CTAs 393 ms.
int tp_comm_sms(int world) {
  static const int forced = [] {
    const char* e = getenv("CB_TP_COMM_SMS");
    return e ? std::max(4, std::min(64, atoi(e))) : 0;
  }();
  return forced ? forced : (world >= 4 ? 32 : 16);
}

template <int BN, class Epi, int LAYOUT>
void set_gemm_attr() {
  cudaFuncSetAttribute(gemm_tn_kernel<BN, Epi, LAYOUT>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                       GemmCfg<BN, false, EpiTmaIn<Epi>::value>::SMEM_BYTES);
}

template <int BN, class Epi, int LAYOUT, bool FIX>
void set_gemm_attr_fix() {
  cudaFuncSetAttribute(gemm_tn_kernel<BN, Epi, LAYOUT, FIX>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                       GemmCfg<BN, false, EpiTmaIn<Epi>::value>::SMEM_BYTES);
}

template <class Epi, int LAYOUT = 0>
void set_gemm_attrs_for() {
  set_gemm_attr<128, Epi, LAYOUT>();
  set_gemm_attr<256, Epi, LAYOUT>();
  cudaFuncSetAttribute(gemm_tn_pair_kernel<Epi, LAYOUT>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                       GemmCfg<256, true, EpiTmaIn<Epi>::value>::SMEM_BYTES);
  if constexpr (EpiCanFix<Epi>::value && LAYOUT == 0) {  // the split-K (SplitFix) variants
    set_gemm_attr_fix<128, Epi, LAYOUT, true>();
    set_gemm_attr_fix<256, Epi, LAYOUT, true>();
    cudaFuncSetAttribute(gemm_tn_pair_kernel<Epi, LAYOUT, true>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         GemmCfg<256, true, EpiTmaIn<Epi>::value>::SMEM_BYTES);
  }
}

void set_all_kernel_attrs() {
  set_gemm_attrs_for<EpiStoreF16>();
  set_gemm_attrs_for<EpiStoreF32>();
  set_gemm_attrs_for<EpiQkvRope>();
  set_gemm_attrs_for<EpiScaledF16>();
  set_gemm_attrs_for<EpiScaledF32>();
  set_gemm_attrs_for<EpiScaledF32Add>();
  set_gemm_attrs_for<EpiStoreF16, GEMM_B_MN>();
  set_gemm_attrs_for<EpiStoreF32, GEMM_B_MN>();
  set_gemm_attrs_for<EpiScaledF32Add, GEMM_B_MN>();
  set_gemm_attrs_for<EpiStoreF16, GEMM_A_MN>();
  set_gemm_attrs_for<EpiStoreF32, GEMM_A_MN>();
  set_gemm_attrs_for<EpiScaledF32Add, GEMM_A_MN>();
  set_gemm_attrs_for<EpiStoreF16, GEMM_A_MN | GEMM_B_MN>();
  // training step (training.cuh)
  set_gemm_attrs_for<EpiSwigluSave>();
  set_gemm_attrs_for<EpiCeBwd>();
  set_gemm_attrs_for<EpiScaledF32, GEMM_B_MN>();
  set_gemm_attrs_for<EpiSwigluBwd, GEMM_B_MN>();
  set_gemm_attrs_for<EpiStoreF16Dsum, GEMM_B_MN>();
  // fused residual + RMSNorm forward
  set_gemm_attrs_for<EpiResidualNorm>();
  set_gemm_attrs_for<RowScaled<EpiQkvRope>>();
  set_gemm_attrs_for<RowScaled<EpiSwiglu>>();
  set_gemm_attrs_for<RowScaled<EpiCrossEntropy>>();
  set_gemm_attrs_for<EpiPartialF32, GEMM_A_MN | GEMM_B_MN>();
  set_gemm_attrs_for<EpiPartialF32>();  // decode (decode.cuh)
  set_gemm_attrs_for<EpiStoreF32, GEMM_A_MN | GEMM_B_MN>();
  set_gemm_attrs_for<EpiScaledF32Add, GEMM_A_MN | GEMM_B_MN>();
  set_gemm_attrs_for<EpiSwiglu>();
  set_gemm_attrs_for<EpiCrossEntropy>();
  cudaFuncSetAttribute(attn_fwd_causal_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       ATT_SMEM);
  cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM);
  cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AB_SMEM);
  cudaFuncSetAttribute(attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM);
}

struct DeviceInfo {
  int sms = 148;
  int pair_clusters = 74;  // CTA pairs of the GEMM that fit on the device at once
};

// Per-device kernel attributes and occupancy, set up once per device.
const DeviceInfo& device_info(int device) {
  static std::mutex mu;
  static DeviceInfo info[64];
  static uint64_t done = 0;
  std::lock_guard<std::mutex> lk(mu);
  if (device < 0 || device >= 64) return info[0];
  if (!(done & (1ull << device))) {
    set_all_kernel_attrs();
    DeviceInfo d;
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device);
    d.pair_clusters = d.sms / 2;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(d.sms & ~1, 1, 1);
    lc.blockDim = dim3(GEMM_THREADS, 1, 1);
    lc.dynamicSmemBytes = GemmCfg<256, true>::SMEM_BYTES;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    lc.attrs = &attr;
    lc.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_tn_pair_kernel<EpiStoreF16>, &lc) ==
            cudaSuccess &&
        n > 0)
      d.pair_clusters = n;
    cudaGetLastError();
    info[device] = d;
    done |= (1ull << device);
  }
  return info[device];
}

void ensure_attrs(int device) { (void)device_info(device); }

int num_sms_of(int device) { return device_info(device).sms; }

// Kernel launch, optionally with programmatic dependent launch (PDL): the kernel's CTAs
// may be scheduled while the previous kernel on the stream finishes, run their setup,
// and wait in pdl_enter() before touching memory. Every kernel launched with pdl = true
// calls pdl_enter() before its first global access. Captured into a CUDA graph the
// attribute becomes a programmatic dependency edge.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// The epilogue's input map (TMA_IN epilogues); the others get a zeroed map they never use.
const CUtensorMap& tc_or_null(const CUtensorMap* tc) {
  static const CUtensorMap zero{};
  return tc ? *tc : zero;
}

template <int BN, class Epi, int LAYOUT = 0>
cudaError_t launch_gemm_bn(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K,
                           int bz, const Epi& epi, int* err, int units, int splits,
                           cudaStream_t st, const CUtensorMap* tc = nullptr,
                           const CUtensorMap* td = nullptr, bool pdl = false,
                           SplitFix fix = SplitFix{}) {
  using Cfg = GemmCfg<BN, false, EpiTmaIn<Epi>::value>;
  const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * ((N + BN - 1) / BN) * splits;
  const int grid = tiles < units ? tiles : units;
  if constexpr (EpiCanFix<Epi>::value && LAYOUT == 0) {
    if (fix.ws && splits > 1)
      return launch_k(gemm_tn_kernel<BN, Epi, LAYOUT, true>, dim3(grid), dim3(GEMM_THREADS),
                      Cfg::SMEM_BYTES, st, pdl, ta, tb, tc_or_null(tc), tc_or_null(td), M, N, K,
                      bz, splits, epi, fix, err);
  }
  return launch_k(gemm_tn_kernel<BN, Epi, LAYOUT>, dim3(grid), dim3(GEMM_THREADS),
                  Cfg::SMEM_BYTES, st, pdl, ta, tb, tc_or_null(tc), tc_or_null(td), M, N, K, bz,
                  splits, epi, SplitFix{}, err);
}

template <class Epi, int LAYOUT = 0>
cudaError_t launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb_half, int M, int N,
                             int K, int bz, const Epi& epi, int* err, int clusters, int splits,
                             cudaStream_t st, const CUtensorMap* tc = nullptr,
                             const CUtensorMap* td = nullptr, bool pdl = false,
                             SplitFix fix = SplitFix{}) {
  using Cfg = GemmCfg<256, true, EpiTmaIn<Epi>::value>;
  const int tiles = ((M + 255) / 256) * ((N + 255) / 256) * splits;
  const int pairs = tiles < clusters ? tiles : clusters;
  if constexpr (EpiCanFix<Epi>::value && LAYOUT == 0) {
    if (fix.ws && splits > 1)
      return launch_k(gemm_tn_pair_kernel<Epi, LAYOUT, true>, dim3(2 * pairs),
                      dim3(GEMM_THREADS), Cfg::SMEM_BYTES, st, pdl, ta, tb_half, tc_or_null(tc),
                      tc_or_null(td), M, N, K, bz, splits, epi, fix, err);
  }
  return launch_k(gemm_tn_pair_kernel<Epi, LAYOUT>, dim3(2 * pairs), dim3(GEMM_THREADS),
                  Cfg::SMEM_BYTES, st, pdl, ta, tb_half, tc_or_null(tc), tc_or_null(td), M, N, K,
                  bz, splits, epi, SplitFix{}, err);
}

// Tile mode for an M x N GEMM: the best of (last-wave fill) x (per-tile operand
// efficiency). A CTA pair moves the fewest operand bytes per FLOP; 128-wide tiles
// fill small problems better. CB_GEMM_MODE=pair|256|128 forces one mode.
int pick_mode(int M, int N, const DeviceInfo& di) {
  static const int forced = [] {
    const char* e = getenv("CB_GEMM_MODE");
    if (!e) return -1;
    if (!strcmp(e, "pair")) return (int)GM_PAIR;
    if (!strcmp(e, "256")) return (int)GM_SINGLE256;
    if (!strcmp(e, "128")) return (int)GM_SINGLE128;
    return -1;
  }();
  auto fill = [](long tiles, long units) {
    long waves = (tiles + units - 1) / units;
    return (double)tiles / (double)(waves * units);
  };
  const bool n256 = (N % 256) == 0;
  if (forced == GM_SINGLE128 || (!n256 && forced != -1)) return GM_SINGLE128;
  if (forced >= 0) return forced;
  const double s_pair = n256 ? fill((long)((M + 255) / 256) * (N / 256), di.pair_clusters) : 0.0;
  const double s_256 = n256 ? 0.85 * fill((long)((M + 127) / 128) * (N / 256), di.sms) : 0.0;
  const double s_128 = 0.78 * fill((long)((M + 127) / 128) * ((N + 127) / 128), di.sms);
  if (s_pair >= s_256 && s_pair >= s_128) return GM_PAIR;
  return s_256 >= s_128 ? GM_SINGLE256 : GM_SINGLE128;
}

int mode_block_n(int mode) { return mode == GM_SINGLE128 ? 128 : 256; }

// tb128: B tensor map with 128-row boxes (single 128-wide tiles and CTA pairs);
// tb256: 256-row boxes (single 256-wide tiles).
// tb128 is B's tensor map with 128-row boxes (1-CTA 128-wide tiles and the CTA pair's
// halves), tb256 the one with 256-row boxes. For an MN-major B (LAYOUT & GEMM_B_MN) both
// are the same 64 x 64-box map.
template <class Epi, int LAYOUT = 0>
cudaError_t launch_gemm(int mode, const CUtensorMap& ta, const CUtensorMap& tb128,
                        const CUtensorMap& tb256, int M, int N, int K, int bz, const Epi& epi,
                        int* err, const DeviceInfo& di, cudaStream_t st, int splits = 1,
                        const CUtensorMap* tc = nullptr, const CUtensorMap* td = nullptr,
                        bool pdl = false, SplitFix fix = SplitFix{}) {
  if (mode == GM_PAIR)
    return launch_gemm_pair<Epi, LAYOUT>(ta, tb128, M, N, K, bz, epi, err, di.pair_clusters,
                                         splits, st, tc, td, pdl, fix);
  if (mode == GM_SINGLE128)
    return launch_gemm_bn<128, Epi, LAYOUT>(ta, tb128, M, N, K, bz, epi, err, di.sms, splits, st,
                                            tc, td, pdl, fix);
  if (EpiTmaIn<Epi>::value)  // 128 x 256 tiles leave no shared memory for the input boxes
    return cudaErrorInvalidConfiguration;
  return launch_gemm_bn<256, Epi, LAYOUT>(ta, tb256, M, N, K, bz, epi, err, di.sms, splits, st,
                                          tc, td, pdl, fix);
}

// Tile mode and K split for a row-parallel projection (O or down) whose epilogue can
// accumulate: split-K = 2 doubles the work units when the tiles alone leave the last
// wave mostly empty (few tokens per GPU). CB_GEMM_SPLIT=1|2 forces the split.
// max_split = 1 when the projection can carry the fused residual + norm epilogue (which
// needs whole sums): the separate norm pass a split would bring back costs about half of
// the down projection's GEMM time, more than a split's fill ever gains.
void pick_projection(int M, int N, int K, const DeviceInfo& di, int* mode, int* splits,
                     int max_split = 2) {
  static const int forced_split = [] {
    const char* e = getenv("CB_GEMM_SPLIT");
    return e ? atoi(e) : 0;
  }();
  auto fill = [](long tiles, long units) {
    long waves = (tiles + units - 1) / units;
    return (double)tiles / (double)(waves * units);
  };
  const bool n256 = (N % 256) == 0;
  const long kb = (K + GEMM_BK - 1) / GEMM_BK;
  double best = -1.0;
  const int sp_max = forced_split ? forced_split : max_split;  // CB_GEMM_SPLIT overrides
  for (int sp = 1; sp <= sp_max; ++sp) {
    if (forced_split && sp != forced_split) continue;
    // The zeroing and the fp32 atomics cost about as much as a 16-k-block half saves:
    // only long reductions (the down projection) split.
    if (!forced_split && sp == 2 && kb < 32) continue;
    const double sp_cost = sp == 2 ? 0.93 : 1.0;  // zeroing + fp32 atomics
    struct Cand { int mode; double score; };
    const Cand cands[3] = {
        {GM_PAIR, n256 ? fill((long)((M + 255) / 256) * (N / 256) * sp, di.pair_clusters) : 0.0},
        {GM_SINGLE256, n256 ? 0.85 * fill((long)((M + 127) / 128) * (N / 256) * sp, di.sms) : 0.0},
        {GM_SINGLE128, 0.78 * fill((long)((M + 127) / 128) * ((N + 127) / 128) * sp, di.sms)}};
    for (const Cand& c : cands)
      if (c.score * sp_cost > best) {
        best = c.score * sp_cost;
        *mode = c.mode;
        *splits = sp;
      }
  }
}

// ------------------------------------------------------- split-K plans (SplitFix)
// Workspace of the last-arrival split-K reduction: fp32 partial slabs (kept small enough
// to stay in L2 between the write and the read) and one arrival counter per tile half.
constexpr size_t FIX_WS_BYTES = 64u << 20;
constexpr int FIX_COUNTERS = 16384;

struct GemmPlan {
  int mode = GM_PAIR;
  int splits = 1;
};

int plan_bm(int mode) { return mode == GM_PAIR ? 256 : 128; }
int plan_bn(int mode) { return mode == GM_SINGLE128 ? 128 : 256; }

// Whether (mode, splits) fits the reduction's workspace: one 128 x BN fp32 slab per unit
// (per CTA of a pair) and one counter per tile half.
bool plan_fits(int mode, int splits, int M, int N) {
  if (splits <= 1) return true;
  const long tiles = (long)((M + plan_bm(mode) - 1) / plan_bm(mode)) *
                     ((N + plan_bn(mode) - 1) / plan_bn(mode));
  const long halves = tiles * (mode == GM_PAIR ? 2 : 1);
  return halves <= FIX_COUNTERS &&
         (size_t)halves * splits * GEMM_BM * plan_bn(mode) * sizeof(float) <= FIX_WS_BYTES;
}

// Estimated duration of an M x N x K GEMM of the fused forward under (mode, splits), in
// units of one SM's time for one 128 x 256 x 64 block of MMAs. A persistent grid runs
// ceil(units / slots) waves of units; a unit costs its k-blocks (128-wide tiles move
// more operand bytes per FLOP; a pair moves the fewest) plus a fixed start-up, and the
// last unit's epilogue is exposed. A split unit also writes its fp32 partial, and the
// tile's last unit reads the other splits' partials before its epilogue.
double plan_cost(int mode, int splits, int M, int N, int K, const DeviceInfo& di, bool tin) {
  const int bm = plan_bm(mode), bn = plan_bn(mode);
  const long tiles = (long)((M + bm - 1) / bm) * ((N + bn - 1) / bn);
  const long units = tiles * splits;
  const long slots = mode == GM_PAIR ? di.pair_clusters : di.sms;
  const long waves = (units + slots - 1) / slots;
  const int kb = (K + GEMM_BK - 1) / GEMM_BK;
  const int kbu = (kb + splits - 1) / splits;
  const double t_kb = mode == GM_PAIR ? 1.0 : (mode == GM_SINGLE256 ? 1.18 : 0.68);
  const double nc = bn / 32.0;
  const double t_start = 3.0;
  const double t_epi = nc * (tin ? 1.0 : 0.6);
  double t_unit = t_start + kbu * t_kb;
  double t_tail = t_epi;
  if (splits > 1) {  // constants from whole-forward graph timings of forced plans
    t_unit += nc * 1.2;                    // the partial written to L2
    t_tail += nc * 1.0 * (splits - 1);     // the last unit's reads of the others
  }
  return waves * t_unit + t_tail;
}

// Tuning override for tests and sweeps: CB_GEMM_PLAN="qkv=128x2,o=pairx1,w13=...,down=...,
// head=..." (mode pair|256|128, x splits). Read on every plan, so a process can switch
// plans between eager (profiled) forwards; captured graphs keep the plan they were built
// with.
bool plan_override(const char* cls, GemmPlan* out) {
  const char* e = getenv("CB_GEMM_PLAN");
  if (!e) return false;
  std::string spec(e), key = std::string(cls) + "=";
  size_t pos = 0;
  while (pos < spec.size()) {
    size_t end = spec.find(',', pos);
    if (end == std::string::npos) end = spec.size();
    const std::string item = spec.substr(pos, end - pos);
    pos = end + 1;
    if (item.compare(0, key.size(), key) != 0) continue;
    const std::string v = item.substr(key.size());
    const size_t x = v.find('x');
    const std::string m = v.substr(0, x);
    GemmPlan p;
    if (m == "pair") p.mode = GM_PAIR;
    else if (m == "256") p.mode = GM_SINGLE256;
    else if (m == "128") p.mode = GM_SINGLE128;
    else return false;
    p.splits = x == std::string::npos ? 1 : std::max(1, atoi(v.c_str() + x + 1));
    *out = p;
    return true;
  }
  return false;
}

// Plan of one GEMM of the fused forward (QKV, O, W1/W3, down, LM head): the cheapest
// (mode, splits) by plan_cost among the tile shapes N allows (a pair and 128 x 256 tiles
// need N % 256 == 0; 128 x 256 tiles have no room for the TMA_IN epilogue's boxes) and
// splits that leave each unit at least 8 k-blocks and fit the reduction's workspace.
// Deterministic: the same shapes always give the same plan, so the summation order and
// the loss bits do not change from call to call.
// The split count the kernel actually runs: with kb_per = ceil(kb / splits) k-blocks per
// unit, ceil(kb / kb_per) units cover K, and every one of them gets at least one k-block
// (a unit with none would hand over an accumulator it never wrote).
int effective_splits(int K, int splits) {
  const int kb = (K + GEMM_BK - 1) / GEMM_BK;
  if (splits <= 1 || kb <= 1) return 1;
  const int kb_per = (kb + splits - 1) / splits;
  return (kb + kb_per - 1) / kb_per;
}

GemmPlan plan_gemm(const char* cls, int M, int N, int K, const DeviceInfo& di, bool tin,
                   bool can_split) {
  GemmPlan best;
  if (plan_override(cls, &best)) {
    if (best.mode != GM_SINGLE128 && N % 256 != 0) best.mode = GM_SINGLE128;
    if (tin && best.mode == GM_SINGLE256) best.mode = GM_SINGLE128;
    best.splits = effective_splits(K, best.splits);
    if (!can_split || !plan_fits(best.mode, best.splits, M, N)) best.splits = 1;
    return best;
  }
  const int kb = (K + GEMM_BK - 1) / GEMM_BK;
  double best_cost = 1e300;
  const int modes[3] = {GM_PAIR, GM_SINGLE256, GM_SINGLE128};
  for (int mode : modes) {
    if (mode != GM_SINGLE128 && N % 256 != 0) continue;
    if (tin && mode == GM_SINGLE256) continue;
    for (int sp = 1; sp <= (can_split ? 8 : 1); ++sp) {
      if (sp > 1 && (kb + sp - 1) / sp < 8) break;
      if (effective_splits(K, sp) != sp) continue;
      if (!plan_fits(mode, sp, M, N)) continue;
      const double c = plan_cost(mode, sp, M, N, K, di, tin);
      if (c < best_cost * 0.97) {  // a split must win clearly
        best_cost = c;
        best.mode = mode;
        best.splits = sp;
      }
    }
  }
  return best;
}

// Causal attention: tcgen05 kernel when seq is a multiple of 128 (tensor maps given),
// otherwise the mma.sync kernel.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// A driver entry point resolved once through the runtime (no -lcuda link).
template <class Fn>
Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    return reinterpret_cast<Fn>(p);
  return nullptr;
}

// The current device and the id of its context as this thread's kernels will see it:
// cudaSetDevice makes the device's primary context current on this thread (creating it if
// needed). Context ids are unique for the life of the process, unlike context handles, so
// a device address cached under an id is never used in a later context (after a
// cudaDeviceReset, say).
cudaError_t current_context_id(int* dev, unsigned long long* id) {
  static const CtxGetCurrentFn get_ctx = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static const CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return e;
  e = cudaSetDevice(*dev);
  if (e != cudaSuccess) return e;
  CUcontext ctx = nullptr;
  if (!get_ctx || !get_id || get_ctx(&ctx) != CUDA_SUCCESS || !ctx ||
      get_id(ctx, id) != CUDA_SUCCESS)
    return cudaErrorContextIsDestroyed;
  return cudaSuccess;
}

// ---------------------------------------------- attention work schedule
// attn_fwd_tc_kernel is persistent (two CTAs per SM) and takes its tiles from a table
// made here once per shape. Tiles that run at the same time should share their K and V
// through L2 (heaviest-first over all heads at once re-read them from HBM for every tile,
// measured 15-20 % slower), and every CTA should end at about the same time. Two
// candidate splits, the one whose last CTA ends first (by the cost model: a tile costs
// its 64-key steps + 1 for its set-up and output) is used, the first on a tie:
//   head-major: the tiles of one head after another, latest query tile first, dealt to
//     the CTAs in rounds that alternate direction (snake);
//   chunked greedy: heads in chunks whose K and V take at most ATTN_CHUNK_MB, within a
//     chunk the latest query tiles of all its heads first, each tile to the CTA with the
//     least work so far (greedy longest-processing-time list scheduling).
// Head-major balances well when every CTA gets many tiles (seq 2048); the chunked greedy
// split when CTAs get few (8-16 sequences of 512: 20-35 % shorter makespan). Both keep
// the tiles that run together within a few MB of K and V. Table: [grid + 1] offsets,
// then the items ((batch * heads + head) * n_qt + query tile) of CTA 0, CTA 1, ...
constexpr double ATTN_CHUNK_MB = 8.0;

std::vector<int> attn_schedule_table(int batch, int heads, int kv_heads, int seq, int grid_max,
                                     int* grid_out) {
  const int n_qt = seq / FA_BQ, hb_count = batch * heads;
  const long n_items = (long)n_qt * hb_count;
  const int grid = (int)std::max<long>(1, std::min<long>(n_items, grid_max));
  auto cost = [&](int w) { return 2L * (w % n_qt + 1) + 1; };
  // head-major, snake
  std::vector<std::vector<int>> hm(grid);
  std::vector<long> hm_load(grid, 0);
  for (long k = 0; k < n_items; ++k) {
    const long rd = k / grid;
    const int c = (int)(rd & 1 ? grid - 1 - k % grid : k % grid);
    const int hb = (int)(k / n_qt), qt = n_qt - 1 - (int)(k % n_qt);
    hm[c].push_back(hb * n_qt + qt);
    hm_load[c] += cost(hb * n_qt + qt);
  }
  // chunked greedy
  const double kv_bytes_per_head = (double)seq * 128 * 2 * 2 / std::max(1, heads / kv_heads);
  const char* env = getenv("CB_ATTN_CHUNK_MB");  // tuning override of the chunk budget
  const double budget_mb = env && atof(env) > 0 ? atof(env) : ATTN_CHUNK_MB;
  const int chunk =
      std::max(1, std::min(hb_count, (int)(budget_mb * (1 << 20) / kv_bytes_per_head)));
  std::vector<std::vector<int>> gr(grid);
  using Slot = std::pair<long, int>;  // (work so far, CTA): the least work, then the lowest CTA
  std::priority_queue<Slot, std::vector<Slot>, std::greater<Slot>> heap;
  for (int c = 0; c < grid; ++c) heap.push({0, c});
  long gr_max = 0;
  for (int c0 = 0; c0 < hb_count; c0 += chunk) {
    const int ce = std::min(chunk, hb_count - c0);
    for (int qt = n_qt - 1; qt >= 0; --qt)
      for (int i = 0; i < ce; ++i) {
        const Slot top = heap.top();
        heap.pop();
        const int w = (c0 + i) * n_qt + qt;
        gr[top.second].push_back(w);
        heap.push({top.first + cost(w), top.second});
        gr_max = std::max(gr_max, top.first + cost(w));
      }
  }
  const long hm_max = *std::max_element(hm_load.begin(), hm_load.end());
  const std::vector<std::vector<int>>& lists = gr_max < hm_max ? gr : hm;
  std::vector<int> table;
  table.reserve(grid + 1 + n_items);
  int off = 0;
  for (int c = 0; c < grid; ++c) {
    table.push_back(off);
    off += (int)lists[c].size();
  }
  table.push_back(off);
  for (int c = 0; c < grid; ++c) table.insert(table.end(), lists[c].begin(), lists[c].end());
  *grid_out = grid;
  return table;
}

struct AttnSched {
  int grid = 0;
  int* table = nullptr;  // device copy of attn_schedule_table
};

std::mutex g_attn_sched_mu;
// keyed by (context id, batch, heads, kv heads, seq)
std::map<std::tuple<unsigned long long, int, int, int, int>, AttnSched> g_attn_sched;

// The schedule of one shape on the current device, made and uploaded on first use. The
// upload cannot happen while `st` is being captured into a graph: forwards prepare their
// shapes before capture (prepare_attention), and a capture that meets an unprepared
// shape fails with cudaErrorStreamCaptureUnsupported.
cudaError_t attn_schedule(int batch, int heads, int kv_heads, int seq, cudaStream_t st,
                          const AttnSched** out) {
  int dev = 0;
  unsigned long long ctx_id = 0;
  cudaError_t e = current_context_id(&dev, &ctx_id);
  if (e != cudaSuccess) return e;
  const std::tuple<unsigned long long, int, int, int, int> key{ctx_id, batch, heads, kv_heads,
                                                                seq};
  std::lock_guard<std::mutex> lock(g_attn_sched_mu);
  auto it = g_attn_sched.find(key);
  if (it != g_attn_sched.end()) {
    *out = &it->second;
    return cudaSuccess;
  }
  if (st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
      return cudaErrorStreamCaptureUnsupported;
  }
  AttnSched s;
  const std::vector<int> table =
      attn_schedule_table(batch, heads, kv_heads, seq, 2 * num_sms_of(dev), &s.grid);
  e = cudaMalloc(&s.table, table.size() * sizeof(int));
  if (e != cudaSuccess) return e;
  e = cudaMemcpy(s.table, table.data(), table.size() * sizeof(int), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(s.table);
    return e;
  }
  *out = &(g_attn_sched[key] = s);
  return cudaSuccess;
}

cudaError_t launch_attention(const CUtensorMap* tq, const CUtensorMap* tk, const CUtensorMap* tv,
                             const __half* q, const __half* k, const __half* v, __half* out,
                             int batch, int heads, int kv_heads, int seq, int* err,
                             cudaStream_t st, float* lse = nullptr) {
  const float scale_log2 = 1.4426950408889634f / sqrtf(128.0f);
  CUtensorMap to;  // the output [batch*seq, heads*128] in 128-query x 64-column boxes
  if (tq && seq % FA_BQ == 0 &&
      make_tmap_rows(&to, out, (uint64_t)heads * 128, (uint64_t)batch * seq, FA_BQ)) {
    const AttnSched* sch = nullptr;
    const cudaError_t e = attn_schedule(batch, heads, kv_heads, seq, st, &sch);
    if (e != cudaSuccess) return e;
    attn_fwd_tc_kernel<<<sch->grid, FA_THREADS, FA_SMEM, st>>>(
        *tq, *tk, *tv, to, seq, heads, kv_heads, sch->table, scale_log2, lse, err);
  } else {
    dim3 grid(seq / ATT_BQ, heads, batch);
    attn_fwd_causal_kernel<<<grid, ATT_THREADS, ATT_SMEM, st>>>(q, k, v, out, seq, heads,
                                                                kv_heads, scale_log2, lse);
  }
  return cudaGetLastError();
}

// Attention backward: D = rowsum(dO o O) (unless the caller computed it: dsum_ready), the
// key-block kernel (dK, dV into dqkv; dQ accumulated in dq32, which this zeroes first),
// then dQ into dqkv.
cudaError_t launch_attention_bwd(const __half* q, const __half* k, const __half* v,
                                 const __half* o, const __half* dout, const float* lse2,
                                 float* dsum, float* dq32, const float2* rope,
                                 const float2* rope_pm, __half* dqkv, int batch, int heads,
                                 int kv_heads, int seq, int sms, cudaStream_t st,
                                 int* err = nullptr, bool dsum_ready = false) {
  const int T = batch * seq;
  const int q_dim = heads * 128, n_qkv = q_dim + 2 * kv_heads * 128;
  const float scale = 1.0f / sqrtf(128.0f);
  const float scale_log2 = 1.4426950408889634f * scale;
  cudaError_t e = cudaMemsetAsync(dq32, 0, (size_t)T * q_dim * sizeof(float), st);
  if (e != cudaSuccess) return e;
  if (!dsum_ready)
    attn_bwd_dsum_kernel<<<(T * heads + 15) / 16, 256, 0, st>>>(o, dout, dsum, T, seq, heads);
  CUtensorMap tq, tk, tv, tdo, tdq, tdkv;
  const bool tc = seq % AT_BK == 0 &&
                  make_tmap_rows(&tdkv, dqkv, (uint64_t)n_qkv, (uint64_t)T, AT_BK) &&
                  make_tmap_qkv(&tq, q, (uint64_t)batch * heads * seq, AT_BQ) &&
                  make_tmap_qkv(&tk, k, (uint64_t)batch * kv_heads * seq, AT_BK) &&
                  make_tmap_qkv(&tv, v, (uint64_t)batch * kv_heads * seq, AT_BK) &&
                  make_tmap_rows(&tdo, dout, (uint64_t)q_dim, (uint64_t)T, AT_BQ) &&
                  make_tmap_f32_rows(&tdq, dq32, (uint64_t)q_dim, (uint64_t)T, 128, AT_BQ);
  if (tc) {  // tcgen05 path
    dim3 grid(seq / AT_BK, kv_heads, batch);
    attn_bwd_tc_kernel<<<grid, AT_THREADS, AT_SMEM, st>>>(tq, tk, tv, tdo, tdq, tdkv, lse2, dsum,
                                                          rope, dq32, seq, heads, kv_heads,
                                                          scale_log2, scale, err);
  } else {
    dim3 grid(seq / AB_BK, kv_heads, batch);
    attn_bwd_kernel<<<grid, AB_THREADS, AB_SMEM, st>>>(q, k, v, dout, lse2, dsum, rope, dq32,
                                                       dqkv, seq, heads, kv_heads, scale_log2,
                                                       scale);
  }
  const size_t groups = (size_t)T * q_dim / 8;
  const int blocks = (int)std::min<size_t>((groups + 255) / 256, (size_t)sms * 16);
  attn_bwd_dq_kernel<<<blocks, 256, 0, st>>>(dq32, rope_pm, dqkv, T, seq, heads, n_qkv, scale);
  return cudaGetLastError();
}

// x = x_in + delta; xn = rmsnorm(x) * gamma (rows kept in registers up to 2048 wide).
// x_in == x is the in-place update; rinv (nullable) receives 1/rms per row.
template <typename DT>
cudaError_t launch_add_rmsnorm(const float* x_in, float* x, const DT* delta, const float* gamma,
                               __half* xn, int T, int d, cudaStream_t st, float* rinv = nullptr) {
  const int blocks = (T + ROW_WARPS - 1) / ROW_WARPS, threads = ROW_WARPS * 32;
  if (d <= 512)
    add_rmsnorm_kernel<2, DT><<<blocks, threads, 0, st>>>(x_in, x, delta, gamma, xn, T, d, rinv);
  else if (d <= 1024)
    add_rmsnorm_kernel<4, DT><<<blocks, threads, 0, st>>>(x_in, x, delta, gamma, xn, T, d, rinv);
  else if (d <= 1536)
    add_rmsnorm_kernel<6, DT><<<blocks, threads, 0, st>>>(x_in, x, delta, gamma, xn, T, d, rinv);
  else if (d <= 2048)
    add_rmsnorm_kernel<8, DT><<<blocks, threads, 0, st>>>(x_in, x, delta, gamma, xn, T, d, rinv);
  else
    add_rmsnorm_long_kernel<DT><<<blocks, threads, 0, st>>>(x_in, x, delta, gamma, xn, T, d, rinv);
  return cudaGetLastError();
}

// ------------------------------------------------------------ kernel classes
enum KClass {
  K_EMBED_NORM = 0,
  K_RMSNORM,
  K_GEMM_QKV,
  K_ATTN,
  K_GEMM_O,
  K_GEMM_W13,
  K_GEMM_W2,
  K_GEMM_HEAD,
  K_CE_FINAL,
  K_LOSS_MEAN,
  K_ALLREDUCE,
  K_RSCATTER,
  K_AGATHER,
  K_NUM
};
const char* kclass_name[K_NUM] = {"embed_rmsnorm", "add_rmsnorm",   "gemm_qkv_rope",
                                  "attention",     "gemm_o",        "gemm_w13_swiglu",
                                  "gemm_w2",       "gemm_lmhead_ce", "ce_finalize",
                                  "loss_mean",     "nccl_allreduce", "nccl_reduce_scatter",
                                  "nccl_all_gather"};

struct KStat {
  int64_t launches = 0;
  double ms = 0, flops = 0, bytes = 0;
};

}  // namespace

// ------------------------------------------------------------ context
struct TrainState;
void free_train_state(TrainState* t);
struct DecodeState;
void free_decode_state(DecodeState* s);

struct cb_ctx {
  cb_model_config cfg{};
  int device = 0;
  int max_batch = 0;
  int num_sms = 148;
  // this rank's share (the whole model unless tensor-parallel)
  int heads_l = 0, kv_heads_l = 0, hidden_l = 0;
  int q_dim = 0, kv_dim = 0, n_qkv = 0;  // local: heads_l*128, kv_heads_l*128, q+2kv
  int q_off = 0, kv_off = 0, hid_off = 0;  // offsets of the share in the full model
  int tp_rank = 0, tp_world = 1;
  ncclComm_t comm = nullptr;
  bool nccl_failed = false;  // the communicator failed or a peer left: no further NCCL call
  std::string nccl_why;      // why
  cudaStream_t comm_stream = nullptr;           // tensor parallel: the all-reduces' stream
  cudaEvent_t tp_ev[4 * 8] = {};                // chunk hand-offs between the two streams
  float* delta32 = nullptr;  // [T, dim] fp32 partial projections, all-reduced across ranks
  cudaStream_t stream = nullptr;
  std::string err;
  bool weights_ready = false;

  // weights
  __half* embed = nullptr;
  __half* wqkv = nullptr;
  __half* wo = nullptr;
  __half* w13 = nullptr;
  __half* w2 = nullptr;
  float* gamma = nullptr;        // [L][2][dim]
  float* gamma_final = nullptr;  // [dim]

  // workspace
  float* x = nullptr;          // [T, dim] fp32 residual stream
  __half* xn = nullptr;        // [T, dim] normalised activations (final: Xf), or fp16(x o gamma)
                               // when the residual add + RMSNorm is fused (ss_part then holds
                               // the rows' partial sums of x^2)
  float* ss_part = nullptr;    // [T, dim/128]
  __half* q = nullptr;         // [B, H, S, 128]
  __half* k = nullptr;
  __half* v = nullptr;
  __half* attn = nullptr;      // [T, q_dim]
  __half* g = nullptr;         // [T, hidden]
  __half* delta = nullptr;     // [T, dim] alpha * (O or down projection), added by add_rmsnorm
  float2* ce_part = nullptr;   // [T, vocab/128]
  float* tgt_logit = nullptr;  // [T]
  float* tok_loss = nullptr;   // [T]
  float* block_sums = nullptr; // [ceil(T/8)]
  float* loss = nullptr;       // [1]
  uint32_t* tokens = nullptr;  // [T]
  uint32_t* targets = nullptr; // [T]
  int64_t* eval_pos = nullptr; // [max_batch] window offsets into a cb_tokens array
  float2* rope = nullptr;      // [64, S] (cos, sin), pair-major
  float2* rope_pm = nullptr;   // [S, 64] the same, position-major
  int* dev_err = nullptr;      // device error flag
  float4* fix_ws = nullptr;    // split-K partial slabs (FIX_WS_BYTES; single-GPU contexts)
  int* fix_cnt = nullptr;      // split-K arrival counters [FIX_COUNTERS], zero between launches
  float* h_loss = nullptr;     // pinned
  int* h_err = nullptr;        // pinned

  // tensor maps (A operands sized for max_batch; B per weight kind, both tile widths)
  CUtensorMap tm_xn, tm_attn, tm_g;
  CUtensorMap tm_x;              // the fp32 residual in 32 x 32 boxes (fused residual epilogue)
  CUtensorMap tm_xh;             // xn as fp16 32 x 32 boxes (its second output)
  CUtensorMap tm_q, tm_k, tm_v;  // attention operands ([B*H*S, 128] rows)
  CUtensorMap tm_wqkv[2], tm_wo[2], tm_w13[2], tm_w2[2], tm_embed[2];  // [0]=BN128 [1]=BN256

  // graphs
  std::map<std::pair<int, uint32_t>, cudaGraphExec_t> graphs;

  // last forward (for sampled logits): its final fp32 residual stream
  int last_batch = 0;
  const float* x_final = nullptr;
  float last_softcap = 0.f;

  // sampled-logit buffers
  __half* samp_a = nullptr;
  float* samp_out = nullptr;
  int samp_cap = 0;

  // profiling
  bool profiling = false;
  KStat stats[K_NUM];
  std::vector<cudaEvent_t> events;
  std::vector<int> ev_class;
  std::vector<double> ev_flops, ev_bytes;
  bool pending_harvest = false;

  // training (cb_enable_training): saved activations, backward scratch, gradients
  TrainState* train = nullptr;
  // decode (cb_prefill / cb_decode_step): KV cache and single-token buffers
  DecodeState* decode = nullptr;

  size_t T_max() const { return (size_t)max_batch * cfg.seq; }
};

namespace {

thread_local std::string g_create_error;

cb_status fail(cb_ctx* c, cb_status code, const std::string& msg) {
  if (c) c->err = msg;
  return code;
}

// ---------------------------------------------- NCCL failure handling (tensor parallel)
// A rank whose peer has left would otherwise wait in a collective for good. The
// communicator is non-blocking: every NCCL call is settled by polling
// ncclCommGetAsyncError, and every wait for a tensor-parallel forward polls the stream
// and the communicator's asynchronous error. On an error, or when nothing completes
// within the deadline ($CB_NCCL_TIMEOUT_MS, default 120 s), or when the caller reports a
// lost peer (cb_tp_peer_lost), the context is marked failed and every later call returns
// CB_ERR_NCCL. The library then makes no further NCCL call on the communicator (no
// ncclCommAbort, no ncclCommDestroy): in two runs on 2 B200 where a peer process had
// exited, the surviving rank's process did not finish within 180 s after
// ncclCommAbort, with collectives in flight and without. The communicator and, if a
// collective still runs, the context's device memory are left to the end of the
// process, which a supervisor then ends. (The reference supervises its workers the same
// way from the host: a child process with a timeout, crates/engine/src/bin/
// theory_runner.rs:9-15.)
int nccl_timeout_ms() {
  const char* e = getenv("CB_NCCL_TIMEOUT_MS");
  const int v = e ? atoi(e) : 0;
  return v > 0 ? v : 120000;
}

void nccl_fail(cb_ctx* c, const std::string& why) {
  c->nccl_failed = true;
  c->nccl_why = why;
  c->err = why;
}

// Waits until the communicator has no operation in progress (the enqueue of a
// non-blocking call, or the set-up of a new communicator); r is the call's own result.
// On an error or after the deadline the context is marked failed. Returns ncclSuccess
// or the failure.
ncclResult_t nccl_settle(cb_ctx* c, ncclResult_t r, const char* what) {
  if (r != ncclSuccess && r != ncclInProgress) {
    nccl_fail(c, std::string(what) + ": " + nccl_api().error_string(r));
    return r;
  }
  const auto t0 = std::chrono::steady_clock::now();
  const auto limit = std::chrono::milliseconds(nccl_timeout_ms());
  for (;;) {
    ncclResult_t state = ncclSuccess;
    const ncclResult_t q = nccl_api().async_error(c->comm, &state);
    if (q != ncclSuccess) state = q;
    if (state == ncclSuccess) return ncclSuccess;
    if (state != ncclInProgress) {
      nccl_fail(c, std::string(what) + ": " + nccl_api().error_string(state));
      return state;
    }
    if (std::chrono::steady_clock::now() - t0 > limit) {
      nccl_fail(c, std::string(what) + ": no progress within " +
                       std::to_string(nccl_timeout_ms()) + " ms");
      return ncclInternalError;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// cudaStreamSynchronize for a context: a tensor-parallel one polls the stream and the
// communicator instead, so that a collective whose peer has left ends in CB_ERR_NCCL.
cb_status sync_ctx_stream(cb_ctx* c, cudaStream_t st) {
  if (c->nccl_failed) {  // failed earlier: never wait for good on what it left behind
    const auto t1 = std::chrono::steady_clock::now();
    while (cudaStreamQuery(st) == cudaErrorNotReady &&
           std::chrono::steady_clock::now() - t1 < std::chrono::seconds(1))
      std::this_thread::sleep_for(std::chrono::microseconds(100));
    return fail(c, CB_ERR_NCCL, "the tensor-parallel communicator has failed: " + c->nccl_why);
  }
  if (c->tp_world == 1 || !c->comm) {
    const cudaError_t e = cudaStreamSynchronize(st);
    return e == cudaSuccess
               ? CB_OK
               : fail(c, CB_ERR_CUDA, std::string("cudaStreamSynchronize: ") + cudaGetErrorString(e));
  }
  const auto t0 = std::chrono::steady_clock::now();
  const auto limit = std::chrono::milliseconds(nccl_timeout_ms());
  std::string why;
  for (;;) {
    const cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) return CB_OK;
    if (q != cudaErrorNotReady)
      return fail(c, CB_ERR_CUDA, std::string("stream: ") + cudaGetErrorString(q));
    ncclResult_t state = ncclSuccess;
    if (nccl_api().async_error(c->comm, &state) == ncclSuccess && state != ncclSuccess &&
        state != ncclInProgress) {
      why = std::string("NCCL asynchronous error: ") + nccl_api().error_string(state);
      break;
    }
    if (std::chrono::steady_clock::now() - t0 > limit) {
      why = "tensor-parallel forward made no progress within " +
            std::to_string(nccl_timeout_ms()) + " ms (a peer rank may have left)";
      break;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  nccl_fail(c, why);
  return fail(c, CB_ERR_NCCL, why);
}

// After a kernel stopped early (an expired wait), split-K arrival counters may be left
// part-way: zero them with the error flag, so the next launch counts from zero.
void reset_split_counters(cb_ctx* c, cudaStream_t st) {
  if (c->fix_cnt) cudaMemsetAsync(c->fix_cnt, 0, FIX_COUNTERS * sizeof(int), st);
}

#define CB_CUDA(call)                                                                  \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess)                                                             \
      return fail(ctx, e_ == cudaErrorMemoryAllocation ? CB_ERR_OUT_OF_MEMORY : CB_ERR_CUDA, \
                  std::string(#call) + ": " + cudaGetErrorString(e_));                 \
  } while (0)

template <class T>
cudaError_t dmalloc(T** p, size_t n) {
  return cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T) + 256);
}

size_t wqkv_layer_elems(const cb_ctx* c) { return (size_t)c->n_qkv * c->cfg.dim; }
size_t wo_layer_elems(const cb_ctx* c) { return (size_t)c->cfg.dim * c->q_dim; }
size_t w13_layer_elems(const cb_ctx* c) { return (size_t)2 * c->hidden_l * c->cfg.dim; }
size_t w2_layer_elems(const cb_ctx* c) { return (size_t)c->cfg.dim * c->hidden_l; }

ShapeInfo shape_of(const cb_ctx* c) {
  ShapeInfo s;
  s.dim = c->cfg.dim;
  s.hidden = c->hidden_l;
  s.q_dim = c->q_dim;
  s.kv_dim = c->kv_dim;
  s.hidden_g = c->cfg.hidden;
  s.q_dim_g = c->cfg.heads * 128;
  s.kv_dim_g = c->cfg.kv_heads * 128;
  s.q_off = c->q_off;
  s.kv_off = c->kv_off;
  s.hid_off = c->hid_off;
  s.vocab = c->cfg.vocab;
  return s;
}

void free_ctx(cb_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
  c->graphs.clear();
  free_train_state(c->train);
  c->train = nullptr;
  free_decode_state(c->decode);
  c->decode = nullptr;
  for (auto e : c->events) cudaEventDestroy(e);
  // after the graphs that hold its collectives; a failed communicator is left alone (no
  // NCCL call once a peer is lost)
  if (c->comm && !c->nccl_failed) nccl_api().destroy(c->comm);
  for (auto ev : c->tp_ev)
    if (ev) cudaEventDestroy(ev);
  if (c->comm_stream) cudaStreamDestroy(c->comm_stream);
  void* ptrs[] = {c->ss_part, c->rope_pm, c->eval_pos, c->delta32, c->delta, c->embed, c->wqkv, c->wo, c->w13, c->w2, c->gamma,
                  c->gamma_final, c->x,  c->xn,    c->q,        c->k,        c->v,
                  c->attn,  c->g,     c->ce_part,  c->tgt_logit, c->tok_loss, c->block_sums,
                  c->loss,  c->tokens, c->targets, c->rope,     c->dev_err,  c->samp_a,
                  c->samp_out, c->fix_ws, c->fix_cnt};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  if (c->h_loss) cudaFreeHost(c->h_loss);
  if (c->h_err) cudaFreeHost(c->h_err);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

#include "tensor_parallel.cuh"

// Per-layer destination of K and V (the decode KV cache): layer l's [batch, kv_heads,
// seq, 128] blocks at k + l * layer_stride and v + l * layer_stride.
struct KvDest {
  __half* k;
  __half* v;
  size_t layer_stride;
};

// Enqueue one forward for `batch` sequences on `st`. When `prof` is set,
// CUDA events bracket every launch (eager mode only). With `kv`, every layer's roped K
// and V are kept (prefill of the decode cache) instead of reusing one buffer.
cudaError_t enqueue_forward(cb_ctx* c, int batch, float softcap, cudaStream_t st, bool prof,
                            const KvDest* kv = nullptr) {
  if (!kv && c->tp_world > 1 && tp_reduce_mode() != TP_ALLREDUCE) {
    // sequence parallel, when every chunk's rows split evenly over the ranks
    const int T = batch * c->cfg.seq;
    int chunks = prof ? 1 : tp_chunks(c, batch);
    if ((T / chunks) % c->tp_world != 0) chunks = 1;
    if (T % c->tp_world == 0)
      return enqueue_forward_tp_sp(c, batch, chunks, softcap, st, prof,
                                   tp_reduce_mode() == TP_SP16);
  }
  if (!prof && !kv && c->tp_world > 1 && c->comm_stream) {
    const int chunks = tp_chunks(c, batch);
    if (chunks > 1) return enqueue_forward_tp_chunked(c, batch, chunks, softcap, st);
  }
  const cb_model_config& cfg = c->cfg;
  const int S = cfg.seq, d = cfg.dim, hid = c->hidden_l, V = cfg.vocab, L = cfg.nlayers;
  const int T = batch * S;
  const float alpha = 1.0f / sqrtf(2.0f * (float)L);  // layer.rs:4420
  const int row_blocks = (T + ROW_WARPS - 1) / ROW_WARPS;
  const bool tp = c->tp_world > 1;
  int ev = 0;
  auto mark = [&](int cls, double flops, double bytes) {
    if (!prof) return;
    c->ev_class.push_back(cls);
    c->ev_flops.push_back(flops);
    c->ev_bytes.push_back(bytes);
    cudaEventRecord(c->events[++ev], st);
  };
  if (prof) {
    c->ev_class.clear();
    c->ev_flops.clear();
    c->ev_bytes.clear();
    cudaEventRecord(c->events[0], st);
  }
  cudaError_t e;
  const double Td = (double)T;

  embed_rmsnorm_kernel<<<row_blocks, ROW_WARPS * 32, 0, st>>>(c->tokens, c->embed, c->gamma, c->x,
                                                                c->xn, T, d, V, c->dev_err);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  mark(K_EMBED_NORM, 0, Td * 4 + Td * d * (2 + 4 + 2));

  const DeviceInfo& di = device_info(c->device);
  // Residual add + RMSNorm: fused into the projection's epilogue (EpiResidualNorm: x +=
  // alpha * acc in place, xn = fp16(x o gamma), per-row partial sums of x^2; the next
  // GEMM applies 1/rms per row, RowScaled) unless the model is tensor parallel (the
  // partials are all-reduced first) or d % 128 != 0; otherwise the projection writes
  // delta and add_rmsnorm does the rest.
  const bool fuse_norm = !tp && d % 128 == 0;
  // Single-GPU GEMMs with too few tiles split K, reduced by the tile's last split
  // (SplitFix), so every fused epilogue still sees whole sums.
  const bool can_fix = !tp && c->fix_ws != nullptr;
  const SplitFix fix{c->fix_ws, c->fix_cnt};
  const GemmPlan p_qkv = plan_gemm("qkv", T, c->n_qkv, d, di, false, can_fix);
  int m_o, s_o, m_2, s_2;
  if (fuse_norm) {
    const GemmPlan po = plan_gemm("o", T, d, c->q_dim, di, true, can_fix);
    const GemmPlan p2 = plan_gemm("down", T, d, hid, di, true, can_fix);
    m_o = po.mode, s_o = po.splits, m_2 = p2.mode, s_2 = p2.splits;
  } else {
    pick_projection(T, d, c->q_dim, di, &m_o, &s_o, 2);
    pick_projection(T, d, hid, di, &m_2, &s_2, 2);
  }
  const GemmPlan p_13 = plan_gemm("w13", T, 2 * hid, d, di, false, can_fix);
  const double attn_flops = 2.0 * 2.0 * (double)batch * c->heads_l * 128.0 * S * (S + 1) / 2.0;

  // GEMMs use programmatic dependent launch (setup overlaps the previous kernel's tail)
  // outside tensor parallelism and eager profiling.
  const bool pdl = !tp && !prof;
  bool fused_last = false;  // the last projection used the fused epilogue
  bool xn_scaled = false;   // xn holds fp16(x o gamma): consumers scale rows by 1/rms
  auto consume = [&](const GemmPlan& plan, const CUtensorMap& tb128, const CUtensorMap& tb256,
                     int N, int layer, const auto& inner) -> cudaError_t {
    using E = std::decay_t<decltype(inner)>;
    const SplitFix f = plan.splits > 1 ? fix : SplitFix{};
    if (xn_scaled) {
      RowScaled<E> ep{inner, c->ss_part, d / 128, (float)d, RMS_EPS, 1.f};
      return launch_gemm(plan.mode, c->tm_xn, tb128, tb256, T, N, d, layer, ep, c->dev_err, di,
                         st, plan.splits, nullptr, nullptr, pdl, f);
    }
    return launch_gemm(plan.mode, c->tm_xn, tb128, tb256, T, N, d, layer, inner, c->dev_err, di,
                       st, plan.splits, nullptr, nullptr, pdl, f);
  };

  // Row-parallel projection (O or down): alpha * A * B^T into the delta buffer. fp16
  // by default; fp32 when K is split in two (atomic adds into a zeroed buffer) or under
  // tensor parallelism, where the fp32 partials are summed across ranks (NCCL).
  // gamma_next: the gain of the RMSNorm that follows (fused epilogue).
  bool delta_f32 = false;
  auto project = [&](int mode, int splits, const CUtensorMap& ta, const CUtensorMap& tb128,
                     const CUtensorMap& tb256, int K, int layer, int cls,
                     const float* gamma_next) -> cudaError_t {
    cudaError_t r;
    fused_last = fuse_norm && (splits == 1 || can_fix);
    delta_f32 = !fused_last && (tp || splits > 1);
    if (fused_last) {
      EpiResidualNorm ep{gamma_next, c->ss_part, d / 128, alpha, 0.f};
      r = launch_gemm(mode, ta, tb128, tb256, T, d, K, layer, ep, c->dev_err, di, st, splits,
                      &c->tm_x, &c->tm_xh, pdl, splits > 1 ? fix : SplitFix{});
      if (r != cudaSuccess) return r;
      mark(cls, 2.0 * Td * d * K,
           Td * K * 2 + (double)d * K * 2 + Td * d * (4 + 4 + 2) + Td * (d / 128) * 4);
      return cudaSuccess;
    }
    if (splits > 1) {
      r = cudaMemsetAsync(c->delta32, 0, (size_t)T * d * sizeof(float), st);
      if (r != cudaSuccess) return r;
      EpiScaledF32Add ep{c->delta32, d, alpha};
      r = launch_gemm(mode, ta, tb128, tb256, T, d, K, layer, ep, c->dev_err, di, st, splits);
    } else if (tp) {
      EpiScaledF32 ep{c->delta32, d, alpha};
      r = launch_gemm(mode, ta, tb128, tb256, T, d, K, layer, ep, c->dev_err, di, st);
    } else {
      EpiScaledF16 ep{c->delta, d, alpha};
      r = launch_gemm(mode, ta, tb128, tb256, T, d, K, layer, ep, c->dev_err, di, st);
    }
    if (r != cudaSuccess) return r;
    mark(cls, 2.0 * Td * d * K,
         Td * K * 2 + (double)d * K * 2 + Td * d * (delta_f32 ? 4 * splits : 2));
    if (tp) {
      ncclResult_t nr = nccl_api().all_reduce(c->delta32, c->delta32, (size_t)T * d, ncclFloat32,
                                              ncclSum, c->comm, st);
      if (nccl_settle(c, nr, "ncclAllReduce") != ncclSuccess) return cudaErrorUnknown;
      mark(K_ALLREDUCE, 0, Td * d * 4);
    }
    return cudaSuccess;
  };
  auto add_norm = [&](const float* gamma) -> cudaError_t {
    xn_scaled = fused_last;
    if (fused_last) return cudaSuccess;  // done by the projection's epilogue
    cudaError_t r = delta_f32 ? launch_add_rmsnorm(c->x, c->x, c->delta32, gamma, c->xn, T, d, st)
                              : launch_add_rmsnorm(c->x, c->x, c->delta, gamma, c->xn, T, d, st);
    if (r == cudaSuccess) mark(K_RMSNORM, 0, Td * d * (4 + (delta_f32 ? 4 : 2) + 4 + 2));
    return r;
  };

  for (int l = 0; l < L; ++l) {
    __half* kl = kv ? kv->k + (size_t)l * kv->layer_stride : c->k;
    __half* vl = kv ? kv->v + (size_t)l * kv->layer_stride : c->v;
    {
      EpiQkvRope ep{c->q, kl, vl, c->rope, S, c->heads_l, c->kv_heads_l};
      e = consume(p_qkv, c->tm_wqkv[0], c->tm_wqkv[1], c->n_qkv, l, ep);
      if (e != cudaSuccess) return e;
      mark(K_GEMM_QKV, 2.0 * Td * c->n_qkv * d,
           Td * d * 2 + (double)c->n_qkv * d * 2 + Td * c->n_qkv * 2);
    }
    CUtensorMap tk = c->tm_k, tv = c->tm_v;
    if (kv && !(make_tmap_qkv(&tk, kl, (uint64_t)T * c->kv_heads_l, FA_BKV) &&
                make_tmap_qkv(&tv, vl, (uint64_t)T * c->kv_heads_l, FA_BKV)))
      return cudaErrorInvalidValue;
    e = launch_attention(&c->tm_q, &tk, &tv, c->q, kl, vl, c->attn, batch, c->heads_l,
                         c->kv_heads_l, S, c->dev_err, st);
    if (e != cudaSuccess) return e;
    mark(K_ATTN, attn_flops, Td * (c->q_dim + 2 * c->kv_dim) * 2 + Td * c->q_dim * 2);
    e = project(m_o, s_o, c->tm_attn, c->tm_wo[0], c->tm_wo[1], c->q_dim, l, K_GEMM_O,
                c->gamma + (size_t)l * 2 * d + d);
    if (e != cudaSuccess) return e;
    if ((e = add_norm(c->gamma + (size_t)l * 2 * d + d)) != cudaSuccess) return e;
    {
      EpiSwiglu ep{c->g, hid};
      e = consume(p_13, c->tm_w13[0], c->tm_w13[1], 2 * hid, l, ep);
      if (e != cudaSuccess) return e;
      mark(K_GEMM_W13, 2.0 * Td * 2 * hid * d, Td * d * 2 + 2.0 * hid * d * 2 + Td * hid * 2);
    }
    const float* g_next = l + 1 < L ? c->gamma + (size_t)(l + 1) * 2 * d : c->gamma_final;
    e = project(m_2, s_2, c->tm_g, c->tm_w2[0], c->tm_w2[1], hid, l, K_GEMM_W2, g_next);
    if (e != cudaSuccess) return e;
    if (l + 1 < L) {  // residual add + RMSNorm(gamma1) of the next layer
      if ((e = add_norm(g_next)) != cudaSuccess) return e;
    }
  }
  if ((e = add_norm(c->gamma_final)) != cudaSuccess) return e;

  const GemmPlan p_head = plan_gemm("head", T, V, d, di, false, can_fix);
  const int nparts = (V + mode_block_n(p_head.mode) - 1) / mode_block_n(p_head.mode);
  {
    EpiCrossEntropy ep{};
    ep.part = c->ce_part;
    ep.nparts = nparts;
    ep.targets = c->targets;
    ep.tgt_logit = c->tgt_logit;
    ep.softcap = softcap;
    e = consume(p_head, c->tm_embed[0], c->tm_embed[1], V, 0, ep);
    if (e != cudaSuccess) return e;
    mark(K_GEMM_HEAD, 2.0 * Td * V * d, Td * d * 2 + (double)V * d * 2 + Td * nparts * 8 + Td * 8);
  }
  ce_finalize_kernel<<<row_blocks, ROW_WARPS * 32, 0, st>>>(c->ce_part, nparts, c->tgt_logit,
                                                            c->tok_loss, c->block_sums, T);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  mark(K_CE_FINAL, 0, Td * nparts * 8 + Td * 8);
  loss_mean_kernel<<<1, 256, 0, st>>>(c->block_sums, row_blocks, T, c->loss);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  mark(K_LOSS_MEAN, 0, row_blocks * 4.0);
  return cudaSuccess;
}

// Upper bound on the profiled launches of one forward: 7 per layer with the separate
// residual + norm pass (5 when it is fused into the projections); under tensor
// parallelism 9 with all-reduces, 11 sequence parallel (2 x (reduce-scatter, norm,
// all-gather)) plus the final all-gather of the residual rows.
int launches_per_forward(const cb_ctx* c) {
  return (c->tp_world > 1 ? 11 : 7) * c->cfg.nlayers + 5;
}

// ---------------------------------------------------------- standalone LM head + CE
struct LmCeScratch {
  float2* part;       // [T, nparts]
  float* tgt;         // [T]
  float* tok;         // [T]   (used when the caller passes no per-token buffer)
  float* blocks;      // [ceil(T / ROW_WARPS)]
  float* loss;        // [1]   (used when the caller passes no loss buffer)
};

int lm_ce_block_n(int vocab) { return (vocab % 256 == 0) ? 256 : 128; }
int lm_ce_nparts(int vocab) { return (vocab + lm_ce_block_n(vocab) - 1) / lm_ce_block_n(vocab); }

size_t lm_ce_scratch_bytes(int T, int vocab) {
  auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t nb = (size_t)(T + ROW_WARPS - 1) / ROW_WARPS;
  return up((size_t)T * lm_ce_nparts(vocab) * sizeof(float2)) + 2 * up((size_t)T * 4) +
         up(nb * 4) + up(4);
}

LmCeScratch lm_ce_carve(void* base, int T, int vocab) {
  auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
  uint8_t* p = static_cast<uint8_t*>(base);
  LmCeScratch s;
  s.part = reinterpret_cast<float2*>(p);
  p += up((size_t)T * lm_ce_nparts(vocab) * sizeof(float2));
  s.tgt = reinterpret_cast<float*>(p);
  p += up((size_t)T * 4);
  s.tok = reinterpret_cast<float*>(p);
  p += up((size_t)T * 4);
  s.blocks = reinterpret_cast<float*>(p);
  p += up((size_t)(T + ROW_WARPS - 1) / ROW_WARPS * 4);
  s.loss = reinterpret_cast<float*>(p);
  return s;
}

bool lm_ce_args_ok(const void* xf, const void* embed, const uint32_t* targets, int T, int d,
                   int V) {
  if (!xf || !embed || !targets || T <= 0 || d <= 0 || V <= 0) return false;
  if (d % 64 != 0 || V % 32 != 0) return false;
  return (((uintptr_t)xf | (uintptr_t)embed) & 15) == 0;
}

// Enqueue the fused head: GEMM with the cross-entropy epilogue, per-token combine,
// fixed-order mean. Target logits start as NaN so an out-of-range target shows.
cudaError_t lm_ce_enqueue(const void* xf, const void* embed, const uint32_t* targets, int T,
                          int d, int V, float softcap, float* per_token_loss, float* loss,
                          const LmCeScratch& s, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const DeviceInfo& di = device_info(dev);
  // 256-wide tiles (CTA pair or single CTA) when the vocab allows, else 128-wide:
  // the partial count always equals lm_ce_nparts(V).
  const int mode = (V % 256 == 0) ? (pick_mode(T, V, di) == GM_PAIR ? GM_PAIR : GM_SINGLE256)
                                  : GM_SINGLE128;
  const int nparts = lm_ce_nparts(V);
  CUtensorMap ta, tb128, tb256;
  if (!make_tmap(&ta, xf, d, T, 1, 128) || !make_tmap(&tb128, embed, d, V, 1, 128) ||
      !make_tmap(&tb256, embed, d, V, 1, 256))
    return cudaErrorInvalidValue;
  e = cudaMemsetAsync(s.tgt, 0xFF, (size_t)T * 4, st);
  if (e != cudaSuccess) return e;
  EpiCrossEntropy ep{};
  ep.part = s.part;
  ep.nparts = nparts;
  ep.targets = targets;
  ep.tgt_logit = s.tgt;
  ep.softcap = softcap;
  e = launch_gemm(mode, ta, tb128, tb256, T, V, d, 0, ep, nullptr, di, st);
  if (e != cudaSuccess) return e;
  const int row_blocks = (T + ROW_WARPS - 1) / ROW_WARPS;
  float* tok = per_token_loss ? per_token_loss : s.tok;
  ce_finalize_kernel<<<row_blocks, ROW_WARPS * 32, 0, st>>>(s.part, nparts, s.tgt, tok, s.blocks,
                                                            T);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  loss_mean_kernel<<<1, 256, 0, st>>>(s.blocks, row_blocks, T, loss ? loss : s.loss);
  return cudaGetLastError();
}

void harvest(cb_ctx* c) {
  if (!c->pending_harvest) return;
  c->pending_harvest = false;
  const int n = (int)c->ev_class.size();
  if (n == 0) return;
  if (cudaEventSynchronize(c->events[n]) != cudaSuccess) return;
  for (int i = 0; i < n; ++i) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, c->events[i], c->events[i + 1]) != cudaSuccess) continue;
    KStat& s = c->stats[c->ev_class[i]];
    s.launches += 1;
    s.ms += ms;
    s.flops += c->ev_flops[i];
    s.bytes += c->ev_bytes[i];
  }
}

cb_status validate_cfg(const cb_model_config* cfg, std::string* why) {
  auto bad = [&](const char* m) {
    *why = m;
    return CB_ERR_INVALID_ARG;
  };
  if (!cfg) return bad("null config");
  if (cfg->hd != 128) return bad("hd must be 128");
  if (cfg->dim <= 0 || cfg->hidden <= 0 || cfg->heads <= 0 || cfg->kv_heads <= 0 ||
      cfg->seq <= 0 || cfg->nlayers <= 0 || cfg->vocab <= 0)
    return bad("non-positive dimension");
  if (cfg->heads % cfg->kv_heads != 0) return bad("heads must be a multiple of kv_heads");
  if (cfg->dim % 256 != 0) return bad("dim must be a multiple of 256");
  if (cfg->hidden % 64 != 0) return bad("hidden must be a multiple of 64");
  if (cfg->seq % 64 != 0) return bad("seq must be a multiple of 64");
  if (cfg->vocab % 32 != 0) return bad("vocab must be a multiple of 32");
  return CB_OK;
}

// Megatron split of one model over tp_world ranks: kv heads (with their query heads)
// and 64-column hidden blocks are divided as evenly as possible, e.g. 52 heads over 8
// ranks = 7,7,7,7,6,6,6,6. info[8] = {tp_rank, tp_world, local heads, local kv heads,
// local hidden, first head, first kv head, first hidden column}.
cb_status tp_partition(const cb_model_config* cfg, int32_t tp_world, int32_t tp_rank,
                       int32_t* info, std::string* why) {
  if (validate_cfg(cfg, why) != CB_OK) return CB_ERR_INVALID_ARG;
  if (tp_world < 1 || tp_rank < 0 || tp_rank >= tp_world) {
    *why = "bad tensor-parallel rank/world";
    return CB_ERR_INVALID_ARG;
  }
  if (tp_world > cfg->kv_heads || tp_world > cfg->hidden / 64) {
    *why = "tensor-parallel world larger than the kv heads or hidden blocks";
    return CB_ERR_INVALID_ARG;
  }
  const int grp = cfg->heads / cfg->kv_heads;
  int kv0, nkv, b0, nb;
  split_even(cfg->kv_heads, tp_world, tp_rank, &kv0, &nkv);
  split_even(cfg->hidden / 64, tp_world, tp_rank, &b0, &nb);
  info[0] = tp_rank;
  info[1] = tp_world;
  info[2] = nkv * grp;
  info[3] = nkv;
  info[4] = nb * 64;
  info[5] = kv0 * grp;
  info[6] = kv0;
  info[7] = b0 * 64;
  return CB_OK;
}

}  // namespace

// ============================================================== C ABI

extern "C" {

const char* cb_version(void) { return CB_VERSION_STR; }

const char* cb_create_error(void) { return g_create_error.c_str(); }

cb_status cb_device_count(int32_t* count) {
  if (!count) return CB_ERR_INVALID_ARG;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;
  *count = n;
  return CB_OK;
}

const char* cb_last_error(const cb_ctx* ctx) {
  if (!ctx) return "null context";
  return ctx->err.c_str();
}

// Shared constructor of cb_create (tp_world == 1) and cb_create_tp.
static cb_status create_ctx(const cb_model_config* cfg, int32_t device, int32_t max_batch,
                            int32_t tp_rank, int32_t tp_world, const void* nccl_id,
                            cb_ctx** out) {
  g_create_error.clear();
  if (!out) {
    g_create_error = "null output pointer";
    return CB_ERR_INVALID_ARG;
  }
  *out = nullptr;
  std::string why;
  if (validate_cfg(cfg, &why) != CB_OK) {
    g_create_error = why;
    return CB_ERR_INVALID_ARG;
  }
  if (max_batch <= 0) {
    g_create_error = "max_batch must be positive";
    return CB_ERR_INVALID_ARG;
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    g_create_error = "no CUDA device";
    return CB_ERR_UNSUPPORTED;
  }
  if (device < 0 || device >= ndev) {
    g_create_error = "device index out of range";
    return CB_ERR_INVALID_ARG;
  }
  cudaDeviceProp prop;
  cudaGetDeviceProperties(&prop, device);
  if (prop.major != 10) {
    g_create_error = std::string("kernels are built for sm_100a; device is ") + prop.name;
    return CB_ERR_UNSUPPORTED;
  }
  if (!encode_fn()) {
    g_create_error = "cuTensorMapEncodeTiled unavailable";
    return CB_ERR_UNSUPPORTED;
  }

  int32_t part[8];
  if (tp_partition(cfg, tp_world, tp_rank, part, &why) != CB_OK) {
    g_create_error = why;
    return CB_ERR_INVALID_ARG;
  }
  if (tp_world > 1 && !nccl_api().ok()) {
    g_create_error = "NCCL unavailable: " + nccl_api().why;
    return CB_ERR_NCCL;
  }

  cb_ctx* ctx = new cb_ctx();
  ctx->cfg = *cfg;
  ctx->device = device;
  ctx->max_batch = max_batch;
  ctx->tp_rank = tp_rank;
  ctx->tp_world = tp_world;
  ctx->heads_l = part[2];
  ctx->kv_heads_l = part[3];
  ctx->hidden_l = part[4];
  ctx->q_off = part[5] * 128;
  ctx->kv_off = part[6] * 128;
  ctx->hid_off = part[7];
  ctx->q_dim = ctx->heads_l * 128;
  ctx->kv_dim = ctx->kv_heads_l * 128;
  ctx->n_qkv = ctx->q_dim + 2 * ctx->kv_dim;

  auto bail = [&](cb_status code, const std::string& m) {
    g_create_error = m;
    free_ctx(ctx);
    return code;
  };
#define CREATE_CUDA(call)                                                                     \
  do {                                                                                        \
    cudaError_t e_ = (call);                                                                  \
    if (e_ != cudaSuccess)                                                                    \
      return bail(e_ == cudaErrorMemoryAllocation ? CB_ERR_OUT_OF_MEMORY : CB_ERR_CUDA,       \
                  std::string(#call) + ": " + cudaGetErrorString(e_));                        \
  } while (0)

  CREATE_CUDA(cudaSetDevice(device));
  ctx->num_sms = num_sms_of(device);
  CREATE_CUDA(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking));
  ensure_attrs(device);

  const int L = cfg->nlayers, d = cfg->dim, hid = ctx->hidden_l, V = cfg->vocab, S = cfg->seq;
  const size_t T = ctx->T_max();
  CREATE_CUDA(dmalloc(&ctx->embed, (size_t)V * d));
  CREATE_CUDA(dmalloc(&ctx->wqkv, (size_t)L * wqkv_layer_elems(ctx)));
  CREATE_CUDA(dmalloc(&ctx->wo, (size_t)L * wo_layer_elems(ctx)));
  CREATE_CUDA(dmalloc(&ctx->w13, (size_t)L * w13_layer_elems(ctx)));
  CREATE_CUDA(dmalloc(&ctx->w2, (size_t)L * w2_layer_elems(ctx)));
  CREATE_CUDA(dmalloc(&ctx->gamma, (size_t)L * 2 * d));
  CREATE_CUDA(dmalloc(&ctx->gamma_final, (size_t)d));
  CREATE_CUDA(dmalloc(&ctx->x, T * d));
  CREATE_CUDA(dmalloc(&ctx->xn, T * d));
  CREATE_CUDA(dmalloc(&ctx->ss_part, T * ((d + 127) / 128)));
  CREATE_CUDA(dmalloc(&ctx->q, T * ctx->q_dim));
  CREATE_CUDA(dmalloc(&ctx->k, T * ctx->kv_dim));
  CREATE_CUDA(dmalloc(&ctx->v, T * ctx->kv_dim));
  CREATE_CUDA(dmalloc(&ctx->attn, T * ctx->q_dim));
  CREATE_CUDA(dmalloc(&ctx->g, T * hid));
  CREATE_CUDA(dmalloc(&ctx->delta, T * d));
  CREATE_CUDA(dmalloc(&ctx->delta32, T * d));
  CREATE_CUDA(dmalloc(&ctx->ce_part, T * ((V + 127) / 128)));
  CREATE_CUDA(dmalloc(&ctx->tgt_logit, T));
  CREATE_CUDA(dmalloc(&ctx->tok_loss, T));
  CREATE_CUDA(dmalloc(&ctx->block_sums, (T + ROW_WARPS - 1) / ROW_WARPS));
  CREATE_CUDA(dmalloc(&ctx->loss, 1));
  CREATE_CUDA(dmalloc(&ctx->tokens, T));
  CREATE_CUDA(dmalloc(&ctx->targets, T));
  CREATE_CUDA(dmalloc(&ctx->eval_pos, (size_t)ctx->max_batch));
  CREATE_CUDA(dmalloc(&ctx->rope, (size_t)S * 64));
  CREATE_CUDA(dmalloc(&ctx->rope_pm, (size_t)S * 64));
  CREATE_CUDA(dmalloc(&ctx->dev_err, 1));
  if (ctx->tp_world == 1) {  // split-K reduction of the fused single-GPU forward
    CREATE_CUDA(dmalloc(&ctx->fix_ws, FIX_WS_BYTES / sizeof(float4)));
    CREATE_CUDA(dmalloc(&ctx->fix_cnt, (size_t)FIX_COUNTERS));
    CREATE_CUDA(cudaMemset(ctx->fix_cnt, 0, FIX_COUNTERS * sizeof(int)));
  }
  CREATE_CUDA(cudaMallocHost(reinterpret_cast<void**>(&ctx->h_loss), sizeof(float)));
  CREATE_CUDA(cudaMallocHost(reinterpret_cast<void**>(&ctx->h_err), sizeof(int)));
  CREATE_CUDA(cudaMemset(ctx->dev_err, 0, sizeof(int)));
  CREATE_CUDA(cudaMemset(ctx->x, 0, T * d * sizeof(float)));
  CREATE_CUDA(cudaMemset(ctx->tgt_logit, 0, T * sizeof(float)));

  // RoPE table [64 pairs][S positions]: theta = p * 10000^(-2i/128) (sdpa_fwd.rs:24-39,
  // layer.rs:645-666), evaluated in double and rounded to f32 (the CPU oracle builds the
  // same values).
  {
    std::vector<float2> tab((size_t)S * 64);
    for (int p = 0; p < S; ++p)
      for (int i = 0; i < 64; ++i) {
        double th = (double)p * std::pow(10000.0, -2.0 * i / 128.0);
        tab[(size_t)i * S + p] = make_float2((float)std::cos(th), (float)std::sin(th));
      }
    CREATE_CUDA(cudaMemcpy(ctx->rope, tab.data(), tab.size() * sizeof(float2),
                           cudaMemcpyHostToDevice));
    std::vector<float2> pm(tab.size());
    for (int p = 0; p < S; ++p)
      for (int i = 0; i < 64; ++i) pm[(size_t)p * 64 + i] = tab[(size_t)i * S + p];
    CREATE_CUDA(cudaMemcpy(ctx->rope_pm, pm.data(), pm.size() * sizeof(float2),
                           cudaMemcpyHostToDevice));
  }

  bool ok = true;
  ok &= make_tmap(&ctx->tm_xn, ctx->xn, d, T, 1, 128);
  ok &= make_tmap_f32_rows(&ctx->tm_x, ctx->x, d, T, 32, 32, /*swizzle128=*/true);
  ok &= make_tmap_h32(&ctx->tm_xh, ctx->xn, d, T);
  ok &= make_tmap(&ctx->tm_attn, ctx->attn, ctx->q_dim, T, 1, 128);
  ok &= make_tmap(&ctx->tm_g, ctx->g, hid, T, 1, 128);
  ok &= make_tmap_qkv(&ctx->tm_q, ctx->q, T * ctx->heads_l, FA_BQ);
  ok &= make_tmap_qkv(&ctx->tm_k, ctx->k, T * ctx->kv_heads_l, FA_BKV);
  ok &= make_tmap_qkv(&ctx->tm_v, ctx->v, T * ctx->kv_heads_l, FA_BKV);
  for (int i = 0; i < 2; ++i) {
    const uint32_t bn = i ? 256 : 128;
    ok &= make_tmap(&ctx->tm_wqkv[i], ctx->wqkv, d, ctx->n_qkv, L, bn);
    ok &= make_tmap(&ctx->tm_wo[i], ctx->wo, ctx->q_dim, d, L, bn);
    ok &= make_tmap(&ctx->tm_w13[i], ctx->w13, d, 2 * hid, L, bn);
    ok &= make_tmap(&ctx->tm_w2[i], ctx->w2, hid, d, L, bn);
    ok &= make_tmap(&ctx->tm_embed[i], ctx->embed, d, V, 1, bn);
  }
  if (!ok) return bail(CB_ERR_UNSUPPORTED, "tensor map encoding failed");

  if (tp_world > 1) {
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof(id));
    // NCCL's all-reduces run beside the GEMMs (tp_chunked_forward): cap them at
    // tp_comm_sms(world) CTAs, the SMs the GEMMs leave free while they overlap.
    // Non-blocking: the set-up (which waits for every rank) is polled with a deadline.
    ncclResult_t nr;
    if (nccl_api().init_rank_config) {
      ncclConfig_t conf = NCCL_CONFIG_INITIALIZER;
      conf.maxCTAs = tp_comm_sms(tp_world);
      conf.blocking = 0;
      nr = nccl_api().init_rank_config(&ctx->comm, tp_world, id, tp_rank, &conf);
      if (ctx->comm) nr = nccl_settle(ctx, nr, "ncclCommInitRankConfig");
    } else {
      nr = nccl_api().init_rank(&ctx->comm, tp_world, id, tp_rank);
    }
    if (nr == ncclSuccess) {
      for (int i = 0; i < 4 * TP_MAX_CHUNKS; ++i)
        CREATE_CUDA(cudaEventCreateWithFlags(&ctx->tp_ev[i], cudaEventDisableTiming));
      CREATE_CUDA(cudaStreamCreateWithFlags(&ctx->comm_stream, cudaStreamNonBlocking));
    }
    if (nr != ncclSuccess) {
      const std::string why = ctx->nccl_failed ? ctx->err : nccl_api().error_string(nr);
      ctx->comm = nullptr;
      return bail(CB_ERR_NCCL, "ncclCommInitRank: " + why);
    }
    // One eager all-reduce so NCCL sets up its connections before any graph capture.
    nr = nccl_api().all_reduce(ctx->delta32, ctx->delta32, 1, ncclFloat32, ncclSum, ctx->comm,
                               ctx->stream);
    if (nccl_settle(ctx, nr, "ncclAllReduce") != ncclSuccess) return bail(CB_ERR_NCCL, ctx->err);
    // Likewise the reduce-scatters and all-gathers of the sequence-parallel forward, at
    // their largest size (the contents are not used).
    const size_t n = T * d / tp_world;
    nr = nccl_api().reduce_scatter(ctx->delta, ctx->delta + (size_t)tp_rank * n, n, ncclHalf,
                                   ncclSum, ctx->comm, ctx->stream);
    if (nccl_settle(ctx, nr, "ncclReduceScatter") != ncclSuccess) return bail(CB_ERR_NCCL, ctx->err);
    nr = nccl_api().reduce_scatter(ctx->delta32, ctx->delta32 + (size_t)tp_rank * n, n,
                                   ncclFloat32, ncclSum, ctx->comm, ctx->stream);
    if (nccl_settle(ctx, nr, "ncclReduceScatter") != ncclSuccess) return bail(CB_ERR_NCCL, ctx->err);
    nr = nccl_api().all_gather(ctx->delta + (size_t)tp_rank * n, ctx->delta, n, ncclHalf,
                               ctx->comm, ctx->stream);
    if (nccl_settle(ctx, nr, "ncclAllGather") != ncclSuccess) return bail(CB_ERR_NCCL, ctx->err);
    nr = nccl_api().all_gather(ctx->delta32 + (size_t)tp_rank * n, ctx->delta32, n, ncclFloat32,
                               ctx->comm, ctx->stream);
    if (nccl_settle(ctx, nr, "ncclAllGather") != ncclSuccess) return bail(CB_ERR_NCCL, ctx->err);
    if (sync_ctx_stream(ctx, ctx->stream) != CB_OK) return bail(CB_ERR_NCCL, ctx->err);
  }

  const int nev = launches_per_forward(ctx) + 1;
  ctx->events.resize(nev);
  for (int i = 0; i < nev; ++i) CREATE_CUDA(cudaEventCreate(&ctx->events[i]));
#undef CREATE_CUDA
  *out = ctx;
  return CB_OK;
}

cb_status cb_create(const cb_model_config* cfg, int32_t device, int32_t max_batch, cb_ctx** out) {
  return create_ctx(cfg, device, max_batch, 0, 1, nullptr, out);
}

cb_status cb_create_tp(const cb_model_config* cfg, int32_t device, int32_t max_batch,
                       int32_t tp_rank, int32_t tp_world, const void* nccl_unique_id,
                       cb_ctx** out) {
  if (tp_world > 1 && !nccl_unique_id) {
    g_create_error = "null NCCL unique id";
    return CB_ERR_INVALID_ARG;
  }
  return create_ctx(cfg, device, max_batch, tp_rank, tp_world, nccl_unique_id, out);
}

cb_status cb_nccl_unique_id(void* out) {
  if (!out) return CB_ERR_INVALID_ARG;
  if (!nccl_api().ok()) {
    g_create_error = "NCCL unavailable: " + nccl_api().why;
    return CB_ERR_NCCL;
  }
  ncclUniqueId id;
  ncclResult_t nr = nccl_api().get_unique_id(&id);
  if (nr != ncclSuccess) {
    g_create_error = std::string("ncclGetUniqueId: ") + nccl_api().error_string(nr);
    return CB_ERR_NCCL;
  }
  std::memcpy(out, &id, sizeof(id));
  return CB_OK;
}

cb_status cb_tp_info(const cb_ctx* ctx, int32_t* info) {
  if (!ctx || !info) return CB_ERR_INVALID_ARG;
  info[0] = ctx->tp_rank;
  info[1] = ctx->tp_world;
  info[2] = ctx->heads_l;
  info[3] = ctx->kv_heads_l;
  info[4] = ctx->hidden_l;
  info[5] = ctx->q_off / 128;
  info[6] = ctx->kv_off / 128;
  info[7] = ctx->hid_off;
  return CB_OK;
}

cb_status cb_tp_peer_lost(cb_ctx* ctx, const char* why) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  if (ctx->tp_world <= 1) return fail(ctx, CB_ERR_INVALID_ARG, "not a tensor-parallel context");
  if (!ctx->nccl_failed)
    nccl_fail(ctx, std::string("a peer rank left: ") + (why ? why : "reported by the caller"));
  return CB_OK;
}

cb_status cb_tp_partition(const cb_model_config* cfg, int32_t tp_world, int32_t tp_rank,
                          int32_t* info) {
  if (!info) return CB_ERR_INVALID_ARG;
  std::string why;
  const cb_status rc = tp_partition(cfg, tp_world, tp_rank, info, &why);
  if (rc != CB_OK) g_create_error = why;  // cb_create_error() tells the caller why
  return rc;
}

cb_status cb_attention_schedule(int32_t batch, int32_t heads, int32_t kv_heads, int32_t seq,
                                int32_t sms, int32_t* table, size_t cap, int32_t* grid,
                                size_t* len) {
  if (!grid || !len || batch < 1 || heads < 1 || kv_heads < 1 || heads % kv_heads != 0 ||
      seq < FA_BQ || seq % FA_BQ != 0 || sms < 1 || (long)batch * heads * (seq / FA_BQ) > (1L << 30))
    return CB_ERR_INVALID_ARG;
  int g = 0;
  const std::vector<int> t = attn_schedule_table(batch, heads, kv_heads, seq, 2 * sms, &g);
  *grid = g;
  *len = t.size();
  if (!table || t.size() > cap) return CB_ERR_INVALID_ARG;
  std::memcpy(table, t.data(), t.size() * sizeof(int));
  return CB_OK;
}

cb_status cb_destroy(cb_ctx* ctx) {
  if (!ctx) return CB_OK;
  cudaSetDevice(ctx->device);
  if (ctx->stream) sync_ctx_stream(ctx, ctx->stream);  // bounded for tensor-parallel contexts
  if (ctx->nccl_failed && ((ctx->stream && cudaStreamQuery(ctx->stream) == cudaErrorNotReady) ||
                           (ctx->comm_stream &&
                            cudaStreamQuery(ctx->comm_stream) == cudaErrorNotReady))) {
    // A collective toward a departed peer is still running: freeing device memory would
    // wait for it. The context's device memory is left to the end of the process.
    g_create_error = "context leaked: a collective of the failed communicator did not end";
    return CB_ERR_NCCL;
  }
  free_ctx(ctx);
  return CB_OK;
}

cb_status cb_init_weights(cb_ctx* ctx, uint64_t seed, int32_t scheme, float sigma) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  if (scheme != CB_INIT_NORMAL && scheme != CB_INIT_REFERENCE)
    return fail(ctx, CB_ERR_INVALID_ARG, "unknown init scheme");
  if (scheme == CB_INIT_NORMAL && !(sigma > 0.f))
    return fail(ctx, CB_ERR_INVALID_ARG, "sigma must be positive");
  CB_CUDA(cudaSetDevice(ctx->device));
  // A failure part-way leaves the weights half overwritten: no forward may run on them.
  ctx->weights_ready = false;
  const cb_model_config& cfg = ctx->cfg;
  InitParams p;
  p.seed = seed;
  p.scheme = scheme;
  p.normal_mul = (float)((double)sigma / CB_IRWIN_HALL4_STD);
  p.scale_embed = 0.005f;
  p.scale_qkv = 1.0f / sqrtf((float)cfg.dim);
  p.scale_ffn = 1.0f / sqrtf((float)cfg.hidden);
  const ShapeInfo s = shape_of(ctx);
  const int grid = ctx->num_sms * 8, block = 256;
  cudaStream_t st = ctx->stream;
  init_weight_kernel<<<grid, block, 0, st>>>(ctx->embed, ST_EMBED, -1, cfg.vocab, cfg.dim, s, p);
  for (int l = 0; l < cfg.nlayers; ++l) {
    init_weight_kernel<<<grid, block, 0, st>>>(ctx->wqkv + l * wqkv_layer_elems(ctx), ST_QKV, l,
                                               ctx->n_qkv, cfg.dim, s, p);
    init_weight_kernel<<<grid, block, 0, st>>>(ctx->wo + l * wo_layer_elems(ctx), ST_WO, l,
                                               cfg.dim, ctx->q_dim, s, p);
    init_weight_kernel<<<grid, block, 0, st>>>(ctx->w13 + l * w13_layer_elems(ctx), ST_W13, l,
                                               2 * ctx->hidden_l, cfg.dim, s, p);
    init_weight_kernel<<<grid, block, 0, st>>>(ctx->w2 + l * w2_layer_elems(ctx), ST_W2, l,
                                               cfg.dim, ctx->hidden_l, s, p);
  }
  fill_f32_kernel<<<grid, block, 0, st>>>(ctx->gamma, (size_t)cfg.nlayers * 2 * cfg.dim, 1.0f);
  fill_f32_kernel<<<grid, block, 0, st>>>(ctx->gamma_final, (size_t)cfg.dim, 1.0f);
  CB_CUDA(cudaGetLastError());
  CB_CUDA(cudaStreamSynchronize(st));
  ctx->weights_ready = true;
  return CB_OK;
}

// Uploads the model's f32 tensors in checkpoint order (train.rs:260-268): embed,
// gamma_final, then per layer wq, wk, wv, wo, w1, w3, w2, gamma1, gamma2.
// fetch(dst, n) enqueues on ctx->stream the copy of the source's next n floats into
// the device buffer dst. Matrices pass through one device staging buffer and are
// rounded to fp16 into their storage slots (each tensor-parallel rank keeps its own
// slice); gains are copied as they are. Returns false with ctx->err set on failure.
static cb_status run_forward(cb_ctx* ctx, int32_t batch, float softcap, cudaStream_t st);

extern "C++" {
template <class Fetch>
bool upload_model(cb_ctx* ctx, Fetch&& fetch) {
  const cb_model_config& cfg = ctx->cfg;
  const ShapeInfo s = shape_of(ctx);
  const size_t d = cfg.dim, hid = cfg.hidden, V = cfg.vocab, hid_l = ctx->hidden_l;
  const size_t qd_g = (size_t)cfg.heads * 128, kvd_g = (size_t)cfg.kv_heads * 128;
  const size_t stage_n = std::max(std::max(V * d, d * hid), std::max(d * qd_g, d * kvd_g));
  float* stage = nullptr;
  if (cudaMalloc(&stage, stage_n * sizeof(float)) != cudaSuccess) {
    ctx->err = "staging allocation failed";
    return false;
  }
  cudaStream_t st = ctx->stream;
  const int grid = ctx->num_sms * 8, block = 256;
  auto mat = [&](size_t n, __half* dst, int kind, int rows, int cols, int sub) -> bool {
    if (!fetch(stage, n)) return false;
    load_weight_kernel<<<grid, block, 0, st>>>(dst, kind, rows, cols, s, sub, stage);
    return cudaGetLastError() == cudaSuccess;
  };
  bool ok = mat(V * d, ctx->embed, ST_EMBED, (int)V, (int)d, -1) && fetch(ctx->gamma_final, d);
  for (int l = 0; ok && l < cfg.nlayers; ++l) {
    __half* qkv = ctx->wqkv + l * wqkv_layer_elems(ctx);
    __half* w13 = ctx->w13 + l * w13_layer_elems(ctx);
    ok = mat(d * qd_g, qkv, ST_QKV, ctx->n_qkv, (int)d, CB_T_WQ) &&
         mat(d * kvd_g, qkv, ST_QKV, ctx->n_qkv, (int)d, CB_T_WK) &&
         mat(d * kvd_g, qkv, ST_QKV, ctx->n_qkv, (int)d, CB_T_WV) &&
         mat(d * qd_g, ctx->wo + l * wo_layer_elems(ctx), ST_WO, (int)d, ctx->q_dim, CB_T_WO) &&
         mat(d * hid, w13, ST_W13, 2 * (int)hid_l, (int)d, CB_T_W1) &&
         mat(d * hid, w13, ST_W13, 2 * (int)hid_l, (int)d, CB_T_W3) &&
         mat(d * hid, ctx->w2 + l * w2_layer_elems(ctx), ST_W2, (int)d, (int)hid_l, CB_T_W2) &&
         fetch(ctx->gamma + (size_t)l * 2 * d, d) && fetch(ctx->gamma + (size_t)l * 2 * d + d, d);
  }
  const cudaError_t e = cudaStreamSynchronize(st);
  cudaFree(stage);
  if (ok && e != cudaSuccess) {
    ctx->err = std::string("weight upload: ") + cudaGetErrorString(e);
    ok = false;
  }
  return ok;
}
}  // extern "C++"

// Number of f32 values of a checkpoint's tensors (train.rs:303-331).
static uint64_t rstk_floats(const cb_model_config& c) {
  const uint64_t d = c.dim, qd = (uint64_t)c.heads * 128, kvd = (uint64_t)c.kv_heads * 128;
  const uint64_t per_layer = d * qd + 2 * d * kvd + qd * d + 3 * d * (uint64_t)c.hidden + 2 * d;
  return (uint64_t)c.vocab * d + d + (uint64_t)c.nlayers * per_layer;
}

cb_status cb_load_weights_f32(cb_ctx* ctx, const float* embed, const float* gamma_final,
                              const cb_layer_weights_f32* layers) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  if (!embed || !gamma_final || !layers)
    return fail(ctx, CB_ERR_INVALID_ARG, "null weight pointer");
  const cb_model_config& cfg = ctx->cfg;
  std::vector<const float*> src = {embed, gamma_final};
  for (int l = 0; l < cfg.nlayers; ++l) {
    const cb_layer_weights_f32& w = layers[l];
    const float* p[9] = {w.wq, w.wk, w.wv, w.wo, w.w1, w.w3, w.w2, w.gamma1, w.gamma2};
    for (const float* q : p) {
      if (!q) return fail(ctx, CB_ERR_INVALID_ARG, "null pointer in layer " + std::to_string(l));
      src.push_back(q);
    }
  }
  CB_CUDA(cudaSetDevice(ctx->device));
  ctx->weights_ready = false;  // as for cb_init_weights: a failed upload leaves none ready
  size_t next = 0;
  auto fetch = [&](float* dst, size_t n) -> bool {
    if (cudaMemcpyAsync(dst, src[next++], n * sizeof(float), cudaMemcpyHostToDevice,
                        ctx->stream) == cudaSuccess)
      return true;
    ctx->err = "host-to-device copy failed";
    return false;
  };
  if (!upload_model(ctx, fetch)) return fail(ctx, CB_ERR_CUDA, "weight upload failed: " + ctx->err);
  ctx->weights_ready = true;
  return CB_OK;
}

namespace {
struct Fd {
  int fd = -1;
  explicit Fd(const char* path) : fd(open(path, O_RDONLY | O_CLOEXEC)) {}
  ~Fd() {
    if (fd >= 0) close(fd);
  }
};
uint32_t le32(const unsigned char* p) {
  return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}
}  // namespace

cb_status cb_load_rstk(cb_ctx* ctx, const char* path, uint32_t* step_out) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  if (!path) return fail(ctx, CB_ERR_INVALID_ARG, "null path");
  Fd f(path);
  if (f.fd < 0) return fail(ctx, CB_ERR_INVALID_ARG, std::string("open ") + path + ": " + strerror(errno));
  struct stat sb;
  if (fstat(f.fd, &sb) != 0 || !S_ISREG(sb.st_mode))
    return fail(ctx, CB_ERR_INVALID_ARG, std::string(path) + " is not a regular file");
  unsigned char h[28];
  if (sb.st_size < 28 || pread(f.fd, h, 28, 0) != 28)
    return fail(ctx, CB_ERR_INVALID_ARG, "checkpoint shorter than its 28-byte header");
  if (std::memcmp(h, "RSTK", 4) != 0) return fail(ctx, CB_ERR_INVALID_ARG, "bad checkpoint magic");
  const uint32_t step = le32(h + 8), dim = le32(h + 12), nl = le32(h + 16), vocab = le32(h + 20);
  const cb_model_config& cfg = ctx->cfg;
  if (dim != (uint32_t)cfg.dim || nl != (uint32_t)cfg.nlayers || vocab != (uint32_t)cfg.vocab)
    return fail(ctx, CB_ERR_INVALID_ARG,
                "checkpoint header dim/nlayers/vocab " + std::to_string(dim) + "/" +
                    std::to_string(nl) + "/" + std::to_string(vocab) + " differ from the config");
  const uint64_t need = 28 + 4 * rstk_floats(cfg);
  if ((uint64_t)sb.st_size < need)
    return fail(ctx, CB_ERR_INVALID_ARG,
                "checkpoint truncated: " + std::to_string(sb.st_size) + " bytes, need " +
                    std::to_string(need));
  CB_CUDA(cudaSetDevice(ctx->device));
  FileStreamer fs(f.fd, ctx->stream);
  if (!fs.ok()) return fail(ctx, CB_ERR_OUT_OF_MEMORY, fs.error());
  uint64_t off = 28;
  auto fetch = [&](float* dst, size_t n) -> bool {
    const bool ok = fs.copy(dst, off, (uint64_t)n * 4);
    off += (uint64_t)n * 4;
    if (!ok) ctx->err = fs.error();
    return ok;
  };
  ctx->weights_ready = false;
  const bool ok = upload_model(ctx, fetch) && fs.finish();
  if (!ok) return fail(ctx, CB_ERR_CUDA, "checkpoint load failed: " + (fs.ok() ? ctx->err : fs.error()));
  if (step_out) *step_out = step;
  ctx->weights_ready = true;
  return CB_OK;
}

struct cb_tokens {
  int device = 0;
  int64_t n = 0;
  uint16_t* data = nullptr;
};

static cb_status tokens_alloc(int64_t n, int32_t device, cb_tokens** out) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    g_create_error = "no CUDA device";
    return CB_ERR_UNSUPPORTED;
  }
  if (device < 0 || device >= count) {
    g_create_error = "device index out of range";
    return CB_ERR_INVALID_ARG;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    g_create_error = "cudaSetDevice failed";
    return CB_ERR_CUDA;
  }
  cb_tokens* t = new cb_tokens;
  t->device = device;
  t->n = n;
  if (cudaMalloc(&t->data, std::max<size_t>(16, (size_t)n * 2)) != cudaSuccess) {
    delete t;
    g_create_error = "device allocation of the token array failed";
    return CB_ERR_OUT_OF_MEMORY;
  }
  *out = t;
  return CB_OK;
}

cb_status cb_tokens_open(const char* path, int32_t device, cb_tokens** out) {
  g_create_error.clear();
  if (!out) {
    g_create_error = "null output pointer";
    return CB_ERR_INVALID_ARG;
  }
  *out = nullptr;
  if (!path) {
    g_create_error = "null path";
    return CB_ERR_INVALID_ARG;
  }
  Fd f(path);
  struct stat sb;
  if (f.fd < 0 || fstat(f.fd, &sb) != 0) {
    g_create_error = std::string("open ") + path + ": " + strerror(errno);
    return CB_ERR_INVALID_ARG;
  }
  if (!S_ISREG(sb.st_mode)) {
    g_create_error = std::string(path) + " is not a regular file";
    return CB_ERR_INVALID_ARG;
  }
  const int64_t n = (int64_t)sb.st_size / 2;  // data.rs:23 n_tokens = len / 2
  cb_tokens* t = nullptr;
  cb_status rc = tokens_alloc(n, device, &t);
  if (rc != CB_OK) return rc;
  cudaStream_t st;
  if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
    cb_tokens_close(t);
    g_create_error = "stream creation failed";
    return CB_ERR_CUDA;
  }
  bool ok;
  std::string why;
  {
    FileStreamer fs(f.fd, st);
    ok = fs.ok() && fs.copy(t->data, 0, (uint64_t)n * 2) && fs.finish();
    why = fs.error();
  }
  cudaStreamDestroy(st);
  if (!ok) {
    cb_tokens_close(t);
    g_create_error = "token file load failed: " + why;
    return CB_ERR_CUDA;
  }
  *out = t;
  return CB_OK;
}

cb_status cb_tokens_from_host(const uint16_t* tokens, int64_t n, int32_t device,
                              cb_tokens** out) {
  g_create_error.clear();
  if (!out || (!tokens && n > 0) || n < 0) {
    g_create_error = "bad token array arguments";
    return CB_ERR_INVALID_ARG;
  }
  *out = nullptr;
  cb_tokens* t = nullptr;
  cb_status rc = tokens_alloc(n, device, &t);
  if (rc != CB_OK) return rc;
  if (n > 0 && cudaMemcpy(t->data, tokens, (size_t)n * 2, cudaMemcpyHostToDevice) != cudaSuccess) {
    cb_tokens_close(t);
    g_create_error = "token upload failed";
    return CB_ERR_CUDA;
  }
  *out = t;
  return CB_OK;
}

cb_status cb_tokens_len(const cb_tokens* data, int64_t* n) {
  if (!data || !n) return CB_ERR_INVALID_ARG;
  *n = data->n;
  return CB_OK;
}

cb_status cb_tokens_close(cb_tokens* data) {
  if (!data) return CB_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(data->device);
  cudaFree(data->data);
  cudaSetDevice(prev);
  delete data;
  return CB_OK;
}

// Gathers `batch` windows (positions already on the device in ctx->eval_pos + first)
// into the context's token/target buffers and runs one forward, all on ctx->stream.
static cb_status windows_forward(cb_ctx* ctx, const cb_tokens* data, size_t first, int32_t batch,
                                 float softcap) {
  const int S = ctx->cfg.seq;
  const int64_t total = (int64_t)batch * S;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)ctx->num_sms * 8);
  gather_windows_kernel<<<grid, 256, 0, ctx->stream>>>(data->data, data->n, ctx->eval_pos + first,
                                                       batch, S, ctx->cfg.vocab, ctx->tokens,
                                                       ctx->targets, ctx->dev_err);
  CB_CUDA(cudaGetLastError());
  return run_forward(ctx, batch, softcap, ctx->stream);
}

static cb_status read_device_error(cb_ctx* ctx) {
  CB_CUDA(cudaMemcpyAsync(ctx->h_err, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost,
                          ctx->stream));
  if (const cb_status rc = sync_ctx_stream(ctx, ctx->stream); rc != CB_OK) return rc;
  if (*ctx->h_err != 0) {
    const int code = *ctx->h_err;
    cudaMemsetAsync(ctx->dev_err, 0, sizeof(int), ctx->stream);
    reset_split_counters(ctx, ctx->stream);
    sync_ctx_stream(ctx, ctx->stream);
    return fail(ctx, code == DEV_ERR_WAIT_TIMEOUT ? CB_ERR_DEVICE_TIMEOUT : CB_ERR_INVALID_ARG,
                code == DEV_ERR_BAD_TOKEN ? "token id out of range in the token data"
                                          : "device error flag " + std::to_string(code));
  }
  return CB_OK;
}

static cb_status check_windows(cb_ctx* ctx, const cb_tokens* data) {
  if (!ctx->weights_ready) return fail(ctx, CB_ERR_NOT_READY, "weights are not loaded");
  if (!data) return fail(ctx, CB_ERR_INVALID_ARG, "null token data");
  if (data->device != ctx->device)
    return fail(ctx, CB_ERR_INVALID_ARG, "token data lives on another device");
  return CB_OK;
}

cb_status cb_forward_loss_windows(cb_ctx* ctx, const cb_tokens* data, const int64_t* positions,
                                  int32_t batch, float softcap, float* loss_out,
                                  float* per_token_loss) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  cb_status rc = check_windows(ctx, data);
  if (rc != CB_OK) return rc;
  if (!positions || !loss_out) return fail(ctx, CB_ERR_INVALID_ARG, "null positions/loss_out");
  if (batch <= 0 || batch > ctx->max_batch)
    return fail(ctx, CB_ERR_INVALID_ARG, "batch " + std::to_string(batch) + " outside [1, " +
                                             std::to_string(ctx->max_batch) + "]");
  const int S = ctx->cfg.seq;
  for (int b = 0; b < batch; ++b)
    if (positions[b] < 0 || positions[b] + S + 1 > data->n)
      return fail(ctx, CB_ERR_INVALID_ARG,
                  "window " + std::to_string(b) + " at " + std::to_string(positions[b]) +
                      " runs past the token data");
  CB_CUDA(cudaSetDevice(ctx->device));
  CB_CUDA(cudaMemcpyAsync(ctx->eval_pos, positions, (size_t)batch * 8, cudaMemcpyHostToDevice,
                          ctx->stream));
  rc = windows_forward(ctx, data, 0, batch, softcap);
  if (rc != CB_OK) return rc;
  const size_t T = (size_t)batch * S;
  CB_CUDA(cudaMemcpyAsync(ctx->h_loss, ctx->loss, sizeof(float), cudaMemcpyDeviceToHost,
                          ctx->stream));
  if (per_token_loss)
    CB_CUDA(cudaMemcpyAsync(per_token_loss, ctx->tok_loss, T * sizeof(float),
                            cudaMemcpyDeviceToHost, ctx->stream));
  rc = read_device_error(ctx);
  if (rc != CB_OK) return rc;
  *loss_out = *ctx->h_loss;
  return CB_OK;
}

cb_status cb_eval_windows(cb_ctx* ctx, const cb_tokens* data, const int32_t* token_bytes,
                          int32_t n_token_bytes, int64_t step_begin, int64_t step_end,
                          float softcap, cb_eval_totals* out) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  cb_status rc = check_windows(ctx, data);
  if (rc != CB_OK) return rc;
  if (!out) return fail(ctx, CB_ERR_INVALID_ARG, "null output");
  if (step_begin < 0 || step_end < step_begin)
    return fail(ctx, CB_ERR_INVALID_ARG, "bad step range");
  if (token_bytes && n_token_bytes <= 0)
    return fail(ctx, CB_ERR_INVALID_ARG, "empty token_bytes table");
  const int S = ctx->cfg.seq;
  const int64_t max_pos = data->n - S - 1;  // train.rs:207
  if (max_pos <= 0)
    return fail(ctx, CB_ERR_INVALID_ARG, "token data shorter than seq + 2 tokens");
  CB_CUDA(cudaSetDevice(ctx->device));
  const int64_t steps = step_end - step_begin;
  std::memset(out, 0, sizeof(*out));
  if (steps == 0) return CB_OK;
  int32_t* d_bytes = nullptr;
  EvalSums* d_sums = nullptr;
  int64_t* d_pos = nullptr;
  std::vector<int64_t> pos((size_t)steps);
  for (int64_t i = 0; i < steps; ++i) pos[(size_t)i] = ((step_begin + i) * S) % max_pos;  // :209
  auto cleanup = [&] {
    cudaFree(d_bytes);
    cudaFree(d_sums);
    cudaFree(d_pos);
  };
  if (cudaMalloc(&d_sums, sizeof(EvalSums)) != cudaSuccess ||
      cudaMalloc(&d_pos, (size_t)steps * 8) != cudaSuccess ||
      (token_bytes && cudaMalloc(&d_bytes, (size_t)n_token_bytes * 4) != cudaSuccess)) {
    cleanup();
    return fail(ctx, CB_ERR_OUT_OF_MEMORY, "evaluation buffers");
  }
  cudaStream_t st = ctx->stream;
  cudaError_t e = cudaMemsetAsync(d_sums, 0, sizeof(EvalSums), st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(d_pos, pos.data(), (size_t)steps * 8, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && token_bytes)
    e = cudaMemcpyAsync(d_bytes, token_bytes, (size_t)n_token_bytes * 4, cudaMemcpyHostToDevice,
                        st);
  if (e != cudaSuccess) {
    cleanup();
    return fail(ctx, CB_ERR_CUDA, std::string("evaluation setup: ") + cudaGetErrorString(e));
  }
  int64_t* saved_pos = ctx->eval_pos;
  ctx->eval_pos = d_pos;
  for (int64_t first = 0; first < steps && rc == CB_OK; first += ctx->max_batch) {
    const int32_t b = (int32_t)std::min<int64_t>(ctx->max_batch, steps - first);
    rc = windows_forward(ctx, data, (size_t)first, b, softcap);
    if (rc == CB_OK) {
      eval_accumulate_kernel<<<1, EVAL_THREADS, 0, st>>>(ctx->tok_loss, ctx->targets, d_bytes,
                                                         n_token_bytes, b * S, d_sums);
      if (cudaGetLastError() != cudaSuccess) rc = fail(ctx, CB_ERR_CUDA, "evaluation launch");
    }
  }
  ctx->eval_pos = saved_pos;
  EvalSums h{};
  if (rc == CB_OK) {
    e = cudaMemcpyAsync(&h, d_sums, sizeof(h), cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) rc = fail(ctx, CB_ERR_CUDA, "evaluation read-back");
  }
  if (rc == CB_OK) rc = read_device_error(ctx);
  sync_ctx_stream(ctx, st);
  cleanup();
  if (rc != CB_OK) return rc;
  out->loss_sum = h.loss_sum;
  out->nats = h.nats;
  out->bytes = h.bytes;
  out->tokens = h.tokens;
  return CB_OK;
}

// Makes the attention schedules a forward of `batch` sequences may launch (also the
// sequence chunks of the tensor-parallel forward) before anything is captured.
cudaError_t prepare_attention(cb_ctx* c, int batch) {
  if (c->cfg.seq % FA_BQ != 0) return cudaSuccess;
  for (int k = 1; k <= 8 && k <= batch; ++k) {
    if (batch % k != 0) continue;
    const AttnSched* s = nullptr;
    const cudaError_t e =
        attn_schedule(batch / k, c->heads_l, c->kv_heads_l, c->cfg.seq, nullptr, &s);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

static cb_status run_forward(cb_ctx* ctx, int32_t batch, float softcap, cudaStream_t st) {
  if (ctx->nccl_failed)
    return fail(ctx, CB_ERR_NCCL, "the tensor-parallel communicator has failed: " + ctx->nccl_why);
  if (ctx->profiling) {
    harvest(ctx);
    cudaError_t e = enqueue_forward(ctx, batch, softcap, st, true);
    if (e != cudaSuccess && ctx->nccl_failed) return fail(ctx, CB_ERR_NCCL, ctx->err);
    if (e != cudaSuccess) return fail(ctx, CB_ERR_CUDA, std::string("forward: ") + cudaGetErrorString(e));
    ctx->pending_harvest = true;
  } else {
    uint32_t sc_bits;
    std::memcpy(&sc_bits, &softcap, 4);
    auto key = std::make_pair((int)batch, sc_bits);
    auto it = ctx->graphs.find(key);
    if (it == ctx->graphs.end()) {
      cudaGraph_t graph = nullptr;
      cudaGraphExec_t exec = nullptr;
      CB_CUDA(prepare_attention(ctx, batch));
      CB_CUDA(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
      cudaError_t e = enqueue_forward(ctx, batch, softcap, ctx->stream, false);
      cudaError_t e2 = cudaStreamEndCapture(ctx->stream, &graph);
      if (e != cudaSuccess || e2 != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        if (ctx->nccl_failed) return fail(ctx, CB_ERR_NCCL, ctx->err);
        return fail(ctx, CB_ERR_CUDA,
                    std::string("graph capture: ") +
                        cudaGetErrorString(e != cudaSuccess ? e : e2));
      }
      e = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      if (e != cudaSuccess)
        return fail(ctx, CB_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
      it = ctx->graphs.emplace(key, exec).first;
    }
    CB_CUDA(cudaGraphLaunch(it->second, st));
  }
  ctx->last_batch = batch;
  ctx->last_softcap = softcap;
  ctx->x_final = ctx->x;
  return CB_OK;
}

static cb_status check_forward_args(cb_ctx* ctx, const void* tokens, const void* targets,
                                    int32_t batch) {
  if (!ctx->weights_ready) return fail(ctx, CB_ERR_NOT_READY, "weights are not loaded");
  if (!tokens || !targets) return fail(ctx, CB_ERR_INVALID_ARG, "null tokens/targets");
  if (batch <= 0 || batch > ctx->max_batch)
    return fail(ctx, CB_ERR_INVALID_ARG,
                "batch " + std::to_string(batch) + " outside [1, " +
                    std::to_string(ctx->max_batch) + "]");
  return CB_OK;
}

cb_status cb_forward_loss(cb_ctx* ctx, const uint32_t* tokens, const uint32_t* targets,
                          int32_t batch, float softcap, float* loss_out, float* per_token_loss) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  cb_status rc = check_forward_args(ctx, tokens, targets, batch);
  if (rc != CB_OK) return rc;
  if (!loss_out) return fail(ctx, CB_ERR_INVALID_ARG, "null loss_out");
  const size_t T = (size_t)batch * ctx->cfg.seq;
  const uint32_t V = (uint32_t)ctx->cfg.vocab;
  for (size_t i = 0; i < T; ++i)
    if (tokens[i] >= V || targets[i] >= V)
      return fail(ctx, CB_ERR_INVALID_ARG, "token id out of range at position " + std::to_string(i));
  CB_CUDA(cudaSetDevice(ctx->device));
  cudaStream_t st = ctx->stream;
  CB_CUDA(cudaMemcpyAsync(ctx->tokens, tokens, T * 4, cudaMemcpyHostToDevice, st));
  CB_CUDA(cudaMemcpyAsync(ctx->targets, targets, T * 4, cudaMemcpyHostToDevice, st));
  rc = run_forward(ctx, batch, softcap, st);
  if (rc != CB_OK) return rc;
  CB_CUDA(cudaMemcpyAsync(ctx->h_loss, ctx->loss, sizeof(float), cudaMemcpyDeviceToHost, st));
  CB_CUDA(cudaMemcpyAsync(ctx->h_err, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost, st));
  if (per_token_loss)
    CB_CUDA(cudaMemcpyAsync(per_token_loss, ctx->tok_loss, T * sizeof(float),
                            cudaMemcpyDeviceToHost, st));
  if ((rc = sync_ctx_stream(ctx, st)) != CB_OK) return rc;
  if (*ctx->h_err != 0) {
    int code = *ctx->h_err;
    cudaMemsetAsync(ctx->dev_err, 0, sizeof(int), st);
    reset_split_counters(ctx, st);
    sync_ctx_stream(ctx, st);
    return fail(ctx, code == DEV_ERR_WAIT_TIMEOUT ? CB_ERR_DEVICE_TIMEOUT : CB_ERR_INVALID_ARG,
                "device error flag " + std::to_string(code));
  }
  *loss_out = *ctx->h_loss;
  return CB_OK;
}

cb_status cb_forward_loss_async(cb_ctx* ctx, const uint32_t* d_tokens, const uint32_t* d_targets,
                                int32_t batch, float softcap, float* d_loss,
                                float* d_per_token_loss, void* stream) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  cb_status rc = check_forward_args(ctx, d_tokens, d_targets, batch);
  if (rc != CB_OK) return rc;
  CB_CUDA(cudaSetDevice(ctx->device));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  const size_t T = (size_t)batch * ctx->cfg.seq;
  if (d_tokens != ctx->tokens)
    CB_CUDA(cudaMemcpyAsync(ctx->tokens, d_tokens, T * 4, cudaMemcpyDeviceToDevice, st));
  if (d_targets != ctx->targets)
    CB_CUDA(cudaMemcpyAsync(ctx->targets, d_targets, T * 4, cudaMemcpyDeviceToDevice, st));
  rc = run_forward(ctx, batch, softcap, st);
  if (rc != CB_OK) return rc;
  if (d_loss)
    CB_CUDA(cudaMemcpyAsync(d_loss, ctx->loss, sizeof(float), cudaMemcpyDeviceToDevice, st));
  if (d_per_token_loss)
    CB_CUDA(cudaMemcpyAsync(d_per_token_loss, ctx->tok_loss, T * sizeof(float),
                            cudaMemcpyDeviceToDevice, st));
  return CB_OK;
}

cb_status cb_check_device_error(cb_ctx* ctx) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  CB_CUDA(cudaSetDevice(ctx->device));
  if (const cb_status rc = sync_ctx_stream(ctx, ctx->stream); rc != CB_OK) return rc;
  CB_CUDA(cudaDeviceSynchronize());
  CB_CUDA(cudaMemcpy(ctx->h_err, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (*ctx->h_err != 0) {
    int code = *ctx->h_err;
    cudaMemset(ctx->dev_err, 0, sizeof(int));
    reset_split_counters(ctx, nullptr);
    return fail(ctx, code == DEV_ERR_WAIT_TIMEOUT ? CB_ERR_DEVICE_TIMEOUT : CB_ERR_INVALID_ARG,
                "device error flag " + std::to_string(code));
  }
  return CB_OK;
}

// Self-test of the bounded device waits: a miniature of the pipeline kernels whose
// producer never produces. Warp 1 owns a TMEM allocation (as the GEMM and attention
// kernels do) and lane 0 of it waits for a "full" barrier nothing arrives on; warps
// 2-3 wait for the barrier that consumer would release. The consumer's wait expires
// after limit_ns and records DEV_ERR_WAIT_TIMEOUT in *err; the other warps see the
// flag and stop waiting too (their own limit is far longer); warp 1 frees its TMEM
// and the kernel returns, leaving the context usable.
__global__ void __launch_bounds__(128) wait_selftest_kernel(uint64_t limit_ns, int* err) {
  __shared__ uint64_t bar_full, bar_done;
  __shared__ uint32_t tmem_slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bar_full, 1);
    mbar_init(&bar_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1 && lane == 0) {
    if (mbar_wait_for(&bar_full, 0, err, limit_ns)) mbar_arrive(&bar_done);
  } else if (warp >= 2) {
    mbar_wait_for(&bar_done, 0, err, 64 * limit_ns);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_slot, 32);
  }
}

cb_status cb_selftest_wait_timeout(cb_ctx* ctx, uint32_t limit_us) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  if (limit_us < 1 || limit_us > 2000000)
    return fail(ctx, CB_ERR_INVALID_ARG, "limit_us must be in [1, 2000000]");
  CB_CUDA(cudaSetDevice(ctx->device));
  if (const cb_status rc = sync_ctx_stream(ctx, ctx->stream); rc != CB_OK) return rc;
  wait_selftest_kernel<<<1, 128, 0, ctx->stream>>>((uint64_t)limit_us * 1000ull, ctx->dev_err);
  CB_CUDA(cudaGetLastError());
  CB_CUDA(cudaMemcpyAsync(ctx->h_err, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost,
                          ctx->stream));
  CB_CUDA(cudaStreamSynchronize(ctx->stream));
  if (*ctx->h_err != 0) {
    const int code = *ctx->h_err;
    CB_CUDA(cudaMemsetAsync(ctx->dev_err, 0, sizeof(int), ctx->stream));
    reset_split_counters(ctx, ctx->stream);
    CB_CUDA(cudaStreamSynchronize(ctx->stream));
    return fail(ctx, code == DEV_ERR_WAIT_TIMEOUT ? CB_ERR_DEVICE_TIMEOUT : CB_ERR_INVALID_ARG,
                "self-test: a device wait expired after " + std::to_string(limit_us) +
                    " us (device error flag " + std::to_string(code) + ")");
  }
  return CB_OK;
}

cb_status cb_sampled_logits(cb_ctx* ctx, const int32_t* rows, int32_t n_rows, float* logits_out) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  if (ctx->last_batch <= 0) return fail(ctx, CB_ERR_NOT_READY, "no forward has run");
  if (!rows || !logits_out || n_rows <= 0)
    return fail(ctx, CB_ERR_INVALID_ARG, "bad sampled-logit arguments");
  const int T = ctx->last_batch * ctx->cfg.seq;
  for (int i = 0; i < n_rows; ++i)
    if (rows[i] < 0 || rows[i] >= T)
      return fail(ctx, CB_ERR_INVALID_ARG, "sampled row out of range");
  CB_CUDA(cudaSetDevice(ctx->device));
  const int d = ctx->cfg.dim, V = ctx->cfg.vocab;
  const int n_pad = (n_rows + 127) / 128 * 128;
  cudaStream_t st = ctx->stream;
  if (const cb_status rc = sync_ctx_stream(ctx, st); rc != CB_OK) return rc;
  if (n_pad > ctx->samp_cap) {
    if (ctx->samp_a) cudaFree(ctx->samp_a);
    if (ctx->samp_out) cudaFree(ctx->samp_out);
    ctx->samp_a = nullptr;
    ctx->samp_out = nullptr;
    ctx->samp_cap = 0;
    CB_CUDA(dmalloc(&ctx->samp_a, (size_t)n_pad * d));
    CB_CUDA(dmalloc(&ctx->samp_out, (size_t)n_pad * V));
    ctx->samp_cap = n_pad;
  }
  int32_t* d_rows = nullptr;
  CB_CUDA(cudaMalloc(&d_rows, n_rows * sizeof(int32_t)));
  cudaError_t e = cudaMemcpyAsync(d_rows, rows, n_rows * sizeof(int32_t), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) {
    gather_norm_rows_kernel<<<n_pad, 128, 0, st>>>(ctx->x_final, d_rows, ctx->gamma_final, n_rows,
                                                   n_pad, d, ctx->samp_a);
    e = cudaGetLastError();
  }
  CUtensorMap ta;
  if (e == cudaSuccess && !make_tmap(&ta, ctx->samp_a, d, n_pad, 1, 128)) e = cudaErrorInvalidValue;
  if (e == cudaSuccess) {
    EpiStoreF32 ep{ctx->samp_out, V, ctx->last_softcap};
    const DeviceInfo& di = device_info(ctx->device);
    e = launch_gemm(pick_mode(n_pad, V, di), ta, ctx->tm_embed[0], ctx->tm_embed[1], n_pad, V, d,
                    0, ep, ctx->dev_err, di, st);
  }
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(logits_out, ctx->samp_out, (size_t)n_rows * V * sizeof(float),
                        cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  cudaFree(d_rows);
  if (e != cudaSuccess)
    return fail(ctx, CB_ERR_CUDA, std::string("sampled logits: ") + cudaGetErrorString(e));
  return CB_OK;
}

cb_status cb_set_profiling(cb_ctx* ctx, int32_t enable) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  if (!enable) harvest(ctx);
  ctx->profiling = enable != 0;
  return CB_OK;
}

cb_status cb_kernel_times(cb_ctx* ctx, cb_kernel_time* out, int32_t max_entries,
                          int32_t* n_entries) {
  if (!ctx || !n_entries) return CB_ERR_INVALID_ARG;
  CB_CUDA(cudaSetDevice(ctx->device));
  harvest(ctx);
  int n = 0;
  for (int i = 0; i < K_NUM; ++i) {
    if (ctx->stats[i].launches == 0) continue;
    if (out && n < max_entries) {
      cb_kernel_time& t = out[n];
      std::memset(&t, 0, sizeof(t));
      std::strncpy(t.name, kclass_name[i], sizeof(t.name) - 1);
      t.launches = ctx->stats[i].launches;
      t.total_ms = ctx->stats[i].ms;
      t.flops = ctx->stats[i].flops;
      t.bytes = ctx->stats[i].bytes;
    }
    ++n;
  }
  *n_entries = n;
  return CB_OK;
}

cb_status cb_reset_kernel_times(cb_ctx* ctx) {
  if (!ctx) return CB_ERR_INVALID_ARG;
  harvest(ctx);
  for (auto& s : ctx->stats) s = KStat();
  return CB_OK;
}

cb_status cb_get_stream(cb_ctx* ctx, void** stream) {
  if (!ctx || !stream) return CB_ERR_INVALID_ARG;
  *stream = ctx->stream;
  return CB_OK;
}

cb_status cb_gemm_f16(const void* A, const void* B, void* C, int32_t M, int32_t N, int32_t K,
                      int32_t out_f32, int32_t block_n, void* stream) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0) return CB_ERR_INVALID_ARG;
  if (K % 64 != 0 || N % 32 != 0 || out_f32 < 0 || out_f32 > 2) return CB_ERR_INVALID_ARG;
  if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)C) & 15) return CB_ERR_INVALID_ARG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CB_ERR_CUDA;
  const DeviceInfo& di = device_info(dev);
  int mode;
  if (block_n == 128) mode = GM_SINGLE128;
  else if (block_n == 256) mode = GM_SINGLE256;
  else if (block_n == 2) mode = GM_PAIR;
  else mode = pick_mode(M, N, di);
  if (mode != GM_SINGLE128 && N % 256 != 0) mode = GM_SINGLE128;
  CUtensorMap ta, tb128, tb256;
  if (!make_tmap(&ta, A, K, M, 1, 128) || !make_tmap(&tb128, B, K, N, 1, 128) ||
      !make_tmap(&tb256, B, K, N, 1, 256))
    return CB_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (out_f32 == 2) {
    EpiScaledF32Add ep{static_cast<float*>(C), N, 1.f};
    e = launch_gemm(mode, ta, tb128, tb256, M, N, K, 0, ep, nullptr, di, st, K >= 128 ? 2 : 1);
  } else if (out_f32) {
    EpiStoreF32 ep{static_cast<float*>(C), N, 0.f};
    e = launch_gemm(mode, ta, tb128, tb256, M, N, K, 0, ep, nullptr, di, st);
  } else {
    EpiStoreF16 ep{static_cast<__half*>(C), N};
    e = launch_gemm(mode, ta, tb128, tb256, M, N, K, 0, ep, nullptr, di, st);
  }
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

extern "C++" {
template <int LAYOUT>
static cudaError_t gemm_layout_launch(int mode, const CUtensorMap& ta, const CUtensorMap& tb128,
                                      const CUtensorMap& tb256, void* C, int M, int N, int K,
                                      int out_mode, const DeviceInfo& di, cudaStream_t st) {
  if (out_mode == 2) {
    EpiScaledF32Add ep{static_cast<float*>(C), N, 1.f};
    return launch_gemm<EpiScaledF32Add, LAYOUT>(mode, ta, tb128, tb256, M, N, K, 0, ep, nullptr,
                                                di, st, K >= 128 ? 2 : 1);
  }
  if (out_mode == 1) {
    EpiStoreF32 ep{static_cast<float*>(C), N, 0.f};
    return launch_gemm<EpiStoreF32, LAYOUT>(mode, ta, tb128, tb256, M, N, K, 0, ep, nullptr, di,
                                            st);
  }
  EpiStoreF16 ep{static_cast<__half*>(C), N};
  return launch_gemm<EpiStoreF16, LAYOUT>(mode, ta, tb128, tb256, M, N, K, 0, ep, nullptr, di, st);
}
}  // extern "C++"

cb_status cb_gemm_f16_layout(const void* A, const void* B, void* C, int32_t M, int32_t N,
                             int32_t K, int32_t layout, int32_t out_f32, int32_t block_n,
                             void* stream) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0 || layout < 0 || layout > 3)
    return CB_ERR_INVALID_ARG;
  if (N % 32 != 0 || out_f32 < 0 || out_f32 > 2) return CB_ERR_INVALID_ARG;
  if ((layout & GEMM_A_MN) ? (M % 64 != 0) : (K % 8 != 0)) return CB_ERR_INVALID_ARG;
  if ((layout & GEMM_B_MN) ? (N % 64 != 0) : (K % 8 != 0)) return CB_ERR_INVALID_ARG;
  if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)C) & 15) return CB_ERR_INVALID_ARG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CB_ERR_CUDA;
  const DeviceInfo& di = device_info(dev);
  int mode;
  if (block_n == 128) mode = GM_SINGLE128;
  else if (block_n == 256) mode = GM_SINGLE256;
  else if (block_n == 2) mode = GM_PAIR;
  else mode = pick_mode(M, N, di);
  if (mode != GM_SINGLE128 && N % 256 != 0) mode = GM_SINGLE128;
  CUtensorMap ta, tb128, tb256;
  const bool a_ok = (layout & GEMM_A_MN) ? make_tmap_mn(&ta, A, M, K, 1)
                                         : make_tmap(&ta, A, K, M, 1, 128);
  bool b_ok;
  if (layout & GEMM_B_MN) {
    b_ok = make_tmap_mn(&tb128, B, N, K, 1);
    tb256 = tb128;
  } else {
    b_ok = make_tmap(&tb128, B, K, N, 1, 128) && make_tmap(&tb256, B, K, N, 1, 256);
  }
  if (!a_ok || !b_ok) return CB_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (layout) {
    case 1: e = gemm_layout_launch<1>(mode, ta, tb128, tb256, C, M, N, K, out_f32, di, st); break;
    case 2: e = gemm_layout_launch<2>(mode, ta, tb128, tb256, C, M, N, K, out_f32, di, st); break;
    case 3: e = gemm_layout_launch<3>(mode, ta, tb128, tb256, C, M, N, K, out_f32, di, st); break;
    default: e = gemm_layout_launch<0>(mode, ta, tb128, tb256, C, M, N, K, out_f32, di, st);
  }
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

cb_status cb_attention_f16(const void* q, const void* k, const void* v, void* out, int32_t batch,
                           int32_t heads, int32_t seq, void* stream) {
  if (!q || !k || !v || !out || batch <= 0 || heads <= 0 || seq <= 0 || seq % 64 != 0)
    return CB_ERR_INVALID_ARG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CB_ERR_CUDA;
  ensure_attrs(dev);
  const uint64_t rows = (uint64_t)batch * heads * seq;
  CUtensorMap tq, tk, tv;
  const bool tc = seq % FA_BQ == 0 && make_tmap_qkv(&tq, q, rows, FA_BQ) &&
                  make_tmap_qkv(&tk, k, rows, FA_BKV) && make_tmap_qkv(&tv, v, rows, FA_BKV);
  cudaError_t e = launch_attention(tc ? &tq : nullptr, &tk, &tv, static_cast<const __half*>(q),
                                   static_cast<const __half*>(k), static_cast<const __half*>(v),
                                   static_cast<__half*>(out), batch, heads, heads, seq, nullptr,
                                   static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

cb_status cb_attention_fwd_lse_f16(const void* q, const void* k, const void* v, void* out,
                                   float* lse, int32_t batch, int32_t heads, int32_t kv_heads,
                                   int32_t seq, void* stream) {
  if (!q || !k || !v || !out || !lse || batch <= 0 || heads <= 0 || kv_heads <= 0 ||
      heads % kv_heads != 0 || seq <= 0 || seq % 64 != 0)
    return CB_ERR_INVALID_ARG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CB_ERR_CUDA;
  ensure_attrs(dev);
  CUtensorMap tq, tk, tv;
  const bool tc = seq % FA_BQ == 0 &&
                  make_tmap_qkv(&tq, q, (uint64_t)batch * heads * seq, FA_BQ) &&
                  make_tmap_qkv(&tk, k, (uint64_t)batch * kv_heads * seq, FA_BKV) &&
                  make_tmap_qkv(&tv, v, (uint64_t)batch * kv_heads * seq, FA_BKV);
  cudaError_t e = launch_attention(tc ? &tq : nullptr, &tk, &tv, static_cast<const __half*>(q),
                                   static_cast<const __half*>(k), static_cast<const __half*>(v),
                                   static_cast<__half*>(out), batch, heads, kv_heads, seq, nullptr,
                                   static_cast<cudaStream_t>(stream), lse);
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

cb_status cb_attention_bwd_f16(const void* q, const void* k, const void* v, const void* o,
                               const void* dout, const float* lse, void* dqkv, int32_t batch,
                               int32_t heads, int32_t kv_heads, int32_t seq, void* stream) {
  if (!q || !k || !v || !o || !dout || !lse || !dqkv || batch <= 0 || heads <= 0 ||
      kv_heads <= 0 || heads % kv_heads != 0 || seq <= 0 || seq % 64 != 0)
    return CB_ERR_INVALID_ARG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CB_ERR_CUDA;
  ensure_attrs(dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t T = (size_t)batch * seq;
  // identity rotation: plain attention gradients
  std::vector<float2> tab((size_t)seq * 64, make_float2(1.f, 0.f));
  void* scratch = nullptr;
  const size_t rope_b = tab.size() * sizeof(float2), dsum_b = T * heads * 4,
               dq_b = T * heads * 128 * 4;
  if (cudaMallocAsync(&scratch, rope_b + dsum_b + dq_b, st) != cudaSuccess) return CB_ERR_OUT_OF_MEMORY;
  char* sp = static_cast<char*>(scratch);
  float2* rope = reinterpret_cast<float2*>(sp);
  float* dsum = reinterpret_cast<float*>(sp + rope_b);
  float* dq32 = reinterpret_cast<float*>(sp + rope_b + dsum_b);
  cudaError_t e = cudaMemcpyAsync(rope, tab.data(), rope_b, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess)
    e = launch_attention_bwd(static_cast<const __half*>(q), static_cast<const __half*>(k),
                             static_cast<const __half*>(v), static_cast<const __half*>(o),
                             static_cast<const __half*>(dout), lse, dsum, dq32, rope, rope,
                             static_cast<__half*>(dqkv), batch, heads, kv_heads, seq,
                             device_info(dev).sms, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);  // the host table must outlive the copy
  cudaFreeAsync(scratch, st);
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

cb_status cb_lm_head_ce_f16(const void* xf, const void* embed, const uint32_t* targets,
                            int32_t T, int32_t dim, int32_t vocab, float softcap,
                            float* per_token_loss, float* loss, void* stream) {
  if (!lm_ce_args_ok(xf, embed, targets, T, dim, vocab)) return CB_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  if (cudaMallocAsync(&scratch, lm_ce_scratch_bytes(T, vocab), st) != cudaSuccess)
    return CB_ERR_OUT_OF_MEMORY;
  const LmCeScratch s = lm_ce_carve(scratch, T, vocab);
  cudaError_t e = lm_ce_enqueue(xf, embed, targets, T, dim, vocab, softcap, per_token_loss, loss,
                                s, st);
  cudaError_t e2 = cudaFreeAsync(scratch, st);
  if (e != cudaSuccess || e2 != cudaSuccess) return CB_ERR_CUDA;
  return CB_OK;
}

}  // extern "C"

// ============================================================================
// LM head + cross-entropy without any device allocation.
//
// Some callers cannot allocate device memory while they run: engines that carve
// all device memory into their own pool at start-up and forbid cudaMalloc in the
// steady state, and latency-critical loops where cudaMalloc/cudaFree would
// synchronise the whole device and stall other streams. This variant of
// cb_lm_head_ce_f16 takes its scratch (the per-tile max/sum-exp partials, the
// target logits, the per-block loss sums) from one fixed array compiled into
// this library instead of from an allocator.
//
// The array is a file-scope static __device__ array of NOALLOC_SCRATCH_BYTES:
// every GPU that loads this library holds it until the process exits. Host code
// may not pass the array's name to a kernel (on the host it is only a stand-in
// symbol), so the first call on each device looks up its device address with
// cudaGetSymbolAddress, with that device current, and caches it together with the
// device's current CUDA context. A caller that resets the device (cudaDeviceReset)
// gets a new primary context in which the array has a new address: the next call
// sees the context change and looks the address up again.
namespace {

constexpr int NOALLOC_MAX_TOKENS = 8192;
constexpr int NOALLOC_MAX_VOCAB = 16384;
// Partials for 8192 tokens x 128 tiles (vocab 16384 with 128-wide tiles) plus
// target logits, per-token losses, block sums and the mean: 8.07 MiB, rounded up.
constexpr size_t NOALLOC_SCRATCH_BYTES = 8u * 1024u * 1024u + 128u * 1024u;

static __device__ __align__(256) unsigned char g_lm_ce_scratch[NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};
unsigned long long g_noalloc_ctx_id[64] = {};

// Device address of g_lm_ce_scratch on the current device: looked up once per device
// and again whenever the device's current context is not the one it was looked up in
// (context ids are unique for the life of the process, unlike context handles).
cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  unsigned long long id = 0;
  cudaError_t e = current_context_id(&dev, &id);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev] || g_noalloc_ctx_id[dev] != id) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_lm_ce_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx_id[dev] = id;
  }
  *out = g_noalloc_addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" cb_status cb_lm_head_ce_f16_noalloc(const void* xf, const void* embed,
                                               const uint32_t* targets, int32_t T, int32_t dim,
                                               int32_t vocab, float softcap,
                                               float* per_token_loss, float* loss,
                                               void* stream) {
  if (!lm_ce_args_ok(xf, embed, targets, T, dim, vocab)) return CB_ERR_INVALID_ARG;
  if (T > NOALLOC_MAX_TOKENS || vocab > NOALLOC_MAX_VOCAB ||
      lm_ce_scratch_bytes(T, vocab) > NOALLOC_SCRATCH_BYTES)
    return CB_ERR_INVALID_ARG;
  void* base = nullptr;
  if (noalloc_scratch(&base) != cudaSuccess) return CB_ERR_CUDA;
  // Every scratch word the kernels read is written earlier in the same call (the
  // target logits are reset to NaN first), so leftovers of a previous call are harmless.
  const LmCeScratch s = lm_ce_carve(base, T, vocab);
  cudaError_t e = lm_ce_enqueue(xf, embed, targets, T, dim, vocab, softcap, per_token_loss, loss,
                                s, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CB_OK : CB_ERR_CUDA;
}

#include "training.cuh"
#include "decode.cuh"
