/*
 * cuda_bridge.h — C ABI of the B200 (sm_100a) forward + loss engine.
 *
 * This library replaces the reference engine's Apple Neural Engine bridge
 * (crates/ane-bridge + the external `ane` crate: Graph/MIL compile,
 * Executable::run_cached_direct, IOSurface TensorData staging) for the
 * transformer forward pass and next-token cross-entropy loss. The engine-level
 * API it serves is kept: ModelConfig (crates/engine/src/model.rs:5-17),
 * ModelWeights / LayerWeights (full_model.rs:19-23, layer.rs:52-63),
 * CompiledKernels::compile_forward_only (layer.rs:967), forward_only_ws /
 * forward_ws / forward (full_model.rs:378,494,915) and forward_losses
 * (full_model.rs:1603).
 *
 * Conventions
 *  - Every call returns a cb_status; none aborts the process. The reference
 *    panics on ANE eval failure (layer.rs:1678, `.expect("ANE eval failed")`);
 *    here the caller receives CB_ERR_* and cb_last_error() describes it.
 *  - One cb_ctx per host thread and device (the reference keeps one
 *    CompiledKernels per worker thread, multistream.rs:70-79). A context is not
 *    thread-safe.
 *  - Layout: row-major, token-major [batch*seq, dim] (the reference is
 *    channel-first [dim, seq] per sequence; its transposes disappear here).
 *  - Host pointers are plain CPU memory (pinned memory makes copies faster).
 *    Functions whose names end in _async take device pointers and a CUDA
 *    stream (cudaStream_t passed as void*; NULL = the context's own stream)
 *    and do not synchronise.
 */
#ifndef RUSTANE_CUDA_BRIDGE_H
#define RUSTANE_CUDA_BRIDGE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t cb_status;
#define CB_OK 0
#define CB_ERR_INVALID_ARG 1   /* bad config, size, pointer or token id */
#define CB_ERR_CUDA 2          /* CUDA runtime/driver error */
#define CB_ERR_OUT_OF_MEMORY 3 /* device allocation failed */
#define CB_ERR_NOT_READY 4     /* weights not loaded */
#define CB_ERR_UNSUPPORTED 5   /* shape or device the kernels do not handle */
#define CB_ERR_DEVICE_TIMEOUT 6 /* a bounded device-side wait expired */
#define CB_ERR_NCCL 7          /* NCCL error (tensor-parallel contexts) */

/* Mirrors ModelConfig (crates/engine/src/model.rs:5-17). q_dim = heads*hd,
 * kv_dim = kv_heads*hd and gqa_ratio = heads/kv_heads are derived. hd must be
 * 128 (the reference fixes head_dim = 128, model.rs presets). */
typedef struct cb_model_config {
  int32_t dim;
  int32_t hidden;
  int32_t heads;
  int32_t kv_heads;
  int32_t hd;
  int32_t seq;
  int32_t nlayers;
  int32_t vocab;
} cb_model_config;

/* Weight init schemes for cb_init_weights. */
#define CB_INIT_NORMAL 0    /* all matrices ~N(0, sigma), RMSNorm gains 1.0 */
#define CB_INIT_REFERENCE 1 /* the reference LCG init: ModelWeights::random
                               (full_model.rs:132-141) + LayerWeights::random
                               (layer.rs:1509-1524); sigma ignored */

/* Per-layer host weights in the reference orientation (layer.rs:52-63):
 * wq [dim, q_dim], wk/wv [dim, kv_dim] (x @ W), wo [q_dim, dim],
 * w1/w3 [dim, hidden], w2 [dim, hidden] (used transposed: gate @ W2^T,
 * ffn_fused.rs:130), gamma1/gamma2 [dim]. */
typedef struct cb_layer_weights_f32 {
  const float* wq;
  const float* wk;
  const float* wv;
  const float* wo;
  const float* w1;
  const float* w3;
  const float* w2;
  const float* gamma1;
  const float* gamma2;
} cb_layer_weights_f32;

/* Per-kernel-class timing collected while profiling is enabled. */
typedef struct cb_kernel_time {
  char name[32];
  int64_t launches;
  double total_ms;      /* sum of CUDA-event durations */
  double flops;         /* algorithmic FLOPs over all launches */
  double bytes;         /* algorithmic HBM bytes over all launches */
} cb_kernel_time;

typedef struct cb_ctx cb_ctx;

/* Library version string. */
const char* cb_version(void);

/* Number of visible CUDA devices (0 when there is none). */
cb_status cb_device_count(int32_t* count);

/* Replaces CompiledKernels::compile_forward_only(&cfg) (layer.rs:967) together
 * with ModelForwardWorkspace::new_lean (full_model.rs:245): allocates device
 * weights and a workspace for up to max_batch sequences of cfg->seq tokens on
 * `device`. Weights are uninitialised until cb_init_weights/cb_load_weights_f32. */
cb_status cb_create(const cb_model_config* cfg, int32_t device, int32_t max_batch,
                    cb_ctx** out);

/* Tensor-parallel context (Megatron split of one model over tp_world GPUs, one
 * process or thread per rank), the CUDA counterpart of the reference's
 * head-sharded attention and hidden-sharded FFN (layer.rs:972-1003, 1906-2053,
 * 4943-5139): rank r holds a near-even share of the kv heads (with their query
 * heads) for Wq/Wk/Wv (column-parallel) and Wo (row-parallel), and of the hidden
 * width in 64-column blocks for W1/W3 (column) and W2 (row). The row-parallel
 * partial outputs are combined by NCCL where the reference summed shard outputs on
 * the CPU (layer.rs:5121, 2018): by default sequence parallel (an fp16 reduce-scatter
 * over the token rows, residual + RMSNorm of each rank's own rows, an all-gather of
 * the normalised rows; $CB_TP_REDUCE=sp32 sends fp32 partial sums, =allreduce uses an
 * fp32 all-reduce with every row replicated). Embedding, the LM head + loss are
 * replicated, so every rank returns the same loss. Every rank passes the same 128-byte
 * NCCL unique id (from cb_nccl_unique_id on one rank) and must run the same sequence
 * of calls. NCCL is loaded at run time ($CB_NCCL_LIB or libnccl.so.2).
 *
 * Failure handling: the communicator is non-blocking. A caller that learns on the host
 * that a peer has left (its own heartbeat or store) calls cb_tp_peer_lost before the
 * next step, so no collective is ever launched toward the missing peer. As a last
 * resort, the communicator's set-up and every wait of a forward also poll the stream
 * and ncclCommGetAsyncError against a host deadline ($CB_NCCL_TIMEOUT_MS, default
 * 120000) and return CB_ERR_NCCL on expiry or an NCCL error. After either, every call on
 * the context returns CB_ERR_NCCL at once and the library makes no further NCCL call on
 * the communicator (ncclCommAbort with a departed peer did not return in tests): the
 * communicator, and the device memory of a context whose collective still runs, stay
 * until the process ends; a rank that lost a peer should destroy the context and exit. */
cb_status cb_create_tp(const cb_model_config* cfg, int32_t device, int32_t max_batch,
                       int32_t tp_rank, int32_t tp_world, const void* nccl_unique_id,
                       cb_ctx** out);

/* Writes a fresh 128-byte NCCL unique id to `out` (for cb_create_tp). */
cb_status cb_nccl_unique_id(void* out);

/* info[8] = {tp_rank, tp_world, local heads, local kv heads, local hidden,
 *            first head, first kv head, first hidden column} of a context. */
cb_status cb_tp_info(const cb_ctx* ctx, int32_t* info);

/* Between steps (none of the context's work in flight): a peer rank has left, as the
 * caller learned on the host. The context is marked failed without any NCCL call, and
 * every later call on it returns CB_ERR_NCCL with `why` (nullable) in cb_last_error. The counterpart of the reference supervisor ending a
 * worker whose peer failed (crates/engine/src/bin/theory_runner.rs:9-15,
 * crates/engine/tests/theory_runner_supervisor.rs:14-74). CB_ERR_INVALID_ARG for a
 * context that is not tensor-parallel. */
cb_status cb_tp_peer_lost(cb_ctx* ctx, const char* why);

/* The same info[8] for rank tp_rank of a tp_world split of `cfg`, without a context
 * or a GPU (the split cb_create_tp uses; host-side sharding code and tests share it).
 * CB_ERR_INVALID_ARG for an invalid config, rank or world (world above the kv heads
 * or the 64-column hidden blocks), with the reason in cb_create_error. */
cb_status cb_tp_partition(const cb_model_config* cfg, int32_t tp_world, int32_t tp_rank,
                          int32_t* info);

/* Frees every device resource of the context. NULL is accepted. Exceptions, for a
 * tensor-parallel context that failed (a peer left, an NCCL error or the deadline): its
 * communicator is not destroyed, and if one of its collectives still runs (a peer left
 * in the middle of a step) its device memory stays until the process ends, since
 * freeing it would wait for that collective; CB_ERR_NCCL is then returned (the reason
 * in cb_create_error). The context is invalid afterwards either way. */
cb_status cb_destroy(cb_ctx* ctx);

/* Generates weights on the device (no host copy of the model is needed).
 * Bit-identical to the CPU oracle's generator for the same (seed, scheme). */
cb_status cb_init_weights(cb_ctx* ctx, uint64_t seed, int32_t scheme, float sigma);

/* Uploads host f32 weights in the reference orientation (ModelWeights,
 * full_model.rs:19-23): embed [vocab, dim], gamma_final [dim], and
 * cfg.nlayers cb_layer_weights_f32. Values are rounded to fp16 on the device;
 * gains stay fp32. */
cb_status cb_load_weights_f32(cb_ctx* ctx, const float* embed, const float* gamma_final,
                              const cb_layer_weights_f32* layers);

/* forward_only_ws / forward_ws (full_model.rs:378,494) for `batch` sequences
 * back to back: tokens/targets are host u32 [batch*seq]. loss_out receives the
 * mean next-token cross-entropy over all batch*seq positions (= the mean of the
 * per-sequence losses). per_token_loss (nullable, host [batch*seq]) receives
 * the per-position losses of forward_losses (full_model.rs:1603). softcap > 0
 * applies logits = softcap*tanh(logits/softcap) (full_model.rs:456-461).
 * Synchronous. */
cb_status cb_forward_loss(cb_ctx* ctx, const uint32_t* tokens, const uint32_t* targets,
                          int32_t batch, float softcap, float* loss_out,
                          float* per_token_loss);

/* Same computation on device buffers, enqueued on `stream` without a host
 * synchronisation. d_loss (device float) and d_per_token_loss (nullable,
 * device [batch*seq]) are written when the stream reaches them. Device-side
 * errors (a bad token id, an expired wait) are reported by the next
 * cb_check_device_error. */
cb_status cb_forward_loss_async(cb_ctx* ctx, const uint32_t* d_tokens, const uint32_t* d_targets,
                                int32_t batch, float softcap, float* d_loss,
                                float* d_per_token_loss, void* stream);

/* Synchronises the context's stream and reports (and clears) a device-side
 * error flag raised by earlier asynchronous forwards. */
cb_status cb_check_device_error(cb_ctx* ctx);

/* Self-test of the bounded device waits that every pipeline kernel uses: runs, on
 * the context's stream, a one-block kernel whose consumer waits for a barrier that
 * nothing arrives on, with a limit of limit_us microseconds (1 .. 2e6; the kernels
 * of the forward use 2 s). The wait expires, the kernel frees its TMEM and returns,
 * and this call returns CB_ERR_DEVICE_TIMEOUT through the same device error flag
 * the forward reports with (then cleared), leaving the context usable. Any other
 * status means the timeout path is broken. No counterpart in the reference (its
 * supervisor timeouts are host-side, tests/theory_runner_supervisor.rs:14-74). */
cb_status cb_selftest_wait_timeout(cb_ctx* ctx, uint32_t limit_us);

/* Logits of selected positions of the LAST forward (row = b*seq + s), the
 * sampled-row dump used for parity checks (the full [T, vocab] logits never
 * reach device memory otherwise). logits_out: host [n_rows * vocab] f32, with
 * the last forward's softcap applied. Synchronous. */
cb_status cb_sampled_logits(cb_ctx* ctx, const int32_t* rows, int32_t n_rows, float* logits_out);

/* ---- Checkpoints and token data (the training binary's I/O:
 * crates/engine/src/bin/train.rs, crates/engine/src/data.rs). ---------------- */

/* Loads an RSTK checkpoint (the format written by save_checkpoint,
 * train.rs:238-273, read by load_checkpoint, train.rs:297-346) straight into the
 * context's fp16 device weights: a 28-byte header (magic "RSTK", then u32 LE
 * version, step, dim, nlayers, vocab, seq) followed by f32 LE tensors in the
 * order embed, gamma_final, then per layer wq, wk, wv, wo, w1, w3, w2, gamma1,
 * gamma2 (reference orientation, as cb_load_weights_f32). The file is streamed
 * through pinned chunks; no host copy of the model is made. Where the reference
 * panics (bad magic) or misreads (header dims that differ from the config, a
 * short file) this returns CB_ERR_INVALID_ARG. Bytes after the last tensor are
 * ignored, as in the reference. step_out (nullable) receives the header step.
 * Tensor-parallel contexts keep their own slice of each tensor. Synchronous. */
cb_status cb_load_rstk(cb_ctx* ctx, const char* path, uint32_t* step_out);

/* A uint16 token array resident in one device's HBM: the B200 form of TokenData
 * (data.rs:11-44), which memory-maps the file. A file of 1e9 tokens takes 2 GB. */
typedef struct cb_tokens cb_tokens;

/* Reads a flat uint16 LE token file (data.rs:17-28; n = file bytes / 2) into
 * device memory on `device`. On failure *out is NULL and cb_create_error()
 * describes it. */
cb_status cb_tokens_open(const char* path, int32_t device, cb_tokens** out);
/* The same from host memory (n tokens). */
cb_status cb_tokens_from_host(const uint16_t* tokens, int64_t n, int32_t device,
                              cb_tokens** out);
cb_status cb_tokens_len(const cb_tokens* data, int64_t* n);
cb_status cb_tokens_close(cb_tokens* data);

/* One forward over `batch` windows of a device token array: sequence b has
 * tokens data[positions[b] .. + seq) and targets data[positions[b] + 1 .. + seq]
 * (train.rs:556-558 `tokens(pos, seq)`, `tokens(pos + 1, seq)`). positions is a
 * host array of `batch` offsets with positions[b] + seq + 1 <= n. The windows
 * are gathered on the device; the data never returns to the host. Token ids >=
 * vocab give CB_ERR_INVALID_ARG. Outputs as cb_forward_loss. Synchronous. */
cb_status cb_forward_loss_windows(cb_ctx* ctx, const cb_tokens* data, const int64_t* positions,
                                  int32_t batch, float softcap, float* loss_out,
                                  float* per_token_loss);

/* Sums of an evaluation pass (all accumulated on the device, fixed order). */
typedef struct cb_eval_totals {
  double loss_sum;   /* sum of the per-token losses */
  double nats;       /* sum of the losses whose target has a positive byte length */
  int64_t bytes;     /* sum of those byte lengths */
  int64_t tokens;    /* positions evaluated */
} cb_eval_totals;

/* The evaluation loop of validate (train.rs:197-236) for validation steps
 * [step_begin, step_end): step vs evaluates the window at
 * pos = (vs * seq) % (n - seq - 1), up to max_batch windows per forward. With
 * token_bytes (host int32 [n_token_bytes], TokenBytes of data.rs:47-73; nullable)
 * the byte-weighted nats of compute_bpb (data.rs:75-91) are summed as well. The
 * caller forms val_loss = loss_sum / tokens and val_bpb = nats / (ln 2 * bytes);
 * data-parallel callers split the step range across ranks and add the totals.
 * Synchronous. */
cb_status cb_eval_windows(cb_ctx* ctx, const cb_tokens* data, const int32_t* token_bytes,
                          int32_t n_token_bytes, int64_t step_begin, int64_t step_end,
                          float softcap, cb_eval_totals* out);

/* ---- Training step: the backward pass (crates/engine/src/full_model.rs:592-702
 * backward_ws; layer.rs:6747-7037). ------------------------------------------- */

/* Gradients in the reference orientation, laid out like cb_layer_weights_f32. */
typedef struct cb_layer_grads_f32 {
  float* wq;
  float* wk;
  float* wv;
  float* wo;
  float* w1;
  float* w3;
  float* w2;
  float* gamma1;
  float* gamma2;
} cb_layer_grads_f32;

/* Allocates what the training step needs on the context's device: every layer's
 * saved activations for max_batch sequences, backward scratch and fp32 gradients
 * for all weights (zeroed). Not available on tensor-parallel contexts. */
cb_status cb_enable_training(cb_ctx* ctx);

/* Zeroes the gradients (ModelGrads::zero_out, full_model.rs:152). */
cb_status cb_zero_grads(cb_ctx* ctx);

/* One training step for `batch` sequences (host tokens/targets as cb_forward_loss):
 * the forward (loss_out = mean loss) followed by the backward, which ADDS into the
 * device gradients, as the reference accumulates ModelGrads over micro-batches. The
 * logits gradient is (softmax - onehot) * loss_scale / seq per position, so each
 * sequence contributes the gradient of its own mean loss, as `batch` calls of
 * forward_ws + backward_ws would. Gradients are bit-reproducible run to run.
 * Synchronous. */
cb_status cb_forward_backward(cb_ctx* ctx, const uint32_t* tokens, const uint32_t* targets,
                              int32_t batch, float softcap, float loss_scale, float* loss_out);

/* Copies the accumulated gradients to host f32 buffers in the reference orientation
 * (d_embed [vocab, dim], d_gamma_final [dim], and cfg.nlayers cb_layer_grads_f32). */
cb_status cb_get_grads_f32(cb_ctx* ctx, float* d_embed, float* d_gamma_final,
                           const cb_layer_grads_f32* layers);

/* ---- Single-token decode with a KV cache (the intent of the reference's
 * metal-decode crate, crates/metal-decode/src/lib.rs:1-4, a placeholder there). -- */

/* Runs the forward over `batch` prompts of `len` tokens each (host u32 [batch*len],
 * 1 <= len <= cfg.seq) and keeps every layer's K and V in the context's KV cache
 * (allocated on first use: 2 * L * max_batch * kv_heads * seq * 128 fp16). logits_out
 * (nullable, host f32 [batch, vocab]) receives the logits of each prompt's last
 * position (softcap applied when > 0). The next decode step writes position len.
 * Synchronous. */
cb_status cb_prefill(cb_ctx* ctx, const uint32_t* tokens, int32_t batch, int32_t len,
                     float softcap, float* logits_out);

/* Advances all `batch` sequences (batch = the prefill's) by one token: tokens (host u32
 * [batch]) are the tokens at the current position; logits_out (nullable, host f32
 * [batch, vocab]) receives the next-token logits and next_out (nullable, host u32
 * [batch]) the greedy choice (largest logit, lowest id on ties). Fails once the position
 * reaches cfg.seq. Synchronous. */
cb_status cb_decode_step(cb_ctx* ctx, const uint32_t* tokens, int32_t batch, float* logits_out,
                         uint32_t* next_out);

/* Position the next cb_decode_step writes (0 before any prefill). */
cb_status cb_decode_position(const cb_ctx* ctx, int32_t* pos);

/* Per-kernel-class CUDA-event timing of forwards run while enabled. */
cb_status cb_set_profiling(cb_ctx* ctx, int32_t enable);
cb_status cb_kernel_times(cb_ctx* ctx, cb_kernel_time* out, int32_t max_entries,
                          int32_t* n_entries);
cb_status cb_reset_kernel_times(cb_ctx* ctx);

/* The context's CUDA stream (cudaStream_t) and device. */
cb_status cb_get_stream(cb_ctx* ctx, void** stream);

/* Human-readable description of the last error on this context (never NULL). */
const char* cb_last_error(const cb_ctx* ctx);

/* Last error of a failed cb_create (no context exists yet). */
const char* cb_create_error(void);

/* ---- Kernel-level entry points (device pointers; used by the tests and the
 * micro-benchmarks; they sit below the model API). -------------------------- */

/* C[M,N] = A[M,K] * B[N,K]^T with fp16 A/B (K contiguous) on the tcgen05 GEMM.
 * out_f32 = 0: C is fp16; 1: C is f32; 2: C is f32 and is accumulated into
 * (C += A * B^T), with K split in two halves whose partial tiles are added
 * atomically (the split-K path of the row-parallel projections; the order of the
 * two adds is not fixed, so results may differ in the last bit between calls).
 * block_n selects the tile: 0 = automatic,
 * 128 or 256 = one CTA per 128 x block_n tile, 2 = a CTA pair per 256 x 256 tile
 * (needs N % 256 == 0, else 128 is used). K % 64 == 0, N % 32 == 0, 16-byte aligned
 * pointers. Enqueued on `stream` (NULL = default stream). */
cb_status cb_gemm_f16(const void* A, const void* B, void* C, int32_t M, int32_t N, int32_t K,
                      int32_t out_f32, int32_t block_n, void* stream);

/* cb_gemm_f16 with either operand stored transposed, the GEMMs of a backward pass:
 * layout bit 0 set = A is stored [K][M] (M contiguous), bit 1 = B is stored [K][N].
 * C[M,N] = A * B^T as in cb_gemm_f16 (out_f32 0, 1 or 2 as there). An operand stored
 * transposed needs its M (or N) % 64 == 0; a K-major one needs K % 8 == 0. */
cb_status cb_gemm_f16_layout(const void* A, const void* B, void* C, int32_t M, int32_t N,
                             int32_t K, int32_t layout, int32_t out_f32, int32_t block_n,
                             void* stream);

/* Causal attention: q/k/v [batch, heads, seq, 128] fp16 -> out [batch*seq,
 * heads*128] fp16, scale 1/sqrt(128). seq % 64 == 0. */
cb_status cb_attention_f16(const void* q, const void* k, const void* v, void* out,
                           int32_t batch, int32_t heads, int32_t seq, void* stream);

/* The work split of the attention kernel (seq % 128 == 0) on a GPU with `sms` SMs,
 * without a GPU: its persistent CTAs (two per SM) take 128-query tiles from this table,
 * made once per shape. Of two splits, the one whose last CTA ends first by a cost model
 * (a tile costs its 64-key steps + 1) is used: head-major (the tiles of one head after
 * another, latest first, dealt in rounds of alternating direction) or chunked greedy
 * (heads in chunks whose K and V take at most 8 MB, the latest query tiles of a chunk
 * first, each to the CTA with the least work so far). Writes into table[cap] (ints): [grid + 1]
 * offsets, then the items ((b * heads + h) * (seq / 128) + query tile) of CTA 0, 1, ...;
 * *grid = the CTA count, *len = the table's length. CB_ERR_INVALID_ARG for an invalid
 * shape or a table longer than cap (*len is set either way). */
cb_status cb_attention_schedule(int32_t batch, int32_t heads, int32_t kv_heads, int32_t seq,
                                int32_t sms, int32_t* table, size_t cap, int32_t* grid,
                                size_t* len);

/* cb_attention_f16 that also writes lse [batch, heads, seq] (f32): the base-2
 * log-sum-exp of each query's scaled scores, lse = log2 sum_k 2^(s_k log2(e)/sqrt(128)),
 * which the backward pass needs. kv_heads divides heads (grouped-query attention). */
cb_status cb_attention_fwd_lse_f16(const void* q, const void* k, const void* v, void* out,
                                   float* lse, int32_t batch, int32_t heads, int32_t kv_heads,
                                   int32_t seq, void* stream);

/* Backward of causal attention (no RoPE): q [batch, heads, seq, 128], k/v [batch,
 * kv_heads, seq, 128], o and dout [batch*seq, heads*128] fp16, lse from
 * cb_attention_fwd_lse_f16 -> dqkv [batch*seq, (heads + 2 kv_heads)*128] fp16 holding
 * dQ, dK, dV side by side per token (the layout of the QKV projection's output
 * gradient). Scratch comes from cudaMallocAsync; returns after the stream finishes. */
cb_status cb_attention_bwd_f16(const void* q, const void* k, const void* v, const void* o,
                               const void* dout, const float* lse, void* dqkv, int32_t batch,
                               int32_t heads, int32_t kv_heads, int32_t seq, void* stream);

/* Tied LM head + next-token cross-entropy on device buffers (the model's final
 * step: full_model.rs:436-471). xf [T, dim] fp16 (final-normalised activations),
 * embed [vocab, dim] fp16, targets [T] u32. Logits = xf * embed^T, softcapped when
 * softcap > 0, are reduced on chip to per-token losses; the [T, vocab] logits are
 * never written. per_token_loss (device [T] f32) and loss (device f32 scalar, mean)
 * are each nullable. A target >= vocab yields NaN for that token. dim % 64 == 0,
 * vocab % 32 == 0, 16-byte aligned pointers. Scratch of about T*vocab/32 bytes comes
 * from the stream-ordered allocator (cudaMallocAsync) and is released on `stream`. */
cb_status cb_lm_head_ce_f16(const void* xf, const void* embed, const uint32_t* targets,
                            int32_t T, int32_t dim, int32_t vocab, float softcap,
                            float* per_token_loss, float* loss, void* stream);

/* cb_lm_head_ce_f16 for callers that cannot allocate device memory during the call:
 * engines that reserve all device memory for their own pool up front and forbid
 * cudaMalloc afterwards, and latency-critical loops where cudaMalloc/cudaFree would
 * synchronise the device. Same arguments, same results; it calls no allocator.
 * Scratch is one fixed array of about 8.1 MiB compiled into this library (a static
 * __device__ array): every GPU that loads the library holds it until the process exits.
 * Limits: T <= 8192 and vocab <= 16384; larger sizes return CB_ERR_INVALID_ARG (split
 * the tokens into chunks of at most 8192).
 * The first call on a device looks up the array's device address with that device
 * current; make that first call before any stream capture on the device. After a
 * cudaDeviceReset the next call sees the new context and looks the address up again
 * (the array's contents do not survive a reset; nothing carries over between calls).
 * All calls share the one array and it keeps the last call's contents: calls that
 * overlap on the GPU (other streams or threads on the same device) race, so the
 * caller must serialise them.
 * No counterpart in the reference (its head and loss run on the CPU). */
cb_status cb_lm_head_ce_f16_noalloc(const void* xf, const void* embed, const uint32_t* targets,
                                    int32_t T, int32_t dim, int32_t vocab, float softcap,
                                    float* per_token_loss, float* loss, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RUSTANE_CUDA_BRIDGE_H */
