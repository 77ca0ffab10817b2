//! Rust bindings to libcudabridge, the B200 (sm_100a) forward + loss engine.
//!
//! This crate takes the place of `crates/ane-bridge` (which re-exports the external
//! `ane` crate: MIL graph compile, `Executable::run_cached_direct`, IOSurface staging)
//! for the transformer forward pass and its next-token cross-entropy loss. The engine
//! keeps its `ModelConfig` / `ModelWeights` / `CompiledKernels` / `forward_only_ws` API
//! (crates/engine/src/{model.rs:5-17, full_model.rs:19-23,378,494,915,1603,
//! layer.rs:52-63,967}); only their bodies call into this crate.
//!
//! `ffi` is one-to-one with `include/cuda_bridge.h`. The safe layer above it owns the
//! handles (`Context`, `DeviceTokens`) and turns every non-zero `cb_status` into an
//! `Error` carrying the library's message. The reference panics when an ANE evaluation
//! fails (layer.rs:1678); callers that want that behaviour `.expect()` the results.

pub mod ffi {
    #![allow(non_camel_case_types)]
    use std::os::raw::{c_char, c_void};

    pub type cb_status = i32;
    pub const CB_OK: cb_status = 0;
    pub const CB_ERR_INVALID_ARG: cb_status = 1;
    pub const CB_ERR_CUDA: cb_status = 2;
    pub const CB_ERR_OUT_OF_MEMORY: cb_status = 3;
    pub const CB_ERR_NOT_READY: cb_status = 4;
    pub const CB_ERR_UNSUPPORTED: cb_status = 5;
    pub const CB_ERR_DEVICE_TIMEOUT: cb_status = 6;
    pub const CB_ERR_NCCL: cb_status = 7;

    pub const CB_INIT_NORMAL: i32 = 0;
    pub const CB_INIT_REFERENCE: i32 = 1;

    #[repr(C)]
    #[derive(Clone, Copy, Debug, PartialEq, Eq)]
    pub struct cb_model_config {
        pub dim: i32,
        pub hidden: i32,
        pub heads: i32,
        pub kv_heads: i32,
        pub hd: i32,
        pub seq: i32,
        pub nlayers: i32,
        pub vocab: i32,
    }

    #[repr(C)]
    pub struct cb_layer_weights_f32 {
        pub wq: *const f32,
        pub wk: *const f32,
        pub wv: *const f32,
        pub wo: *const f32,
        pub w1: *const f32,
        pub w3: *const f32,
        pub w2: *const f32,
        pub gamma1: *const f32,
        pub gamma2: *const f32,
    }

    #[repr(C)]
    pub struct cb_layer_grads_f32 {
        pub wq: *mut f32,
        pub wk: *mut f32,
        pub wv: *mut f32,
        pub wo: *mut f32,
        pub w1: *mut f32,
        pub w3: *mut f32,
        pub w2: *mut f32,
        pub gamma1: *mut f32,
        pub gamma2: *mut f32,
    }

    #[repr(C)]
    #[derive(Clone, Copy)]
    pub struct cb_kernel_time {
        pub name: [c_char; 32],
        pub launches: i64,
        pub total_ms: f64,
        pub flops: f64,
        pub bytes: f64,
    }

    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default)]
    pub struct cb_eval_totals {
        pub loss_sum: f64,
        pub nats: f64,
        pub bytes: i64,
        pub tokens: i64,
    }

    pub enum cb_ctx {}
    pub enum cb_tokens {}

    unsafe extern "C" {
        pub fn cb_version() -> *const c_char;
        pub fn cb_device_count(count: *mut i32) -> cb_status;
        pub fn cb_create(cfg: *const cb_model_config, device: i32, max_batch: i32, out: *mut *mut cb_ctx) -> cb_status;
        pub fn cb_create_tp(cfg: *const cb_model_config, device: i32, max_batch: i32, tp_rank: i32, tp_world: i32, nccl_unique_id: *const c_void, out: *mut *mut cb_ctx) -> cb_status;
        pub fn cb_nccl_unique_id(out128: *mut c_void) -> cb_status;
        pub fn cb_tp_info(ctx: *const cb_ctx, info: *mut i32) -> cb_status;
        pub fn cb_tp_peer_lost(ctx: *mut cb_ctx, why: *const c_char) -> cb_status;
        pub fn cb_tp_partition(cfg: *const cb_model_config, tp_world: i32, tp_rank: i32, info: *mut i32) -> cb_status;
        pub fn cb_destroy(ctx: *mut cb_ctx) -> cb_status;
        pub fn cb_init_weights(ctx: *mut cb_ctx, seed: u64, scheme: i32, sigma: f32) -> cb_status;
        pub fn cb_load_weights_f32(ctx: *mut cb_ctx, embed: *const f32, gamma_final: *const f32, layers: *const cb_layer_weights_f32) -> cb_status;
        pub fn cb_forward_loss(ctx: *mut cb_ctx, tokens: *const u32, targets: *const u32, batch: i32, softcap: f32, loss_out: *mut f32, per_token_loss: *mut f32) -> cb_status;
        pub fn cb_forward_loss_async(ctx: *mut cb_ctx, d_tokens: *const u32, d_targets: *const u32, batch: i32, softcap: f32, d_loss: *mut f32, d_per_token_loss: *mut f32, stream: *mut c_void) -> cb_status;
        pub fn cb_check_device_error(ctx: *mut cb_ctx) -> cb_status;
        pub fn cb_selftest_wait_timeout(ctx: *mut cb_ctx, limit_us: u32) -> cb_status;
        pub fn cb_sampled_logits(ctx: *mut cb_ctx, rows: *const i32, n_rows: i32, logits_out: *mut f32) -> cb_status;
        pub fn cb_load_rstk(ctx: *mut cb_ctx, path: *const c_char, step_out: *mut u32) -> cb_status;
        pub fn cb_tokens_open(path: *const c_char, device: i32, out: *mut *mut cb_tokens) -> cb_status;
        pub fn cb_tokens_from_host(tokens: *const u16, n: i64, device: i32, out: *mut *mut cb_tokens) -> cb_status;
        pub fn cb_tokens_len(data: *const cb_tokens, n: *mut i64) -> cb_status;
        pub fn cb_tokens_close(data: *mut cb_tokens) -> cb_status;
        pub fn cb_forward_loss_windows(ctx: *mut cb_ctx, data: *const cb_tokens, positions: *const i64, batch: i32, softcap: f32, loss_out: *mut f32, per_token_loss: *mut f32) -> cb_status;
        pub fn cb_eval_windows(ctx: *mut cb_ctx, data: *const cb_tokens, token_bytes: *const i32, n_token_bytes: i32, step_begin: i64, step_end: i64, softcap: f32, out: *mut cb_eval_totals) -> cb_status;
        pub fn cb_enable_training(ctx: *mut cb_ctx) -> cb_status;
        pub fn cb_zero_grads(ctx: *mut cb_ctx) -> cb_status;
        pub fn cb_forward_backward(ctx: *mut cb_ctx, tokens: *const u32, targets: *const u32, batch: i32, softcap: f32, loss_scale: f32, loss_out: *mut f32) -> cb_status;
        pub fn cb_get_grads_f32(ctx: *mut cb_ctx, d_embed: *mut f32, d_gamma_final: *mut f32, layers: *const cb_layer_grads_f32) -> cb_status;
        pub fn cb_prefill(ctx: *mut cb_ctx, tokens: *const u32, batch: i32, len: i32, softcap: f32, logits_out: *mut f32) -> cb_status;
        pub fn cb_decode_step(ctx: *mut cb_ctx, tokens: *const u32, batch: i32, logits_out: *mut f32, next_out: *mut u32) -> cb_status;
        pub fn cb_decode_position(ctx: *const cb_ctx, pos: *mut i32) -> cb_status;
        pub fn cb_set_profiling(ctx: *mut cb_ctx, enable: i32) -> cb_status;
        pub fn cb_kernel_times(ctx: *mut cb_ctx, out: *mut cb_kernel_time, max_entries: i32, n_entries: *mut i32) -> cb_status;
        pub fn cb_reset_kernel_times(ctx: *mut cb_ctx) -> cb_status;
        pub fn cb_get_stream(ctx: *mut cb_ctx, stream: *mut *mut c_void) -> cb_status;
        pub fn cb_last_error(ctx: *const cb_ctx) -> *const c_char;
        pub fn cb_create_error() -> *const c_char;
        pub fn cb_gemm_f16(a: *const c_void, b: *const c_void, c: *mut c_void, m: i32, n: i32, k: i32, out_f32: i32, block_n: i32, stream: *mut c_void) -> cb_status;
        pub fn cb_gemm_f16_layout(a: *const c_void, b: *const c_void, c: *mut c_void, m: i32, n: i32, k: i32, layout: i32, out_f32: i32, block_n: i32, stream: *mut c_void) -> cb_status;
        pub fn cb_attention_f16(q: *const c_void, k: *const c_void, v: *const c_void, out: *mut c_void, batch: i32, heads: i32, seq: i32, stream: *mut c_void) -> cb_status;
        pub fn cb_attention_schedule(batch: i32, heads: i32, kv_heads: i32, seq: i32, sms: i32, table: *mut i32, cap: usize, grid: *mut i32, len: *mut usize) -> cb_status;
        pub fn cb_attention_fwd_lse_f16(q: *const c_void, k: *const c_void, v: *const c_void, out: *mut c_void, lse: *mut f32, batch: i32, heads: i32, kv_heads: i32, seq: i32, stream: *mut c_void) -> cb_status;
        pub fn cb_attention_bwd_f16(q: *const c_void, k: *const c_void, v: *const c_void, o: *const c_void, dout: *const c_void, lse: *const f32, dqkv: *mut c_void, batch: i32, heads: i32, kv_heads: i32, seq: i32, stream: *mut c_void) -> cb_status;
        pub fn cb_lm_head_ce_f16(xf: *const c_void, embed: *const c_void, targets: *const u32, t: i32, dim: i32, vocab: i32, softcap: f32, per_token_loss: *mut f32, loss: *mut f32, stream: *mut c_void) -> cb_status;
        pub fn cb_lm_head_ce_f16_noalloc(xf: *const c_void, embed: *const c_void, targets: *const u32, t: i32, dim: i32, vocab: i32, softcap: f32, per_token_loss: *mut f32, loss: *mut f32, stream: *mut c_void) -> cb_status;
    }
}

use std::ffi::{CStr, CString};
use std::fmt;
use std::ptr;

/// A failed bridge call: the `cb_status` and the library's description of it.
#[derive(Debug, Clone)]
pub struct Error {
    pub status: ffi::cb_status,
    pub message: String,
}

impl fmt::Display for Error {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "cuda-bridge status {}: {}", self.status, self.message)
    }
}

impl std::error::Error for Error {}

pub type Result<T> = std::result::Result<T, Error>;

fn message(p: *const std::os::raw::c_char) -> String {
    if p.is_null() {
        String::new()
    } else {
        unsafe { CStr::from_ptr(p) }.to_string_lossy().into_owned()
    }
}

fn check(status: ffi::cb_status, ctx: *const ffi::cb_ctx) -> Result<()> {
    if status == ffi::CB_OK {
        return Ok(());
    }
    let text = if ctx.is_null() {
        message(unsafe { ffi::cb_create_error() })
    } else {
        message(unsafe { ffi::cb_last_error(ctx) })
    };
    Err(Error { status, message: text })
}

/// Model hyper-parameters in the engine's terms (ModelConfig, model.rs:5-17).
pub fn model_config(dim: usize, hidden: usize, heads: usize, kv_heads: usize, hd: usize,
                    seq: usize, nlayers: usize, vocab: usize) -> ffi::cb_model_config {
    ffi::cb_model_config {
        dim: dim as i32,
        hidden: hidden as i32,
        heads: heads as i32,
        kv_heads: kv_heads as i32,
        hd: hd as i32,
        seq: seq as i32,
        nlayers: nlayers as i32,
        vocab: vocab as i32,
    }
}

/// Host f32 weights of one layer in the reference orientation (LayerWeights,
/// layer.rs:52-63): wq [dim, q_dim], wk / wv [dim, kv_dim], wo [q_dim, dim],
/// w1 / w3 / w2 [dim, hidden], gains [dim].
pub struct LayerWeightsRef<'a> {
    pub wq: &'a [f32],
    pub wk: &'a [f32],
    pub wv: &'a [f32],
    pub wo: &'a [f32],
    pub w1: &'a [f32],
    pub w3: &'a [f32],
    pub w2: &'a [f32],
    pub gamma1: &'a [f32],
    pub gamma2: &'a [f32],
}

/// One device context: weights, workspace and captured forward graphs for up to
/// `max_batch` sequences on one GPU (the compile-once handle of
/// `CompiledKernels::compile_forward_only`, layer.rs:967). Not `Sync`: one per thread,
/// as the reference keeps one `CompiledKernels` per worker (multistream.rs:70-79).
pub struct Context {
    raw: *mut ffi::cb_ctx,
    cfg: ffi::cb_model_config,
}

unsafe impl Send for Context {}

impl Context {
    pub fn new(cfg: ffi::cb_model_config, device: i32, max_batch: i32) -> Result<Self> {
        let mut raw = ptr::null_mut();
        check(unsafe { ffi::cb_create(&cfg, device, max_batch, &mut raw) }, ptr::null())?;
        Ok(Self { raw, cfg })
    }

    /// A tensor-parallel rank: heads and hidden columns split over `tp_world` GPUs,
    /// partial sums all-reduced with NCCL. Every rank passes the same 128-byte id.
    pub fn new_tensor_parallel(cfg: ffi::cb_model_config, device: i32, max_batch: i32,
                               tp_rank: i32, tp_world: i32, nccl_id: &[u8; 128]) -> Result<Self> {
        let mut raw = ptr::null_mut();
        check(unsafe {
            ffi::cb_create_tp(&cfg, device, max_batch, tp_rank, tp_world,
                              nccl_id.as_ptr().cast(), &mut raw)
        }, ptr::null())?;
        Ok(Self { raw, cfg })
    }

    pub fn raw(&self) -> *mut ffi::cb_ctx {
        self.raw
    }

    fn ok(&self, status: ffi::cb_status) -> Result<()> {
        check(status, self.raw)
    }

    /// Device-side weights: `CB_INIT_REFERENCE` regenerates the reference's own LCG
    /// init (ModelWeights::random, full_model.rs:132-141) bit for bit in fp16;
    /// `CB_INIT_NORMAL` draws N(0, sigma).
    pub fn init_weights(&mut self, seed: u64, scheme: i32, sigma: f32) -> Result<()> {
        self.ok(unsafe { ffi::cb_init_weights(self.raw, seed, scheme, sigma) })
    }

    /// Uploads host f32 weights (reference orientation); the library rounds them to
    /// fp16 and lays them out on the device. Every slice length is checked against the
    /// config first: the C call reads a fixed number of floats from each pointer.
    pub fn load_weights_f32(&mut self, embed: &[f32], gamma_final: &[f32],
                            layers: &[LayerWeightsRef<'_>]) -> Result<()> {
        let c = self.cfg;
        let (d, h) = (c.dim as usize, c.hidden as usize);
        let (qd, kvd) = ((c.heads * c.hd) as usize, (c.kv_heads * c.hd) as usize);
        let bad = |what: String| Error { status: ffi::CB_ERR_INVALID_ARG, message: what };
        if layers.len() != c.nlayers as usize {
            return Err(bad(format!("{} layers given, the config has {}", layers.len(), c.nlayers)));
        }
        if embed.len() != c.vocab as usize * d || gamma_final.len() != d {
            return Err(bad("embed or gamma_final size differs from the config".into()));
        }
        let mut arr = Vec::with_capacity(layers.len());
        for (i, l) in layers.iter().enumerate() {
            let sizes = [(l.wq.len(), d * qd), (l.wk.len(), d * kvd), (l.wv.len(), d * kvd),
                         (l.wo.len(), qd * d), (l.w1.len(), d * h), (l.w3.len(), d * h),
                         (l.w2.len(), d * h), (l.gamma1.len(), d), (l.gamma2.len(), d)];
            if sizes.iter().any(|(got, want)| got != want) {
                return Err(bad(format!("layer {i}: a weight size differs from the config")));
            }
            arr.push(ffi::cb_layer_weights_f32 {
                wq: l.wq.as_ptr(), wk: l.wk.as_ptr(), wv: l.wv.as_ptr(), wo: l.wo.as_ptr(),
                w1: l.w1.as_ptr(), w3: l.w3.as_ptr(), w2: l.w2.as_ptr(),
                gamma1: l.gamma1.as_ptr(), gamma2: l.gamma2.as_ptr(),
            });
        }
        self.ok(unsafe {
            ffi::cb_load_weights_f32(self.raw, embed.as_ptr(), gamma_final.as_ptr(), arr.as_ptr())
        })
    }

    /// Mean next-token cross-entropy over whole sequences held back to back
    /// (forward_only_ws, full_model.rs:378). With `per_token`, every position's loss
    /// as well (forward_losses, full_model.rs:1603).
    pub fn forward_loss(&mut self, tokens: &[u32], targets: &[u32], softcap: f32,
                        per_token: Option<&mut Vec<f32>>) -> Result<f32> {
        let seq = self.cfg.seq as usize;
        if tokens.len() != targets.len() || tokens.is_empty() || tokens.len() % seq != 0 {
            return Err(Error { status: ffi::CB_ERR_INVALID_ARG,
                               message: "tokens/targets must hold whole sequences".into() });
        }
        let mut loss = 0.0f32;
        let ptl = match per_token {
            Some(v) => {
                v.resize(tokens.len(), 0.0);
                v.as_mut_ptr()
            }
            None => ptr::null_mut(),
        };
        self.ok(unsafe {
            ffi::cb_forward_loss(self.raw, tokens.as_ptr(), targets.as_ptr(),
                                 (tokens.len() / seq) as i32, softcap, &mut loss, ptl)
        })?;
        Ok(loss)
    }

    /// Logits of rows (b * seq + s) of the last forward, [rows.len() * vocab].
    pub fn sampled_logits(&mut self, rows: &[i32]) -> Result<Vec<f32>> {
        let mut out = vec![0.0f32; rows.len() * self.cfg.vocab as usize];
        self.ok(unsafe {
            ffi::cb_sampled_logits(self.raw, rows.as_ptr(), rows.len() as i32, out.as_mut_ptr())
        })?;
        Ok(out)
    }

    /// Streams an RSTK checkpoint (bin/train.rs:238-346) into the device weights;
    /// returns the step recorded in its header.
    pub fn load_checkpoint(&mut self, path: &str) -> Result<u32> {
        let c = CString::new(path).map_err(|_| Error {
            status: ffi::CB_ERR_INVALID_ARG, message: "path contains a NUL byte".into() })?;
        let mut step = 0u32;
        self.ok(unsafe { ffi::cb_load_rstk(self.raw, c.as_ptr(), &mut step) })?;
        Ok(step)
    }

    /// One forward over windows of a device token array: sequence b reads
    /// data[positions[b] ..][..seq] and the targets one position later.
    pub fn forward_loss_windows(&mut self, data: &DeviceTokens, positions: &[i64],
                                softcap: f32) -> Result<f32> {
        let mut loss = 0.0f32;
        self.ok(unsafe {
            ffi::cb_forward_loss_windows(self.raw, data.raw, positions.as_ptr(),
                                         positions.len() as i32, softcap, &mut loss,
                                         ptr::null_mut())
        })?;
        Ok(loss)
    }

    /// Device sums of validation steps [step_begin, step_end) (validate,
    /// bin/train.rs:197-236); `token_bytes` enables the val_bpb sums (data.rs:75-91).
    pub fn eval_windows(&mut self, data: &DeviceTokens, token_bytes: Option<&[i32]>,
                        step_begin: i64, step_end: i64, softcap: f32)
                        -> Result<ffi::cb_eval_totals> {
        let mut t = ffi::cb_eval_totals::default();
        let (tb, n) = token_bytes.map_or((ptr::null(), 0), |b| (b.as_ptr(), b.len() as i32));
        self.ok(unsafe {
            ffi::cb_eval_windows(self.raw, data.raw, tb, n, step_begin, step_end, softcap, &mut t)
        })?;
        Ok(t)
    }

    /// One training step (forward_ws + backward_ws, full_model.rs:494,592-702):
    /// returns the loss; gradients accumulate on the device until `zero_grads`.
    pub fn forward_backward(&mut self, tokens: &[u32], targets: &[u32], softcap: f32,
                            loss_scale: f32) -> Result<f32> {
        self.ok(unsafe { ffi::cb_enable_training(self.raw) })?;
        let mut loss = 0.0f32;
        self.ok(unsafe {
            ffi::cb_forward_backward(self.raw, tokens.as_ptr(), targets.as_ptr(),
                                     (tokens.len() / self.cfg.seq as usize) as i32, softcap,
                                     loss_scale, &mut loss)
        })?;
        Ok(loss)
    }

    pub fn zero_grads(&mut self) -> Result<()> {
        self.ok(unsafe { ffi::cb_zero_grads(self.raw) })
    }

    /// Runs `batch` equal-length prompts into the KV cache; returns each prompt's
    /// last-position logits [batch * vocab].
    pub fn prefill(&mut self, prompts: &[u32], batch: i32, softcap: f32) -> Result<Vec<f32>> {
        let mut out = vec![0.0f32; batch as usize * self.cfg.vocab as usize];
        let len = (prompts.len() / batch.max(1) as usize) as i32;
        self.ok(unsafe {
            ffi::cb_prefill(self.raw, prompts.as_ptr(), batch, len, softcap, out.as_mut_ptr())
        })?;
        Ok(out)
    }

    /// Advances every sequence by one token; returns the greedy next tokens.
    /// Between steps: a peer rank of this tensor-parallel context has left (learned by
    /// the caller's own heartbeat or store). The context is marked failed without any
    /// NCCL call; every later call returns an error, and the process should exit.
    pub fn tp_peer_lost(&mut self, why: &str) -> Result<()> {
        let c = CString::new(why).unwrap_or_default();
        self.ok(unsafe { ffi::cb_tp_peer_lost(self.raw, c.as_ptr()) })
    }

    pub fn decode_step(&mut self, tokens: &[u32], logits: Option<&mut Vec<f32>>)
                       -> Result<Vec<u32>> {
        let mut next = vec![0u32; tokens.len()];
        let lp = match logits {
            Some(v) => {
                v.resize(tokens.len() * self.cfg.vocab as usize, 0.0);
                v.as_mut_ptr()
            }
            None => ptr::null_mut(),
        };
        self.ok(unsafe {
            ffi::cb_decode_step(self.raw, tokens.as_ptr(), tokens.len() as i32, lp,
                                next.as_mut_ptr())
        })?;
        Ok(next)
    }
}

impl Drop for Context {
    fn drop(&mut self) {
        unsafe {
            ffi::cb_destroy(self.raw);
        }
    }
}

/// A uint16 token array resident in one GPU's HBM (TokenData, data.rs:11-44).
pub struct DeviceTokens {
    raw: *mut ffi::cb_tokens,
}

unsafe impl Send for DeviceTokens {}

impl DeviceTokens {
    pub fn open(path: &str, device: i32) -> Result<Self> {
        let c = CString::new(path).map_err(|_| Error {
            status: ffi::CB_ERR_INVALID_ARG, message: "path contains a NUL byte".into() })?;
        let mut raw = ptr::null_mut();
        check(unsafe { ffi::cb_tokens_open(c.as_ptr(), device, &mut raw) }, ptr::null())?;
        Ok(Self { raw })
    }

    pub fn from_host(tokens: &[u16], device: i32) -> Result<Self> {
        let mut raw = ptr::null_mut();
        check(unsafe {
            ffi::cb_tokens_from_host(tokens.as_ptr(), tokens.len() as i64, device, &mut raw)
        }, ptr::null())?;
        Ok(Self { raw })
    }

    pub fn len(&self) -> i64 {
        let mut n = 0i64;
        unsafe {
            ffi::cb_tokens_len(self.raw, &mut n);
        }
        n
    }

    pub fn is_empty(&self) -> bool {
        self.len() == 0
    }
}

impl Drop for DeviceTokens {
    fn drop(&mut self) {
        unsafe {
            ffi::cb_tokens_close(self.raw);
        }
    }
}

/// Number of CUDA devices visible to the library.
pub fn device_count() -> Result<i32> {
    let mut n = 0i32;
    check(unsafe { ffi::cb_device_count(&mut n) }, ptr::null())?;
    Ok(n)
}

/// The library's build string (names the sm_100a target).
pub fn version() -> String {
    message(unsafe { ffi::cb_version() })
}
