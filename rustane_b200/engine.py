"""Engine-level forward/loss API over the CUDA bridge.

Names and argument meaning follow the reference engine so callers switch
without changes:
  CompiledKernels.compile_forward_only(cfg)      layer.rs:967
  ModelWeights (random / from host arrays)        full_model.rs:19-23,132-141
  ModelForwardWorkspace.new / new_lean            full_model.rs:221-263
  forward_only_ws / forward_ws / forward          full_model.rs:378,494,915
  forward_losses                                  full_model.rs:1603
  ForwardScheduler (sequence-parallel workers)    multistream.rs:54-161
Errors raise CudaBridgeError (the reference panics on ANE eval failure,
layer.rs:1678).
"""
from __future__ import annotations

import ctypes as C
import threading
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import bridge as B
from .model import ModelConfig


def _cfg_struct(cfg: ModelConfig) -> B.cb_model_config:
    return B.cb_model_config(cfg.dim, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.hd, cfg.seq,
                             cfg.nlayers, cfg.vocab)


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


@dataclass
class LayerWeights:
    """Host f32 layer weights in the reference orientation (layer.rs:52-63)."""
    wq: np.ndarray
    wk: np.ndarray
    wv: np.ndarray
    wo: np.ndarray
    w1: np.ndarray
    w3: np.ndarray
    w2: np.ndarray
    gamma1: np.ndarray
    gamma2: np.ndarray


@dataclass
class ModelWeights:
    """Model weights. Either host f32 arrays (embed/layers/gamma_final) or a
    device-side generator spec (scheme, seed, sigma) the bridge expands on the
    GPU without a host copy of the model."""
    embed: Optional[np.ndarray] = None
    layers: Optional[list] = None
    gamma_final: Optional[np.ndarray] = None
    scheme: Optional[int] = None
    seed: int = 0
    sigma: float = 0.02
    generation: int = field(default_factory=lambda: ModelWeights._next_gen())

    _gen_lock = threading.Lock()
    _gen_counter = [0]

    @staticmethod
    def _next_gen() -> int:
        with ModelWeights._gen_lock:
            ModelWeights._gen_counter[0] += 1
            return ModelWeights._gen_counter[0]

    @classmethod
    def random(cls, cfg: ModelConfig) -> "ModelWeights":
        """The reference's own init (ModelWeights::random, full_model.rs:132-141)."""
        return cls(scheme=B.CB_INIT_REFERENCE)

    @classmethod
    def normal(cls, cfg: ModelConfig, seed: int = 0, sigma: float = 0.02) -> "ModelWeights":
        """All matrices ~N(0, sigma), gains 1.0 (the benchmark init)."""
        return cls(scheme=B.CB_INIT_NORMAL, seed=seed, sigma=sigma)

    def touch(self) -> None:
        """A new generation: a context uploads a ModelWeights once and skips later loads
        of the same generation, so call this after changing the arrays in place."""
        self.generation = ModelWeights._next_gen()

    @classmethod
    def from_arrays(cls, embed, layers: Sequence[LayerWeights], gamma_final) -> "ModelWeights":
        return cls(embed=np.ascontiguousarray(embed, np.float32), layers=list(layers),
                   gamma_final=np.ascontiguousarray(gamma_final, np.float32))


@dataclass
class LayerGrads:
    """Host f32 layer gradients, reference orientation (layer.rs:66-76)."""
    dwq: np.ndarray
    dwk: np.ndarray
    dwv: np.ndarray
    dwo: np.ndarray
    dw1: np.ndarray
    dw3: np.ndarray
    dw2: np.ndarray
    dgamma1: np.ndarray
    dgamma2: np.ndarray


@dataclass
class ModelGrads:
    """Host f32 gradients of all weights (full_model.rs:26-30)."""
    dembed: np.ndarray
    layers: list
    dgamma_final: np.ndarray

    @classmethod
    def zeros(cls, cfg: ModelConfig) -> "ModelGrads":
        d, h = cfg.dim, cfg.hidden
        qd, kvd = cfg.heads * cfg.hd, cfg.kv_heads * cfg.hd
        z = lambda *s: np.zeros(s, np.float32)  # noqa: E731
        return cls(z(cfg.vocab, d),
                   [LayerGrads(z(d, qd), z(d, kvd), z(d, kvd), z(qd, d), z(d, h), z(d, h),
                               z(d, h), z(d), z(d)) for _ in range(cfg.nlayers)], z(d))

    def zero_out(self) -> None:
        """ModelGrads::zero_out (full_model.rs:152)."""
        self.dembed[...] = 0
        self.dgamma_final[...] = 0
        for lg in self.layers:
            for a in vars(lg).values():
                a[...] = 0

    def add_(self, other: "ModelGrads") -> None:
        self.dembed += other.dembed
        self.dgamma_final += other.dgamma_final
        for a, b in zip(self.layers, other.layers):
            for k in vars(a):
                getattr(a, k)[...] += getattr(b, k)


class ModelForwardWorkspace:
    """Accepted for API compatibility. The device workspace lives inside
    CompiledKernels (sized by its max_batch); nothing is allocated here."""

    def __init__(self, cfg: ModelConfig):
        self.cfg = cfg

    @classmethod
    def new(cls, cfg: ModelConfig) -> "ModelForwardWorkspace":
        return cls(cfg)

    @classmethod
    def new_lean(cls, cfg: ModelConfig) -> "ModelForwardWorkspace":
        return cls(cfg)


class CompiledKernels:
    """Owns one cb_ctx: device weights, workspace and captured forward graphs
    for `max_batch` sequences on one GPU. Not thread-safe (one per thread)."""

    def __init__(self, cfg: ModelConfig, device: int = 0, max_batch: int = 1,
                 tp_rank: int = 0, tp_world: int = 1, nccl_id: Optional[bytes] = None):
        self.lib = B.load_library()
        self.cfg = cfg
        self.device = device
        self.max_batch = max_batch
        self.tp_rank, self.tp_world = tp_rank, tp_world
        h = C.c_void_p()
        if tp_world == 1:
            B.check(self.lib.cb_create(C.byref(_cfg_struct(cfg)), device, max_batch, C.byref(h)))
        else:
            if nccl_id is None or len(nccl_id) != 128:
                raise ValueError("tensor parallelism needs the 128-byte NCCL unique id")
            buf = C.create_string_buffer(bytes(nccl_id), 128)
            B.check(self.lib.cb_create_tp(C.byref(_cfg_struct(cfg)), device, max_batch, tp_rank,
                                          tp_world, buf, C.byref(h)))
        self._h = h
        self._loaded_generation: Optional[int] = None

    @classmethod
    def compile_forward_only(cls, cfg: ModelConfig, device: int = 0,
                             max_batch: int = 1) -> "CompiledKernels":
        return cls(cfg, device, max_batch)

    compile = compile_forward_only

    # ---- lifecycle
    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.cb_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self) -> C.c_void_p:
        if not self._h:
            raise RuntimeError("CompiledKernels is closed")
        return self._h

    def _check(self, status: int) -> None:
        B.check(status, self._h)

    # ---- weights
    def init_weights(self, seed: int = 0, scheme: int = B.CB_INIT_NORMAL,
                     sigma: float = 0.02) -> None:
        self._loaded_generation = None
        self._check(self.lib.cb_init_weights(self.handle, seed, scheme, sigma))

    def load_weights(self, w: ModelWeights) -> None:
        if self._loaded_generation == w.generation:
            return
        if w.scheme is not None:
            self.init_weights(w.seed, w.scheme, w.sigma)
        else:
            cfg = self.cfg
            if w.layers is None or len(w.layers) != cfg.nlayers:
                raise ValueError("layer count does not match the config")
            d, h = cfg.dim, cfg.hidden
            qd, kvd = cfg.heads * cfg.hd, cfg.kv_heads * cfg.hd
            sizes = dict(wq=d * qd, wk=d * kvd, wv=d * kvd, wo=qd * d, w1=d * h, w3=d * h,
                         w2=d * h, gamma1=d, gamma2=d)

            def f32(a, n, what):
                # the C call reads exactly n floats from each pointer
                a = np.ascontiguousarray(a, np.float32)
                if a.size != n:
                    raise ValueError(f"{what} holds {a.size} values, the config needs {n}")
                return a

            keep = [f32(w.embed, cfg.vocab * d, "embed"),
                    f32(w.gamma_final, d, "gamma_final")]
            arr = (B.cb_layer_weights_f32 * cfg.nlayers)()
            for i, lw in enumerate(w.layers):
                fields = {}
                for name, n in sizes.items():
                    a = f32(getattr(lw, name), n, f"layer {i} {name}")
                    keep.append(a)
                    fields[name] = _fptr(a)
                arr[i] = B.cb_layer_weights_f32(**fields)
            # a failed upload leaves the device weights half written: forget the old
            # generation first, so a retry with the same ModelWeights uploads again
            self._loaded_generation = None
            self._check(self.lib.cb_load_weights_f32(self.handle, _fptr(keep[0]),
                                                     _fptr(keep[1]), arr))
        self._loaded_generation = w.generation

    # ---- training (backward pass)
    def enable_training(self) -> None:
        """Allocate saved activations, backward scratch and gradients on the device."""
        if not getattr(self, "_training", False):
            self._check(self.lib.cb_enable_training(self.handle))
            self._training = True

    def zero_grads(self) -> None:
        self._check(self.lib.cb_zero_grads(self.handle))

    def forward_backward(self, tokens, targets, softcap: float = 0.0,
                         loss_scale: float = 1.0) -> float:
        """One training step: returns the mean loss; gradients accumulate on the device."""
        self.enable_training()
        t, g, batch = self._tokens(tokens, targets)
        loss = C.c_float()
        self._check(self.lib.cb_forward_backward(
            self.handle, t.ctypes.data_as(C.POINTER(C.c_uint32)),
            g.ctypes.data_as(C.POINTER(C.c_uint32)), batch, softcap, loss_scale, C.byref(loss)))
        return loss.value

    def grads(self, out: Optional["ModelGrads"] = None) -> "ModelGrads":
        """The accumulated device gradients in the reference orientation (host f32)."""
        cfg = self.cfg
        if out is None:
            out = ModelGrads.zeros(cfg)
        arr = (B.cb_layer_grads_f32 * cfg.nlayers)()
        for i, lg in enumerate(out.layers):
            arr[i] = B.cb_layer_grads_f32(*[_fptr(getattr(lg, k)) for k in (
                "dwq", "dwk", "dwv", "dwo", "dw1", "dw3", "dw2", "dgamma1", "dgamma2")])
        self._check(self.lib.cb_get_grads_f32(self.handle, _fptr(out.dembed),
                                              _fptr(out.dgamma_final), arr))
        return out

    # ---- decode (KV cache)
    def prefill(self, prompts, softcap: float = 0.0) -> np.ndarray:
        """Run `batch` prompts of equal length (array [batch, len]) into the KV cache;
        returns the logits of each prompt's last position, [batch, vocab]."""
        p = np.ascontiguousarray(np.asarray(prompts, dtype=np.uint32))
        if p.ndim == 1:
            p = p[None, :]
        batch, length = p.shape
        out = np.empty((batch, self.cfg.vocab), np.float32)
        self._check(self.lib.cb_prefill(self.handle, p.ctypes.data_as(C.POINTER(C.c_uint32)),
                                        batch, length, softcap, _fptr(out)))
        return out

    def decode_step(self, tokens, logits: bool = True):
        """Feed one token per sequence at the current position; returns (logits
        [batch, vocab], greedy next tokens [batch]), or (None, next tokens) with
        logits=False (the logits then stay on the device)."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32).reshape(-1))
        z = np.empty((t.size, self.cfg.vocab), np.float32) if logits else None
        nxt = np.empty(t.size, np.uint32)
        self._check(self.lib.cb_decode_step(
            self.handle, t.ctypes.data_as(C.POINTER(C.c_uint32)), t.size,
            _fptr(z) if logits else None, nxt.ctypes.data_as(C.POINTER(C.c_uint32))))
        return z, nxt

    def decode_position(self) -> int:
        p = C.c_int32()
        self._check(self.lib.cb_decode_position(self.handle, C.byref(p)))
        return p.value

    def generate(self, prompts, n_new: int, softcap: float = 0.0) -> np.ndarray:
        """Greedy continuation of equal-length prompts: [batch, n_new] new tokens."""
        first = self.prefill(prompts, softcap)
        cur = first.argmax(axis=1).astype(np.uint32)
        out = [cur]
        for _ in range(n_new - 1):
            _, cur = self.decode_step(cur)
            out.append(cur)
        return np.stack(out, axis=1)

    def load_checkpoint(self, path) -> int:
        """Stream an RSTK checkpoint (train.rs:238-346) into the device weights;
        returns the step recorded in its header."""
        step = C.c_uint32()
        self._check(self.lib.cb_load_rstk(self.handle, str(path).encode(), C.byref(step)))
        self._loaded_generation = None
        return step.value

    # ---- forward
    def _tokens(self, tokens, targets):
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32).reshape(-1))
        g = np.ascontiguousarray(np.asarray(targets, dtype=np.uint32).reshape(-1))
        if t.size != g.size or t.size % self.cfg.seq != 0:
            raise ValueError("tokens/targets must hold whole sequences of cfg.seq")
        return t, g, t.size // self.cfg.seq

    def forward_loss(self, tokens, targets, softcap: float = 0.0,
                     per_token: bool = False):
        t, g, batch = self._tokens(tokens, targets)
        loss = C.c_float()
        ptl = np.empty(t.size, np.float32) if per_token else None
        self._check(self.lib.cb_forward_loss(
            self.handle, t.ctypes.data_as(C.POINTER(C.c_uint32)),
            g.ctypes.data_as(C.POINTER(C.c_uint32)), batch, softcap, C.byref(loss),
            _fptr(ptl) if ptl is not None else None))
        return (loss.value, ptl) if per_token else loss.value

    def forward_loss_async(self, d_tokens: int, d_targets: int, batch: int, softcap: float,
                           d_loss: int, d_per_token: int = 0, stream: int = 0) -> None:
        """Device-pointer variant (ints are raw device addresses)."""
        self._check(self.lib.cb_forward_loss_async(
            self.handle, C.c_void_p(d_tokens), C.c_void_p(d_targets), batch, softcap,
            C.c_void_p(d_loss), C.c_void_p(d_per_token or None), C.c_void_p(stream or None)))

    def forward_loss_windows(self, data, positions, softcap: float = 0.0,
                             per_token: bool = False):
        """Forward over windows of a DeviceTokens array: sequence b has tokens
        data[positions[b]:+seq] and targets data[positions[b]+1:+seq+1]."""
        pos = np.ascontiguousarray(np.asarray(positions, dtype=np.int64).reshape(-1))
        loss = C.c_float()
        ptl = np.empty(pos.size * self.cfg.seq, np.float32) if per_token else None
        self._check(self.lib.cb_forward_loss_windows(
            self.handle, data.handle, pos.ctypes.data_as(C.POINTER(C.c_int64)), pos.size,
            softcap, C.byref(loss), _fptr(ptl) if ptl is not None else None))
        return (loss.value, ptl) if per_token else loss.value

    def eval_windows(self, data, token_bytes, step_begin: int, step_end: int,
                     softcap: float = 0.0) -> dict:
        """Device sums of validation steps [step_begin, step_end) (train.rs:197-236)."""
        tb = None
        if token_bytes is not None:
            tb = np.ascontiguousarray(token_bytes.bytes, dtype=np.int32)
        out = B.cb_eval_totals()
        self._check(self.lib.cb_eval_windows(
            self.handle, data.handle,
            tb.ctypes.data_as(C.POINTER(C.c_int32)) if tb is not None else None,
            tb.size if tb is not None else 0, step_begin, step_end, softcap, C.byref(out)))
        return dict(loss_sum=out.loss_sum, nats=out.nats, bytes=out.bytes, tokens=out.tokens)

    def check_device_error(self) -> None:
        self._check(self.lib.cb_check_device_error(self.handle))

    def selftest_wait_timeout(self, limit_us: int = 1000) -> int:
        """Runs the bounded-wait self-test kernel (a wait nothing ever completes, with a
        limit of limit_us) and returns its status without raising: CB_ERR_DEVICE_TIMEOUT
        when the expiry path works. The context stays usable afterwards."""
        return int(self.lib.cb_selftest_wait_timeout(self.handle, int(limit_us)))

    def sampled_logits(self, rows) -> np.ndarray:
        r = np.ascontiguousarray(np.asarray(rows, dtype=np.int32).reshape(-1))
        out = np.empty((r.size, self.cfg.vocab), np.float32)
        self._check(self.lib.cb_sampled_logits(
            self.handle, r.ctypes.data_as(C.POINTER(C.c_int32)), r.size, _fptr(out)))
        return out

    # ---- profiling
    def set_profiling(self, enable: bool) -> None:
        self._check(self.lib.cb_set_profiling(self.handle, 1 if enable else 0))

    def reset_kernel_times(self) -> None:
        self._check(self.lib.cb_reset_kernel_times(self.handle))

    def kernel_times(self) -> dict:
        arr = (B.cb_kernel_time * 32)()
        n = C.c_int32()
        self._check(self.lib.cb_kernel_times(self.handle, arr, 32, C.byref(n)))
        return {arr[i].name.decode(): dict(launches=arr[i].launches, total_ms=arr[i].total_ms,
                                           flops=arr[i].flops, bytes=arr[i].bytes)
                for i in range(n.value)}

    def tp_peer_lost(self, why: str = "a peer rank left") -> None:
        """Between steps: a peer rank has left (learned on the host). The context is marked
        failed without any NCCL call; later calls raise CudaBridgeError (CB_ERR_NCCL), and
        the process should close the context and exit."""
        self._check(self.lib.cb_tp_peer_lost(self.handle, why.encode()))

    def tp_info(self) -> dict:
        a = (C.c_int32 * 8)()
        self._check(self.lib.cb_tp_info(self.handle, a))
        keys = ("rank", "world", "heads", "kv_heads", "hidden", "head0", "kv_head0", "hidden0")
        return dict(zip(keys, list(a)))

    def stream(self) -> int:
        s = C.c_void_p()
        self._check(self.lib.cb_get_stream(self.handle, C.byref(s)))
        return s.value or 0


def forward_backward(cfg: ModelConfig, kernels: "CompiledKernels", weights: ModelWeights,
                     tokens, targets, softcap: float = 0.0, loss_scale: float = 1.0,
                     grads: Optional[ModelGrads] = None) -> float:
    """forward_ws followed by backward_ws (full_model.rs:494, 592-702): returns the loss
    and ADDS this call's gradients into `grads` (host, reference orientation), as the
    reference accumulates ModelGrads across micro-batches. The device keeps its own
    running sum too (CompiledKernels.grads / zero_grads)."""
    kernels.load_weights(weights)
    kernels.enable_training()
    if grads is None:
        return kernels.forward_backward(tokens, targets, softcap, loss_scale)
    kernels.zero_grads()
    loss = kernels.forward_backward(tokens, targets, softcap, loss_scale)
    grads.add_(kernels.grads())
    return loss


def nccl_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id for CompiledKernels(..., tp_world > 1)."""
    lib = B.load_library()
    buf = C.create_string_buffer(128)
    B.check(lib.cb_nccl_unique_id(buf))
    return buf.raw


# ---------------------------------------------------------------- model API

@dataclass
class ForwardResult:
    """Forward outputs. The reference's ForwardResult (full_model.rs:121-129)
    also carries backward caches; training is not part of this engine."""
    loss: float
    per_token_loss: Optional[np.ndarray] = None


def forward_only_ws(cfg: ModelConfig, kernels: CompiledKernels, weights: ModelWeights,
                    tokens, targets, softcap: float = 0.0,
                    ws: Optional[ModelForwardWorkspace] = None) -> float:
    """Mean next-token cross-entropy (full_model.rs:378). tokens/targets hold one
    or more sequences of cfg.seq back to back."""
    if kernels.cfg != cfg:
        raise ValueError("kernels were compiled for a different config")
    kernels.load_weights(weights)
    return kernels.forward_loss(tokens, targets, softcap)


forward_ws = forward_only_ws


def forward(cfg: ModelConfig, kernels: CompiledKernels, weights: ModelWeights, tokens,
            targets, softcap: float = 0.0) -> ForwardResult:
    kernels.load_weights(weights)
    loss, ptl = kernels.forward_loss(tokens, targets, softcap, per_token=True)
    return ForwardResult(loss, ptl)


def forward_losses(cfg: ModelConfig, kernels: CompiledKernels, weights: ModelWeights, tokens,
                   targets, softcap: float = 0.0) -> np.ndarray:
    """Per-position losses (full_model.rs:1603)."""
    kernels.load_weights(weights)
    return kernels.forward_loss(tokens, targets, softcap, per_token=True)[1]


class ForwardScheduler:
    """Sequence-parallel forward workers (multistream.rs:54-161): one
    CompiledKernels per worker (here: per GPU), each on its own host thread,
    pulling whole sequences; results return in request order. No communication
    between workers."""

    def __init__(self, cfg: ModelConfig, weights: ModelWeights, devices: Sequence[int],
                 max_batch: int = 1):
        self.cfg = cfg
        self.workers = [CompiledKernels(cfg, d, max_batch) for d in devices]
        for w in self.workers:
            w.load_weights(weights)

    def run_batch(self, requests: Sequence[tuple], softcap: float = 0.0) -> list:
        """requests: [(tokens, targets)] one sequence each -> [loss] in order."""
        out = [None] * len(requests)
        errors = []
        lock = threading.Lock()
        nxt = [0]

        def work(k: CompiledKernels):
            while True:
                with lock:
                    i = nxt[0]
                    nxt[0] += 1
                if i >= len(requests):
                    return
                try:
                    out[i] = k.forward_loss(requests[i][0], requests[i][1], softcap)
                except Exception as e:  # propagate after join
                    errors.append(e)
                    return

        threads = [threading.Thread(target=work, args=(k,)) for k in self.workers]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]
        return out

    def close(self) -> None:
        for w in self.workers:
            w.close()
