"""ctypes binding of include/cuda_bridge.h (libcudabridge.so).

This is the Python-side view of the C ABI; the Rust engine binds the same
symbols through the cuda-bridge crate (crates/cuda-bridge/src/lib.rs). There is no
CPU fallback: if the library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libcudabridge.so"

CB_OK = 0
CB_ERR_INVALID_ARG = 1
CB_ERR_CUDA = 2
CB_ERR_OUT_OF_MEMORY = 3
CB_ERR_NOT_READY = 4
CB_ERR_UNSUPPORTED = 5
CB_ERR_DEVICE_TIMEOUT = 6
CB_ERR_NCCL = 7

CB_INIT_NORMAL = 0
CB_INIT_REFERENCE = 1

STATUS_NAMES = {
    CB_OK: "CB_OK",
    CB_ERR_INVALID_ARG: "CB_ERR_INVALID_ARG",
    CB_ERR_CUDA: "CB_ERR_CUDA",
    CB_ERR_OUT_OF_MEMORY: "CB_ERR_OUT_OF_MEMORY",
    CB_ERR_NOT_READY: "CB_ERR_NOT_READY",
    CB_ERR_UNSUPPORTED: "CB_ERR_UNSUPPORTED",
    CB_ERR_DEVICE_TIMEOUT: "CB_ERR_DEVICE_TIMEOUT",
    CB_ERR_NCCL: "CB_ERR_NCCL",
}

# Every symbol include/cuda_bridge.h declares (checked by the CPU test suite).
EXPORTED = [
    "cb_version", "cb_device_count", "cb_create", "cb_create_tp", "cb_nccl_unique_id",
    "cb_tp_info", "cb_tp_peer_lost", "cb_tp_partition", "cb_destroy", "cb_init_weights",
    "cb_load_weights_f32", "cb_forward_loss", "cb_forward_loss_async",
    "cb_check_device_error", "cb_selftest_wait_timeout", "cb_sampled_logits",
    "cb_set_profiling", "cb_kernel_times",
    "cb_reset_kernel_times", "cb_get_stream", "cb_last_error", "cb_create_error",
    "cb_gemm_f16", "cb_gemm_f16_layout", "cb_attention_f16", "cb_attention_schedule",
    "cb_attention_fwd_lse_f16",
    "cb_attention_bwd_f16", "cb_lm_head_ce_f16",
    "cb_lm_head_ce_f16_noalloc", "cb_load_rstk", "cb_tokens_open", "cb_tokens_from_host",
    "cb_tokens_len", "cb_tokens_close", "cb_forward_loss_windows", "cb_eval_windows",
    "cb_enable_training", "cb_zero_grads", "cb_forward_backward", "cb_get_grads_f32",
    "cb_prefill", "cb_decode_step", "cb_decode_position",
]


class CudaBridgeError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class cb_model_config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in
                ("dim", "hidden", "heads", "kv_heads", "hd", "seq", "nlayers", "vocab")]


class cb_layer_weights_f32(C.Structure):
    _fields_ = [(n, C.POINTER(C.c_float)) for n in
                ("wq", "wk", "wv", "wo", "w1", "w3", "w2", "gamma1", "gamma2")]


class cb_kernel_time(C.Structure):
    _fields_ = [("name", C.c_char * 32), ("launches", C.c_int64), ("total_ms", C.c_double),
                ("flops", C.c_double), ("bytes", C.c_double)]


class cb_layer_grads_f32(C.Structure):
    _fields_ = [(n, C.POINTER(C.c_float)) for n in
                ("wq", "wk", "wv", "wo", "w1", "w3", "w2", "gamma1", "gamma2")]


class cb_eval_totals(C.Structure):
    _fields_ = [("loss_sum", C.c_double), ("nats", C.c_double), ("bytes", C.c_int64),
                ("tokens", C.c_int64)]


_lib = None


def load_library(path: Path | None = None) -> C.CDLL:
    """Load libcudabridge.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} not found: build the CUDA bridge first (python -m rustane_b200.build)")
    lib = C.CDLL(str(p))
    vp, i32, i64, u64, f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_float
    pf, pu32, pi32 = C.POINTER(C.c_float), C.POINTER(C.c_uint32), C.POINTER(C.c_int32)
    sig = {
        "cb_version": (C.c_char_p, []),
        "cb_device_count": (i32, [pi32]),
        "cb_create": (i32, [C.POINTER(cb_model_config), i32, i32, C.POINTER(vp)]),
        "cb_create_tp": (i32, [C.POINTER(cb_model_config), i32, i32, i32, i32, vp,
                               C.POINTER(vp)]),
        "cb_nccl_unique_id": (i32, [vp]),
        "cb_tp_info": (i32, [vp, pi32]),
        "cb_tp_peer_lost": (i32, [vp, C.c_char_p]),
        "cb_tp_partition": (i32, [C.POINTER(cb_model_config), i32, i32, pi32]),
        "cb_destroy": (i32, [vp]),
        "cb_init_weights": (i32, [vp, u64, i32, f32]),
        "cb_load_weights_f32": (i32, [vp, pf, pf, C.POINTER(cb_layer_weights_f32)]),
        "cb_forward_loss": (i32, [vp, pu32, pu32, i32, f32, pf, pf]),
        "cb_forward_loss_async": (i32, [vp, vp, vp, i32, f32, vp, vp, vp]),
        "cb_check_device_error": (i32, [vp]),
        "cb_selftest_wait_timeout": (i32, [vp, C.c_uint32]),
        "cb_sampled_logits": (i32, [vp, pi32, i32, pf]),
        "cb_set_profiling": (i32, [vp, i32]),
        "cb_kernel_times": (i32, [vp, C.POINTER(cb_kernel_time), i32, pi32]),
        "cb_reset_kernel_times": (i32, [vp]),
        "cb_get_stream": (i32, [vp, C.POINTER(vp)]),
        "cb_last_error": (C.c_char_p, [vp]),
        "cb_create_error": (C.c_char_p, []),
        "cb_gemm_f16": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, vp]),
        "cb_gemm_f16_layout": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]),
        "cb_attention_f16": (i32, [vp, vp, vp, vp, i32, i32, i32, vp]),
        "cb_attention_schedule": (i32, [i32, i32, i32, i32, i32, vp, C.c_size_t, vp, vp]),
        "cb_attention_fwd_lse_f16": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]),
        "cb_attention_bwd_f16": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]),
        "cb_lm_head_ce_f16": (i32, [vp, vp, vp, i32, i32, i32, f32, vp, vp, vp]),
        "cb_lm_head_ce_f16_noalloc": (i32, [vp, vp, vp, i32, i32, i32, f32, vp, vp, vp]),
        "cb_load_rstk": (i32, [vp, C.c_char_p, pu32]),
        "cb_tokens_open": (i32, [C.c_char_p, i32, C.POINTER(vp)]),
        "cb_tokens_from_host": (i32, [C.POINTER(C.c_uint16), i64, i32, C.POINTER(vp)]),
        "cb_tokens_len": (i32, [vp, C.POINTER(i64)]),
        "cb_tokens_close": (i32, [vp]),
        "cb_forward_loss_windows": (i32, [vp, vp, C.POINTER(i64), i32, f32, pf, pf]),
        "cb_eval_windows": (i32, [vp, vp, pi32, i32, i64, i64, f32, C.POINTER(cb_eval_totals)]),
        "cb_enable_training": (i32, [vp]),
        "cb_zero_grads": (i32, [vp]),
        "cb_forward_backward": (i32, [vp, pu32, pu32, i32, f32, f32, pf]),
        "cb_get_grads_f32": (i32, [vp, pf, pf, C.POINTER(cb_layer_grads_f32)]),
        "cb_prefill": (i32, [vp, pu32, i32, i32, f32, pf]),
        "cb_decode_step": (i32, [vp, pu32, i32, pf, pu32]),
        "cb_decode_position": (i32, [vp, pi32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, ctx=None) -> None:
    if status != CB_OK:
        lib = load_library()
        msg = (lib.cb_last_error(ctx) if ctx else lib.cb_create_error()) or b""
        raise CudaBridgeError(status, msg.decode())
