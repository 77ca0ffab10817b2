"""CPU ORACLE wrapper — test infrastructure only.

Loads oracle/liboracle.so (forward_ref.cpp: a same-math fp32 restatement of the
reference forward + loss, crates/engine/src/full_model.rs:378-472 and the ops it
calls). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs may use this module, and only as the checker or the CPU
baseline — never as the product path.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

SCHEME_NORMAL = 0
SCHEME_REFERENCE = 1


class orc_config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in
                ("dim", "hidden", "heads", "kv_heads", "hd", "seq", "nlayers", "vocab")]


class orc_layer(C.Structure):
    _fields_ = [(n, C.POINTER(C.c_float)) for n in
                ("wq", "wk", "wv", "wo", "w1", "w3", "w2", "gamma1", "gamma2")]


_lib = None


def build() -> Path:
    r = subprocess.run(["make", "-s", "-C", str(HERE)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        pf = C.POINTER(C.c_float)
        L.orc_gen_weights.restype = C.c_int
        L.orc_gen_weights.argtypes = [C.POINTER(orc_config), C.c_uint64, C.c_int, C.c_float, pf,
                                      pf, C.POINTER(orc_layer)]
        L.orc_forward.restype = C.c_int
        L.orc_forward.argtypes = [C.POINTER(orc_config), pf, pf, C.POINTER(orc_layer),
                                  C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.c_int,
                                  C.c_float, pf, pf, C.POINTER(C.c_int32), C.c_int, pf]
        L.orc_forward_backward.restype = C.c_int
        L.orc_forward_backward.argtypes = [C.POINTER(orc_config), pf, pf, C.POINTER(orc_layer),
                                           C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                           C.c_int, C.c_float, C.c_float, pf, pf, pf,
                                           C.POINTER(orc_layer)]
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_max_threads.restype = C.c_int
        L.orc_f32_to_f16_bits.restype = C.c_uint16
        L.orc_f32_to_f16_bits.argtypes = [C.c_float]
        L.orc_f16_bits_to_f32.restype = C.c_float
        L.orc_f16_bits_to_f32.argtypes = [C.c_uint16]
        L.orc_lcg_jump.restype = C.c_uint64
        L.orc_lcg_jump.argtypes = [C.c_uint64, C.c_uint64]
        L.orc_lcg_value.restype = C.c_float
        L.orc_lcg_value.argtypes = [C.c_uint64, C.c_float]
        _lib = L
    return _lib


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


class OracleModel:
    """Host f32 weights (reference orientation) + the oracle forward."""

    LAYER_FIELDS = ("wq", "wk", "wv", "wo", "w1", "w3", "w2", "gamma1", "gamma2")

    def __init__(self, cfg, seed: int = 0, scheme: int = SCHEME_NORMAL, sigma: float = 0.02,
                 arrays: dict | None = None):
        self.cfg = cfg
        self.c = orc_config(cfg.dim, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.hd, cfg.seq,
                            cfg.nlayers, cfg.vocab)
        d, h, qd, kvd = cfg.dim, cfg.hidden, cfg.heads * cfg.hd, cfg.kv_heads * cfg.hd
        shapes = dict(wq=(d, qd), wk=(d, kvd), wv=(d, kvd), wo=(qd, d), w1=(d, h), w3=(d, h),
                      w2=(d, h), gamma1=(d,), gamma2=(d,))
        if arrays is None:
            self.embed = np.empty((cfg.vocab, d), np.float32)
            self.gamma_final = np.empty((d,), np.float32)
            self.layers = [{k: np.empty(s, np.float32) for k, s in shapes.items()}
                           for _ in range(cfg.nlayers)]
        else:
            self.embed = np.ascontiguousarray(arrays["embed"], np.float32)
            self.gamma_final = np.ascontiguousarray(arrays["gamma_final"], np.float32)
            self.layers = [{k: np.ascontiguousarray(lw[k], np.float32) for k in shapes}
                           for lw in arrays["layers"]]
        self._layer_arr = (orc_layer * cfg.nlayers)()
        for i, lw in enumerate(self.layers):
            self._layer_arr[i] = orc_layer(*[_fp(lw[k]) for k in self.LAYER_FIELDS])
        if arrays is None:
            rc = lib().orc_gen_weights(C.byref(self.c), seed, scheme, sigma, _fp(self.embed),
                                       _fp(self.gamma_final), self._layer_arr)
            if rc != 0:
                raise RuntimeError(f"orc_gen_weights failed: {rc}")

    def forward(self, tokens, targets, softcap: float = 0.0, sample_rows=None):
        t = np.ascontiguousarray(np.asarray(tokens, np.uint32).reshape(-1))
        g = np.ascontiguousarray(np.asarray(targets, np.uint32).reshape(-1))
        batch = t.size // self.cfg.seq
        loss = C.c_float()
        ptl = np.empty(t.size, np.float32)
        rows = None
        samp = None
        if sample_rows is not None:
            rows = np.ascontiguousarray(np.asarray(sample_rows, np.int32).reshape(-1))
            samp = np.empty((rows.size, self.cfg.vocab), np.float32)
        rc = lib().orc_forward(
            C.byref(self.c), _fp(self.embed), _fp(self.gamma_final), self._layer_arr,
            t.ctypes.data_as(C.POINTER(C.c_uint32)), g.ctypes.data_as(C.POINTER(C.c_uint32)),
            batch, softcap, C.byref(loss), _fp(ptl),
            rows.ctypes.data_as(C.POINTER(C.c_int32)) if rows is not None else None,
            0 if rows is None else rows.size, _fp(samp) if samp is not None else None)
        if rc != 0:
            raise RuntimeError(f"orc_forward failed: {rc}")
        return loss.value, ptl, samp


    def forward_backward(self, tokens, targets, softcap: float = 0.0, loss_scale: float = 1.0):
        """(loss, grads): grads = {"embed", "gamma_final", "layers": [dict]} in the
        reference orientation, the gradients of one training step (orc_forward_backward)."""
        t = np.ascontiguousarray(np.asarray(tokens, np.uint32).reshape(-1))
        g = np.ascontiguousarray(np.asarray(targets, np.uint32).reshape(-1))
        batch = t.size // self.cfg.seq
        d_embed = np.zeros_like(self.embed)
        d_gf = np.zeros_like(self.gamma_final)
        d_layers = [{k: np.zeros_like(v) for k, v in lw.items()} for lw in self.layers]
        arr = (orc_layer * self.cfg.nlayers)()
        for i, lw in enumerate(d_layers):
            arr[i] = orc_layer(*[_fp(lw[k]) for k in self.LAYER_FIELDS])
        loss = C.c_float()
        rc = lib().orc_forward_backward(
            C.byref(self.c), _fp(self.embed), _fp(self.gamma_final), self._layer_arr,
            t.ctypes.data_as(C.POINTER(C.c_uint32)), g.ctypes.data_as(C.POINTER(C.c_uint32)),
            batch, softcap, loss_scale, C.byref(loss), _fp(d_embed), _fp(d_gf), arr)
        if rc != 0:
            raise RuntimeError(f"orc_forward_backward failed: {rc}")
        return loss.value, {"embed": d_embed, "gamma_final": d_gf, "layers": d_layers}


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


def max_threads() -> int:
    return lib().orc_max_threads()


def reference_tokens(seq: int, vocab: int):
    """Tokens/targets of the reference forward benchmarks:
    tokens[i] = (i*31+7) % V, targets = tokens shifted by one
    (crates/engine/tests/bench_fwd_only_scale.rs:110-115)."""
    tokens = np.array([(i * 31 + 7) % vocab for i in range(seq)], np.uint32)
    targets = np.array([(i * 31 + 7) % vocab for i in range(1, seq + 1)], np.uint32)
    return tokens, targets
