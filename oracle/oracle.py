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
        pu = C.POINTER(C.c_uint32)
        for name, args in (
                ("orc_op_embedding", [pf, C.c_int, C.c_int, pu, C.c_int, pf]),
                ("orc_op_embedding_backward", [pf, C.c_int, C.c_int, pu, C.c_int, pf]),
                ("orc_op_rmsnorm", [pf, pf, pf, pf, C.c_int, C.c_int]),
                ("orc_op_rmsnorm_backward", [pf, pf, pf, pf, pf, pf, C.c_int, C.c_int]),
                ("orc_op_silu_gate", [pf, pf, pf, C.c_int64]),
                ("orc_op_silu_gate_backward", [pf, pf, pf, pf, pf, C.c_int64]),
                ("orc_op_cross_entropy", [pf, pu, C.c_int, C.c_int, C.c_float, C.c_float, pf,
                                          pf]),
                ("orc_op_sgemm", [C.c_int, C.c_int, C.c_int, pf, pf, C.c_int, pf])):
            getattr(L, name).restype = C.c_int
            getattr(L, name).argtypes = args
        _lib = L
    return _lib


# ---- the oracle's single ops (the functions its forward and backward use), for the
# ports of the reference's CPU-op unit tests. Float arrays are float32, rows token-major.

def _f32(a):
    return np.ascontiguousarray(a, np.float32)


def _u32p(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


def _check(rc, name):
    if rc != 0:
        raise ValueError(f"{name} failed: {rc}")


def op_embedding(table, ids):
    """out[t] = table[ids[t]] (cpu/embedding.rs:8-17); table [V, d]."""
    table = _f32(table)
    ids = np.ascontiguousarray(ids, np.uint32).reshape(-1)
    out = np.empty((ids.size, table.shape[1]), np.float32)
    _check(lib().orc_op_embedding(_fp(table), table.shape[0], table.shape[1], _u32p(ids),
                                  ids.size, _fp(out)), "orc_op_embedding")
    return out


def op_embedding_backward(dout, ids, vocab):
    """dtable [vocab, d] with dtable[ids[t]] += dout[t] (cpu/embedding.rs:20-44)."""
    dout = _f32(dout)
    ids = np.ascontiguousarray(ids, np.uint32).reshape(-1)
    dtable = np.zeros((vocab, dout.shape[1]), np.float32)
    _check(lib().orc_op_embedding_backward(_fp(dout), vocab, dout.shape[1], _u32p(ids),
                                           ids.size, _fp(dtable)),
           "orc_op_embedding_backward")
    return dtable


def op_rmsnorm(x, gamma):
    """(out, rinv) per row of x [n, d] (cpu/rmsnorm.rs:15-42, 83-107)."""
    x, gamma = _f32(np.atleast_2d(x)), _f32(gamma)
    out = np.empty_like(x)
    rinv = np.empty(x.shape[0], np.float32)
    _check(lib().orc_op_rmsnorm(_fp(x), _fp(gamma), _fp(out), _fp(rinv), x.shape[0],
                                x.shape[1]), "orc_op_rmsnorm")
    return out, rinv


def op_rmsnorm_backward(dy, x, gamma, rinv):
    """(dx, dgamma) (cpu/rmsnorm.rs:44-81, 109-147); dgamma sums over the rows."""
    dy, x, gamma, rinv = _f32(np.atleast_2d(dy)), _f32(np.atleast_2d(x)), _f32(gamma), _f32(rinv)
    dx = np.empty_like(x)
    dgamma = np.zeros(x.shape[1], np.float32)
    _check(lib().orc_op_rmsnorm_backward(_fp(dy), _fp(x), _fp(gamma), _fp(rinv), _fp(dx),
                                         _fp(dgamma), x.shape[0], x.shape[1]),
           "orc_op_rmsnorm_backward")
    return dx, dgamma


def op_silu_gate(gate, up):
    """silu(gate) * up (cpu/silu.rs:37-46)."""
    gate, up = _f32(gate), _f32(up)
    out = np.empty_like(gate)
    _check(lib().orc_op_silu_gate(_fp(gate), _fp(up), _fp(out), gate.size), "orc_op_silu_gate")
    return out


def op_silu_gate_backward(dout, gate, up):
    """(dgate, dup) of out = silu(gate) * up (cpu/silu.rs:23-34)."""
    dout, gate, up = _f32(dout), _f32(gate), _f32(up)
    dgate, dup = np.empty_like(gate), np.empty_like(up)
    _check(lib().orc_op_silu_gate_backward(_fp(dout), _fp(gate), _fp(up), _fp(dgate), _fp(dup),
                                           gate.size), "orc_op_silu_gate_backward")
    return dgate, dup


def op_cross_entropy(logits, targets, softcap=0.0, scale=1.0, grad=True):
    """(losses [n], dlogits [n, V] or None) of raw logits [n, V]
    (cpu/cross_entropy.rs:13-96; softcap full_model.rs:456-461)."""
    z = _f32(np.atleast_2d(logits))
    t = np.ascontiguousarray(targets, np.uint32).reshape(-1)
    losses = np.empty(z.shape[0], np.float32)
    dl = np.empty_like(z) if grad else None
    _check(lib().orc_op_cross_entropy(_fp(z), _u32p(t), z.shape[0], z.shape[1], softcap, scale,
                                      _fp(losses), _fp(dl) if grad else None),
           "orc_op_cross_entropy")
    return losses, dl


def op_sgemm(a, b, b_trans=False):
    """a [M, K] @ b [K, N], or a @ b.T for b [N, K] when b_trans (the oracle's GEMM)."""
    a, b = _f32(a), _f32(b)
    M, K = a.shape
    N = b.shape[0] if b_trans else b.shape[1]
    c = np.empty((M, N), np.float32)
    _check(lib().orc_op_sgemm(M, N, K, _fp(a), _fp(b), int(b_trans), _fp(c)), "orc_op_sgemm")
    return c


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
