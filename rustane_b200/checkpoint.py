"""RSTK checkpoints (crates/engine/src/bin/train.rs:238-346).

Layout: 28-byte header — magic b"RSTK", then u32 LE version (1), step, dim,
nlayers, vocab, seq — followed by f32 LE tensors in the reference orientation:
embed [vocab, dim], gamma_final [dim], then per layer wq, wk, wv, wo, w1, w3, w2,
gamma1, gamma2.

save_checkpoint / load_checkpoint are host mirrors of the training binary's
functions (numpy, for writing checkpoints and reading them on the CPU).
CompiledKernels.load_checkpoint streams a file straight into device weights
(cb_load_rstk) without a host copy of the model.
"""
from __future__ import annotations

import struct
from pathlib import Path
from typing import Tuple

import numpy as np

from .engine import LayerWeights, ModelWeights
from .model import ModelConfig

MAGIC = b"RSTK"
VERSION = 1
HEADER_BYTES = 28
LAYER_TENSORS = ("wq", "wk", "wv", "wo", "w1", "w3", "w2", "gamma1", "gamma2")


def layer_shapes(cfg: ModelConfig) -> dict:
    """Element counts of one layer's tensors (train.rs:303-311), as 2-D shapes in
    the reference orientation (x @ W; w2 is [dim, hidden] and used transposed)."""
    d, qd, kvd, h = cfg.dim, cfg.heads * cfg.hd, cfg.kv_heads * cfg.hd, cfg.hidden
    return {"wq": (d, qd), "wk": (d, kvd), "wv": (d, kvd), "wo": (qd, d), "w1": (d, h),
            "w3": (d, h), "w2": (d, h), "gamma1": (d,), "gamma2": (d,)}


def checkpoint_bytes(cfg: ModelConfig) -> int:
    n = cfg.vocab * cfg.dim + cfg.dim
    n += cfg.nlayers * sum(int(np.prod(s)) for s in layer_shapes(cfg).values())
    return HEADER_BYTES + 4 * n


def save_checkpoint(cfg: ModelConfig, weights: ModelWeights, step: int, directory) -> Path:
    """Write ckpt_{step:06}.bin into `directory` (train.rs:238-273). `weights`
    must hold host arrays (ModelWeights.from_arrays)."""
    if weights.embed is None:
        raise ValueError("save_checkpoint needs host weight arrays")
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    path = d / f"ckpt_{step:06d}.bin"
    shapes = layer_shapes(cfg)
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<6I", VERSION, step, cfg.dim, cfg.nlayers, cfg.vocab, cfg.seq))
        f.write(np.ascontiguousarray(weights.embed, dtype="<f4").tobytes())
        f.write(np.ascontiguousarray(weights.gamma_final, dtype="<f4").tobytes())
        for lw in weights.layers:
            for name in LAYER_TENSORS:
                a = np.ascontiguousarray(getattr(lw, name), dtype="<f4")
                if a.size != int(np.prod(shapes[name])):
                    raise ValueError(f"{name} has {a.size} values, expected {shapes[name]}")
                f.write(a.tobytes())
    return path


def read_header(path) -> dict:
    with open(path, "rb") as f:
        h = f.read(HEADER_BYTES)
    if len(h) < HEADER_BYTES or h[:4] != MAGIC:
        raise ValueError("bad checkpoint magic")
    version, step, dim, nlayers, vocab, seq = struct.unpack("<6I", h[4:])
    return dict(version=version, step=step, dim=dim, nlayers=nlayers, vocab=vocab, seq=seq)


def load_checkpoint(path, cfg: ModelConfig) -> Tuple[int, ModelWeights]:
    """(step, host ModelWeights) from an RSTK file (train.rs:297-346). Tensor
    sizes come from `cfg`, as in the reference."""
    step = read_header(path)["step"]
    raw = np.memmap(path, dtype="<f4", mode="r", offset=HEADER_BYTES)
    off = 0

    def take(shape):
        nonlocal off
        n = int(np.prod(shape))
        if off + n > raw.size:
            raise ValueError("checkpoint truncated")
        a = np.array(raw[off:off + n], dtype=np.float32).reshape(shape)
        off += n
        return a

    embed = take((cfg.vocab, cfg.dim))
    gamma_final = take((cfg.dim,))
    shapes = layer_shapes(cfg)
    layers = [LayerWeights(**{name: take(shapes[name]) for name in LAYER_TENSORS})
              for _ in range(cfg.nlayers)]
    return step, ModelWeights.from_arrays(embed, layers, gamma_final)
