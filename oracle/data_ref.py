"""CPU ORACLE for the token-data, val_bpb and checkpoint rows — test
infrastructure only (tests/ may use it as the checker; the product never does).

Plain-Python restatements, element by element, of:
  data.rs:17-28   TokenData::open        n_tokens = file bytes / 2, u16 LE
  data.rs:34-43   token / tokens         u16 -> u32
  data.rs:52-68   TokenBytes::load       i32 LE array
  data.rs:75-91   compute_bpb            f32 running sum over byte-bearing targets
  data.rs:93-99   random_position        u64 wrapping LCG-style offset
  train.rs:197-236 validate              pos = (vs * seq) % (n - seq - 1)
  train.rs:238-273 save_checkpoint       28-byte header + f32 LE tensors
  train.rs:297-346 load_checkpoint
The reference's own tests hold no golden vectors for these functions; the
restatements are checked against byte strings built by hand in the tests.
"""
from __future__ import annotations

import struct

import numpy as np

U64 = (1 << 64) - 1


def read_tokens(raw: bytes) -> list:
    n = len(raw) // 2
    return [raw[2 * i] | (raw[2 * i + 1] << 8) for i in range(n)]


def read_token_bytes(raw: bytes) -> list:
    n = len(raw) // 4
    return [struct.unpack_from("<i", raw, 4 * i)[0] for i in range(n)]


def compute_bpb(losses, targets, token_bytes):
    total_nats = np.float32(0.0)
    total_bytes = 0
    for loss, tok in zip(losses, targets):
        bl = token_bytes[int(tok)]
        if bl > 0:
            total_nats = np.float32(total_nats + np.float32(loss))
            total_bytes += bl
    if total_bytes > 0:
        bpb = np.float32(total_nats / np.float32(np.float32(0.6931471805599453) *
                                                 np.float32(total_bytes)))
    else:
        bpb = np.float32(0.0)
    return float(bpb), float(total_nats), total_bytes


def random_position(step: int, micro: int, max_pos: int) -> int:
    seed = ((step * 7919) & U64)
    seed = (seed + ((micro * 104729) & U64)) & U64
    return seed % max_pos


def validation_windows(tokens: list, seq: int, steps: int):
    """[(input, target)] of validate's loop (train.rs:207-211)."""
    max_pos = len(tokens) - seq - 1
    out = []
    for vs in range(steps):
        pos = (vs * seq) % max_pos
        out.append((tokens[pos:pos + seq], tokens[pos + 1:pos + 1 + seq]))
    return out


def layer_counts(dim, hidden, heads, kv_heads, hd=128):
    qd, kvd = heads * hd, kv_heads * hd
    return [dim * qd, dim * kvd, dim * kvd, qd * dim, dim * hidden, dim * hidden,
            dim * hidden, dim, dim]


def write_checkpoint(step, dim, nlayers, vocab, seq, tensors) -> bytes:
    """Bytes of save_checkpoint: `tensors` is the flat list of f32 arrays in file
    order (embed, gamma_final, then 9 per layer)."""
    out = bytearray(b"RSTK")
    for v in (1, step, dim, nlayers, vocab, seq):
        out += struct.pack("<I", v)
    for t in tensors:
        for x in np.asarray(t, np.float32).reshape(-1).tolist():
            out += struct.pack("<f", x)
    return bytes(out)


def read_checkpoint(raw: bytes, dim, hidden, heads, kv_heads, nlayers, vocab):
    """(step, flat list of tensors) as load_checkpoint reads them."""
    assert raw[0:4] == b"RSTK", "bad checkpoint magic"
    step = struct.unpack_from("<I", raw, 8)[0]
    off = 28
    counts = [vocab * dim, dim] + layer_counts(dim, hidden, heads, kv_heads) * nlayers
    tensors = []
    for n in counts:
        tensors.append(np.array(struct.unpack_from(f"<{n}f", raw, off), np.float32))
        off += 4 * n
    return step, tensors
