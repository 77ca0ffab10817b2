"""Token data, val_bpb and the evaluation loop of the training binary.

Host-side mirrors of crates/engine/src/data.rs:
  TokenData (mmap'd uint16 token file)          data.rs:10-44
  TokenBytes (int32 byte length per token id)    data.rs:46-73
  compute_bpb                                    data.rs:75-91
  random_position                                data.rs:93-99
and the device path that replaces them on the GPU:
  DeviceTokens: the whole token file resident in HBM (cb_tokens_open); windows
  are gathered on the device, so a forward over file data copies no tokens.
  validate(): train.rs:197-236 over DeviceTokens, evaluated max_batch windows per
  forward with the loss and byte sums accumulated on the device (cb_eval_windows);
  under torch.distributed the validation steps are split across ranks.
"""
from __future__ import annotations

import ctypes as C
import math
from pathlib import Path
from typing import Optional, Tuple

import numpy as np

from . import bridge as B


class TokenData:
    """A flat uint16 little-endian token file, memory-mapped (data.rs:10-44)."""

    def __init__(self, array: np.ndarray):
        self._tokens = array

    @classmethod
    def open(cls, path) -> "TokenData":
        p = Path(path)
        n = p.stat().st_size // 2  # data.rs:23 n_tokens = len / 2
        arr = np.memmap(p, dtype="<u2", mode="r", shape=(n,)) if n else np.zeros(0, "<u2")
        return cls(arr)

    def len(self) -> int:
        return int(self._tokens.shape[0])

    __len__ = len

    def token(self, pos: int) -> int:
        return int(self._tokens[pos])

    def tokens(self, start: int, length: int) -> np.ndarray:
        """tokens[start, start + length) as u32 (data.rs:40-43)."""
        if start < 0 or start + length > self.len():
            raise IndexError("token range past the end of the data")
        return np.asarray(self._tokens[start:start + length], dtype=np.uint32)

    @property
    def array(self) -> np.ndarray:
        return self._tokens


class TokenBytes:
    """Byte length of every token id, 0 for special tokens (data.rs:46-73)."""

    def __init__(self, table: np.ndarray):
        self.bytes = np.ascontiguousarray(table, dtype=np.int32)

    @classmethod
    def load(cls, path) -> "TokenBytes":
        raw = Path(path).read_bytes()
        return cls(np.frombuffer(raw[:len(raw) // 4 * 4], dtype="<i4"))

    def byte_len(self, token_id: int) -> int:
        return int(self.bytes[token_id])


def compute_bpb(losses, targets, token_bytes: TokenBytes) -> Tuple[float, float, int]:
    """(val_bpb, total_nats, total_bytes) from per-token losses in nats
    (data.rs:75-91): only targets with a positive byte length count. The nats
    are summed in f32 in position order, as the reference does."""
    losses = np.asarray(losses, dtype=np.float32).reshape(-1)
    targets = np.asarray(targets).reshape(-1)
    bl = token_bytes.bytes[targets]
    keep = bl > 0
    total_bytes = int(bl[keep].astype(np.int64).sum())
    picked = losses[keep]
    total_nats = np.float32(np.cumsum(picked, dtype=np.float32)[-1]) if picked.size else np.float32(0)
    if total_bytes == 0:
        return 0.0, float(total_nats), 0
    bpb = np.float32(total_nats) / (np.float32(math.log(2)) * np.float32(total_bytes))
    return float(bpb), float(total_nats), total_bytes


def random_position(step: int, micro: int, max_pos: int) -> int:
    """(step * 7919 + micro * 104729) mod max_pos with u64 wrapping (data.rs:93-99);
    the training loop's window offset (train.rs:556)."""
    m = (1 << 64) - 1
    seed = ((step * 7919) & m) + ((micro * 104729) & m)
    return (seed & m) % max_pos


def validation_positions(n_tokens: int, seq: int, step_begin: int, step_end: int) -> np.ndarray:
    """Window offsets of validation steps [step_begin, step_end):
    (vs * seq) % (n - seq - 1) (train.rs:207-209)."""
    max_pos = n_tokens - seq - 1
    if max_pos <= 0:
        raise ValueError("token data shorter than seq + 2 tokens")
    vs = np.arange(step_begin, step_end, dtype=np.int64)
    return (vs * seq) % max_pos


class DeviceTokens:
    """A uint16 token array resident in one GPU's HBM (cb_tokens)."""

    def __init__(self, handle: C.c_void_p, device: int):
        self.lib = B.load_library()
        self._h = handle
        self.device = device

    @classmethod
    def open(cls, path, device: int = 0) -> "DeviceTokens":
        lib = B.load_library()
        h = C.c_void_p()
        B.check(lib.cb_tokens_open(str(path).encode(), device, C.byref(h)))
        return cls(h, device)

    @classmethod
    def from_array(cls, tokens, device: int = 0) -> "DeviceTokens":
        lib = B.load_library()
        a = np.ascontiguousarray(np.asarray(tokens).reshape(-1))
        if a.size and (a.min() < 0 or a.max() > 0xFFFF):
            raise ValueError("token ids must fit in uint16")
        a = a.astype("<u2")
        h = C.c_void_p()
        B.check(lib.cb_tokens_from_host(a.ctypes.data_as(C.POINTER(C.c_uint16)), a.size, device,
                                        C.byref(h)))
        return cls(h, device)

    @property
    def handle(self) -> C.c_void_p:
        if not self._h:
            raise RuntimeError("DeviceTokens is closed")
        return self._h

    def len(self) -> int:
        n = C.c_int64()
        B.check(self.lib.cb_tokens_len(self.handle, C.byref(n)))
        return n.value

    __len__ = len

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.cb_tokens_close(self._h)
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


def split_steps(steps: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous, near-even share [begin, end) of `steps` validation steps."""
    base, extra = divmod(steps, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def _sum_over_ranks(values, device=None):
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(values)
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.tolist()


def validate(cfg, kernels, weights, val_data: DeviceTokens,
             token_bytes: Optional[TokenBytes], steps: int, softcap: float = 0.0,
             distributed: bool = True) -> Tuple[float, float]:
    """(val_loss, val_bpb) of `steps` validation windows (train.rs:197-236).
    val_bpb is 0.0 without a token_bytes table, as in the reference. With an
    initialised torch.distributed default group (and distributed=True) each rank
    evaluates its share of the steps and the sums are added over ranks. weights=None
    evaluates what the context holds (e.g. after CompiledKernels.load_checkpoint)."""
    if weights is not None:
        kernels.load_weights(weights)
    rank, world, dev = 0, 1, None
    if distributed:
        try:
            import torch.distributed as dist
            if dist.is_available() and dist.is_initialized():
                rank, world = dist.get_rank(), dist.get_world_size()
                if dist.get_backend() == "nccl":
                    dev = f"cuda:{kernels.device}"
        except ImportError:
            pass
    begin, end = split_steps(steps, rank, world)
    tot = kernels.eval_windows(val_data, token_bytes, begin, end, softcap)
    loss_sum, nats, nbytes, ntok = _sum_over_ranks(
        [tot["loss_sum"], tot["nats"], tot["bytes"], tot["tokens"]], dev)
    val_loss = loss_sum / ntok if ntok else 0.0
    bpb = nats / (math.log(2) * nbytes) if (token_bytes is not None and nbytes > 0) else 0.0
    return float(np.float32(val_loss)), float(np.float32(bpb))
