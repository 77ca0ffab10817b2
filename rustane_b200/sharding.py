"""Work partitioning across GPUs.

Two pieces, both host logic:

* Shard-count resolution, mirroring crates/engine/src/sharding.rs:162-307: a
  requested shard count for an axis (attention head groups, FFN hidden width)
  must divide that axis; policy FailFast rejects an invalid request, policy
  AutoAdjustNearest replaces it with the nearest valid divisor (ties go to the
  smaller one) and records the adjustment.
* Sequence sharding (the reference's data parallelism, multistream.rs:54-161):
  the global batch of independent sequences is split into equal contiguous
  slices, one per rank; ranks never exchange activations. Only the scalar
  results (time, loss) are combined, on the host side of the job.
* The tensor-parallel split (`tp_partition`), answered by the bridge library
  itself (cb_tp_partition), so host code sees exactly the split cb_create_tp uses.
* The token rows a tensor-parallel rank owns in the sequence-parallel forward
  (`sequence_parallel_rows`): the rows whose residual it keeps, adds its reduce-scattered
  projection sums to and normalises before the all-gather.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field
from math import gcd
from typing import List, Optional, Tuple

import numpy as np


class ShardPolicy(enum.Enum):
    FAIL_FAST = "fail_fast"
    AUTO_ADJUST_NEAREST = "auto_adjust_nearest"


@dataclass(frozen=True)
class ModeAdjustment:
    axis: str
    requested: int
    applied: int
    reason: str


def divisors(value: int) -> List[int]:
    """Sorted divisors of value (sharding.rs:286-300)."""
    out = []
    i = 1
    while i * i <= value:
        if value % i == 0:
            out.append(i)
            if i != value // i:
                out.append(value // i)
        i += 1
    return sorted(out)


def nearest_divisor(divs: List[int], requested: int) -> int:
    """Closest divisor to `requested`; the smaller one on a tie (sharding.rs:302-307)."""
    return min(divs, key=lambda d: (abs(requested - d), d))


def resolve_axis(axis: str, shape_name: str, shape_value: int, requested: Optional[int],
                 policy: ShardPolicy, adjustments: List[ModeAdjustment]) -> int:
    """sharding.rs:227-260: None -> 1 shard; a divisor -> itself; otherwise per policy."""
    if requested is None:
        return 1
    if requested <= 0:
        raise ValueError(f"{axis} must be positive")
    valid = divisors(shape_value)
    if requested in valid:
        return requested
    if policy is ShardPolicy.FAIL_FAST:
        raise ValueError(f"{axis}={requested} is invalid for {shape_name}={shape_value}; "
                         f"valid divisors: {', '.join(map(str, valid))}")
    applied = nearest_divisor(valid, requested)
    adjustments.append(ModeAdjustment(axis, requested, applied,
                                      f"nearest valid divisor for {shape_name}={shape_value}"))
    return applied


@dataclass
class ModeResolution:
    attn_shards: int
    ffn_shards: int
    adjustments: List[ModeAdjustment] = field(default_factory=list)


def resolve_modes(cfg, attn_request: Optional[int], ffn_request: Optional[int],
                  policy: ShardPolicy = ShardPolicy.FAIL_FAST) -> ModeResolution:
    """Forward shard counts for attention (head groups) and FFN (hidden width),
    as resolve_modes (sharding.rs:162-213) does for its forward axes."""
    adj: List[ModeAdjustment] = []
    groups = gcd(cfg.heads, cfg.kv_heads)
    attn = resolve_axis("ATTN_FWD_SHARDS", "attention group count", groups, attn_request,
                        policy, adj)
    ffn = resolve_axis("FFN_FWD_SHARDS", "hidden width", cfg.hidden, ffn_request, policy, adj)
    return ModeResolution(attn, ffn, adj)


# ------------------------------------------------------------- sequence sharding

def shard_sequences(global_batch: int, world: int) -> int:
    """Sequences per rank. The global batch must divide evenly (FailFast)."""
    if global_batch <= 0 or world <= 0:
        raise ValueError("global batch and world size must be positive")
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} does not divide over {world} ranks; "
                         f"valid rank counts: {', '.join(map(str, divisors(global_batch)))}")
    return global_batch // world


def global_tokens(vocab: int, seq: int, global_batch: int, seed: int) -> Tuple[np.ndarray,
                                                                                np.ndarray]:
    """Uniform random tokens/targets of the whole job (independent of the rank count)."""
    rng = np.random.default_rng(seed)
    tok = rng.integers(0, vocab, global_batch * seq, dtype=np.int64).astype(np.uint32)
    tgt = rng.integers(0, vocab, global_batch * seq, dtype=np.int64).astype(np.uint32)
    return tok, tgt


def rank_shard(tokens: np.ndarray, targets: np.ndarray, seq: int, rank: int,
               per_rank: int) -> Tuple[np.ndarray, np.ndarray]:
    """Contiguous slice of whole sequences owned by `rank`."""
    a, b = rank * per_rank * seq, (rank + 1) * per_rank * seq
    if b > tokens.size:
        raise ValueError("rank slice beyond the global batch")
    return tokens[a:b], targets[a:b]


@dataclass(frozen=True)
class TpPartition:
    """Rank `rank` of a `world`-way Megatron split: query heads [head0, head0 + heads),
    kv heads [kv_head0, kv_head0 + kv_heads) and hidden columns [hidden0, hidden0 +
    hidden) (layer.rs:972-1003, 1906-2053: head-sharded attention, hidden-sharded FFN)."""
    rank: int
    world: int
    heads: int
    kv_heads: int
    hidden: int
    head0: int
    kv_head0: int
    hidden0: int


def tp_partition(cfg, world: int, rank: int) -> TpPartition:
    """The split cb_create_tp uses (no GPU needed); raises ValueError when the config,
    rank or world is invalid for tensor parallelism."""
    import ctypes as C

    from . import bridge as B
    lib = B.load_library()
    c = B.cb_model_config(cfg.dim, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.hd, cfg.seq,
                          cfg.nlayers, cfg.vocab)
    info = (C.c_int32 * 8)()
    rc = lib.cb_tp_partition(C.byref(c), world, rank, info)
    if rc != B.CB_OK:
        raise ValueError(f"no {world}-way tensor-parallel split of this config (rank {rank})")
    return TpPartition(*list(info))


def sequence_parallel_chunks(batch: int, seq: int, world: int, chunks: int = 2) -> int:
    """Chunks the sequence-parallel forward splits a batch into: the requested count
    (CB_TP_CHUNKS, default 2) lowered until it divides the batch, and 1 when a chunk's
    rows would not split evenly over the ranks (the rule of enqueue_forward in bridge.cu)."""
    n = max(1, min(chunks, 8))
    while n > 1 and batch % n:
        n -= 1
    if (batch * seq // n) % world:
        n = 1
    return n


def sequence_parallel_rows(batch: int, seq: int, world: int, rank: int,
                           chunks: int = 2) -> List[Tuple[int, int]]:
    """[start, stop) token-row ranges rank `rank` owns in the sequence-parallel forward:
    the batch's rows in chunks of Tc rows, and within chunk j the rank's contiguous slice
    of Tc / world rows (NCCL's reduce-scatter / all-gather layout)."""
    T = batch * seq
    if T % world:
        raise ValueError(f"{T} token rows do not split over {world} ranks")
    n = sequence_parallel_chunks(batch, seq, world, chunks)
    tc = T // n
    tl = tc // world
    return [(j * tc + rank * tl, j * tc + (rank + 1) * tl) for j in range(n)]


def reduce_max(value: float, device=None) -> float:
    """Max over ranks of the default process group (identity without one)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_mean(value: float, device=None) -> float:
    """Mean over ranks of the default process group (identity without one)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item()) / dist.get_world_size()
