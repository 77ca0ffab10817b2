"""The benchmark runner of the reference engine (crates/engine/src/parallel_bench.rs):
`ParallelBenchRunner.compile(cfg, request)` resolves the requested attention / FFN
shard counts exactly as the reference does (environment parsing, FailFast or
AutoAdjustNearest, mode labels), compiles the forward, and `forward_loss(...)` runs
one forward + loss (parallel_bench.rs:239-289), the call the reference's benchmarks
time.

On one B200 every mode runs the same single-context forward: the reference's shard
modes split a layer's heads and hidden columns into separate ANE programs run side by
side, while here every head and hidden column of a layer is already in flight inside
one kernel, so the resolved mode is recorded (labels, notes) but changes no launch.
Splitting a model over several GPUs is tensor parallelism (`CompiledKernels(...,
tp_rank=, tp_world=, nccl_id=)`, i.e. cb_create_tp).
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

from .engine import CompiledKernels, ModelForwardWorkspace, ModelWeights, forward_only_ws
from .model import ModelConfig
from .sharding import ShardPolicy, resolve_modes


class ParallelBenchError(ValueError):
    """ParallelBenchError (parallel_bench.rs:90-108)."""


def _parse_env_count(var: str) -> Optional[int]:
    """A positive integer from the environment, or None when unset
    (parse_env_count, sharding.rs:216-228)."""
    raw = os.environ.get(var)
    if raw is None:
        return None
    try:
        value = int(raw)
    except ValueError:
        raise ParallelBenchError(f"{var} must be an integer, got '{raw}'") from None
    if value <= 0:
        raise ParallelBenchError(f"{var} must be positive")
    return value


@dataclass(frozen=True)
class ParallelBenchRequest:
    """Requested forward shard counts (parallel_bench.rs:24-39)."""
    attn_request: Optional[int] = None
    ffn_request: Optional[int] = None
    policy: ShardPolicy = ShardPolicy.FAIL_FAST

    @classmethod
    def from_env(cls, policy: ShardPolicy = ShardPolicy.FAIL_FAST) -> "ParallelBenchRequest":
        """ATTN_FWD_SHARDS / FFN_FWD_SHARDS, or the ATTN_SHARDS / FFN_SHARDS shorthand
        (not both for one axis), as ShardRequest::from_env (sharding.rs:64-100) reads
        them for the forward."""
        req = {}
        for axis in ("ATTN", "FFN"):
            short = _parse_env_count(f"{axis}_SHARDS")
            fwd = _parse_env_count(f"{axis}_FWD_SHARDS")
            bwd = _parse_env_count(f"{axis}_BWD_SHARDS")
            if short is not None and (fwd is not None or bwd is not None):
                name = "attention" if axis == "ATTN" else "FFN"
                raise ParallelBenchError(
                    f"{axis}_SHARDS={short} conflicts with per-direction {name} shard vars; "
                    "use per-direction vars or the shorthand, not both")
            req[axis] = short if short is not None else fwd
        return cls(req["ATTN"], req["FFN"], policy)


@dataclass
class ResolvedParallelBenchConfig:
    """What a request resolved to (parallel_bench.rs:57-88)."""
    requested_attn: Optional[int]
    requested_ffn: Optional[int]
    applied_attn: int
    applied_ffn: int
    notes: List[str] = field(default_factory=list)

    def mode_label(self) -> str:
        a, f = self.applied_attn > 1, self.applied_ffn > 1
        if a and f:
            return f"attn{self.applied_attn}_ffn{self.applied_ffn}"
        if a:
            return f"attn{self.applied_attn}"
        if f:
            return f"ffn{self.applied_ffn}"
        return "baseline"

    def benchmark_suffix(self) -> str:
        label = self.mode_label()
        return "" if label == "baseline" else f"_{label}"


def resolve_parallel_bench_config(cfg: ModelConfig,
                                  request: ParallelBenchRequest) -> ResolvedParallelBenchConfig:
    """resolve_parallel_bench_config (parallel_bench.rs:316-364)."""
    try:
        res = resolve_modes(cfg, request.attn_request, request.ffn_request, request.policy)
    except ValueError as e:
        raise ParallelBenchError(str(e)) from None
    notes = [f"requested {a.axis}={a.requested}, applied {a.applied} ({a.reason})"
             for a in res.adjustments]
    return ResolvedParallelBenchConfig(request.attn_request, request.ffn_request,
                                       res.attn_shards, res.ffn_shards, notes)


class ParallelBenchRunner:
    """ParallelBenchRunner (parallel_bench.rs:110-290) on one B200."""

    def __init__(self, cfg: ModelConfig, resolved: ResolvedParallelBenchConfig,
                 kernels: CompiledKernels, use_lean_workspace: bool):
        self.cfg = cfg
        self._resolved = resolved
        self.kernels = kernels
        self.use_lean_workspace = use_lean_workspace

    @classmethod
    def compile(cls, cfg: ModelConfig, request: Optional[ParallelBenchRequest] = None,
                use_lean_workspace: bool = True, device: int = 0,
                max_batch: int = 1) -> Tuple["ParallelBenchRunner", float]:
        """(runner, compile seconds), as ParallelBenchRunner::compile
        (parallel_bench.rs:165-233); an invalid request raises ParallelBenchError
        before anything is compiled."""
        resolved = resolve_parallel_bench_config(cfg, request or ParallelBenchRequest())
        t0 = time.perf_counter()
        kernels = CompiledKernels(cfg, device, max_batch)
        return cls(cfg, resolved, kernels, use_lean_workspace), time.perf_counter() - t0

    def resolved(self) -> ResolvedParallelBenchConfig:
        return self._resolved

    def forward_loss(self, weights: ModelWeights, tokens, targets, softcap: float = 0.0,
                     ws: Optional[ModelForwardWorkspace] = None) -> float:
        """Mean next-token loss of the sequences in tokens/targets
        (parallel_bench.rs:239-289)."""
        return forward_only_ws(self.cfg, self.kernels, weights, tokens, targets, softcap, ws)

    def close(self) -> None:
        self.kernels.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
