"""The benchmark runner's host logic (parallel_bench.rs): request parsing from the
environment, mode resolution and labels, and (on a GPU) that its forward_loss is the
engine's forward."""
import numpy as np
import pytest

from rustane_b200 import (CudaBridgeError, ModelWeights, ParallelBenchError,
                          ParallelBenchRequest, ParallelBenchRunner)
from rustane_b200.model import ModelConfig, custom_config
from rustane_b200.parallel_bench import resolve_parallel_bench_config
from rustane_b200.sharding import ShardPolicy

ENV = ("ATTN_SHARDS", "FFN_SHARDS", "ATTN_FWD_SHARDS", "FFN_FWD_SHARDS", "ATTN_BWD_SHARDS",
       "FFN_BWD_SHARDS")


@pytest.fixture
def clean_env(monkeypatch):
    for v in ENV:
        monkeypatch.delenv(v, raising=False)
    return monkeypatch


def test_request_from_env(clean_env):
    assert ParallelBenchRequest.from_env() == ParallelBenchRequest(None, None)
    clean_env.setenv("ATTN_FWD_SHARDS", "4")
    clean_env.setenv("FFN_SHARDS", "8")
    r = ParallelBenchRequest.from_env(ShardPolicy.AUTO_ADJUST_NEAREST)
    assert (r.attn_request, r.ffn_request, r.policy) == (4, 8, ShardPolicy.AUTO_ADJUST_NEAREST)


@pytest.mark.parametrize("env,msg", [
    ({"ATTN_FWD_SHARDS": "x"}, "must be an integer"),
    ({"FFN_FWD_SHARDS": "0"}, "must be positive"),
    ({"ATTN_SHARDS": "2", "ATTN_BWD_SHARDS": "2"}, "conflicts"),
])
def test_request_from_env_errors(clean_env, env, msg):
    for k, v in env.items():
        clean_env.setenv(k, v)
    with pytest.raises(ParallelBenchError, match=msg):
        ParallelBenchRequest.from_env()


def test_resolution_labels_and_notes():
    cfg = ModelConfig.target_600m()  # 12 heads, hidden 4096
    base = resolve_parallel_bench_config(cfg, ParallelBenchRequest())
    assert (base.mode_label(), base.benchmark_suffix()) == ("baseline", "")
    both = resolve_parallel_bench_config(cfg, ParallelBenchRequest(4, 8))
    assert (both.mode_label(), both.benchmark_suffix()) == ("attn4_ffn8", "_attn4_ffn8")
    assert resolve_parallel_bench_config(cfg, ParallelBenchRequest(2, None)).mode_label() == "attn2"
    assert resolve_parallel_bench_config(cfg, ParallelBenchRequest(None, 2)).mode_label() == "ffn2"
    adj = resolve_parallel_bench_config(
        cfg, ParallelBenchRequest(5, None, ShardPolicy.AUTO_ADJUST_NEAREST))
    assert adj.applied_attn == 4 and adj.requested_attn == 5
    assert adj.notes and "applied 4" in adj.notes[0]
    with pytest.raises(ParallelBenchError, match="valid divisors"):
        resolve_parallel_bench_config(cfg, ParallelBenchRequest(5, None))


def test_compile_resolves_before_touching_a_device(bridge_lib):
    cfg = ModelConfig.target_600m()
    with pytest.raises(ParallelBenchError):
        ParallelBenchRunner.compile(cfg, ParallelBenchRequest(7, None))
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(CudaBridgeError):
        ParallelBenchRunner.compile(cfg)


@pytest.mark.gpu
def test_runner_forward_loss_is_the_engine_forward(bridge_lib):
    cfg = custom_config(256, 512, 2, 2, 128)
    rng = np.random.default_rng(4)
    tok = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
    w = ModelWeights.normal(cfg, seed=9, sigma=0.05)
    runner, compile_s = ParallelBenchRunner.compile(cfg, ParallelBenchRequest(2, 2))
    with runner:
        assert compile_s >= 0 and runner.resolved().mode_label() == "attn2_ffn2"
        loss = runner.forward_loss(w, tok, tgt)
        assert loss == runner.kernels.forward_loss(tok, tgt)
        assert 0 < loss < 20  # the reference's sanity bound (phase4_training.rs:106-124)


ODD = ModelConfig(256, 768, 1, 1, 128, 16, 2, 256)  # test_combined_forward_correctness.rs:245-257


def test_odd_config_single_head_falls_back_to_baseline():
    """One attention group: a request for 8 attention shards adjusts to 1, i.e. the
    baseline mode (test_combined_forward_correctness.rs:245-268)."""
    r = resolve_parallel_bench_config(ODD, ParallelBenchRequest(8, None,
                                                                ShardPolicy.AUTO_ADJUST_NEAREST))
    assert (r.applied_attn, r.mode_label()) == (1, "baseline")
