"""CPU tests of the multi-rank host logic (gloo, world size 2) and of the
shard-count policy ported from crates/engine/src/sharding.rs.

The data-parallel forward shards whole sequences over ranks with no data-path
collective; only scalars (times, losses) are reduced. Here each rank runs the
CPU oracle on its shard and the reduced mean loss must equal the single-process
loss on the whole batch."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from rustane_b200.model import ModelConfig, custom_config
from rustane_b200.sharding import (ShardPolicy, divisors, global_tokens, nearest_divisor,
                                   rank_shard, resolve_modes, shard_sequences)

CFG = custom_config(256, 512, 2, 2, 64, 512)
GLOBAL_BATCH = 4
SEED = 11


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import torch.distributed as dist
    from oracle.oracle import OracleModel
    from rustane_b200.sharding import reduce_max, reduce_mean
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        per = shard_sequences(GLOBAL_BATCH, world)
        tok, tgt = global_tokens(CFG.vocab, CFG.seq, GLOBAL_BATCH, SEED)
        my_tok, my_tgt = rank_shard(tok, tgt, CFG.seq, rank, per)
        loss = OracleModel(CFG, seed=3, sigma=0.05).forward(my_tok, my_tgt)[0]
        mean = reduce_mean(loss)
        mx = reduce_max(float(rank * 10 + 1))
        out[rank] = (mean, mx, per)
    finally:
        dist.destroy_process_group()


def test_sequence_sharded_loss_equals_single_process(oracle_lib):
    from oracle.oracle import OracleModel
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), out), nprocs=world, join=True,
                       start_method="spawn")
    tok, tgt = global_tokens(CFG.vocab, CFG.seq, GLOBAL_BATCH, SEED)
    full = OracleModel(CFG, seed=3, sigma=0.05).forward(tok, tgt)[0]
    for r in range(world):
        mean, mx, per = out[r]
        assert per == GLOBAL_BATCH // world
        assert abs(mean - full) < 1e-5
        assert mx == 11.0


def test_shard_sequences_rules():
    assert shard_sequences(64, 8) == 8
    assert shard_sequences(64, 1) == 64
    with pytest.raises(ValueError, match="valid rank counts"):
        shard_sequences(64, 3)
    tok, tgt = global_tokens(512, 4, 6, 0)
    parts = [rank_shard(tok, tgt, 4, r, 2)[0] for r in range(3)]
    assert np.array_equal(np.concatenate(parts), tok)
    # the global batch does not depend on the rank count
    assert np.array_equal(global_tokens(512, 4, 6, 0)[0], tok)


def test_divisors_and_nearest_match_reference_rules():
    # sharding.rs:326-368: divisors sorted; nearest prefers the smaller on ties
    assert divisors(12) == [1, 2, 3, 4, 6, 12]
    assert divisors(52) == [1, 2, 4, 13, 26, 52]
    assert nearest_divisor(divisors(12), 5) == 4
    assert nearest_divisor(divisors(52), 8) == 4


def test_resolve_modes_fail_fast_and_auto_adjust():
    cfg = ModelConfig.target_600m()  # 12 heads, hidden 4096
    ok = resolve_modes(cfg, 4, 8)
    assert (ok.attn_shards, ok.ffn_shards, ok.adjustments) == (4, 8, [])
    with pytest.raises(ValueError, match="valid divisors"):
        resolve_modes(cfg, 5, None, ShardPolicy.FAIL_FAST)
    adj = resolve_modes(cfg, 5, 3, ShardPolicy.AUTO_ADJUST_NEAREST)
    assert adj.attn_shards == 4 and adj.ffn_shards == 2
    assert [a.axis for a in adj.adjustments] == ["ATTN_FWD_SHARDS", "FFN_FWD_SHARDS"]
    none = resolve_modes(cfg, None, None)
    assert (none.attn_shards, none.ffn_shards) == (1, 1)
