"""CPU tests of the multi-rank host logic (gloo, world size 2) and of the
shard-count policy ported from crates/engine/src/sharding.rs; the tensor-parallel
split of cb_create_tp is checked by emulating its ranks on the CPU.

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


# ---- tensor parallelism: the Megatron split cb_create_tp uses, checked on CPU ranks

TP_CASES = {
    # 3 heads over 2 ranks (2 + 1), hidden 320 = 5 blocks of 64 (3 + 2)
    "uneven": custom_config(256, 320, 3, 2, 64),
    # grouped-query: 4 query heads on 2 kv heads, one kv head (two query heads) per rank
    "gqa": custom_config(256, 384, 4, 2, 64).replace(kv_heads=2),
}


def _tp_forward64(m, part, tokens, targets, all_reduce, seq_parallel=None):
    """One rank's Megatron forward in float64: Wq/Wk/Wv and W1/W3 column slices of its
    heads and hidden columns, Wo and W2 row slices, the partial O and down outputs summed
    over the ranks (where the GPU contexts call an NCCL all-reduce), everything else
    replicated (layer.rs:1906-2053, 4943-5139).

    With seq_parallel = (rows, reduce_scatter, all_gather) the partial outputs are
    reduce-scattered instead: the rank adds the sums of its own token rows (`rows`, from
    sequence_parallel_rows) to its residual rows, normalises them, and all-gathers the
    normalised rows (and, at the end, the residual rows), as the sequence-parallel GPU
    forward does."""
    import torch
    cfg = m.cfg
    S, hd = cfg.seq, cfg.hd
    f = lambda a: torch.from_numpy(np.asarray(a, np.float64))  # noqa: E731
    q0, q1 = part.head0 * hd, (part.head0 + part.heads) * hd
    k0, k1 = part.kv_head0 * hd, (part.kv_head0 + part.kv_heads) * hd
    c0, c1 = part.hidden0, part.hidden0 + part.hidden
    E = f(m.embed)
    x = E[torch.from_numpy(np.asarray(tokens, np.int64)).view(-1, S)]
    alpha = 1.0 / np.sqrt(2.0 * cfg.nlayers)
    p = torch.arange(S, dtype=torch.float64)[:, None]
    i = torch.arange(hd // 2, dtype=torch.float64)[None, :]
    th = p * torch.pow(torch.tensor(10000.0, dtype=torch.float64), -2.0 * i / hd)
    cos, sin = torch.cos(th)[None, :, None, :], torch.sin(th)[None, :, None, :]

    def norm(v, g):
        return v / torch.sqrt((v * v).mean(-1, keepdim=True) + 1e-5) * f(g)

    def rope(v):
        w = v.view(v.shape[0], S, -1, hd // 2, 2)
        a, b = w[..., 0], w[..., 1]
        return torch.stack([a * cos - b * sin, b * cos + a * sin], -1).view(v.shape)

    mask = torch.triu(torch.ones(S, S, dtype=torch.bool), 1)
    B0, d = x.shape[0], x.shape[-1]

    def combine(x, partial, gamma):
        """x + alpha * (sum over ranks of partial) and its normalised rows"""
        if seq_parallel is None:
            x = x + alpha * all_reduce(partial)
            return x, norm(x, gamma)
        rows, reduce_scatter, all_gather = seq_parallel
        flat, xf = partial.reshape(B0 * S, d), x.reshape(B0 * S, d).clone()
        xn_own = []
        for (r0, r1), chunk in zip(rows, _chunks_of(flat, rows)):
            mine = reduce_scatter(chunk)
            xf[r0:r1] = xf[r0:r1] + alpha * mine
            xn_own.append(norm(xf[r0:r1], gamma))
        xn = torch.cat([all_gather(o) for o in xn_own]).reshape(B0, S, d)
        # rows of other ranks are not kept: poison them so a missed row shows
        keep = torch.zeros(B0 * S, dtype=torch.bool)
        for r0, r1 in rows:
            keep[r0:r1] = True
        xf[~keep] = float("nan")
        return xf.reshape(B0, S, d), xn

    xn = norm(x, m.layers[0]["gamma1"]) if m.layers else None
    for li, lw in enumerate(m.layers):
        q = rope(xn @ f(lw["wq"])[:, q0:q1])
        k = rope(xn @ f(lw["wk"])[:, k0:k1])
        v = xn @ f(lw["wv"])[:, k0:k1]
        B_ = q.shape[0]
        q = q.view(B_, S, part.heads, hd).transpose(1, 2)
        k = k.view(B_, S, part.kv_heads, hd).transpose(1, 2)
        v = v.view(B_, S, part.kv_heads, hd).transpose(1, 2)
        grp = part.heads // part.kv_heads
        k, v = k.repeat_interleave(grp, dim=1), v.repeat_interleave(grp, dim=1)
        sc = (q @ k.transpose(-1, -2) / np.sqrt(float(hd))).masked_fill(mask, float("-inf"))
        a = (torch.softmax(sc, -1) @ v).transpose(1, 2).reshape(B_, S, -1)
        x, xn = combine(x, a @ f(lw["wo"])[q0:q1, :], lw["gamma2"])
        h1, h3 = xn @ f(lw["w1"])[:, c0:c1], xn @ f(lw["w3"])[:, c0:c1]
        g_next = m.layers[li + 1]["gamma1"] if li + 1 < len(m.layers) else m.gamma_final
        x, xn = combine(x, (h1 * torch.sigmoid(h1) * h3) @ f(lw["w2"])[:, c0:c1].T, g_next)
    if seq_parallel is not None:  # the final residual rows are gathered too
        rows, _, all_gather = seq_parallel
        xf = x.reshape(B0 * S, d)
        x = torch.cat([all_gather(xf[r0:r1]) for r0, r1 in rows]).reshape(B0, S, d)
    z = norm(x, m.gamma_final) @ E.T
    tgt = torch.from_numpy(np.asarray(targets, np.int64)).view(-1, S)
    ptl = torch.logsumexp(z, -1) - torch.gather(z, -1, tgt[..., None])[..., 0]
    return ptl.reshape(-1).numpy()


def _chunks_of(flat, rows):
    """The chunks of rows that the ranks' slices `rows` belong to (all ranks' rows)."""
    n = len(rows)
    tc = flat.shape[0] // n
    return [flat[j * tc:(j + 1) * tc] for j in range(n)]


def _tp_rank_main(rank, world, port, case, out, seq_parallel=False):
    import torch.distributed as dist
    from oracle.oracle import OracleModel
    from rustane_b200.sharding import tp_partition
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = TP_CASES[case]
        m = OracleModel(cfg, seed=5, sigma=0.05)
        tok, tgt = global_tokens(cfg.vocab, cfg.seq, 2, SEED)

        def all_reduce(t):
            t = t.contiguous()
            dist.all_reduce(t)
            return t

        sp = None
        if seq_parallel:
            import torch
            from rustane_b200.sharding import sequence_parallel_rows

            def reduce_scatter(t):
                o = torch.empty((t.shape[0] // world,) + tuple(t.shape[1:]), dtype=t.dtype)
                dist.reduce_scatter_tensor(o, t.contiguous())
                return o

            def all_gather(t):
                o = torch.empty((t.shape[0] * world,) + tuple(t.shape[1:]), dtype=t.dtype)
                dist.all_gather_into_tensor(o, t.contiguous())
                return o

            sp = (sequence_parallel_rows(2, cfg.seq, world, rank), reduce_scatter, all_gather)
        part = tp_partition(cfg, world, rank)
        out[rank] = (part, _tp_forward64(m, part, tok, tgt, all_reduce, sp))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("seq_parallel", [False, True], ids=["allreduce", "seqpar"])
@pytest.mark.parametrize("case", sorted(TP_CASES))
def test_tensor_parallel_split_equals_single_process(oracle_lib, bridge_lib, case,
                                                     seq_parallel):
    """Two gloo ranks, each holding only its cb_tp_partition share of the heads and
    hidden columns, reproduce the single-process forward (float64, so the only
    difference is summation order): with all-reduced projections, and sequence parallel
    (reduce-scatter to the rows sequence_parallel_rows gives the rank, residual and norm
    on those rows only, all-gather of the normalised rows)."""
    from oracle import torch_ref
    from oracle.oracle import OracleModel
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_tp_rank_main, args=(world, _free_port(), case, out, seq_parallel),
                       nprocs=world, join=True, start_method="spawn")
    cfg = TP_CASES[case]
    parts = [out[r][0] for r in range(world)]
    # the shares tile the heads, kv heads and hidden columns exactly once
    assert sum(p.heads for p in parts) == cfg.heads
    assert sum(p.kv_heads for p in parts) == cfg.kv_heads
    assert sum(p.hidden for p in parts) == cfg.hidden
    assert [p.head0 for p in parts] == [0, parts[0].heads]
    assert [p.hidden0 for p in parts] == [0, parts[0].hidden]
    tok, tgt = global_tokens(cfg.vocab, cfg.seq, 2, SEED)
    _, want, _ = torch_ref.forward(OracleModel(cfg, seed=5, sigma=0.05), tok, tgt)
    for r in range(world):
        np.testing.assert_allclose(out[r][1], want, rtol=0, atol=1e-10)


def test_tp_partition_matches_the_split_rule(bridge_lib):
    """52 heads over 8 ranks = 7,7,7,7,6,6,6,6; 17920 hidden = 280 blocks = 35 each."""
    from rustane_b200.model import CONFIGS
    from rustane_b200.sharding import tp_partition
    parts = [tp_partition(CONFIGS["32B"], 8, r) for r in range(8)]
    assert [p.heads for p in parts] == [7, 7, 7, 7, 6, 6, 6, 6]
    assert [p.head0 for p in parts] == [0, 7, 14, 21, 28, 34, 40, 46]
    assert all(p.hidden == 2240 for p in parts)
    with pytest.raises(ValueError):
        tp_partition(CONFIGS["600m-A"], 13, 0)  # more ranks than kv heads
    with pytest.raises(ValueError):
        tp_partition(CONFIGS["600m-A"], 2, 2)  # rank out of range


def test_tp_partition_properties(bridge_lib):
    """For every valid split the ranks' shares tile the kv heads (with their query heads)
    and the 64-column hidden blocks exactly once, in rank order, each share within one
    unit of the others."""
    from hypothesis import given, settings
    from hypothesis import strategies as st
    from rustane_b200.sharding import tp_partition

    @settings(max_examples=200, deadline=None)
    @given(kv=st.integers(1, 64), grp=st.sampled_from([1, 2, 4, 8]),
           blocks=st.integers(1, 400), data=st.data())
    def check(kv, grp, blocks, data):
        cfg = ModelConfig(256, 64 * blocks, kv * grp, kv, 128, 64, 1, 1024)
        world = data.draw(st.integers(1, min(kv, blocks)))
        parts = [tp_partition(cfg, world, r) for r in range(world)]
        head0 = kv0 = col0 = 0
        for p in parts:
            assert (p.head0, p.kv_head0, p.hidden0) == (head0, kv0, col0)
            assert p.heads == p.kv_heads * grp and p.kv_heads >= 1 and p.hidden >= 64
            head0, kv0, col0 = head0 + p.heads, kv0 + p.kv_heads, col0 + p.hidden
        assert (head0, kv0, col0) == (cfg.heads, cfg.kv_heads, cfg.hidden)
        assert max(p.kv_heads for p in parts) - min(p.kv_heads for p in parts) <= 1
        assert max(p.hidden for p in parts) - min(p.hidden for p in parts) <= 64

    check()


def test_sequence_parallel_rows_tile_the_batch():
    """The ranks' sequence-parallel rows cover every token row exactly once, in equal
    slices, for the chunk counts the forward picks."""
    from rustane_b200.sharding import sequence_parallel_chunks, sequence_parallel_rows
    for batch, seq, world in [(2, 64, 2), (16, 2048, 8), (4, 512, 2), (3, 512, 2), (1, 128, 4)]:
        T = batch * seq
        seen = np.zeros(T, np.int32)
        n = sequence_parallel_chunks(batch, seq, world)
        for r in range(world):
            rows = sequence_parallel_rows(batch, seq, world, r)
            assert len(rows) == n
            for r0, r1 in rows:
                assert r1 - r0 == T // n // world
                seen[r0:r1] += 1
        assert (seen == 1).all()
    assert sequence_parallel_chunks(3, 512, 2) == 1   # 3 sequences do not split in 2
    assert sequence_parallel_chunks(16, 2048, 8) == 2
    with pytest.raises(ValueError):
        sequence_parallel_rows(1, 63, 2, 0)
