"""Tensor parallelism on 2 GPUs (Megatron split; the row-parallel partial sums combined
by a sequence-parallel fp16 or fp32 reduce-scatter + all-gather, or by an fp32 all-reduce)
against the single-GPU forward on the same weights and tokens.

Thresholds are the reference's own sharded-vs-baseline equivalence bounds
(crates/engine/tests/test_combined_forward_correctness.rs:13-14 and
parallel_bench_forward.rs:5-8): per-token loss max-abs <= 2e-2, cosine >= 0.999,
|delta loss| <= 1e-4. Skipped with fewer than 2 GPUs."""
import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from rustane_b200.model import CONFIGS, custom_config

pytestmark = pytest.mark.gpu

needs2 = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")


def _tokens(cfg, batch, seed):
    rng = np.random.default_rng(seed)
    return (rng.integers(0, cfg.vocab, batch * cfg.seq).astype(np.uint32),
            rng.integers(0, cfg.vocab, batch * cfg.seq).astype(np.uint32))


SAMPLE_ROWS = [0, 5, 511, 700]


def _tp_rank(rank, world, cfg, batch, seed, nccl_id, out, mode=None):
    import os
    if mode:
        os.environ["CB_TP_REDUCE"] = mode  # read on the first forward of the process
    from rustane_b200 import CB_INIT_NORMAL, CompiledKernels
    tok, tgt = _tokens(cfg, batch, seed)
    rows = [r for r in SAMPLE_ROWS if r < batch * cfg.seq]
    with CompiledKernels(cfg, rank, batch, tp_rank=rank, tp_world=world, nccl_id=nccl_id) as k:
        k.init_weights(seed, CB_INIT_NORMAL, 0.02)
        loss, ptl = k.forward_loss(tok, tgt, per_token=True)
        z = k.sampled_logits(rows)
        loss2 = k.forward_loss(tok, tgt)  # graph replay
        out[rank] = (loss, ptl, loss2, k.tp_info())
        out[f"logits{rank}"] = z


def _single(cfg, batch, seed, out):
    from rustane_b200 import CB_INIT_NORMAL, CompiledKernels
    tok, tgt = _tokens(cfg, batch, seed)
    rows = [r for r in SAMPLE_ROWS if r < batch * cfg.seq]
    with CompiledKernels(cfg, 0, batch) as k:
        k.init_weights(seed, CB_INIT_NORMAL, 0.02)
        out["single"] = k.forward_loss(tok, tgt, per_token=True)
        out["logits_single"] = k.sampled_logits(rows)


def _run(cfg, batch, seed, mode=None):
    from rustane_b200 import nccl_unique_id
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    p = ctx.Process(target=_single, args=(cfg, batch, seed, out))
    p.start()
    p.join(600)
    assert p.exitcode == 0
    nid = nccl_unique_id()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, cfg, batch, seed, nid, out, mode))
             for r in range(2)]
    for q in procs:
        q.start()
    for q in procs:
        q.join(600)
        assert q.exitcode == 0
    return out


def _check(out):
    l1, p1 = out["single"]
    z1 = out["logits_single"]
    for r in range(2):
        loss, ptl, loss2, info = out[r]
        assert loss == loss2
        assert abs(loss - l1) <= 1e-4, (loss, l1)
        assert np.max(np.abs(ptl - p1)) <= 2e-2
        cos = float(np.dot(ptl, p1) / (np.linalg.norm(ptl) * np.linalg.norm(p1)))
        assert cos >= 0.999
        # the final residual rows reach every rank (sequence parallel: all-gathered)
        assert np.max(np.abs(out[f"logits{r}"] - z1)) <= 2e-2
    # every rank returns the same losses
    assert out[0][0] == out[1][0]
    np.testing.assert_array_equal(out[0][1], out[1][1])
    return [out[r][3] for r in range(2)]


@needs2
@pytest.mark.parametrize("mode", ["sp16", "sp32", "allreduce"])
def test_tp2_matches_single_gpu_600m_shape(bridge_lib, mode):
    cfg = CONFIGS["600m-A"].replace(nlayers=4)
    infos = _check(_run(cfg, 2, 21, mode))
    assert [i["heads"] for i in infos] == [6, 6]
    assert [i["hidden"] for i in infos] == [2048, 2048]


@needs2
def test_tp2_matches_single_gpu_32b_shape(bridge_lib):
    """~32B shape: 52 heads, hidden 17920, seq 2048 (two layers)."""
    cfg = CONFIGS["32B"].replace(nlayers=2)
    infos = _check(_run(cfg, 1, 22))
    assert [i["heads"] for i in infos] == [26, 26]
    assert sum(i["hidden"] for i in infos) == 17920


@needs2
def test_tp2_uneven_split(bridge_lib):
    """5 heads and 5 hidden blocks over 2 ranks: shares 3/2."""
    cfg = custom_config(512, 320, 5, 2, 128, 1024)
    infos = _check(_run(cfg, 2, 23))
    assert [i["heads"] for i in infos] == [3, 2]
    assert [i["hidden"] for i in infos] == [192, 128]


def _tp_rank_env(rank, world, cfg, batch, seed, nccl_id, chunks, out, mode):
    import os
    os.environ["CB_TP_CHUNKS"] = str(chunks)  # read on the first forward of the process
    _tp_rank(rank, world, cfg, batch, seed, nccl_id, out, mode)


@needs2
@pytest.mark.parametrize("mode", ["sp16", "allreduce"])
def test_tp2_two_stream_chunks_equal_one_stream(bridge_lib, mode):
    """The chunked forward (collectives on their own stream, overlapping the next chunk's
    GEMMs) gives the same losses as the one-stream forward. With two ranks every element
    is the sum of two partials, which does not depend on which rank adds them, so the
    sequence-parallel forward matches too although chunking changes the rows a rank owns."""
    from rustane_b200 import nccl_unique_id
    cfg = CONFIGS["600m-A"].replace(nlayers=3)
    ctx = mp.get_context("spawn")
    res = {}
    for chunks in (1, 4):
        out = ctx.Manager().dict()
        nid = nccl_unique_id()
        procs = [ctx.Process(target=_tp_rank_env,
                             args=(r, 2, cfg, 4, 31, nid, chunks, out, mode))
                 for r in range(2)]
        for q in procs:
            q.start()
        for q in procs:
            q.join(600)
            assert q.exitcode == 0
        res[chunks] = out[0]
    l1, p1, _, _ = res[1]
    l4, p4, _, _ = res[4]
    assert abs(l1 - l4) <= 1e-6 * l1
    np.testing.assert_allclose(p4, p1, rtol=0, atol=1e-5)


def _tp_rank_profiled(rank, world, cfg, batch, seed, nccl_id, out):
    from rustane_b200 import CB_INIT_NORMAL, CompiledKernels
    tok, tgt = _tokens(cfg, batch, seed)
    with CompiledKernels(cfg, rank, batch, tp_rank=rank, tp_world=world, nccl_id=nccl_id) as k:
        k.init_weights(seed, CB_INIT_NORMAL, 0.02)
        loss = k.forward_loss(tok, tgt)
        k.set_profiling(True)
        k.reset_kernel_times()
        loss_prof = k.forward_loss(tok, tgt)
        times = k.kernel_times()
        k.set_profiling(False)
        out[rank] = (loss, loss_prof, times)


@needs2
def test_tp2_sequence_parallel_profiled_pass(bridge_lib):
    """The eager profiled pass of the sequence-parallel forward (one stream, one chunk)
    times each collective separately and returns the graph forward's loss."""
    from rustane_b200 import nccl_unique_id
    cfg = CONFIGS["600m-A"].replace(nlayers=2)
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    nid = nccl_unique_id()
    procs = [ctx.Process(target=_tp_rank_profiled, args=(r, 2, cfg, 2, 51, nid, out))
             for r in range(2)]
    for q in procs:
        q.start()
    for q in procs:
        q.join(600)
        assert q.exitcode == 0
    for r in range(2):
        loss, loss_prof, times = out[r]
        assert abs(loss_prof - loss) <= 1e-6 * loss
        L = cfg.nlayers
        assert times["nccl_reduce_scatter"]["launches"] == 2 * L
        assert times["nccl_all_gather"]["launches"] == 2 * L + 1
        assert times["add_rmsnorm"]["launches"] == 2 * L
        assert "nccl_allreduce" not in times


def test_peer_lost_is_refused_on_a_single_gpu_context(bridge_lib):
    """cb_tp_peer_lost on a context that is not tensor-parallel is an argument error and
    leaves the context usable."""
    from rustane_b200 import CB_INIT_NORMAL, CompiledKernels, CudaBridgeError
    from rustane_b200 import bridge as B
    cfg = custom_config(256, 512, 2, 1, 128, 512)
    tok, tgt = _tokens(cfg, 1, 3)
    with CompiledKernels(cfg, 0, 1) as k:
        k.init_weights(3, CB_INIT_NORMAL, 0.02)
        with pytest.raises(CudaBridgeError) as e:
            k.tp_peer_lost("no peers here")
        assert e.value.status == B.CB_ERR_INVALID_ARG
        assert np.isfinite(k.forward_loss(tok, tgt))
