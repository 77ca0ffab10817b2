"""Tensor parallelism on 2 GPUs (Megatron split with NCCL all-reduce) against the
single-GPU forward on the same weights and tokens.

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


def _tp_rank(rank, world, cfg, batch, seed, nccl_id, out):
    from rustane_b200 import CB_INIT_NORMAL, CompiledKernels
    tok, tgt = _tokens(cfg, batch, seed)
    with CompiledKernels(cfg, rank, batch, tp_rank=rank, tp_world=world, nccl_id=nccl_id) as k:
        k.init_weights(seed, CB_INIT_NORMAL, 0.02)
        loss, ptl = k.forward_loss(tok, tgt, per_token=True)
        loss2 = k.forward_loss(tok, tgt)  # graph replay
        out[rank] = (loss, ptl, loss2, k.tp_info())


def _single(cfg, batch, seed, out):
    from rustane_b200 import CB_INIT_NORMAL, CompiledKernels
    tok, tgt = _tokens(cfg, batch, seed)
    with CompiledKernels(cfg, 0, batch) as k:
        k.init_weights(seed, CB_INIT_NORMAL, 0.02)
        out["single"] = k.forward_loss(tok, tgt, per_token=True)


def _run(cfg, batch, seed):
    from rustane_b200 import nccl_unique_id
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    p = ctx.Process(target=_single, args=(cfg, batch, seed, out))
    p.start()
    p.join(600)
    assert p.exitcode == 0
    nid = nccl_unique_id()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, cfg, batch, seed, nid, out))
             for r in range(2)]
    for q in procs:
        q.start()
    for q in procs:
        q.join(600)
        assert q.exitcode == 0
    return out


def _check(out):
    l1, p1 = out["single"]
    for r in range(2):
        loss, ptl, loss2, info = out[r]
        assert loss == loss2
        assert abs(loss - l1) <= 1e-4, (loss, l1)
        assert np.max(np.abs(ptl - p1)) <= 2e-2
        cos = float(np.dot(ptl, p1) / (np.linalg.norm(ptl) * np.linalg.norm(p1)))
        assert cos >= 0.999
    return [out[r][3] for r in range(2)]


@needs2
def test_tp2_matches_single_gpu_600m_shape(bridge_lib):
    cfg = CONFIGS["600m-A"].replace(nlayers=4)
    infos = _check(_run(cfg, 2, 21))
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


def _tp_rank_env(rank, world, cfg, batch, seed, nccl_id, chunks, out):
    import os
    os.environ["CB_TP_CHUNKS"] = str(chunks)  # read on the first forward of the process
    _tp_rank(rank, world, cfg, batch, seed, nccl_id, out)


@needs2
def test_tp2_two_stream_chunks_equal_one_stream(bridge_lib):
    """The chunked forward (all-reduces on their own stream, overlapping the next chunk's
    GEMMs) gives the same losses as the one-stream forward."""
    from rustane_b200 import nccl_unique_id
    cfg = CONFIGS["600m-A"].replace(nlayers=3)
    ctx = mp.get_context("spawn")
    res = {}
    for chunks in (1, 4):
        out = ctx.Manager().dict()
        nid = nccl_unique_id()
        procs = [ctx.Process(target=_tp_rank_env, args=(r, 2, cfg, 4, 31, nid, chunks, out))
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


def _tp_rank_leaves(rank, nccl_id, left, out):
    """Rank 1 runs one forward and exits between steps (nothing of it in flight); rank 0
    then runs its next forward, whose all-reduce has no peer."""
    import os
    import time
    os.environ["NCCL_NVLS_ENABLE"] = "0"     # no multicast objects bound to a leaving rank
    os.environ["CB_NCCL_TIMEOUT_MS"] = "5000"
    from rustane_b200 import CB_INIT_NORMAL, CompiledKernels, CudaBridgeError
    from rustane_b200 import bridge as B
    cfg = custom_config(512, 1024, 4, 2, 256, 2048)
    tok, tgt = _tokens(cfg, 2, 41)
    k = CompiledKernels(cfg, rank, 2, tp_rank=rank, tp_world=2, nccl_id=nccl_id)
    k.init_weights(41, CB_INIT_NORMAL, 0.02)
    out[f"loss{rank}"] = k.forward_loss(tok, tgt)
    if rank == 1:
        left.set()
        os._exit(0)  # leaves without any clean-up, like a worker that died between steps
    left.wait(60)
    time.sleep(2.0)  # the peer process is gone
    t0 = time.perf_counter()
    try:
        k.forward_loss(tok, tgt)
        out["status"] = B.CB_OK
    except CudaBridgeError as e:
        out["status"] = e.status
        out["message"] = str(e)
    out["seconds"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    try:
        k.forward_loss(tok, tgt)
        out["again"] = B.CB_OK
    except CudaBridgeError as e:
        out["again"] = e.status
    out["again_seconds"] = time.perf_counter() - t0
    k.close()


@needs2
def test_tp2_peer_leaving_gives_nccl_error_within_deadline(bridge_lib):
    """A tensor-parallel rank whose peer has left gets CB_ERR_NCCL from its next forward
    within the NCCL deadline (5 s here): the bridge polls the stream and the
    communicator's asynchronous error and aborts the communicator, instead of waiting in
    the all-reduce for good; the context then refuses further forwards at once."""
    from rustane_b200 import bridge as B
    from rustane_b200 import nccl_unique_id
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    left = ctx.Event()
    nid = nccl_unique_id()
    procs = [ctx.Process(target=_tp_rank_leaves, args=(r, nid, left, out)) for r in range(2)]
    for q in procs:
        q.start()
    for q in procs:
        q.join(180)
        assert q.exitcode == 0, q.exitcode
    assert abs(out["loss0"] - out["loss1"]) <= 1e-6 * out["loss0"]
    assert out["status"] == B.CB_ERR_NCCL, out.get("message")
    assert out["seconds"] < 5.0 + 15.0, out["seconds"]
    assert out["again"] == B.CB_ERR_NCCL and out["again_seconds"] < 1.0
