"""CPU tests of the token-data, val_bpb and RSTK checkpoint host logic against
the oracle restatements (oracle/data_ref.py) and hand-built byte strings."""
import multiprocessing as mp
import os
import struct

import numpy as np
import pytest

from oracle import data_ref as R
from rustane_b200 import LayerWeights, ModelWeights
from rustane_b200.checkpoint import (checkpoint_bytes, load_checkpoint, read_header,
                                     save_checkpoint)
from rustane_b200.data import (TokenBytes, TokenData, compute_bpb, random_position,
                               split_steps, validate, validation_positions)
from rustane_b200.model import custom_config


def test_token_file_layout(tmp_path):
    # u16 little endian; an odd trailing byte is ignored (n = len / 2)
    raw = bytes([0x01, 0x00, 0xFF, 0x1F, 0x34, 0x12, 0x07])
    p = tmp_path / "tok.bin"
    p.write_bytes(raw)
    td = TokenData.open(p)
    assert len(td) == 3 == len(R.read_tokens(raw))
    assert [td.token(i) for i in range(3)] == R.read_tokens(raw) == [1, 0x1FFF, 0x1234]
    assert td.tokens(1, 2).dtype == np.uint32
    assert td.tokens(1, 2).tolist() == [0x1FFF, 0x1234]
    with pytest.raises(IndexError):
        td.tokens(2, 2)


def test_empty_token_file(tmp_path):
    p = tmp_path / "empty.bin"
    p.write_bytes(b"")
    assert len(TokenData.open(p)) == 0


def test_token_bytes_layout(tmp_path):
    table = [0, 1, 3, -1, 7]
    p = tmp_path / "token_bytes.bin"
    p.write_bytes(b"".join(struct.pack("<i", v) for v in table) + b"\x00")
    tb = TokenBytes.load(p)
    assert tb.bytes.tolist() == R.read_token_bytes(p.read_bytes()) == table
    assert tb.byte_len(2) == 3


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_compute_bpb_matches_oracle_bit_exact(seed):
    rng = np.random.default_rng(seed)
    V, T = 300, 5000
    table = rng.integers(0, 6, V).astype(np.int32)
    table[:7] = 0  # special tokens carry no bytes
    losses = (rng.random(T) * 9).astype(np.float32)
    targets = rng.integers(0, V, T).astype(np.uint32)
    got = compute_bpb(losses, targets, TokenBytes(table))
    want = R.compute_bpb(losses.tolist(), targets.tolist(), table.tolist())
    assert got == want


def test_compute_bpb_without_bytes_is_zero():
    tb = TokenBytes(np.zeros(8, np.int32))
    assert compute_bpb(np.ones(4, np.float32), np.arange(4), tb) == (0.0, 0.0, 0)
    assert R.compute_bpb([1.0] * 4, [0, 1, 2, 3], [0] * 8) == (0.0, 0.0, 0)


@pytest.mark.parametrize("step,micro,max_pos", [
    (0, 0, 1000), (5, 3, 999_983), (123456, 7, 1 << 30),
    ((1 << 64) // 7919 + 5, 1, 1_000_003),        # step * 7919 wraps
    (3, (1 << 64) // 104729 + 9, 65_537),          # micro * 104729 wraps
    ((1 << 64) - 1, (1 << 64) - 1, 97),            # the sum wraps
])
def test_random_position_matches_oracle(step, micro, max_pos):
    assert random_position(step, micro, max_pos) == R.random_position(step, micro, max_pos)


def test_validation_positions_match_oracle():
    toks = list(range(1000))
    seq = 64
    pos = validation_positions(len(toks), seq, 0, 40)
    win = R.validation_windows(toks, seq, 40)
    for p, (inp, tgt) in zip(pos.tolist(), win):
        assert toks[p:p + seq] == inp and toks[p + 1:p + 1 + seq] == tgt
    assert validation_positions(len(toks), seq, 10, 40).tolist() == pos[10:].tolist()
    with pytest.raises(ValueError):
        validation_positions(seq + 1, seq, 0, 1)


@pytest.mark.parametrize("steps,world", [(10, 1), (10, 3), (2, 4), (0, 2), (17, 8)])
def test_split_steps_partitions(steps, world):
    seen = []
    for r in range(world):
        a, b = split_steps(steps, r, world)
        assert 0 <= a <= b <= steps
        seen.extend(range(a, b))
    assert seen == list(range(steps))


def _tiny_cfg():
    return custom_config(256, 512, 2, 2, 128, 64).replace(vocab=96)


def _random_weights(cfg, seed):
    rng = np.random.default_rng(seed)
    d, h, qd = cfg.dim, cfg.hidden, cfg.heads * cfg.hd
    kvd = cfg.kv_heads * cfg.hd
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    layers = [LayerWeights(wq=f(d, qd), wk=f(d, kvd), wv=f(d, kvd), wo=f(qd, d), w1=f(d, h),
                           w3=f(d, h), w2=f(d, h), gamma1=f(d), gamma2=f(d))
              for _ in range(cfg.nlayers)]
    return ModelWeights.from_arrays(f(cfg.vocab, d), layers, f(d))


def _flat(w):
    out = [w.embed, w.gamma_final]
    for lw in w.layers:
        out += [getattr(lw, k) for k in ("wq", "wk", "wv", "wo", "w1", "w3", "w2", "gamma1",
                                         "gamma2")]
    return out


def test_checkpoint_bytes_match_oracle_writer(tmp_path):
    cfg = _tiny_cfg()
    w = _random_weights(cfg, 0)
    path = save_checkpoint(cfg, w, 1234, tmp_path)
    assert path.name == "ckpt_001234.bin"
    raw = path.read_bytes()
    assert len(raw) == checkpoint_bytes(cfg)
    assert raw == R.write_checkpoint(1234, cfg.dim, cfg.nlayers, cfg.vocab, cfg.seq, _flat(w))
    assert read_header(path) == dict(version=1, step=1234, dim=cfg.dim, nlayers=cfg.nlayers,
                                     vocab=cfg.vocab, seq=cfg.seq)


def test_checkpoint_round_trip(tmp_path):
    cfg = _tiny_cfg()
    w = _random_weights(cfg, 1)
    path = save_checkpoint(cfg, w, 7, tmp_path)
    step, w2 = load_checkpoint(path, cfg)
    assert step == 7
    for a, b in zip(_flat(w), _flat(w2)):
        assert a.shape == b.shape and np.array_equal(a, b)
    step_o, flat_o = R.read_checkpoint(path.read_bytes(), cfg.dim, cfg.hidden, cfg.heads,
                                       cfg.kv_heads, cfg.nlayers, cfg.vocab)
    assert step_o == 7
    for a, b in zip(_flat(w), flat_o):
        assert np.array_equal(a.reshape(-1), b)


def test_checkpoint_rejects_bad_magic_and_truncation(tmp_path):
    cfg = _tiny_cfg()
    path = save_checkpoint(cfg, _random_weights(cfg, 2), 1, tmp_path)
    raw = path.read_bytes()
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"XXXX" + raw[4:])
    with pytest.raises(ValueError, match="magic"):
        read_header(bad)
    short = tmp_path / "short.bin"
    short.write_bytes(raw[:-4])
    with pytest.raises(ValueError, match="truncated"):
        load_checkpoint(short, cfg)


class _FakeKernels:
    """Stands in for CompiledKernels.eval_windows: per-step losses from a table."""
    device = 0

    def __init__(self, per_step_loss, per_step_nats, per_step_bytes, seq):
        self.l, self.n, self.b, self.seq = per_step_loss, per_step_nats, per_step_bytes, seq

    def load_weights(self, w):
        pass

    def eval_windows(self, data, token_bytes, begin, end, softcap):
        return dict(loss_sum=float(sum(self.l[begin:end])), nats=float(sum(self.n[begin:end])),
                    bytes=int(sum(self.b[begin:end])), tokens=(end - begin) * self.seq)


def _fake():
    rng = np.random.default_rng(5)
    steps = 11
    return (_FakeKernels(rng.random(steps) * 500, rng.random(steps) * 400,
                         rng.integers(100, 200, steps), 64), steps)


def _validate_rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        k, steps = _fake()
        q.put((rank, validate(None, k, None, None, TokenBytes(np.ones(4, np.int32)), steps)))
    finally:
        dist.destroy_process_group()


def test_validate_sums_over_gloo_ranks():
    """validate() splits the validation steps across ranks and adds the sums: two
    gloo ranks give the single-process (val_loss, val_bpb)."""
    k, steps = _fake()
    want = validate(None, k, None, None, TokenBytes(np.ones(4, np.int32)), steps,
                    distributed=False)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_validate_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == got[1]
    np.testing.assert_allclose(got[0], want, rtol=1e-6)
