"""GPU tests of the checkpoint and token-data rows through the C ABI: RSTK files
streamed into device weights, windows gathered from an HBM-resident token array,
and the device-side validation sums, each against the host path and the oracle."""
import numpy as np
import pytest

from oracle import data_ref as R
from oracle.oracle import OracleModel, SCHEME_NORMAL
from rustane_b200 import (CompiledKernels, CudaBridgeError, DeviceTokens, LayerWeights,
                          ModelWeights, TokenBytes, validate)
from rustane_b200 import bridge as B
from rustane_b200.checkpoint import save_checkpoint
from rustane_b200.data import validation_positions
from rustane_b200.model import custom_config

pytestmark = pytest.mark.gpu


def _cfg():
    return custom_config(512, 1024, 4, 2, 128, 2048).replace(kv_heads=2)


def _oracle_weights(cfg, seed=3, sigma=0.05):
    ora = OracleModel(cfg, seed=seed, scheme=SCHEME_NORMAL, sigma=sigma)
    rng = np.random.default_rng(seed)
    for lw in ora.layers:  # non-unit gains, so their place in the file matters
        lw["gamma1"][:] = 1 + 0.1 * rng.standard_normal(cfg.dim)
        lw["gamma2"][:] = 1 + 0.1 * rng.standard_normal(cfg.dim)
    ora.gamma_final[:] = 1 + 0.1 * rng.standard_normal(cfg.dim)
    w = ModelWeights.from_arrays(ora.embed, [LayerWeights(**lw) for lw in ora.layers],
                                 ora.gamma_final)
    return ora, w


def test_rstk_load_matches_host_upload_and_oracle(tmp_path):
    cfg = _cfg()
    ora, w = _oracle_weights(cfg)
    path = save_checkpoint(cfg, w, 4242, tmp_path)
    rng = np.random.default_rng(0)
    tok = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    l_ref = ora.forward(tok, tgt)[0]
    with CompiledKernels(cfg, 0, 2) as k:
        k.load_weights(w)
        l_host, p_host = k.forward_loss(tok, tgt, per_token=True)
        assert k.load_checkpoint(path) == 4242
        l_file, p_file = k.forward_loss(tok, tgt, per_token=True)
    assert l_file == l_host and np.array_equal(p_file, p_host)  # same fp16 rounding
    assert abs(l_file - l_ref) / l_ref <= 1e-3


def test_rstk_errors_leave_context_usable(tmp_path):
    cfg = _cfg()
    _, w = _oracle_weights(cfg)
    good = save_checkpoint(cfg, w, 1, tmp_path / "good")
    raw = good.read_bytes()
    cases = {
        "magic": b"XSTK" + raw[4:],
        "dims": raw[:12] + (cfg.dim * 2).to_bytes(4, "little") + raw[16:],
        "short": raw[:-8],
        "header": raw[:20],
    }
    tok = np.arange(cfg.seq, dtype=np.uint32) % cfg.vocab
    with CompiledKernels(cfg, 0, 1) as k:
        k.load_checkpoint(good)
        base = k.forward_loss(tok, tok)
        for name, data in cases.items():
            p = tmp_path / f"{name}.bin"
            p.write_bytes(data)
            with pytest.raises(CudaBridgeError) as e:
                k.load_checkpoint(p)
            assert e.value.status == B.CB_ERR_INVALID_ARG, name
        with pytest.raises(CudaBridgeError):
            k.load_checkpoint(tmp_path / "missing.bin")
        # trailing bytes are ignored, as in the reference
        p = tmp_path / "trailing.bin"
        p.write_bytes(raw + b"\0" * 12)
        assert k.load_checkpoint(p) == 1
        assert k.forward_loss(tok, tok) == base


def _token_file(tmp_path, cfg, n, seed):
    rng = np.random.default_rng(seed)
    toks = rng.integers(0, cfg.vocab, n).astype("<u2")
    p = tmp_path / "tokens.bin"
    p.write_bytes(toks.tobytes())
    return p, toks


def test_windows_forward_equals_host_tokens(tmp_path):
    cfg = _cfg()
    path, toks = _token_file(tmp_path, cfg, 20_000, 1)
    pos = np.array([0, 777, 20_000 - cfg.seq - 1], np.int64)
    inp = np.concatenate([toks[p:p + cfg.seq] for p in pos]).astype(np.uint32)
    tgt = np.concatenate([toks[p + 1:p + 1 + cfg.seq] for p in pos]).astype(np.uint32)
    with CompiledKernels(cfg, 0, 4) as k, DeviceTokens.open(path) as data:
        assert len(data) == 20_000
        k.init_weights(2, B.CB_INIT_NORMAL, 0.05)
        want, pw = k.forward_loss(inp, tgt, per_token=True)
        got, pg = k.forward_loss_windows(data, pos, per_token=True)
        assert got == want and np.array_equal(pg, pw)
        # from host memory gives the same device array
        with DeviceTokens.from_array(toks) as d2:
            assert k.forward_loss_windows(d2, pos) == want


def test_windows_reject_bad_windows_and_ids(tmp_path):
    cfg = _cfg()
    path, toks = _token_file(tmp_path, cfg, 5000, 2)
    bad = toks.copy()
    bad[100] = cfg.vocab  # out of range id inside the second window
    with CompiledKernels(cfg, 0, 2) as k, DeviceTokens.open(path) as data, \
            DeviceTokens.from_array(bad) as bad_data:
        k.init_weights(0, B.CB_INIT_NORMAL, 0.02)
        ok = k.forward_loss_windows(data, [0])
        with pytest.raises(CudaBridgeError) as e:
            k.forward_loss_windows(data, [5000 - cfg.seq])  # target runs past the end
        assert e.value.status == B.CB_ERR_INVALID_ARG
        with pytest.raises(CudaBridgeError) as e:
            k.forward_loss_windows(data, [0, 0, 0])  # more windows than max_batch
        assert e.value.status == B.CB_ERR_INVALID_ARG
        with pytest.raises(CudaBridgeError) as e:
            k.forward_loss_windows(bad_data, [0, 64])
        assert e.value.status == B.CB_ERR_INVALID_ARG
        assert k.forward_loss_windows(data, [0]) == ok  # the context stays usable


def test_tokens_open_errors(tmp_path):
    with pytest.raises(CudaBridgeError):
        DeviceTokens.open(tmp_path / "missing.bin")
    with pytest.raises(CudaBridgeError):
        DeviceTokens.open(tmp_path, device=0)  # a directory
    p = tmp_path / "odd.bin"
    p.write_bytes(b"\x01\x00\x02")
    with DeviceTokens.open(p) as d:
        assert len(d) == 1


def test_validate_matches_host_loop_and_oracle_bpb(tmp_path):
    cfg = _cfg()
    path, toks = _token_file(tmp_path, cfg, 30_000, 3)
    rng = np.random.default_rng(4)
    table = rng.integers(1, 5, cfg.vocab).astype(np.int32)
    table[:50] = 0  # special tokens
    tb = TokenBytes(table)
    steps = 7  # max_batch 3: forwards of 3, 3 and 1 windows
    w = ModelWeights.normal(cfg, seed=6, sigma=0.05)
    with CompiledKernels(cfg, 0, 3) as k, DeviceTokens.open(path) as data:
        val_loss, val_bpb = validate(cfg, k, w, data, tb, steps)
        # host loop of train.rs:205-233: one window per forward, per-token losses back
        losses, targets = [], []
        for p in validation_positions(len(toks), cfg.seq, 0, steps):
            inp = toks[p:p + cfg.seq].astype(np.uint32)
            tgt = toks[p + 1:p + 1 + cfg.seq].astype(np.uint32)
            losses.append(k.forward_loss(inp, tgt, per_token=True)[1])
            targets.append(tgt)
        tot = k.eval_windows(data, tb, 0, steps)
        no_bytes = validate(cfg, k, w, data, None, steps)
    losses, targets = np.concatenate(losses), np.concatenate(targets)
    want_bpb, want_nats, want_bytes = R.compute_bpb(losses.tolist(), targets.tolist(),
                                                    table.tolist())
    assert tot["bytes"] == want_bytes and tot["tokens"] == steps * cfg.seq
    assert abs(tot["nats"] - want_nats) / want_nats < 1e-5
    assert abs(val_bpb - want_bpb) / want_bpb < 1e-5
    assert abs(val_loss - float(np.mean(losses, dtype=np.float64))) < 1e-5
    assert no_bytes == (val_loss, 0.0)


def test_validate_loss_matches_oracle():
    cfg = custom_config(256, 512, 2, 2, 128, 1024)
    rng = np.random.default_rng(9)
    toks = rng.integers(0, cfg.vocab, 3 * cfg.seq).astype(np.uint16)
    ora = OracleModel(cfg, seed=1, scheme=SCHEME_NORMAL, sigma=0.05)
    steps = 3
    want = []
    for inp, tgt in R.validation_windows(toks.tolist(), cfg.seq, steps):
        want.append(ora.forward(np.array(inp, np.uint32), np.array(tgt, np.uint32))[0])
    with CompiledKernels(cfg, 0, 2) as k, DeviceTokens.from_array(toks) as data:
        val_loss, _ = validate(cfg, k, ModelWeights.normal(cfg, seed=1, sigma=0.05), data, None,
                               steps)
    assert abs(val_loss - np.mean(want)) / np.mean(want) <= 1e-3
