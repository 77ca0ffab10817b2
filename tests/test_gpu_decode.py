"""GPU tests of single-token decode with a KV cache (cb_prefill / cb_decode_step)
against the CPU oracle's forward logits at the same positions (a decode step for the
token at position p yields the logits the full causal forward has at row p). Tolerance:
the forward's 2e-2 max-abs on logits."""
import numpy as np
import pytest

from oracle.oracle import OracleModel, SCHEME_NORMAL
from rustane_b200 import CB_INIT_NORMAL, CompiledKernels, CudaBridgeError
from rustane_b200 import bridge as B
from rustane_b200.model import custom_config

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-2


def _oracle_logits(cfg, seqs, rows_per_seq, seed, sigma, softcap):
    """Oracle logits [batch, len(rows), vocab] at the given positions of each sequence."""
    batch = seqs.shape[0]
    tok = np.zeros((batch, cfg.seq), np.uint32)
    tok[:, :seqs.shape[1]] = seqs
    rows = [b * cfg.seq + r for b in range(batch) for r in rows_per_seq]
    ora = OracleModel(cfg, seed=seed, scheme=SCHEME_NORMAL, sigma=sigma)
    _, _, z = ora.forward(tok.reshape(-1), np.zeros(batch * cfg.seq, np.uint32), softcap,
                          sample_rows=rows)
    return z.reshape(batch, len(rows_per_seq), cfg.vocab)


@pytest.mark.parametrize("kv_heads,softcap", [(2, 0.0), (1, 10.0)])
def test_decode_matches_oracle_forward(bridge_lib, kv_heads, softcap):
    cfg = custom_config(256, 512, 2, 2, 128, 512).replace(kv_heads=kv_heads)
    seed, sigma = 4, 0.05
    rng = np.random.default_rng(1)
    batch, plen, steps = 3, 37, 20
    seqs = rng.integers(0, cfg.vocab, (batch, plen + steps)).astype(np.uint32)
    want = _oracle_logits(cfg, seqs, list(range(plen - 1, plen + steps)), seed, sigma, softcap)
    with CompiledKernels(cfg, 0, 4) as k:
        k.init_weights(seed, CB_INIT_NORMAL, sigma)
        first = k.prefill(seqs[:, :plen], softcap)
        assert k.decode_position() == plen
        got = [first]
        for j in range(steps):
            logits, nxt = k.decode_step(seqs[:, plen + j])
            assert np.array_equal(nxt, logits.argmax(axis=1))
            got.append(logits)
        assert k.decode_position() == plen + steps
    got = np.stack(got, axis=1)
    assert np.max(np.abs(got - want)) <= LOGIT_ATOL, np.max(np.abs(got - want))


def test_decode_to_the_end_of_the_window(bridge_lib):
    """Prefill of seq - 4 tokens, then the last 4 positions; a further step is refused."""
    cfg = custom_config(256, 512, 2, 1, 128, 256)
    rng = np.random.default_rng(2)
    seqs = rng.integers(0, cfg.vocab, (2, cfg.seq)).astype(np.uint32)
    want = _oracle_logits(cfg, seqs, list(range(cfg.seq - 5, cfg.seq)), 3, 0.05, 0.0)
    with CompiledKernels(cfg, 0, 2) as k:
        k.init_weights(3, CB_INIT_NORMAL, 0.05)
        got = [k.prefill(seqs[:, :cfg.seq - 4])]
        for p in range(cfg.seq - 4, cfg.seq):
            got.append(k.decode_step(seqs[:, p])[0])
        with pytest.raises(CudaBridgeError) as e:
            k.decode_step(seqs[:, 0])
        assert e.value.status == B.CB_ERR_INVALID_ARG
    assert np.max(np.abs(np.stack(got, 1) - want)) <= LOGIT_ATOL


def test_greedy_generation_is_consistent(bridge_lib):
    """generate() feeds back its own argmax: re-running the oracle forward over the
    generated sequence gives the same argmax at every generated position."""
    cfg = custom_config(256, 512, 2, 2, 128, 512)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, cfg.vocab, (2, 16)).astype(np.uint32)
    with CompiledKernels(cfg, 0, 2) as k:
        k.init_weights(6, CB_INIT_NORMAL, 0.05)
        gen = k.generate(prompt, 12)
    full = np.concatenate([prompt, gen], axis=1)
    z = _oracle_logits(cfg, full, list(range(15, 15 + 12)), 6, 0.05, 0.0)
    top2 = np.sort(z, axis=2)[..., -2:]
    confident = (top2[..., 1] - top2[..., 0]) > 2 * LOGIT_ATOL  # skip near-ties
    assert np.array_equal(z.argmax(axis=2)[confident], gen[confident])


def test_decode_errors(bridge_lib):
    cfg = custom_config(256, 512, 2, 1, 128, 256)
    with CompiledKernels(cfg, 0, 2) as k:
        k.init_weights(0, CB_INIT_NORMAL, 0.02)
        with pytest.raises(CudaBridgeError) as e:
            k.decode_step([1, 2])
        assert e.value.status == B.CB_ERR_NOT_READY
        k.prefill(np.ones((2, 10), np.uint32))
        with pytest.raises(CudaBridgeError) as e:
            k.decode_step([1, 2, 3])  # batch differs from the prefill
        assert e.value.status == B.CB_ERR_INVALID_ARG
        with pytest.raises(CudaBridgeError) as e:
            k.decode_step([1, cfg.vocab])
        assert e.value.status == B.CB_ERR_INVALID_ARG
        with pytest.raises(CudaBridgeError):
            k.prefill(np.ones((2, cfg.seq + 1), np.uint32))
        logits, _ = k.decode_step([1, 2])  # still usable
        assert np.isfinite(logits).all()


def test_decode_bench_width_64_sequences_matches_oracle(bridge_lib):
    """The decode bench's GEMM shapes (600m-A width: d 1536, hidden 4096, 12 heads,
    vocab 8192, 64 sequences: the split-K counts and element-wise kernels the bench
    runs), two layers and a 128-token window."""
    cfg = custom_config(1536, 4096, 12, 2, 128, 8192)
    seed, sigma = 8, 0.02
    rng = np.random.default_rng(9)
    batch, plen, steps = 64, 29, 3
    seqs = rng.integers(0, cfg.vocab, (batch, plen + steps)).astype(np.uint32)
    want = _oracle_logits(cfg, seqs, list(range(plen, plen + steps)), seed, sigma, 0.0)
    with CompiledKernels(cfg, 0, batch) as k:
        k.init_weights(seed, CB_INIT_NORMAL, sigma)
        k.prefill(seqs[:, :plen], 0.0)
        got = []
        for j in range(steps):
            logits, nxt = k.decode_step(seqs[:, plen + j])
            assert np.array_equal(nxt, logits.argmax(axis=1))
            got.append(logits)
    got = np.stack(got, axis=1)
    assert np.max(np.abs(got - want)) <= LOGIT_ATOL, np.max(np.abs(got - want))
