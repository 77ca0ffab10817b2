"""GPU parity at the exact shapes bench.py times, through the public API.

Tile modes (CTA pair, 128 x 256 or 128 x 128 tiles, K splits) and the fused
residual/norm epilogues are chosen per GEMM from the token count, so the 64-sequence
600m-A forward, the 8-sequence 7B / 13B forwards and the 16 x 2048 ~32B forward each
run a graph that the batch-1 parity tests never build. Here the GPU runs the whole
batch in one call; the CPU oracle runs only a few of its sequences (sequences are
independent), and those sequences' per-token losses and sampled logits are compared.

Tolerances (the target spec's): the mean loss of the checked sequences within 1e-3
relative; logits at sampled positions within 2e-2 max-abs; every per-token loss of
the checked sequences within 5e-2 (as in test_gpu_forward.py)."""
import numpy as np
import pytest

from oracle.oracle import OracleModel, SCHEME_NORMAL
from rustane_b200 import CB_INIT_NORMAL, CompiledKernels
from rustane_b200.model import CONFIGS
from rustane_b200.sharding import global_tokens

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-3
LOGIT_ATOL = 2e-2
PTL_ATOL = 5e-2


def _check_sequences(cfg, batch, seqs, seed=0, n_rows_per_seq=3):
    # the bench's own token generator (bench.py: global_tokens(vocab, seq, batch, seed))
    tok, tgt = global_tokens(cfg.vocab, cfg.seq, batch, seed)
    S = cfg.seq
    local_rows = np.linspace(0, S - 1, n_rows_per_seq).astype(np.int32)
    gpu_rows = np.concatenate([b * S + local_rows for b in seqs]).astype(np.int32)
    with CompiledKernels(cfg, 0, batch) as k:
        k.init_weights(seed, CB_INIT_NORMAL, 0.02)
        loss_all, ptl = k.forward_loss(tok, tgt, per_token=True)
        z = k.sampled_logits(gpu_rows)
    assert np.isfinite(loss_all)
    assert abs(float(np.mean(ptl)) - loss_all) <= 1e-5 * loss_all
    sel = np.concatenate([np.arange(b * S, (b + 1) * S) for b in seqs])
    ora_rows = np.concatenate([i * S + local_rows for i in range(len(seqs))]).astype(np.int32)
    ora = OracleModel(cfg, seed=seed, scheme=SCHEME_NORMAL, sigma=0.02)
    l_ref, p_ref, z_ref = ora.forward(tok[sel], tgt[sel], 0.0, sample_rows=ora_rows)
    l_gpu = float(np.mean(ptl[sel]))
    assert abs(l_gpu - l_ref) / abs(l_ref) <= LOSS_RTOL, (l_gpu, l_ref)
    assert float(np.max(np.abs(ptl[sel] - p_ref))) <= PTL_ATOL
    dz = float(np.max(np.abs(z - z_ref)))
    assert dz <= LOGIT_ATOL, dz
    return l_gpu, l_ref, dz


def test_600m_bench_batch_64(bridge_lib):
    """BASELINE config 1 on one GPU: 64 sequences in one forward (the bench's graph)."""
    _check_sequences(CONFIGS["600m-A"], 64, [0, 31, 63])


@pytest.mark.parametrize("per_gpu", [8, 16, 32])
def test_600m_bench_shard_batches(bridge_lib, per_gpu):
    """The per-GPU shares of the 2-, 4- and 8-GPU scaling runs (64 / N sequences)."""
    _check_sequences(CONFIGS["600m-A"], per_gpu, [0, per_gpu - 1])


@pytest.mark.parametrize("name", ["7B", "13B"])
def test_large_config_bench_batch_8(bridge_lib, name):
    """BASELINE configs 2 and 3 at their benchmark batch of 8, two layers (every layer
    takes the same tile modes, so depth does not change the graph's kernels)."""
    _check_sequences(CONFIGS[name].replace(nlayers=2), 8, [0, 7])


def test_32b_bench_shape_one_layer(bridge_lib):
    """BASELINE config 4's single-GPU shape: 16 sequences of 2048 tokens, one layer; the
    oracle checks the last sequence (its attention spans all 2048 keys)."""
    _check_sequences(CONFIGS["32B"].replace(nlayers=1), 16, [15], n_rows_per_seq=4)
