"""GPU test of the sequence-parallel forward workers (ForwardScheduler, the
reference's multistream.rs:54-161): worker contexts on their own host threads pull
whole sequences, with no communication between them."""
import numpy as np
import pytest

from rustane_b200 import CompiledKernels, ForwardScheduler, ModelWeights
from rustane_b200.model import custom_config

pytestmark = pytest.mark.gpu


def _tokens(cfg, seed):
    rng = np.random.default_rng(seed)
    return (rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32),
            rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32))


def test_forward_scheduler_returns_losses_in_request_order(bridge_lib):
    """Two worker contexts (both on GPU 0 here; one per GPU in a multi-GPU job): every
    loss comes back in request order and equals one context's forward of that
    sequence."""
    cfg = custom_config(256, 512, 2, 2, 128)
    w = ModelWeights.normal(cfg, seed=13, sigma=0.05)
    reqs = [_tokens(cfg, 40 + i) for i in range(5)]
    with CompiledKernels(cfg, 0, 1) as k:
        k.load_weights(w)
        want = [k.forward_loss(t, g) for t, g in reqs]
    sched = ForwardScheduler(cfg, w, devices=[0, 0])
    try:
        got = sched.run_batch(reqs)
    finally:
        sched.close()
    assert len(set(round(x, 6) for x in want)) == len(want)  # distinct sequences
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-6)
