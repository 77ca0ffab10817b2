"""The bounded device waits, made to expire on purpose in an allowed form.

Every mbarrier wait of the pipeline kernels gives up after a time limit, records
DEV_ERR_WAIT_TIMEOUT in the context's device error flag, frees its TMEM and returns;
the host then reports CB_ERR_DEVICE_TIMEOUT. cb_selftest_wait_timeout runs a miniature
of those kernels whose producer never produces (a barrier nothing arrives on) with a
short limit, so the expiry path runs without any fault, trap or hang. Afterwards the
same context must still run a forward that matches the CPU oracle."""
import time

import numpy as np
import pytest

from oracle.oracle import OracleModel, SCHEME_NORMAL
from rustane_b200 import CB_INIT_NORMAL, CompiledKernels
from rustane_b200 import bridge as B
from rustane_b200.model import custom_config

pytestmark = pytest.mark.gpu


def test_expired_wait_is_reported_and_the_context_recovers(bridge_lib):
    cfg = custom_config(256, 512, 2, 2, 128, 1024)
    rng = np.random.default_rng(31)
    tok = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    ref = OracleModel(cfg, seed=3, scheme=SCHEME_NORMAL, sigma=0.05).forward(tok, tgt)[0]
    with CompiledKernels(cfg, 0, 2) as k:
        k.init_weights(3, CB_INIT_NORMAL, 0.05)
        before = k.forward_loss(tok, tgt)
        for limit_us in (1000, 20000):  # twice: the flag is cleared after each report
            t0 = time.perf_counter()
            rc = k.selftest_wait_timeout(limit_us)
            dt = time.perf_counter() - t0
            assert rc == B.CB_ERR_DEVICE_TIMEOUT, rc
            assert b"expired" in bridge_lib.cb_last_error(k.handle)
            # the short limit, not the kernels' 2 s one, ended the wait
            assert limit_us * 1e-6 <= dt < 1.0, dt
        k.check_device_error()  # nothing left in the flag
        after = k.forward_loss(tok, tgt)
    assert after == before
    assert abs(after - ref) / ref <= 1e-3


def test_selftest_rejects_limits_out_of_range(bridge_lib):
    cfg = custom_config(256, 512, 2, 1, 128, 1024)
    with CompiledKernels(cfg, 0, 1) as k:
        assert k.selftest_wait_timeout(0) == B.CB_ERR_INVALID_ARG
        assert k.selftest_wait_timeout(2_000_001) == B.CB_ERR_INVALID_ARG
