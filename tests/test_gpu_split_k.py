"""Split-K with the last-arrival reduction (SplitFix in gemm_tc.cuh) on the fused forward.

A GEMM with too few tiles to fill the GPU splits K: every split writes its fp32 partial,
and the tile's last split to arrive adds all partials in split order and runs the fused
epilogue (RoPE, SwiGLU, residual + RMSNorm, cross-entropy). The plans are forced here
through CB_GEMM_PLAN (read whenever a forward is planned, so each new context picks it
up), covering every fused epilogue under 1-CTA 128- and 256-wide tiles and CTA pairs,
with up to 8 splits. Each plan must match the CPU oracle with the parity tolerances
(loss 1e-3 relative, sampled logits 2e-2) and give the same bits on every call."""
import os

import numpy as np
import pytest

from oracle.oracle import OracleModel, SCHEME_NORMAL
from rustane_b200 import CB_INIT_NORMAL, CompiledKernels
from rustane_b200.model import CONFIGS, custom_config

pytestmark = pytest.mark.gpu

PLANS = [
    "qkv=128x3,o=128x2,w13=pairx2,down=128x4,head=pairx3",
    "qkv=pairx2,o=pairx4,w13=128x5,down=pairx2,head=128x2",
    "qkv=256x8,o=128x8,w13=256x4,down=128x8,head=256x8",
]


@pytest.fixture
def plan_env():
    old = os.environ.get("CB_GEMM_PLAN")
    yield
    if old is None:
        os.environ.pop("CB_GEMM_PLAN", None)
    else:
        os.environ["CB_GEMM_PLAN"] = old


def _tokens(cfg, batch, seed):
    rng = np.random.default_rng(seed)
    return (rng.integers(0, cfg.vocab, batch * cfg.seq).astype(np.uint32),
            rng.integers(0, cfg.vocab, batch * cfg.seq).astype(np.uint32))


@pytest.mark.parametrize("plan", PLANS)
def test_forced_split_plans_match_oracle(bridge_lib, plan_env, plan):
    cfg = custom_config(512, 1024, 4, 2, 256, 2048).replace(kv_heads=2)
    tok, tgt = _tokens(cfg, 3, 41)
    rows = np.array([0, 255, 256, 700], np.int32)
    l_ref, p_ref, z_ref = OracleModel(cfg, seed=8, scheme=SCHEME_NORMAL, sigma=0.05).forward(
        tok, tgt, 0.0, sample_rows=rows)
    os.environ["CB_GEMM_PLAN"] = plan
    with CompiledKernels(cfg, 0, 3) as k:
        k.init_weights(8, CB_INIT_NORMAL, 0.05)
        l1, p1 = k.forward_loss(tok, tgt, per_token=True)
        z = k.sampled_logits(rows)
        l2, p2 = k.forward_loss(tok, tgt, per_token=True)
        k.set_profiling(True)  # the eager path plans the same way
        l3 = k.forward_loss(tok, tgt)
    assert l1 == l2 == l3 and np.array_equal(p1, p2)
    assert abs(l1 - l_ref) / l_ref <= 1e-3, (l1, l_ref)
    assert float(np.max(np.abs(z - z_ref))) <= 2e-2
    assert float(np.max(np.abs(p1 - p_ref))) <= 5e-2


def test_600m_batch1_split_plan_matches_oracle(bridge_lib, plan_env):
    """BASELINE config 0's shape (one 512-token sequence, all 20 layers) with every
    fused GEMM split (a plan the planner may pick for few tokens)."""
    cfg = CONFIGS["600m-A"]
    tok, tgt = _tokens(cfg, 1, 42)
    rows = np.array([0, 311, 511], np.int32)
    l_ref, _, z_ref = OracleModel(cfg, seed=0, scheme=SCHEME_NORMAL, sigma=0.02).forward(
        tok, tgt, 0.0, sample_rows=rows)
    os.environ["CB_GEMM_PLAN"] = "qkv=128x2,o=128x4,w13=pairx2,down=128x6,head=pairx2"
    with CompiledKernels(cfg, 0, 1) as k:
        k.init_weights(0, CB_INIT_NORMAL, 0.02)
        loss = k.forward_loss(tok, tgt)
        z = k.sampled_logits(rows)
        assert k.forward_loss(tok, tgt) == loss
    assert abs(loss - l_ref) / l_ref <= 1e-3, (loss, l_ref)
    assert float(np.max(np.abs(z - z_ref))) <= 2e-2
