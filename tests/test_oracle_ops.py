"""The reference's CPU-op unit tests, run against the oracle's own single ops (the
functions its forward and backward use): cpu/embedding.rs:47-95, cpu/rmsnorm.rs:241-400,
cpu/silu.rs:48-110, cpu/cross_entropy.rs:98-156 and the GEMM of cpu/vdsp.rs:354-376.
Same inputs and bounds as the reference's tests; the reference's channel-first layout
checks become token-major row checks."""
import numpy as np
import pytest

from oracle import oracle as orc

EPS = 1e-5  # cpu/rmsnorm.rs:10


# ---- embedding (cpu/embedding.rs tests)

def test_embedding_forward_lookup(oracle_lib):
    table = np.array([[1, 2], [3, 4], [5, 6]], np.float32)
    out = orc.op_embedding(table, [2, 0, 1])
    np.testing.assert_array_equal(out.reshape(-1), [5, 6, 1, 2, 3, 4])


def test_embedding_backward_scatter_add(oracle_lib):
    d_out = np.array([[0.1, 0.2], [0.3, 0.4], [0.5, 0.6]], np.float32)
    d_table = orc.op_embedding_backward(d_out, [1, 1, 2], vocab=3)
    np.testing.assert_array_equal(d_table[0], [0, 0])
    np.testing.assert_allclose(d_table[1], [0.4, 0.6], atol=1e-6)
    np.testing.assert_allclose(d_table[2], [0.5, 0.6], atol=1e-6)


def test_embedding_roundtrip_identity(oracle_lib):
    table = np.array([[10, 20], [30, 40]], np.float32)
    np.testing.assert_array_equal(orc.op_embedding(table, [0, 1]), table)


def test_embedding_rejects_out_of_range_id(oracle_lib):
    with pytest.raises(ValueError):
        orc.op_embedding(np.zeros((3, 2), np.float32), [3])


# ---- RMSNorm (cpu/rmsnorm.rs tests)

def test_rmsnorm_forward_unit_gamma(oracle_lib):
    out, rinv = orc.op_rmsnorm([3.0, 4.0], [1.0, 1.0])
    rms = np.sqrt(np.float32(12.5) + np.float32(EPS))
    assert abs(rinv[0] - 1 / rms) < 1e-5
    np.testing.assert_allclose(out[0], [3 / rms, 4 / rms], atol=1e-5)


def test_rmsnorm_forward_with_gamma(oracle_lib):
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    out, rinv = orc.op_rmsnorm(x, [0.5] * 4)
    expect_rinv = 1 / np.sqrt(7.5 + EPS)
    assert abs(rinv[0] - expect_rinv) < 1e-5
    np.testing.assert_allclose(out[0], x * expect_rinv * 0.5, atol=1e-5)


def test_rmsnorm_backward_numerical_gradient(oracle_lib):
    x = np.array([1.0, -2.0, 3.0, -0.5], np.float32)
    gamma = np.array([1.0, 0.5, 2.0, 1.5], np.float32)
    dy = np.ones(4, np.float32)
    _, rinv = orc.op_rmsnorm(x, gamma)
    dx, _ = orc.op_rmsnorm_backward(dy, x, gamma, rinv)
    h = 1e-4
    for i in range(4):
        xp, xm = x.copy(), x.copy()
        xp[i] += h
        xm[i] -= h
        num = (orc.op_rmsnorm(xp, gamma)[0].sum() - orc.op_rmsnorm(xm, gamma)[0].sum()) / (2 * h)
        assert abs(dx[0, i] - num) < 1e-2, (i, dx[0, i], num)


def _ref_pattern(n, mul, add):
    """The reference's deterministic test inputs: ((i * mul + add) % 100) * 0.01 - 0.5."""
    return np.array([((i * mul + add) % 100) * 0.01 - 0.5 for i in range(n)], np.float32)


def test_rmsnorm_rows_match_single_rows(oracle_lib):
    """channel_first_matches_batch: a [seq, dim] batch gives each row's own result."""
    dim, seq = 4, 3
    gamma = np.array([1.5, 0.5, 2.0, 0.8], np.float32)
    x = _ref_pattern(dim * seq, 17, 3).reshape(dim, seq).T.copy()  # channel-first -> rows
    out, rinv = orc.op_rmsnorm(x, gamma)
    for s in range(seq):
        o1, r1 = orc.op_rmsnorm(x[s], gamma)
        assert abs(rinv[s] - r1[0]) < 1e-5
        np.testing.assert_allclose(out[s], o1[0], atol=1e-5)


def test_rmsnorm_backward_rows_match_single_rows(oracle_lib):
    """channel_first_backward_matches_batch: dx per row, dgamma summed over rows."""
    dim, seq = 4, 3
    gamma = np.array([1.5, 0.5, 2.0, 0.8], np.float32)
    x = _ref_pattern(dim * seq, 17, 3).reshape(dim, seq).T.copy()
    dy = _ref_pattern(dim * seq, 13, 7).reshape(dim, seq).T.copy()
    _, rinv = orc.op_rmsnorm(x, gamma)
    dx, dgamma = orc.op_rmsnorm_backward(dy, x, gamma, rinv)
    dg_sum = np.zeros(dim, np.float32)
    for s in range(seq):
        dx1, dg1 = orc.op_rmsnorm_backward(dy[s], x[s], gamma, rinv[s:s + 1])
        np.testing.assert_allclose(dx[s], dx1[0], atol=1e-5)
        dg_sum += dg1
    np.testing.assert_allclose(dgamma, dg_sum, atol=1e-5)


# ---- SiLU (cpu/silu.rs tests); silu(x) = silu_gate(x, 1)

def test_silu_forward_zero(oracle_lib):
    assert abs(orc.op_silu_gate([0.0], [1.0])[0]) < 1e-6


def test_silu_forward_positive(oracle_lib):
    sig = 1 / (1 + np.exp(np.float32(-2.0)))
    assert abs(orc.op_silu_gate([2.0], [1.0])[0] - 2 * sig) < 1e-6


def test_silu_backward_numerical(oracle_lib):
    x = np.array([-1.0, 0.0, 0.5, 2.0], np.float32)
    one = np.ones(4, np.float32)
    dx, _ = orc.op_silu_gate_backward(one, x, one)
    h = 1e-4
    num = (orc.op_silu_gate(x + h, one) - orc.op_silu_gate(x - h, one)) / (2 * h)
    np.testing.assert_allclose(dx, num, atol=1e-3)


def test_silu_gate_matches_manual(oracle_lib):
    gate, up = np.array([1.0, 2.0], np.float32), np.array([3.0, 4.0], np.float32)
    silu = orc.op_silu_gate(gate, np.ones(2, np.float32))
    np.testing.assert_allclose(orc.op_silu_gate(gate, up), silu * up, atol=1e-6)


def test_silu_gate_backward_up_is_silu(oracle_lib):
    gate = np.array([-3.0, -0.25, 0.75, 4.0], np.float32)
    up = np.array([0.5, -2.0, 1.5, 3.0], np.float32)
    dout = np.array([1.0, -1.0, 0.5, 2.0], np.float32)
    dgate, dup = orc.op_silu_gate_backward(dout, gate, up)
    np.testing.assert_allclose(dup, dout * orc.op_silu_gate(gate, np.ones(4, np.float32)),
                               atol=1e-6)
    h = 1e-3
    num = (orc.op_silu_gate(gate + h, up) - orc.op_silu_gate(gate - h, up)) / (2 * h) * dout
    np.testing.assert_allclose(dgate, num, atol=2e-3)


# ---- cross-entropy (cpu/cross_entropy.rs tests)

def test_ce_loss_is_positive(oracle_lib):
    loss, _ = orc.op_cross_entropy([1.0, 2.0, 3.0, 4.0], [3], grad=False)
    assert 0 < loss[0] < 2


def test_ce_loss_decreases_with_confidence(oracle_lib):
    low, _ = orc.op_cross_entropy([1.0, 1.0, 1.0, 1.0], [3], grad=False)
    high, _ = orc.op_cross_entropy([0.0, 0.0, 0.0, 10.0], [3], grad=False)
    assert high[0] < low[0]


def test_ce_gradients_sum_to_zero(oracle_lib):
    _, dl = orc.op_cross_entropy([1.0, 2.0, 3.0], [1])
    assert abs(dl.sum()) < 1e-5


@pytest.mark.parametrize("softcap", [0.0, 2.5])
def test_ce_numerical_gradient(oracle_lib, softcap):
    logits = np.array([2.0, -1.0, 0.5, 1.5], np.float32)
    _, dl = orc.op_cross_entropy(logits, [2], softcap=softcap)
    h = 1e-3
    for i in range(4):
        p, m = logits.copy(), logits.copy()
        p[i] += h
        m[i] -= h
        lp, _ = orc.op_cross_entropy(p, [2], softcap=softcap, grad=False)
        lm, _ = orc.op_cross_entropy(m, [2], softcap=softcap, grad=False)
        assert abs(dl[0, i] - (lp[0] - lm[0]) / (2 * h)) < 5e-3


def test_ce_batch_scale_and_known_value(oracle_lib):
    """forward_backward_batch: per-row losses, gradients scaled by inv_seq."""
    rng = np.random.default_rng(0)
    z = rng.standard_normal((5, 64)).astype(np.float32) * 3
    t = rng.integers(0, 64, 5)
    loss, dl = orc.op_cross_entropy(z, t, scale=1 / 5)
    z64 = z.astype(np.float64)
    lse = np.log(np.exp(z64 - z64.max(1, keepdims=True)).sum(1)) + z64.max(1)
    np.testing.assert_allclose(loss, lse - z64[np.arange(5), t], rtol=1e-6)
    sm = np.exp(z64 - lse[:, None])
    sm[np.arange(5), t] -= 1
    np.testing.assert_allclose(dl, sm / 5, atol=1e-7)


# ---- the oracle's GEMM (the LM head's sgemm_at form is b_trans)

@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (7, 33, 19), (50, 130, 300), (97, 16, 513)])
@pytest.mark.parametrize("b_trans", [False, True])
def test_sgemm_matches_numpy(oracle_lib, M, N, K, b_trans):
    rng = np.random.default_rng(M * 1000 + N + K)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((N, K) if b_trans else (K, N)).astype(np.float32)
    want = a.astype(np.float64) @ (b.T if b_trans else b).astype(np.float64)
    np.testing.assert_allclose(orc.op_sgemm(a, b, b_trans), want, rtol=1e-4,
                               atol=1e-4 * np.sqrt(K))
