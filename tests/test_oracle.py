"""CPU tests of the oracle: pinned against the reference's published losses,
cross-checked against an independent torch float64 forward, and its shared
weight generator checked bit-for-bit."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import torch_ref
from oracle.oracle import (OracleModel, SCHEME_NORMAL, SCHEME_REFERENCE, lib, reference_tokens)
from rustane_b200.model import custom_config

GOLDEN = Path(__file__).with_name("golden") / "reference_kat.json"


def _kat_entries():
    seen, out = set(), []
    for e in json.loads(GOLDEN.read_text()):
        key = (e["dim"], e["hidden"], e["heads"], e["seq"])
        if key in seen:
            continue
        seen.add(key)
        out.append(e)
    return out


@pytest.mark.parametrize("e", _kat_entries(), ids=lambda e: e["name"])
def test_reference_init_known_answer(oracle_lib, e):
    """Reference init zeroes Wo/W2, so every layer is an identity and one layer
    stands for all of them; the loss must match the published value (the
    reference returned x_next through fp16 on the ANE: allow 1e-4)."""
    cfg = custom_config(e["dim"], e["hidden"], e["heads"], 1, e["seq"], e["vocab"])
    m = OracleModel(cfg, scheme=SCHEME_REFERENCE)
    tok, tgt = reference_tokens(cfg.seq, cfg.vocab)
    loss, ptl, _ = m.forward(tok, tgt)
    assert abs(loss - e["loss"]) <= 1e-4, (loss, e["loss"])
    assert np.all(ptl > 0)


def test_reference_init_layers_are_identity(oracle_lib):
    cfg1 = custom_config(256, 512, 2, 1, 128, 1024)
    cfg3 = cfg1.replace(nlayers=3)
    tok, tgt = reference_tokens(128, 1024)
    l1 = OracleModel(cfg1, scheme=SCHEME_REFERENCE).forward(tok, tgt)[0]
    l3 = OracleModel(cfg3, scheme=SCHEME_REFERENCE).forward(tok, tgt)[0]
    assert l1 == l3


def test_lcg_matches_reference_recurrence(oracle_lib):
    """The jump-ahead LCG equals the sequential recurrence of random_vec
    (full_model.rs:1473-1484): seed = 42 + n, step before each element."""
    L = lib()
    n = 1000
    s = (42 + n) & (2**64 - 1)
    a, c = 6364136223846793005, 1442695040888963407
    scale = np.float32(0.005)
    for i in range(300):
        s = (s * a + c) & (2**64 - 1)
        assert L.orc_lcg_jump(42 + n, i + 1) == s
        hi = np.float32(s >> 32)
        r = np.float32(np.float32(hi / np.float32(4294967295.0)) * np.float32(2.0)) - np.float32(1.0)
        expect = np.float32(r * scale)
        assert L.orc_lcg_value(s, 0.005) == expect


def test_f16_conversion_matches_ieee(oracle_lib):
    L = lib()
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(2000).astype(np.float32) * 0.02,
        rng.standard_normal(500).astype(np.float32) * 1e-5,       # subnormal halves
        rng.standard_normal(500).astype(np.float32) * 3e4,        # near overflow
        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e-8, 2.0**-25, 2.0**-24,
                  3 * 2.0**-26, np.inf, -np.inf], np.float32),
    ])
    with np.errstate(over="ignore"):  # values past the fp16 range round to inf on purpose
        for v in vals:
            bits = L.orc_f32_to_f16_bits(float(v))
            assert bits == int(np.float16(v).view(np.uint16)), v
            assert L.orc_f16_bits_to_f32(bits) == np.float32(np.float16(v))


def test_normal_init_statistics(oracle_lib):
    cfg = custom_config(256, 512, 2, 1, 64, 1024)
    m = OracleModel(cfg, seed=7, scheme=SCHEME_NORMAL, sigma=0.02)
    w = m.layers[0]["w1"]
    assert abs(float(w.mean())) < 1e-3
    assert abs(float(w.std()) - 0.02) < 1e-3
    # values are exactly fp16-representable
    assert np.array_equal(w, w.astype(np.float16).astype(np.float32))
    m2 = OracleModel(cfg, seed=8, scheme=SCHEME_NORMAL, sigma=0.02)
    assert not np.array_equal(m.embed, m2.embed)


def _torch_forward64(m: OracleModel, tokens, targets, softcap=0.0):
    """Independent float64 restatement (torch) of the same forward."""
    return torch_ref.forward(m, tokens, targets, softcap, dtype=torch.float64)


def test_torch_fp32_fused_attention_matches_float64(oracle_lib):
    """The bench's torch-CPU figure (float32, fused causal attention) computes the
    same forward."""
    cfg = custom_config(256, 512, 2, 2, 64, 512)
    m = OracleModel(cfg, seed=5, scheme=SCHEME_NORMAL, sigma=0.05)
    rng = np.random.default_rng(3)
    tok = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
    l64, p64, _ = _torch_forward64(m, tok, tgt)
    l32, p32, _ = torch_ref.forward(m, tok, tgt, dtype=torch.float32, fused_attention=True)
    assert abs(l32 - l64) / l64 < 1e-5
    np.testing.assert_allclose(p32, p64, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("softcap", [0.0, 15.0])
def test_oracle_matches_float64_torch(oracle_lib, softcap):
    cfg = custom_config(256, 512, 2, 2, 64, 512)
    m = OracleModel(cfg, seed=3, scheme=SCHEME_NORMAL, sigma=0.05)
    rng = np.random.default_rng(1)
    tok = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    rows = [0, 5, 63, 64, 127]
    loss, ptl, samp = m.forward(tok, tgt, softcap, sample_rows=rows)
    l64, p64, z64 = _torch_forward64(m, tok, tgt, softcap)
    assert abs(loss - l64) / l64 < 1e-5
    np.testing.assert_allclose(ptl, p64, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(samp, z64[rows], rtol=1e-4, atol=1e-4)


def test_oracle_gqa_matches_float64_torch(oracle_lib):
    cfg = custom_config(256, 512, 4, 1, 64, 512).replace(kv_heads=2)
    m = OracleModel(cfg, seed=4, scheme=SCHEME_NORMAL, sigma=0.05)
    rng = np.random.default_rng(2)
    tok = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
    loss, _, _ = m.forward(tok, tgt)
    l64, _, _ = _torch_forward64(m, tok, tgt)
    assert abs(loss - l64) / l64 < 1e-5


def test_init_loss_near_log_vocab(oracle_lib):
    """At N(0, 0.02) init the loss is about ln V (phase4_training.rs:106-124)."""
    cfg = custom_config(256, 512, 2, 2, 64, 8192)
    m = OracleModel(cfg, seed=0)
    rng = np.random.default_rng(0)
    tok = rng.integers(0, 8192, 64).astype(np.uint32)
    tgt = rng.integers(0, 8192, 64).astype(np.uint32)
    loss = m.forward(tok, tgt)[0]
    assert 0 < loss < 20
    assert abs(loss - np.log(8192)) < 0.5


def _torch_params64(m: OracleModel):
    f = lambda a: torch.tensor(np.asarray(a, np.float64), requires_grad=True)  # noqa: E731
    return {"embed": f(m.embed), "gamma_final": f(m.gamma_final),
            "layers": [{k: f(v) for k, v in lw.items()} for lw in m.layers]}


def _torch_seq_loss64(cfg, P, tokens, targets, softcap=0.0):
    """Sum over sequences of each sequence's mean token loss, float64 autograd."""
    S = cfg.seq
    tok = torch.from_numpy(np.asarray(tokens, np.int64)).view(-1, S)
    x = P["embed"][tok]
    alpha = 1.0 / np.sqrt(2.0 * cfg.nlayers)
    p = torch.arange(S, dtype=torch.float64)[:, None]
    i = torch.arange(64, dtype=torch.float64)[None, :]
    th = p * torch.pow(torch.tensor(10000.0, dtype=torch.float64), -2.0 * i / 128.0)
    cos, sin = torch.cos(th), torch.sin(th)

    def norm(v, g):
        return v / torch.sqrt((v * v).mean(-1, keepdim=True) + 1e-5) * g

    def rope(v):
        B_ = v.shape[0]
        v = v.view(B_, S, -1, 64, 2)
        a, b = v[..., 0], v[..., 1]
        c, s = cos[None, :, None, :], sin[None, :, None, :]
        return torch.stack([a * c - b * s, b * c + a * s], -1).view(B_, S, -1)

    for lw in P["layers"]:
        xn = norm(x, lw["gamma1"])
        q, k, v = rope(xn @ lw["wq"]), rope(xn @ lw["wk"]), xn @ lw["wv"]
        B_ = q.shape[0]
        q = q.view(B_, S, cfg.heads, 128).transpose(1, 2)
        k = k.view(B_, S, cfg.kv_heads, 128).transpose(1, 2).repeat_interleave(cfg.gqa_ratio, 1)
        v = v.view(B_, S, cfg.kv_heads, 128).transpose(1, 2).repeat_interleave(cfg.gqa_ratio, 1)
        sc = q @ k.transpose(-1, -2) / np.sqrt(128.0)
        sc = sc.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool), 1), float("-inf"))
        a = (torch.softmax(sc, -1) @ v).transpose(1, 2).reshape(B_, S, -1)
        x = x + alpha * (a @ lw["wo"])
        xn = norm(x, lw["gamma2"])
        h1, h3 = xn @ lw["w1"], xn @ lw["w3"]
        x = x + alpha * ((h1 * torch.sigmoid(h1) * h3) @ lw["w2"].T)
    z = norm(x, P["gamma_final"]) @ P["embed"].T
    if softcap > 0:
        z = softcap * torch.tanh(z / softcap)
    tgt = torch.from_numpy(np.asarray(targets, np.int64)).view(-1, S)
    ptl = torch.logsumexp(z, -1) - torch.gather(z, -1, tgt[..., None])[..., 0]
    return ptl.mean(-1).sum(), ptl.mean().item()


def _grad_close(got, want, rtol):
    """Max-abs error relative to the tensor's largest gradient."""
    want = want.detach().numpy()
    scale = max(np.abs(want).max(), 1e-12)
    err = np.abs(got.astype(np.float64) - want).max()
    assert err <= rtol * scale, (err, scale)


@pytest.mark.parametrize("softcap,kv_heads", [(0.0, 2), (12.0, 1)])
def test_oracle_backward_matches_float64_autograd(oracle_lib, softcap, kv_heads):
    """orc_forward_backward (the reference's backward restated in fp32) against float64
    autograd of the same forward, with non-unit gains and GQA."""
    cfg = custom_config(256, 512, 2, 2, 64, 384).replace(kv_heads=kv_heads)
    m = OracleModel(cfg, seed=11, scheme=SCHEME_NORMAL, sigma=0.08)
    rng = np.random.default_rng(3)
    for lw in m.layers:
        lw["gamma1"][:] = 1 + 0.2 * rng.standard_normal(cfg.dim)
        lw["gamma2"][:] = 1 + 0.2 * rng.standard_normal(cfg.dim)
        lw["wo"][:] = 0.08 * rng.standard_normal(lw["wo"].shape)
        lw["w2"][:] = 0.08 * rng.standard_normal(lw["w2"].shape)
    m.gamma_final[:] = 1 + 0.2 * rng.standard_normal(cfg.dim)
    tok = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    loss_scale = 4.0
    loss, g = m.forward_backward(tok, tgt, softcap, loss_scale)
    P = _torch_params64(m)
    total, mean = _torch_seq_loss64(cfg, P, tok, tgt, softcap)
    (loss_scale * total).backward()
    assert abs(loss - mean) / mean < 1e-5
    _grad_close(g["embed"], P["embed"].grad, 1e-4)
    _grad_close(g["gamma_final"], P["gamma_final"].grad, 1e-4)
    for gl, pl in zip(g["layers"], P["layers"]):
        for k in OracleModel.LAYER_FIELDS:
            _grad_close(gl[k], pl[k].grad, 1e-4)


def test_oracle_backward_accumulates(oracle_lib):
    """Two sequences in one call give the sum of the two single-sequence gradients."""
    cfg = custom_config(256, 512, 2, 1, 64, 256)
    m = OracleModel(cfg, seed=2, scheme=SCHEME_NORMAL, sigma=0.05)
    rng = np.random.default_rng(8)
    tok = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    _, g2 = m.forward_backward(tok, tgt)
    _, ga = m.forward_backward(tok[:64], tgt[:64])
    _, gb = m.forward_backward(tok[64:], tgt[64:])
    np.testing.assert_allclose(g2["embed"], ga["embed"] + gb["embed"], rtol=1e-4, atol=1e-7)
    np.testing.assert_allclose(g2["layers"][0]["w1"], ga["layers"][0]["w1"] + gb["layers"][0]["w1"],
                               rtol=1e-4, atol=1e-7)


def test_oracle_odd_config_matches_float64_torch(oracle_lib):
    """The reference's odd test shape (test_combined_forward_correctness.rs:245-257: one
    head, hidden 768, seq 16, vocab 256, 2 layers) through the oracle and torch float64."""
    cfg = custom_config(256, 768, 1, 2, 16, 256)
    m = OracleModel(cfg, seed=8, scheme=SCHEME_NORMAL, sigma=0.05)
    rng = np.random.default_rng(8)
    tok = rng.integers(0, cfg.vocab, 3 * cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, 3 * cfg.seq).astype(np.uint32)
    loss, ptl, _ = m.forward(tok, tgt)
    l64, p64, _ = _torch_forward64(m, tok, tgt)
    assert abs(loss - l64) / l64 < 1e-5
    np.testing.assert_allclose(ptl, p64, rtol=1e-4, atol=1e-4)
