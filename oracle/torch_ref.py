"""Torch CPU restatement of the forward + loss: test infrastructure, like the rest of
this package, and never part of the product path.

Two uses:
- float64 with an explicit masked softmax: an independent cross-check of the C
  oracle (``forward_ref.cpp``) on tiny configurations;
- float32 with torch's fused causal attention: the optional second CPU figure of
  the bench (torch's own MKL/oneDNN kernels on the host cores), beside the C
  oracle's.

The math follows the reference engine's forward (crates/engine/src/full_model.rs:
378-472, layer flow layer.rs:4409-4624 with alpha = 1/sqrt(2L) at :4420; RoPE on
interleaved pairs, kernels/sdpa_fwd.rs:24-60; SwiGLU with W2 used transposed,
kernels/ffn_fused.rs:105-154; RMSNorm eps 1e-5, cpu/rmsnorm.rs:10,149-183; CE with
the mean over all tokens, cpu/cross_entropy.rs:58-96).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def forward(m, tokens, targets, softcap: float = 0.0, dtype=torch.float64,
            fused_attention: bool = False):
    """(mean loss, per-token losses [T], logits [T, V]) of the model ``m`` (an object
    with ``cfg``, ``embed``, ``gamma_final`` and ``layers``: dicts of reference-
    orientation arrays, as ``oracle.OracleModel`` holds them). With ``dtype``
    float32 the numpy weights are shared, not copied."""
    cfg = m.cfg
    S = cfg.seq

    def f(a):
        return torch.from_numpy(np.asarray(a, np.float64 if dtype == torch.float64
                                           else np.float32))

    E = f(m.embed)
    tok = torch.from_numpy(np.asarray(tokens, np.int64)).view(-1, S)
    x = E[tok]  # [B, S, d]
    alpha = 1.0 / np.sqrt(2.0 * cfg.nlayers)
    p = torch.arange(S, dtype=torch.float64)[:, None]
    i = torch.arange(cfg.hd // 2, dtype=torch.float64)[None, :]
    th = p * torch.pow(torch.tensor(10000.0, dtype=torch.float64), -2.0 * i / cfg.hd)
    cos, sin = torch.cos(th).to(dtype), torch.sin(th).to(dtype)

    def norm(v, g):
        return v / torch.sqrt((v * v).mean(-1, keepdim=True) + 1e-5) * f(g)

    def rope(v):  # [B, S, n*hd]
        B_ = v.shape[0]
        v = v.view(B_, S, -1, cfg.hd // 2, 2)
        a, b = v[..., 0], v[..., 1]
        c, s = cos[None, :, None, :], sin[None, :, None, :]
        return torch.stack([a * c - b * s, b * c + a * s], -1).view(B_, S, -1)

    mask = torch.triu(torch.ones(S, S, dtype=torch.bool), 1)
    for lw in m.layers:
        xn = norm(x, lw["gamma1"])
        q, k, v = rope(xn @ f(lw["wq"])), rope(xn @ f(lw["wk"])), xn @ f(lw["wv"])
        B_ = q.shape[0]
        q = q.view(B_, S, cfg.heads, cfg.hd).transpose(1, 2)
        k = k.view(B_, S, cfg.kv_heads, cfg.hd).transpose(1, 2)
        v = v.view(B_, S, cfg.kv_heads, cfg.hd).transpose(1, 2)
        if cfg.gqa_ratio > 1:
            k = k.repeat_interleave(cfg.gqa_ratio, dim=1)
            v = v.repeat_interleave(cfg.gqa_ratio, dim=1)
        if fused_attention:
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        else:
            sc = (q @ k.transpose(-1, -2) / np.sqrt(float(cfg.hd))).masked_fill(
                mask, float("-inf"))
            a = torch.softmax(sc, -1) @ v
        a = a.transpose(1, 2).reshape(B_, S, -1)
        x = x + alpha * (a @ f(lw["wo"]))
        xn = norm(x, lw["gamma2"])
        h1, h3 = xn @ f(lw["w1"]), xn @ f(lw["w3"])
        x = x + alpha * ((h1 * torch.sigmoid(h1) * h3) @ f(lw["w2"]).T)
    xf = norm(x, m.gamma_final)
    z = xf @ E.T
    if softcap > 0:
        z = softcap * torch.tanh(z / softcap)
    tgt = torch.from_numpy(np.asarray(targets, np.int64)).view(-1, S)
    ptl = torch.logsumexp(z, -1) - torch.gather(z, -1, tgt[..., None])[..., 0]
    return ptl.mean().item(), ptl.reshape(-1).numpy(), z.reshape(-1, cfg.vocab).numpy()
