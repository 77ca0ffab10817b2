"""GPU tests of the individual kernels through the C ABI, against plain
PyTorch fp32 references of the same op."""
import ctypes as C
import math

import pytest
import torch

from rustane_b200 import bridge as B

pytestmark = pytest.mark.gpu


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("M,N,K,bn", [
    (128, 128, 64, 128),
    (128, 256, 64, 256),
    (256, 512, 128, 256),
    (200, 384, 192, 128),       # ragged M (TMA zero fill + row masking)
    (1000, 1536, 1536, 256),
    (1024, 4608, 1536, 0),      # QKV shape, automatic tile choice
    (512, 1536, 4096, 0),       # down-projection shape
    (4096, 8192, 1536, 256),
    (256, 256, 64, 2),          # one CTA-pair tile
    (200, 512, 192, 2),         # ragged M: the odd CTA of the pair is out of bounds
    (1000, 1536, 1536, 2),
    (4096, 8192, 1536, 2),
    (32768, 4608, 1536, 0),     # full 600m-A QKV shape, automatic choice
])
def test_gemm_matches_torch(bridge_lib, M, N, K, bn):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    a = (torch.randn(M, K, device="cuda", generator=g) / K ** 0.25).half()
    b = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.25).half()
    ref = a.float() @ b.float().T
    c32 = torch.empty(M, N, device="cuda", dtype=torch.float32)
    assert bridge_lib.cb_gemm_f16(_ptr(a), _ptr(b), _ptr(c32), M, N, K, 1, bn, _stream()) == 0
    c16 = torch.empty(M, N, device="cuda", dtype=torch.float16)
    assert bridge_lib.cb_gemm_f16(_ptr(a), _ptr(b), _ptr(c16), M, N, K, 0, bn, _stream()) == 0
    torch.cuda.synchronize()
    torch.testing.assert_close(c32, ref, rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(c16.float(), ref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("M,N,K,bn", [
    (128, 128, 128, 128),       # two k-blocks: one per half
    (300, 256, 192, 256),       # odd k-block count: halves of 2 and 1, ragged M
    (4096, 1536, 1536, 2),      # the O projection at 4096 tokens per GPU
    (4096, 1536, 4096, 0),      # the down projection, automatic tile
    (1000, 1536, 4096, 2),      # ragged M on the CTA pair
])
def test_gemm_split_k_accumulates(bridge_lib, M, N, K, bn):
    """out_f32 = 2: C += A * B^T with the K range split across two work units per tile."""
    g = torch.Generator(device="cuda").manual_seed(M + 3 * N + K)
    a = (torch.randn(M, K, device="cuda", generator=g) / K ** 0.25).half()
    b = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.25).half()
    c0 = torch.randn(M, N, device="cuda", generator=g)
    ref = c0 + a.float() @ b.float().T
    c = c0.clone()
    assert bridge_lib.cb_gemm_f16(_ptr(a), _ptr(b), _ptr(c), M, N, K, 2, bn, _stream()) == 0
    torch.cuda.synchronize()
    torch.testing.assert_close(c, ref, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("layout", [1, 2, 3])
@pytest.mark.parametrize("M,N,K,bn", [
    (128, 128, 64, 128),
    (256, 256, 200, 2),          # ragged K (zero-filled boxes)
    (320, 512, 1000, 256),       # ragged M on a 1-CTA tile, K not a multiple of 64
    (1536, 1536, 4096, 0),       # a weight-gradient shape: K = tokens
    (4096, 4608, 1536, 2),       # dX of the QKV projection: B = Wqkv as stored
])
def test_gemm_transposed_operands(bridge_lib, layout, M, N, K, bn):
    """cb_gemm_f16_layout: A stored [K][M] (bit 0) and/or B stored [K][N] (bit 1)."""
    g = torch.Generator(device="cuda").manual_seed(M + N + K + layout)
    a = (torch.randn(M, K, device="cuda", generator=g) / K ** 0.25).half()
    b = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.25).half()
    ref = a.float() @ b.float().T
    a_arg = a.t().contiguous() if layout & 1 else a
    b_arg = b.t().contiguous() if layout & 2 else b
    c32 = torch.empty(M, N, device="cuda", dtype=torch.float32)
    assert bridge_lib.cb_gemm_f16_layout(_ptr(a_arg), _ptr(b_arg), _ptr(c32), M, N, K, layout, 1,
                                         bn, _stream()) == 0
    c16 = torch.empty(M, N, device="cuda", dtype=torch.float16)
    assert bridge_lib.cb_gemm_f16_layout(_ptr(a_arg), _ptr(b_arg), _ptr(c16), M, N, K, layout, 0,
                                         bn, _stream()) == 0
    acc = torch.ones(M, N, device="cuda", dtype=torch.float32)
    assert bridge_lib.cb_gemm_f16_layout(_ptr(a_arg), _ptr(b_arg), _ptr(acc), M, N, K, layout, 2,
                                         bn, _stream()) == 0
    torch.cuda.synchronize()
    torch.testing.assert_close(c32, ref, rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(c16.float(), ref, rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(acc, ref + 1, rtol=1e-4, atol=1e-3)


def test_gemm_rejects_bad_shapes(bridge_lib):
    a = torch.zeros(128, 96, device="cuda", dtype=torch.float16)
    assert bridge_lib.cb_gemm_f16(_ptr(a), _ptr(a), _ptr(a), 128, 128, 96, 0, 0, None) == \
        B.CB_ERR_INVALID_ARG


# The tcgen05 kernel gives each CTA a block of two 128-query tiles (2m, 2m+1); seq 128,
# 384 and 640 end in a block with one tile.
@pytest.mark.parametrize("batch,heads,seq", [(1, 1, 64), (2, 3, 128), (1, 2, 384), (1, 12, 512),
                                             (2, 3, 640), (2, 4, 2048)])
def test_attention_matches_torch(bridge_lib, batch, heads, seq):
    g = torch.Generator(device="cuda").manual_seed(seq + heads)
    q, k, v = (torch.randn(batch, heads, seq, 128, device="cuda", generator=g).half()
               for _ in range(3))
    out = torch.empty(batch * seq, heads * 128, device="cuda", dtype=torch.float16)
    assert bridge_lib.cb_attention_f16(_ptr(q), _ptr(k), _ptr(v), _ptr(out), batch, heads, seq,
                                       _stream()) == 0
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(),
                                                           is_causal=True)
    ref = ref.transpose(1, 2).reshape(batch * seq, heads * 128)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=3e-3)


def test_gemm_positive_sum_bias_matches_cublas(bridge_lib):
    """Long all-positive dot products: our tcgen05 GEMM and cuBLAS show the same
    small low bias against float64 (tensor-core fp32 accumulation truncates)."""
    M, N, K = 512, 512, 5120
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.rand(M, K, device="cuda", generator=g).half()
    b = torch.rand(N, K, device="cuda", generator=g).half()
    ref = a.double() @ b.double().T
    ours = torch.empty(M, N, device="cuda", dtype=torch.float32)
    assert bridge_lib.cb_gemm_f16(_ptr(a), _ptr(b), _ptr(ours), M, N, K, 1, 0, _stream()) == 0
    torch.cuda.synchronize()
    rel_ours = ((ours.double() - ref) / ref).mean().item()
    # cuBLAS fp16 GEMM with fp32 accumulation and fp32 output (when torch exposes it)
    try:
        cub = torch.mm(a, b.T, out_dtype=torch.float32)
    except (TypeError, RuntimeError):
        cub = None
    assert abs(rel_ours) < 2e-4
    if cub is not None:
        rel_cub = ((cub.double() - ref) / ref).mean().item()
        print(f"mean relative error vs float64: ours {rel_ours:.3e}, cuBLAS {rel_cub:.3e}")
        assert abs(rel_ours - rel_cub) < max(5e-5, 0.5 * abs(rel_cub))


def _lm_head_ce_torch(xf, emb, tgt, softcap):
    z = xf.float() @ emb.float().T
    if softcap > 0:
        z = softcap * torch.tanh(z / softcap)
    return torch.logsumexp(z, -1) - z.gather(1, tgt.long()[:, None])[:, 0]


@pytest.mark.parametrize("T,d,V,softcap", [(512, 1536, 8192, 0.0), (300, 256, 1024, 15.0),
                                           (1024, 512, 4000, 0.0)])
def test_lm_head_ce_matches_torch(bridge_lib, T, d, V, softcap):
    g = torch.Generator(device="cuda").manual_seed(T + V)
    xf = torch.randn(T, d, device="cuda", generator=g).half()
    emb = (torch.randn(V, d, device="cuda", generator=g) * 0.02).half()
    tgt = torch.randint(0, V, (T,), device="cuda", generator=g).to(torch.int32)
    ptl = torch.empty(T, device="cuda", dtype=torch.float32)
    loss = torch.empty(1, device="cuda", dtype=torch.float32)
    assert bridge_lib.cb_lm_head_ce_f16(_ptr(xf), _ptr(emb), _ptr(tgt), T, d, V, softcap,
                                        _ptr(ptl), _ptr(loss), _stream()) == 0
    ref = _lm_head_ce_torch(xf, emb, tgt, softcap)
    torch.cuda.synchronize()
    torch.testing.assert_close(ptl, ref, rtol=1e-4, atol=1e-4)
    assert abs(loss.item() - ref.mean().item()) < 1e-4
    # nullable outputs
    assert bridge_lib.cb_lm_head_ce_f16(_ptr(xf), _ptr(emb), _ptr(tgt), T, d, V, softcap,
                                        None, _ptr(loss), _stream()) == 0
    torch.cuda.synchronize()
    assert abs(loss.item() - ref.mean().item()) < 1e-4


def test_lm_head_ce_bad_target_is_nan(bridge_lib):
    T, d, V = 128, 256, 1024
    xf = torch.randn(T, d, device="cuda").half()
    emb = torch.randn(V, d, device="cuda").half()
    tgt = torch.zeros(T, device="cuda", dtype=torch.int32)
    tgt[5] = V
    ptl = torch.empty(T, device="cuda", dtype=torch.float32)
    assert bridge_lib.cb_lm_head_ce_f16(_ptr(xf), _ptr(emb), _ptr(tgt), T, d, V, 0.0, _ptr(ptl),
                                        None, _stream()) == 0
    torch.cuda.synchronize()
    assert torch.isnan(ptl[5]) and torch.isfinite(ptl[:5]).all()
    assert bridge_lib.cb_lm_head_ce_f16(_ptr(xf), _ptr(emb), _ptr(tgt), T, 100, V, 0.0, _ptr(ptl),
                                        None, _stream()) == B.CB_ERR_INVALID_ARG


@pytest.mark.parametrize("batch,heads,kv_heads,seq", [(1, 8, 2, 640), (2, 6, 3, 2048),
                                                      (3, 2, 1, 128)])
def test_attention_gqa_forward_and_lse_match_torch(bridge_lib, batch, heads, kv_heads, seq):
    """Grouped-query attention forward with the base-2 log-sum-exp it keeps for the
    backward pass, against float32 torch."""
    g = torch.Generator(device="cuda").manual_seed(seq + 7 * heads + kv_heads)
    q = torch.randn(batch, heads, seq, 128, device="cuda", generator=g).half()
    k = torch.randn(batch, kv_heads, seq, 128, device="cuda", generator=g).half()
    v = torch.randn(batch, kv_heads, seq, 128, device="cuda", generator=g).half()
    out = torch.empty(batch * seq, heads * 128, device="cuda", dtype=torch.float16)
    lse = torch.empty(batch, heads, seq, device="cuda", dtype=torch.float32)
    assert bridge_lib.cb_attention_fwd_lse_f16(_ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(lse),
                                               batch, heads, kv_heads, seq, _stream()) == 0
    grp = heads // kv_heads
    kk, vv = k.float().repeat_interleave(grp, 1), v.float().repeat_interleave(grp, 1)
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), kk, vv, is_causal=True)
    ref = ref.transpose(1, 2).reshape(batch * seq, heads * 128)
    s = (q.float() @ kk.transpose(-1, -2)) / 128 ** 0.5
    mask = torch.ones(seq, seq, device="cuda", dtype=torch.bool).triu(1)
    lse_ref = torch.logsumexp(s.masked_fill(mask, float("-inf")), dim=-1) / math.log(2)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=3e-3)
    torch.testing.assert_close(lse, lse_ref, rtol=0, atol=2e-3)


def _attn_ref(q, k, v, group):
    """float32 causal attention with autograd (K/V heads repeated for GQA)."""
    kk = k.repeat_interleave(group, dim=1)
    vv = v.repeat_interleave(group, dim=1)
    return torch.nn.functional.scaled_dot_product_attention(q, kk, vv, is_causal=True)


@pytest.mark.parametrize("batch,heads,kv_heads,seq", [
    (1, 1, 1, 64), (2, 3, 3, 128), (1, 4, 2, 256), (2, 2, 1, 512), (1, 2, 2, 192)])
def test_attention_backward_matches_torch(bridge_lib, batch, heads, kv_heads, seq):
    g = torch.Generator(device="cuda").manual_seed(seq * 3 + heads + kv_heads)
    q = torch.randn(batch, heads, seq, 128, device="cuda", generator=g).half()
    k = torch.randn(batch, kv_heads, seq, 128, device="cuda", generator=g).half()
    v = torch.randn(batch, kv_heads, seq, 128, device="cuda", generator=g).half()
    dout = (torch.randn(batch * seq, heads * 128, device="cuda", generator=g) * 0.1).half()
    T = batch * seq
    out = torch.empty(T, heads * 128, device="cuda", dtype=torch.float16)
    lse = torch.empty(batch, heads, seq, device="cuda", dtype=torch.float32)
    assert bridge_lib.cb_attention_fwd_lse_f16(_ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(lse),
                                               batch, heads, kv_heads, seq, _stream()) == 0
    n_qkv = (heads + 2 * kv_heads) * 128
    dqkv = torch.empty(T, n_qkv, device="cuda", dtype=torch.float16)
    assert bridge_lib.cb_attention_bwd_f16(_ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(dout),
                                           _ptr(lse), _ptr(dqkv), batch, heads, kv_heads, seq,
                                           _stream()) == 0
    qf, kf, vf = (t.float().requires_grad_() for t in (q, k, v))
    ref = _attn_ref(qf, kf, vf, heads // kv_heads)
    # lse against the float32 scores: log2 sum_k 2^(s_k log2(e) / sqrt(128))
    s = (qf.detach() @ kf.detach().repeat_interleave(heads // kv_heads, 1).transpose(-1, -2))
    s = s / 128 ** 0.5
    mask = torch.ones(seq, seq, device="cuda", dtype=torch.bool).triu(1)
    lse_ref = torch.logsumexp(s.masked_fill(mask, float("-inf")), dim=-1) / math.log(2)
    do4 = dout.float().reshape(batch, seq, heads, 128).transpose(1, 2)
    ref.backward(do4)
    torch.cuda.synchronize()
    torch.testing.assert_close(lse, lse_ref, rtol=0, atol=2e-3)
    d = dqkv.float().reshape(batch, seq, heads + 2 * kv_heads, 128).transpose(1, 2)
    dq, dk, dv = d[:, :heads], d[:, heads:heads + kv_heads], d[:, heads + kv_heads:]
    for got, want in ((dq, qf.grad), (dk, kf.grad), (dv, vf.grad)):
        err = (got - want).abs().max().item()
        scale = want.abs().max().item()
        assert err <= 2e-2 * scale + 1e-3, (err, scale)
        cos = torch.nn.functional.cosine_similarity(got.flatten(), want.flatten(), dim=0).item()
        assert cos >= 0.999, cos
