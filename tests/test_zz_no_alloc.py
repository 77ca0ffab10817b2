"""GPU test of cb_lm_head_ce_f16_noalloc, the LM head + cross-entropy entry point
for callers that cannot allocate device memory during the call (engines that own
all device memory through their own pool, loops where a cudaMalloc would
synchronise the device). Its scratch is a fixed array inside the library.

It must give the same per-token and mean losses as the allocating entry point
cb_lm_head_ce_f16, on two calls in a row (the second reuses the array the first
left behind). This file sorts last so a run that stops at the first failure has
already run every other test; it also passes alone in a fresh process."""
import ctypes as C

import pytest
import torch

from rustane_b200 import bridge as B

pytestmark = pytest.mark.gpu


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _inputs(T, d, V, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    xf = torch.randn(T, d, device="cuda", generator=g).half()
    emb = (torch.randn(V, d, device="cuda", generator=g) * 0.02).half()
    tgt = torch.randint(0, V, (T,), device="cuda", generator=g).to(torch.int32)
    return xf, emb, tgt


def _run(fn, xf, emb, tgt, T, d, V, softcap):
    ptl = torch.full((T,), float("nan"), device="cuda")
    loss = torch.full((1,), float("nan"), device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = fn(_ptr(xf), _ptr(emb), _ptr(tgt), T, d, V, softcap, _ptr(ptl), _ptr(loss), stream)
    torch.cuda.synchronize()
    return rc, ptl, loss


def test_no_alloc_matches_allocating_entry_point_twice(bridge_lib):
    cases = [(4096, 1536, 8192, 0.0, 1), (1000, 512, 4000, 15.0, 2)]
    for T, d, V, softcap, seed in cases:  # two calls in a row, different shapes
        xf, emb, tgt = _inputs(T, d, V, seed)
        rc_ref, ptl_ref, loss_ref = _run(bridge_lib.cb_lm_head_ce_f16, xf, emb, tgt, T, d, V,
                                         softcap)
        rc, ptl, loss = _run(bridge_lib.cb_lm_head_ce_f16_noalloc, xf, emb, tgt, T, d, V,
                             softcap)
        assert rc_ref == B.CB_OK and rc == B.CB_OK
        torch.testing.assert_close(ptl, ptl_ref, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(loss, loss_ref, rtol=1e-5, atol=1e-5)
        assert torch.isfinite(ptl).all()


def test_no_alloc_rejects_sizes_beyond_its_array(bridge_lib):
    xf, emb, tgt = _inputs(8200, 256, 1024, 3)
    rc, _, _ = _run(bridge_lib.cb_lm_head_ce_f16_noalloc, xf, emb, tgt, 8200, 256, 1024, 0.0)
    assert rc == B.CB_ERR_INVALID_ARG
    xf, emb, tgt = _inputs(128, 256, 16416, 4)
    rc, _, _ = _run(bridge_lib.cb_lm_head_ce_f16_noalloc, xf, emb, tgt, 128, 256, 16416, 0.0)
    assert rc == B.CB_ERR_INVALID_ARG
