"""qkv_attention_noalloc, the entry point for callers that cannot allocate device memory
(FFI hosts without a CUDA allocator, engines whose HBM is reserved by a fixed pool): it must
give the same answer as qkv_attention with a caller-owned workspace, on two calls in a row
that share its static scratch, and refuse calls whose partials exceed that scratch.

This file is collected last on purpose; it also passes when run alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL_MAX, TOL_MEAN = 2e-2, 2e-3  # the tolerance the attention parity tests use


def _case(seed, bits, n, hq=32, hkv=4, D=128):
    from chad_b200.cache import QuantizedKVCache

    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn((1, hkv, n, D), generator=g, device="cuda")
    k[..., [3, 37, 70, 101]] *= 8.0
    v = torch.randn((1, hkv, n, D), generator=g, device="cuda")
    q = torch.randn((1, hq, 1, D), generator=g, device="cuda").to(torch.bfloat16)
    c = QuantizedKVCache(group_size=64, bits=bits)
    c.update_and_fetch(k.to(torch.bfloat16), v.to(torch.bfloat16))
    return q, c


def _noalloc(lib, q, c, n, out, splits=0):
    kw, ks, kb = c.keys
    vw, vs, vb = c.values
    B, HQ, S, D = q.shape
    return lib.qkv_attention_noalloc(
        q.data_ptr(), kw.data_ptr(), ks.data_ptr(), kb.data_ptr(), vw.data_ptr(),
        vs.data_ptr(), vb.data_ptr(), out.data_ptr(), B, HQ, kw.shape[1], S, D, kw.shape[2], n,
        None, None, None, c.bits, 64, 0, D ** -0.5, 0, None, 0, 0, 0, 0, 0, splits,
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    from chad_b200 import _lib, ops

    lib = _lib.load()
    cases = [(11, 4, 32768), (12, 8, 5000)]
    outs = []
    for seed, bits, n in cases:  # two calls in a row through the shared scratch
        q, c = _case(seed, bits, n)
        out = torch.empty_like(q)
        assert _noalloc(lib, q, c, n, out) == _lib.QKV_OK, lib.qkv_last_error()
        outs.append((q, c, n, out))
    torch.cuda.synchronize()
    for q, c, n, out in outs:
        want = ops.attention(q, c.keys, c.values, q.shape[-1] ** -0.5, n, c.bits)
        err = (out.float() - want.float()).abs()
        assert torch.isfinite(out.float()).all()
        assert err.max().item() < TOL_MAX and err.mean().item() < TOL_MEAN


def test_noalloc_rejects_partials_beyond_the_scratch():
    from chad_b200 import _lib

    lib = _lib.load()
    q, c = _case(13, 4, 1024)
    big = torch.empty((1, 32, 512, 128), dtype=torch.bfloat16, device="cuda")
    rc = lib.qkv_attention_noalloc(
        big.data_ptr(), *(t.data_ptr() for t in c.keys), *(t.data_ptr() for t in c.values),
        big.data_ptr(), 1, 32, 4, 512, 128, c.keys[0].shape[2], 1024, None, None, None, 4, 64,
        0, 0.1, 1, None, 0, 0, 0, 0, 0, 64, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.QKV_EWORKSPACE
    msg = lib.qkv_last_error().decode()
    assert "static scratch" in msg and str(4 << 20) in msg
    assert ctypes.c_int(rc).value < 0
    assert np.isscalar(rc)
