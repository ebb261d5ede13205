"""qkv_attention_noalloc, the entry point for callers that cannot allocate device memory
(FFI hosts without a CUDA allocator, engines whose HBM is reserved by a fixed pool): it must
give the same answer as qkv_attention with a caller-owned workspace, and the oracle's, on
calls in a row that share its static scratch (decode, the tensor-core verify path, ragged
batches), and refuse calls whose partials exceed that scratch.

This file is collected last on purpose; it also passes when run alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest

from oracle import qkv_oracle as orc
from tests.helpers import f32_of, make_case, torch_from_f32

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL_MAX, TOL_MEAN = 2e-2, 2e-3  # the tolerance the attention parity tests use


def _case(seed, bits, n, hq=32, hkv=4, D=128, S=1, B=1):
    """q and a cache over n keys, plus the oracle's quantized tuples."""
    from chad_b200.cache import QuantizedKVCache

    q, k, v = make_case(seed, B, hq, hkv, S, D, n, "bf16", outliers=True)
    c = QuantizedKVCache(group_size=64, bits=bits)
    c.update_and_fetch(torch_from_f32(k, "bf16"), torch_from_f32(v, "bf16"))
    kq = orc.affine_quantize(k, bits, 64, "bf16")
    vq = orc.affine_quantize(v, bits, 64, "bf16")
    return q, c, kq, vq


def _noalloc(lib, q, c, n, out, lens=None, mask=0, splits=0):
    kw, ks, kb = c.keys
    vw, vs, vb = c.values
    B, HQ, S, D = q.shape
    return lib.qkv_attention_noalloc(
        q.data_ptr(), kw.data_ptr(), ks.data_ptr(), kb.data_ptr(), vw.data_ptr(),
        vs.data_ptr(), vb.data_ptr(), out.data_ptr(), B, HQ, kw.shape[1], S, D, kw.shape[2], n,
        None if lens is None else lens.data_ptr(), None, None, c.bits, 64, 0, D ** -0.5, mask,
        None, 0, 0, 0, 0, 0, splits, torch.cuda.current_stream().cuda_stream)


def _check(out, want_gpu, ref):
    got = out.float()
    assert torch.isfinite(got).all()
    err = (got - want_gpu.float()).abs()
    assert err.max().item() < TOL_MAX and err.mean().item() < TOL_MEAN
    e2 = np.abs(f32_of(out) - ref)
    assert e2.max() < TOL_MAX and e2.mean() < TOL_MEAN, (e2.max(), e2.mean())


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    from chad_b200 import _lib, ops

    lib = _lib.load()
    cases = [(11, 4, 32768), (12, 8, 5000)]
    outs = []
    for seed, bits, n in cases:  # two calls in a row through the shared scratch
        q, c, kq, vq = _case(seed, bits, n)
        tq = torch_from_f32(q, "bf16")
        out = torch.empty_like(tq)
        assert _noalloc(lib, tq, c, n, out) == _lib.QKV_OK, lib.qkv_last_error()
        outs.append((q, tq, c, kq, vq, n, out))
    torch.cuda.synchronize()
    for q, tq, c, kq, vq, n, out in outs:
        ws = torch.zeros(ops.workspace_size(1, 32, 4, 1, 128, n, c.bits), dtype=torch.uint8,
                         device="cuda")
        want = ops.attention(tq, c.keys, c.values, 128 ** -0.5, n, c.bits, workspace=ws)
        ref = orc.attention_quantized_fp32(q, kq, vq, 128 ** -0.5, n, c.bits)
        _check(out, want, ref)


def test_noalloc_across_paths_shares_a_clean_scratch():
    """A verify block on the tensor-core path (its combine clears the scratch), then a
    ragged batch on the balanced decode plan, then a plain decode: each through the static
    scratch, each equal to the caller-workspace result and to the oracle."""
    from chad_b200 import _lib, ops

    lib = _lib.load()
    # 1) S=8 causal verify block at GQA 8 (64 query rows): tensor-core path, key splits
    q, c, kq, vq = _case(21, 4, 1000, S=8)
    tq = torch_from_f32(q, "bf16")
    out = torch.empty_like(tq)
    assert _noalloc(lib, tq, c, 1000, out, mask=1) == _lib.QKV_OK, lib.qkv_last_error()
    want = ops.attention(tq, c.keys, c.values, 128 ** -0.5, 1000, 4, mask="causal",
                         workspace=torch.zeros(16 << 20, dtype=torch.uint8, device="cuda"))
    _check(out, want, orc.attention_quantized_fp32(q, kq, vq, 128 ** -0.5, 1000, 4, 64,
                                                   "causal"))
    # 2) ragged batch: three sequences of different lengths in one cache
    lens_l = [700, 3000, 1500]
    q, c, kq, vq = _case(22, 8, 3000, B=3)
    tq = torch_from_f32(q, "bf16")
    lens = torch.tensor(lens_l, dtype=torch.int32, device="cuda")
    out = torch.empty_like(tq)
    assert _noalloc(lib, tq, c, 3000, out, lens=lens) == _lib.QKV_OK, lib.qkv_last_error()
    want = ops.attention(tq, c.keys, c.values, 128 ** -0.5, 3000, 8, lens=lens,
                         workspace=torch.zeros(16 << 20, dtype=torch.uint8, device="cuda"))
    _check(out, want, orc.attention_quantized_fp32(q, kq, vq, 128 ** -0.5, lens_l, 8))
    # 3) plain decode
    q, c, kq, vq = _case(23, 4, 9000)
    tq = torch_from_f32(q, "bf16")
    out = torch.empty_like(tq)
    assert _noalloc(lib, tq, c, 9000, out) == _lib.QKV_OK, lib.qkv_last_error()
    want = ops.attention(tq, c.keys, c.values, 128 ** -0.5, 9000, 4,
                         workspace=torch.zeros(16 << 20, dtype=torch.uint8, device="cuda"))
    _check(out, want, orc.attention_quantized_fp32(q, kq, vq, 128 ** -0.5, 9000, 4))
    assert ops.device_status() == 0


def test_noalloc_rejects_partials_beyond_the_scratch():
    from chad_b200 import _lib

    lib = _lib.load()
    _, c, _, _ = _case(13, 4, 1024)
    big = torch.empty((1, 32, 512, 128), dtype=torch.bfloat16, device="cuda")
    rc = lib.qkv_attention_noalloc(
        big.data_ptr(), *(t.data_ptr() for t in c.keys), *(t.data_ptr() for t in c.values),
        big.data_ptr(), 1, 32, 4, 512, 128, c.keys[0].shape[2], 1024, None, None, None, 4, 64,
        0, 0.1, 1, None, 0, 0, 0, 0, 0, 64, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.QKV_EWORKSPACE
    msg = lib.qkv_last_error().decode()
    assert "static scratch" in msg and str(4 << 20) in msg
    assert ctypes.c_int(rc).value < 0
