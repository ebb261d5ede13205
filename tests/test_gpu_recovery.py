"""Bounded waits: a merge that gives up reports QKV_EDEVICE, and the library recovers.

Every spin-wait in libqkv gives up after a bounded time, records a status word and lets the
kernel wind down instead of hanging the GPU. This drives that path in the one form that
faults nothing: a test hook makes the decode merge wait for a partial set that no CTA ever
writes (a flag that nothing sets), with the wait shortened to 200 us. The kernel must
return, the status word must read QKV_EDEVICE, the host side must zero the workspace it
caches (and the library its static scratch), and the next call must match the oracle.
"""

import numpy as np
import pytest

from oracle import qkv_oracle as orc
from tests.helpers import f32_of, make_case, torch_from_f32

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SPIN_NS = 200_000  # the shortened bound on the merge's wait


def _case(seed=41, n=4096, bits=4):
    from chad_b200.cache import QuantizedKVCache

    q, k, v = make_case(seed, 1, 32, 4, 1, 128, n, "bf16", outliers=True)
    c = QuantizedKVCache(group_size=64, bits=bits)
    c.update_and_fetch(torch_from_f32(k, "bf16"), torch_from_f32(v, "bf16"))
    kq = orc.affine_quantize(k, bits, 64, "bf16")
    vq = orc.affine_quantize(v, bits, 64, "bf16")
    ref = orc.attention_quantized_fp32(q, kq, vq, 128 ** -0.5, n, bits)
    return torch_from_f32(q, "bf16"), c, ref


def _close(out, ref):
    g = f32_of(out)
    err = np.abs(g - ref)
    return np.isfinite(g).all() and err.max() < 2e-2 and err.mean() < 2e-3


@pytest.fixture
def hooks():
    from chad_b200 import _lib

    lib = _lib.load()
    yield lib
    assert lib.qkv_test_hooks(0, 0) == _lib.QKV_OK
    torch.cuda.synchronize()


def test_merge_timeout_reports_and_workspace_recovers(hooks):
    from chad_b200 import _lib, ops

    lib = hooks
    dev = torch.device("cuda", torch.cuda.current_device())
    q, c, ref = _case()
    n = 4096
    assert ops.device_status() == 0
    ws = ops._workspace(dev, 64 << 20)  # the cached workspace, with room for the extra set
    assert lib.qkv_test_hooks(1, SPIN_NS) == _lib.QKV_OK
    ops.attention(q, c.keys, c.values, 128 ** -0.5, n, 4)
    torch.cuda.synchronize()  # the kernel returned: the wait was bounded
    assert lib.qkv_test_hooks(0, 0) == _lib.QKV_OK
    with pytest.raises(ops.DeviceWaitError):
        ops.check_device()
    assert int(torch.count_nonzero(ws)) == 0
    assert ops.device_status() == 0  # the word was cleared by the check
    out = ops.attention(q, c.keys, c.values, 128 ** -0.5, n, 4)
    assert _close(out, ref)
    assert ops.device_status() == 0


def test_noalloc_timeout_then_reset_recovers(hooks):
    from chad_b200 import _lib, ops

    lib = hooks
    q, c, ref = _case(seed=42, n=3000, bits=8)
    n = 3000
    st = torch.cuda.current_stream().cuda_stream

    def call(out):
        kw, ks, kb = c.keys
        vw, vs, vb = c.values
        return lib.qkv_attention_noalloc(
            q.data_ptr(), kw.data_ptr(), ks.data_ptr(), kb.data_ptr(), vw.data_ptr(),
            vs.data_ptr(), vb.data_ptr(), out.data_ptr(), 1, 32, 4, 1, 128, kw.shape[2], n,
            None, None, None, 8, 64, 0, 128 ** -0.5, 0, None, 0, 0, 0, 0, 0, 0, st)

    out = torch.empty_like(q)
    assert lib.qkv_test_hooks(1, SPIN_NS) == _lib.QKV_OK
    assert call(out) == _lib.QKV_OK, lib.qkv_last_error()
    assert lib.qkv_test_hooks(0, 0) == _lib.QKV_OK
    status = lib.qkv_device_status(st, 1)  # synchronizes, clears, zeroes the static scratch
    assert status <= _lib.QKV_EDEVICE * 1000, status
    assert lib.qkv_device_status(st, 0) == 0
    out2 = torch.empty_like(q)
    assert call(out2) == _lib.QKV_OK, lib.qkv_last_error()
    torch.cuda.synchronize()
    assert _close(out2, ref)
    assert ops.device_status() == 0
