"""libqkv.so loads, exports every symbol include/qkv.h declares, and rejects bad arguments
with status codes before touching a GPU (so these run on CPU-only machines too)."""

import ctypes
import os
import re

import pytest

from chad_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "qkv.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qkv_[a-z_]+)\s*\(", src)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("qkv_attention", "qkv_partials", "qkv_combine", "qkv_prefill",
                 "qkv_quantize_append", "qkv_dequantize", "qkv_workspace_size",
                 "qkv_last_error", "qkv_version", "qkv_device_status"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_workspace_size():
    lib = _lib.load()
    assert lib.qkv_version() == 100
    assert lib.qkv_workspace_size(1, 32, 4, 1, 128, 32768, 4, 64) > 0
    assert lib.qkv_workspace_size(1, 30, 4, 1, 128, 32768, 4, 64) == 0  # HQ % HKV


@pytest.mark.parametrize("B,HQ,HKV,S,D,bits", [
    (1, 32, 4, 1, 128, 4), (1, 32, 4, 1, 128, 8), (4, 32, 4, 1, 128, 4), (1, 16, 2, 1, 256, 8),
    (1, 32, 4, 8, 128, 4), (1, 32, 4, 2048, 128, 4), (2, 8, 8, 4, 64, 8), (3, 32, 2, 2, 128, 4),
])
def test_workspace_need_never_shrinks_as_keys_grow(B, HQ, HKV, S, D, bits):
    """ops.workspace_size asks the library for the next power of two of the key count, which
    is only safe if the need never shrinks as the key count grows."""
    lib = _lib.load()
    prev = 0
    n = 1
    while n <= 1 << 20:
        need = lib.qkv_workspace_size(B, HQ, HKV, S, D, n, bits, 64)
        assert need >= prev, (n, need, prev)
        prev = need
        n = n * 3 // 2 + 1


def _attn(lib, **over):
    a = dict(q=16, kw=16, ks=16, kb=16, vw=16, vs=16, vb=16, out=16, B=1, HQ=16, HKV=2, S=1,
             D=128, NP=512, n=100, lens=None, pos_base=None, total_lens=None, bits=4, gs=64,
             dtype=0, scale=0.1, mask_kind=0, mask=None, mask_nk=0, sb=0, sh=0, sq=0,
             out_kind=0, splits=0, ws=16, ws_bytes=1 << 20, stream=None)
    a.update(over)
    return lib.qkv_attention(*a.values())


@pytest.mark.parametrize("over,code", [
    (dict(bits=5), _lib.QKV_EUNSUPPORTED),
    (dict(gs=32), _lib.QKV_EUNSUPPORTED),
    (dict(D=96), _lib.QKV_EUNSUPPORTED),
    (dict(q=None), _lib.QKV_EINVAL),
    (dict(HQ=15), _lib.QKV_EINVAL),
    (dict(n=600), _lib.QKV_EINVAL),
    (dict(NP=500, n=100), _lib.QKV_EALIGN),
    (dict(kw=18), _lib.QKV_EALIGN),
    (dict(mask_kind=2), _lib.QKV_EINVAL),
    (dict(mask_kind=7), _lib.QKV_EINVAL),
    (dict(out_kind=3), _lib.QKV_EINVAL),
    (dict(dtype=2), _lib.QKV_EINVAL),
])
def test_attention_rejects_bad_arguments(over, code):
    lib = _lib.load()
    assert _attn(lib, **over) == code
    assert lib.qkv_last_error()  # a message was set


def test_quantize_and_dequantize_reject_bad_arguments():
    lib = _lib.load()
    assert lib.qkv_quantize_append(16, 0, 16, 16, 16, 1, 2, 10, 128, 8, 0, 4, 64, 0, None) \
        == _lib.QKV_EINVAL  # offset + S > NP
    assert lib.qkv_quantize_append(16, 5, 16, 16, 16, 1, 2, 1, 128, 8, 0, 4, 64, 0, None) \
        == _lib.QKV_EINVAL
    assert lib.qkv_dequantize(16, 16, 16, 16, 4, 128, 3, 64, 0, 0, None) == _lib.QKV_EUNSUPPORTED
    assert lib.qkv_dequantize(16, 16, 16, 16, 4, 128, 4, 64, 0, 2, None) == _lib.QKV_EINVAL
    n = ctypes.c_int(0)
    assert lib.qkv_partials(16, 16, 16, 16, 16, 16, 16, 16, 1 << 20, None, 1, 16, 2, 1, 128,
                            512, 10, None, None, None, 4, 64, 0, 0.1, 0, None, 0, 0, 0, 0, 0,
                            None) == _lib.QKV_EINVAL  # n_parts null
    assert lib.qkv_combine(None, 2, 4, 128, 16, 0, 0, None) == _lib.QKV_EINVAL
    assert n.value == 0


def test_check_raises_with_message():
    lib = _lib.load()
    rc = lib.qkv_dequantize(16, 16, 16, 16, 4, 100, 4, 64, 0, 0, None)
    with pytest.raises(_lib.QKVError) as e:
        _lib.check(rc)
    assert "head_dim" in str(e.value)


@pytest.mark.parametrize("B,HQ,HKV,S,D,bits", [
    (1, 32, 4, 1, 128, 8), (1, 32, 4, 8, 128, 4), (1, 32, 4, 16, 128, 8), (4, 32, 4, 1, 128, 4),
    (1, 32, 4, 2048, 128, 4), (2, 64, 8, 8, 128, 4),
])
def test_python_workspace_estimate_covers_every_key_count(B, HQ, HKV, S, D, bits):
    """ops.workspace_size memoizes by power-of-two key count: its answer must cover the
    library's exact need at every key count below that power of two."""
    from chad_b200 import ops

    lib = _lib.load()
    for n in list(range(1, 40000, 97)) + [8191, 8192, 8193, 8696, 16384, 16385, 131072]:
        assert ops.workspace_size(B, HQ, HKV, S, D, n, bits) >= \
            lib.qkv_workspace_size(B, HQ, HKV, S, D, n, bits, 64), n


def test_test_hook_arguments_are_checked():
    lib = _lib.load()
    assert lib.qkv_test_hooks(-1, 0) == _lib.QKV_EINVAL
    assert lib.qkv_test_hooks(0, -5) == _lib.QKV_EINVAL
    assert lib.qkv_test_hooks(0, 0) == _lib.QKV_OK


def test_kv_append_rejects_bad_arguments():
    lib = _lib.load()
    # offset + S beyond the padded length, then a bad x dtype
    assert lib.qkv_quantize_append_kv(16, 16, 0, 16, 16, 16, 16, 16, 16, 1, 2, 10, 128, 8, 0, 4,
                                      64, 0, None) == _lib.QKV_EINVAL
    assert lib.qkv_quantize_append_kv(16, 16, 7, 16, 16, 16, 16, 16, 16, 1, 2, 1, 128, 8, 0, 4,
                                      64, 0, None) == _lib.QKV_EINVAL


def test_gather_buffer_size_and_argument_checks():
    lib = _lib.load()
    rows, D, W = 96, 128, 4
    # data [2][world][rows][D+4] 64-bit words (flag, float), seen [rows] u32
    assert lib.qkv_gather_buffer_size(rows, D, W) == 2 * W * rows * (D + 4) * 8 + rows * 4
    assert lib.qkv_gather_buffer_size(rows, 100, W) == 0
    assert lib.qkv_gather_buffer_size(0, D, W) == 0
    E = _lib.QKV_EINVAL

    def call(parts=16, n=rows, d=D, peers=16, mine=16, world=2, rank=0, out=16, dt=0, kind=0):
        return lib.qkv_gather_combine(parts, n, d, peers, mine, world, rank, out, dt, kind, None)

    assert call(parts=None) == E
    assert call(peers=None) == E
    assert call(rank=2) == E
    assert call(world=0) == E
    assert call(world=129, rank=0) == E
    assert call(n=0) == E
    assert call(d=100) == _lib.QKV_EUNSUPPORTED
    assert call(dt=2) == E
    assert call(kind=3) == E
    assert call(parts=8) == _lib.QKV_EALIGN
    p = ctypes.c_void_p()
    assert lib.qkv_peer_alloc(0, ctypes.byref(p), None) == E
    assert lib.qkv_peer_open(None, ctypes.byref(p)) == E
    assert lib.qkv_peer_free(None, 0) == _lib.QKV_OK


def test_python_bindings_match_the_ctypes_table():
    """The CPython bindings of the per-layer calls are built, bound to the loaded library,
    and return the library's own status codes (argument checks run before any GPU work)."""
    ext = _lib.ext()
    assert ext is not None, "chad_b200._qkvext was not built"
    for name, attr in _lib.EXT_BOUND.items():
        assert _lib.fn(name) is getattr(ext, attr)
    lib = _lib.load()
    args = (16, 16, 16, 16, 16, 16, 16, 16, 1, 32, 4, 1, 100, 512, 10, None, None, None, 4, 64,
            0, 0.1, 0, None, 0, 0, 0, 0, 0, 0, 16, 1 << 20, None)  # head_dim 100
    assert ext.attention(*args) == lib.qkv_attention(*args) == _lib.QKV_EUNSUPPORTED
    bad_kind = args[:28] + (7,) + args[29:]
    assert ext.attention(*bad_kind) == lib.qkv_attention(*bad_kind) == _lib.QKV_EINVAL
    assert ext.combine(None, 2, 4, 128, 16, 0, 0, None) == _lib.QKV_EINVAL
    assert ext.gather_combine(None, 4, 128, 16, 16, 2, 0, 16, 0, 0, None) == _lib.QKV_EINVAL
    assert ext.quantize_append_kv(16, 16, 7, 16, 16, 16, 16, 16, 16, 1, 2, 1, 128, 8, 0, 4, 64,
                                  0, None) == _lib.QKV_EINVAL
    with pytest.raises(TypeError):
        ext.attention(*args[:-1])
    with pytest.raises(OverflowError):
        ext.combine(None, 1 << 40, 4, 128, 16, 0, 0, None)
