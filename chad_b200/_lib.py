"""ctypes binding of libqkv.so (the C ABI declared in include/qkv.h).

The shared library is the only compute path: if it is missing this module raises, it never
substitutes anything else.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqkv.so")

QKV_OK = 0
QKV_EINVAL = -1
QKV_EUNSUPPORTED = -2
QKV_ECUDA = -3
QKV_EWORKSPACE = -4
QKV_EALIGN = -5
QKV_EDEVICE = -6

QKV_BF16, QKV_F16, QKV_F32 = 0, 1, 2
QKV_MASK_NONE, QKV_MASK_CAUSAL, QKV_MASK_BOOL, QKV_MASK_ADDITIVE = 0, 1, 2, 3
QKV_OUT_NORMALIZED, QKV_OUT_PARTIAL = 0, 1
QKV_IPC_HANDLE_BYTES = 64  # size of a CUDA IPC memory handle (qkv_peer_alloc)

# every symbol include/qkv.h declares, with (restype, argtypes)
_vp, _i, _ll, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "qkv_version": (_i, []),
    "qkv_last_error": (ctypes.c_char_p, []),
    "qkv_device_status": (_i, [_vp, _i]),
    "qkv_test_hooks": (_i, [_i, _ll]),
    "qkv_quantize_append": (_i, [_vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "qkv_quantize_append_kv": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp,
                                    _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "qkv_dequantize": (_i, [_vp, _vp, _vp, _vp, _ll, _i, _i, _i, _i, _i, _vp]),
    "qkv_workspace_size": (_sz, [_i, _i, _i, _i, _i, _i, _i, _i]),
    "qkv_attention": (
        _i,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,  # q, kw, ks, kb, vw, vs, vb, out
         _i, _i, _i, _i, _i, _i, _i,  # B HQ HKV S D NP n
         _vp, _vp, _vp,  # lens pos_base total_lens
         _i, _i, _i, _f,  # bits group_size dtype scale
         _i, _vp, _i, _ll, _ll, _ll,  # mask_kind mask mask_nk strides
         _i, _i, _vp, _sz, _vp],  # out_kind splits workspace ws_bytes stream
    ),
    "qkv_partials": (
        _i,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp,  # q, kw, ks, kb, vw, vs, vb
         _vp, _sz, ctypes.POINTER(ctypes.c_int),  # parts parts_bytes n_parts
         _i, _i, _i, _i, _i, _i, _i,  # B HQ HKV S D NP n
         _vp, _vp, _vp,  # lens pos_base total_lens
         _i, _i, _i, _f,  # bits group_size dtype scale
         _i, _vp, _i, _ll, _ll, _ll,  # mask
         _i, _vp],  # splits stream
    ),
    "qkv_attention_noalloc": (
        _i,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,  # q, kw, ks, kb, vw, vs, vb, out
         _i, _i, _i, _i, _i, _i, _i,  # B HQ HKV S D NP n
         _vp, _vp, _vp,  # lens pos_base total_lens
         _i, _i, _i, _f,  # bits group_size dtype scale
         _i, _vp, _i, _ll, _ll, _ll,  # mask_kind mask mask_nk strides
         _i, _i, _vp],  # out_kind splits stream
    ),
    "qkv_combine": (_i, [_vp, _i, _ll, _i, _vp, _i, _i, _vp]),
    "qkv_gather_buffer_size": (_sz, [_ll, _i, _i]),
    "qkv_gather_combine": (_i, [_vp, _ll, _i, _vp, _vp, _i, _i, _vp, _i, _i, _vp]),
    "qkv_peer_alloc": (_i, [_sz, _vp, _vp]),
    "qkv_peer_open": (_i, [_vp, _vp]),
    "qkv_peer_free": (_i, [_vp, _i]),
    "qkv_prefill": (
        _i,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
         _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _sz, _vp],
    ),
}

_lib = None
_ext = None
_lock = threading.Lock()
# entry points with CPython bindings (chad_b200._qkvext): the per-layer calls
EXT_BOUND = {"qkv_attention": "attention", "qkv_prefill": "prefill",
             "qkv_quantize_append_kv": "quantize_append_kv", "qkv_combine": "combine",
             "qkv_gather_combine": "gather_combine"}


class QKVError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"libqkv error {code}: {msg}")
        self.code = code


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libqkv.so once; raise if it is absent (there is no other implementation)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(
                    f"{path} is missing: build it with `python -m chad_b200.build` "
                    "(the quantized-KV attention path has no non-CUDA implementation)")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _bind_ext(lib)
            _lib = lib
    return _lib


def _bind_ext(lib) -> None:
    """Point the CPython bindings at this library instance (same ABI as the ctypes table,
    a fraction of its per-call cost); without them every call goes through ctypes."""
    global _ext
    try:
        from . import _qkvext
    except ImportError:
        _ext = None
        return
    for name in EXT_BOUND:
        _qkvext.bind(name, ctypes.cast(getattr(lib, name), ctypes.c_void_p).value)
    _ext = _qkvext


def fn(name: str):
    """The callable for entry point `name`: its CPython binding when built, else ctypes."""
    lib = load()
    if _ext is not None and name in EXT_BOUND:
        return getattr(_ext, EXT_BOUND[name])
    return getattr(lib, name)


def ext():
    """The CPython bindings module bound to the loaded library, or None if not built."""
    load()
    return _ext


def check(rc: int) -> None:
    if rc != QKV_OK:
        msg = load().qkv_last_error()
        raise QKVError(rc, msg.decode() if msg else "")
