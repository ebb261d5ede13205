"""Torch-tensor front end of the C ABI (libqkv.so).

Tensors only carry device memory and streams here: every function passes raw pointers to
the CUDA library and enqueues on torch's current stream.
"""

from __future__ import annotations

import contextlib
import ctypes
import functools
import math
import os
from typing import Optional, Sequence, Tuple, Union

import torch

from . import _lib
from ._lib import check

GROUP_SIZE = 64
# Opt-in: read the device status word after every attention call (synchronizes the stream;
# for debugging — the default reads it only when device_status()/check_device() is called).
CHECK_EACH_CALL = bool(os.environ.get("CHAD_QKV_CHECK"))


class DeviceWaitError(RuntimeError):
    """A kernel gave up on a bounded wait (QKV_EDEVICE): its output is not trustworthy.
    The cached workspaces of the device have been zeroed again, so later calls are."""
_DT = {torch.bfloat16: _lib.QKV_BF16, torch.float16: _lib.QKV_F16, torch.float32: _lib.QKV_F32}

QuantTuple = Tuple[torch.Tensor, torch.Tensor, torch.Tensor]


def dtype_code(t: Union[torch.Tensor, torch.dtype]) -> int:
    dt = t.dtype if isinstance(t, torch.Tensor) else t
    if dt not in _DT:
        raise TypeError(f"unsupported dtype {dt}")
    return _DT[dt]


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    # the raw handle of torch's current stream, without building a Stream object per call
    if _RAW_STREAM is not None:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return _RAW_STREAM(idx)
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


_DEVICES = {}


def _need_cuda(*ts: torch.Tensor) -> torch.device:
    idx = None
    for t in ts:
        if t is None:
            continue
        d = t.get_device()  # -1 on the CPU; an int compare is cheaper than torch.device objects
        if d < 0:
            raise ValueError("libqkv operates on CUDA tensors only")
        if idx is None:
            idx = d
        elif d != idx:
            raise ValueError("tensors are on different devices")
    if idx is None:
        return None
    dev = _DEVICES.get(idx)
    if dev is None:
        dev = _DEVICES[idx] = torch.device("cuda", idx)
    return dev


def _on(dev: torch.device):
    """Context making `dev` current; a no-op when it already is (the common case: switching
    devices on every call costs more than the rest of the host-side work)."""
    if dev.index is None or dev.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(dev)


def _contig(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


# --------------------------------------------------------------------------------------
# quantization
# --------------------------------------------------------------------------------------

def quantize_append(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor,
                    biases: torch.Tensor, offset: int, bits: int,
                    group_size: int = GROUP_SIZE) -> None:
    """Quantize x (B, H, S, D) into the padded cache buffers at positions [offset, offset+S)."""
    dev = _need_cuda(x, w, scales, biases)
    _contig(x, "x"), _contig(w, "w"), _contig(scales, "scales"), _contig(biases, "biases")
    b, h, s, d = x.shape
    np_ = w.shape[2]
    lib = _lib.load()
    with _on(dev):
        check(lib.qkv_quantize_append(x.data_ptr(), dtype_code(x), w.data_ptr(),
                                      scales.data_ptr(), biases.data_ptr(), b, h, s, d, np_,
                                      offset, bits, group_size, dtype_code(scales),
                                      _stream(dev)))


def quantize_append_kv(k: torch.Tensor, v: torch.Tensor, k_quant: Sequence[torch.Tensor],
                       v_quant: Sequence[torch.Tensor], offset: int, bits: int,
                       group_size: int = GROUP_SIZE) -> None:
    """Quantize k and v (B, H, S, D) into their cache buffers at [offset, offset+S), one
    launch for both."""
    dev = _need_cuda(k, v, *k_quant, *v_quant)
    for t, nm in ((k, "k"), (v, "v"), *((t, "cache") for t in (*k_quant, *v_quant))):
        _contig(t, nm)
    if k.shape != v.shape or k.dtype != v.dtype:
        raise ValueError("k and v must share shape and dtype")
    b, h, s, d = k.shape
    np_ = k_quant[0].shape[2]
    kw, ks, kb = k_quant
    vw, vs, vb = v_quant
    with _on(dev):
        check(_lib.fn("qkv_quantize_append_kv")(
            k.data_ptr(), v.data_ptr(), dtype_code(k), kw.data_ptr(), ks.data_ptr(),
            kb.data_ptr(), vw.data_ptr(), vs.data_ptr(), vb.data_ptr(), b, h, s, d, np_, offset,
            bits, group_size, dtype_code(ks), _stream(dev)))


def quantize(x: torch.Tensor, bits: int, group_size: int = GROUP_SIZE,
             scale_dtype: Optional[torch.dtype] = None) -> QuantTuple:
    """mx.quantize equivalent on the GPU: (w uint32, scales, biases) for x (..., D)."""
    *lead, d = x.shape
    rows = int(math.prod(lead)) if lead else 1
    sd = scale_dtype or (x.dtype if x.dtype != torch.float32 else torch.bfloat16)
    x4 = x.reshape(1, 1, rows, d).contiguous()
    w = torch.empty((1, 1, rows, d * bits // 32), dtype=torch.int32, device=x.device)
    sc = torch.empty((1, 1, rows, d // group_size), dtype=sd, device=x.device)
    bi = torch.empty_like(sc)
    quantize_append(x4, w, sc, bi, 0, bits, group_size)
    return (w.view(*lead, -1), sc.view(*lead, -1), bi.view(*lead, -1))


def dequantize(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, bits: int,
               group_size: int = GROUP_SIZE, round_mode: int = 0) -> torch.Tensor:
    """mx.dequantize equivalent: values in the scale dtype, shape (..., D)."""
    dev = _need_cuda(w, scales, biases)
    d = w.shape[-1] * 32 // bits
    rows = w.numel() // w.shape[-1]
    out = torch.empty((*w.shape[:-1], d), dtype=scales.dtype, device=w.device)
    lib = _lib.load()
    with _on(dev):
        check(lib.qkv_dequantize(_contig(w, "w").data_ptr(), _contig(scales, "scales").data_ptr(),
                                 _contig(biases, "biases").data_ptr(), out.data_ptr(), rows, d,
                                 bits, group_size, dtype_code(scales), round_mode, _stream(dev)))
    return out


# --------------------------------------------------------------------------------------
# attention
# --------------------------------------------------------------------------------------

_WS = {}


def workspace_size(B: int, HQ: int, HKV: int, S: int, D: int, n_max: int, bits: int,
                   group_size: int = GROUP_SIZE, device: Optional[int] = None) -> int:
    """Workspace bytes for calls with up to n_max keys. The need grows with n_max, so it is
    asked for the next power of two: a decode loop, whose key count grows by one per step,
    hits the memoized value instead of calling into the library every step."""
    if device is None:
        device = torch.cuda.current_device() if torch.cuda.is_available() else -1
    n = max(256, 1 << (max(n_max, 1) - 1).bit_length())  # next power of two, at least 256
    return _workspace_size(device, B, HQ, HKV, S, D, n, bits, group_size)


@functools.lru_cache(maxsize=4096)
def _workspace_size(device: int, B: int, HQ: int, HKV: int, S: int, D: int, n_max: int,
                    bits: int, group_size: int) -> int:
    # the split plan depends on the current device's SM count: memoized per device
    return int(_lib.load().qkv_workspace_size(B, HQ, HKV, S, D, n_max, bits, group_size))


def _workspace(dev: torch.device, nbytes: int) -> torch.Tensor:
    key = (dev.type, dev.index)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        # zeroed once: the in-kernel merge reads a zero word as "not yet written" (every
        # call leaves the workspace zero again)
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _WS[key] = ws
    return ws


def _mask_args(mask, q: torch.Tensor, n_keys: int):
    """-> (kind, tensor or None, mask_nk, sb, sh, sq)."""
    if mask is None:
        return _lib.QKV_MASK_NONE, None, 0, 0, 0, 0
    if isinstance(mask, str):
        if mask != "causal":
            raise ValueError(f"unknown mask {mask!r}")
        return _lib.QKV_MASK_CAUSAL, None, 0, 0, 0, 0
    m = mask
    if m.dtype == torch.bool:
        m = m.to(torch.uint8)
        kind = _lib.QKV_MASK_BOOL
    else:
        m = m.to(q.dtype)
        kind = _lib.QKV_MASK_ADDITIVE
    while m.dim() < 4:
        m = m.unsqueeze(0)
    if m.stride(-1) != 1:
        m = m.contiguous()
    b, hq, s, _ = q.shape
    sb = m.stride(0) if m.shape[0] > 1 else 0
    sh = m.stride(1) if m.shape[1] > 1 else 0
    sq = m.stride(2) if m.shape[2] > 1 else 0
    if (m.shape[0] not in (1, b)) or (m.shape[1] not in (1, hq)) or (m.shape[2] not in (1, s)):
        raise ValueError(f"mask shape {tuple(mask.shape)} does not broadcast to {(b, hq, s, n_keys)}")
    if m.shape[3] < n_keys:
        raise ValueError(f"mask covers {m.shape[3]} keys < {n_keys}")
    return kind, m, m.shape[3], sb, sh, sq


def attention(q: torch.Tensor, k_quant: Sequence[torch.Tensor], v_quant: Sequence[torch.Tensor],
              scale: float, n: int, bits: int, *, lens: Optional[torch.Tensor] = None,
              mask=None, out: Optional[torch.Tensor] = None, out_kind: int = 0,
              pos_base: Optional[torch.Tensor] = None, total_lens: Optional[torch.Tensor] = None,
              splits: int = 0, group_size: int = GROUP_SIZE,
              workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention of q (B, HQ, S, D) over full padded cache tuples (w, scales, biases).

    n: valid key count (the upper bound of `lens` when per-batch lengths are given).
    out_kind 0 returns (B, HQ, S, D) in q's dtype; 1 returns fp32 partial rows
    (B, HQ, S, D+4) = [out(D), max (log2 units), sum, 0, 0].
    """
    kw, ks, kb = k_quant
    vw, vs, vb = v_quant
    dev = _need_cuda(q, kw, ks, kb, vw, vs, vb, lens, pos_base, total_lens)
    if not (q.is_contiguous() and kw.is_contiguous() and ks.is_contiguous()
            and kb.is_contiguous() and vw.is_contiguous() and vs.is_contiguous()
            and vb.is_contiguous()):
        raise ValueError("q and the quantized cache tensors must be contiguous")
    B, HQ, S, D = q.shape
    _, HKV, NP = kw.shape[:3]
    if out is None:
        if out_kind == _lib.QKV_OUT_NORMALIZED:
            out = torch.empty_like(q)
        else:
            out = torch.empty((B, HQ, S, D + 4), dtype=torch.float32, device=q.device)
    kind, m, mnk, sb, sh, sq = _mask_args(mask, q, n)
    for t in (lens, pos_base, total_lens):
        if t is not None and t.dtype != torch.int32:
            raise TypeError("lens/pos_base/total_lens must be int32")
    idx = dev.index
    if workspace is None:
        need = workspace_size(B, HQ, HKV, S, D, max(n, 1), bits, group_size, idx)
        if splits:
            # forced split count: rows of at most D + 16 floats per split (D + 2*D/32 merged)
            need = max(need, splits * B * HQ * S * (D + 16) * 4 + (1 << 16))
        workspace = _workspace(dev, need)
    fn = _lib.fn("qkv_attention")
    switch = idx != torch.cuda.current_device()
    with (torch.cuda.device(dev) if switch else contextlib.nullcontext()):
        check(fn(q.data_ptr(), kw.data_ptr(), ks.data_ptr(), kb.data_ptr(), vw.data_ptr(),
                 vs.data_ptr(), vb.data_ptr(), out.data_ptr(), B, HQ, HKV, S, D, NP, n,
                 _ptr(lens), _ptr(pos_base), _ptr(total_lens), bits, group_size, dtype_code(q),
                 float(scale), kind, _ptr(m), mnk, sb, sh, sq, out_kind, splits,
                 workspace.data_ptr(), workspace.numel(),
                 _RAW_STREAM(idx) if _RAW_STREAM is not None else _stream(dev)))
        if CHECK_EACH_CALL:
            check_device()
    return out


def partials(q: torch.Tensor, k_quant: Sequence[torch.Tensor], v_quant: Sequence[torch.Tensor],
             scale: float, n: int, bits: int, *, lens: Optional[torch.Tensor] = None,
             mask=None, parts: Optional[torch.Tensor] = None, splits: int = 0,
             pos_base: Optional[torch.Tensor] = None, total_lens: Optional[torch.Tensor] = None,
             group_size: int = GROUP_SIZE) -> torch.Tensor:
    """Pass 1 only: per-split partial rows (P, B, HQ, S, D+4) fp32, un-merged."""
    kw, ks, kb = k_quant
    vw, vs, vb = v_quant
    dev = _need_cuda(q, kw, ks, kb, vw, vs, vb, lens, pos_base, total_lens)
    B, HQ, S, D = q.shape
    HKV, NP = kw.shape[1], kw.shape[2]
    need = workspace_size(B, HQ, HKV, S, D, max(n, 1), bits, group_size, dev.index)
    if splits:
        # forced split count: rows of at most D + 16 floats per split (D + 2*D/32 merged)
        need = max(need, splits * B * HQ * S * (D + 16) * 4 + (1 << 16))
    if parts is None:
        parts = torch.empty(need // 4, dtype=torch.float32, device=q.device)
    kind, m, mnk, sb, sh, sq = _mask_args(mask, q, n)
    np_out = ctypes.c_int(0)
    with _on(dev):
        check(_lib.load().qkv_partials(
            q.data_ptr(), kw.data_ptr(), ks.data_ptr(), kb.data_ptr(), vw.data_ptr(),
            vs.data_ptr(), vb.data_ptr(), parts.data_ptr(), parts.numel() * parts.element_size(),
            ctypes.byref(np_out), B, HQ, HKV, S, D, NP, n, _ptr(lens), _ptr(pos_base),
            _ptr(total_lens), bits, group_size, dtype_code(q), float(scale), kind, _ptr(m), mnk,
            sb, sh, sq, splits, _stream(dev)))
    p = np_out.value
    return parts.view(-1)[: p * B * HQ * S * (D + 4)].view(p, B, HQ, S, D + 4)


def combine(parts: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16,
            out_kind: int = 0) -> torch.Tensor:
    """LSE-merge partial rows: parts (P, rows..., D+4) fp32 -> (rows..., D) or a merged partial."""
    dev = _need_cuda(parts)
    _contig(parts, "parts")
    p = parts.shape[0]
    d = parts.shape[-1] - 4
    rows = parts[0].numel() // (d + 4)
    if out_kind == _lib.QKV_OUT_NORMALIZED:
        out = torch.empty((*parts.shape[1:-1], d), dtype=out_dtype, device=parts.device)
    else:
        out = torch.empty(parts.shape[1:], dtype=torch.float32, device=parts.device)
    with _on(dev):
        check(_lib.fn("qkv_combine")(parts.data_ptr(), p, rows, d, out.data_ptr(),
                                      dtype_code(out_dtype), out_kind, _stream(dev)))
    return out


def prefill(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
            k_quant: Sequence[torch.Tensor], v_quant: Sequence[torch.Tensor], offset: int,
            bits: int, scale: float, group_size: int = GROUP_SIZE,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Quantize-append the new chunk at [offset, offset+S) then attend causally over all keys
    (one library call; S = 1 is a decode step)."""
    # one call per layer per decode step: the host work here is kept to plain attribute reads
    kw, ks, kb = k_quant
    vw, vs, vb = v_quant
    dev = _need_cuda(q, k_new, v_new, kw)
    if not (q.is_contiguous() and k_new.is_contiguous() and v_new.is_contiguous()):
        raise ValueError("q, k_new and v_new must be contiguous")
    B, HQ, S, D = q.shape
    _, HKV, NP = kw.shape[:3]
    if out is None:
        out = torch.empty_like(q)
    idx = dev.index
    dt = _DT.get(q.dtype)
    if dt is None:
        raise TypeError(f"unsupported dtype {q.dtype}")
    ws = _workspace(dev, workspace_size(B, HQ, HKV, S, D, offset + S, bits, group_size, idx))
    fn = _lib.fn("qkv_prefill")
    switch = idx != torch.cuda.current_device()
    with (torch.cuda.device(dev) if switch else contextlib.nullcontext()):
        check(fn(q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), kw.data_ptr(), ks.data_ptr(),
                 kb.data_ptr(), vw.data_ptr(), vs.data_ptr(), vb.data_ptr(), out.data_ptr(), B,
                 HQ, HKV, S, D, NP, offset, bits, group_size, dt, float(scale), ws.data_ptr(),
                 ws.numel(), _RAW_STREAM(idx) if _RAW_STREAM is not None else _stream(dev)))
        if CHECK_EACH_CALL:
            check_device()
    return out


def device_status(reset: bool = True) -> int:
    """Device status word of the current device (0 = no kernel gave up on a bounded wait).
    Synchronizes torch's current stream. With reset, a non-zero word is cleared and every
    workspace this module cached for the device is zeroed again (a merge that gave up may
    have left partial words behind, which the next call would read as written); the library
    zeroes the static scratch of qkv_attention_noalloc itself."""
    dev = torch.device("cuda", torch.cuda.current_device())
    v = int(_lib.load().qkv_device_status(_stream(dev), 1 if reset else 0))
    if v < 0 and v > -1000:  # the call itself failed (not a status word)
        check(v)
    if v != 0 and reset:
        ws = _WS.get((dev.type, dev.index))
        if ws is not None:
            ws.zero_()
    return v


def check_device() -> None:
    """Raise DeviceWaitError if a kernel on the current device gave up on a bounded wait
    since the last check (after resetting the status and zeroing the cached workspaces)."""
    v = device_status(reset=True)
    if v != 0:
        raise DeviceWaitError(
            f"a libqkv kernel gave up on a bounded wait (status {v}): outputs since the last "
            "check are not trustworthy; the workspace has been zeroed")
