"""Fused quantized-KV attention on B200 — the host-side mirror of the reference's
``src/chad/mlx_qsdpa.py`` (same names, argument meaning and error behaviour).

* ``qsdpa(q, k_quant, v_quant, scale, n)`` — attention of q over the FULL padded cache
  buffers with a runtime valid length, as at mlx_qsdpa.py:572-630. Any S (decode, verify,
  prefill) and any GQA; the kernels live in libqkv.so.
* ``covers(head_dim, gqa)`` / ``_eligible(q, cache, mask)`` — the contract gate
  (mlx_qsdpa.py:485-488, 633-658), widened to what the B200 kernels handle: head_dim 64,
  128 or 256, 4- or 8-bit group-64 codes, fp16/bf16, any GQA, S >= 1, mask None /
  "causal" / bool / additive arrays.
* ``kernel_healthy()`` — one-time numeric self-check (mlx_qsdpa.py:661-719): the same six
  probe shapes, compared against a dequantize -> fp32 torch reference on the GPU. A failed
  or NaN-producing kernel makes ``install()`` refuse.
* ``install()`` — replaces ``chad_b200.attention.scaled_dot_product_attention`` and every
  module-level binding of it under ``chad_b200.`` with the fused router; idempotent;
  returns False under ``CHAD_NO_QSDPA`` or when the self-check fails (mlx_qsdpa.py:722-782).

Deliberate difference from the reference: when a fused kernel reports an error the router
raises instead of silently dropping to the stock path, so a broken CUDA library can never
hide behind a fallback. Ineligible calls (non-quantized caches, sinks, unsupported shapes)
go to the stock seam exactly as in the reference.
"""

from __future__ import annotations

import logging
import os
import sys
from typing import Any, Optional

import torch

from . import attention as _attention
from . import ops

log = logging.getLogger("chad")

_GQAS_REF = (4, 8)   # the reference's covered GQA factors, kept for _pick_blocks' table
_DIMS = (64, 128, 256)
_BITS = (4, 8)


def _flag(name: str) -> bool:
    """A CHAD_* boolean: truthy iff set to a non-empty value (src/chad/config.py:20-25)."""
    return bool(os.environ.get(name))


def covers(head_dim: int, gqa: int, bits: int = 8) -> bool:
    """True iff the B200 kernels handle this attention shape."""
    return head_dim in _DIMS and gqa >= 1 and bits in _BITS


def _pick_blocks(n: int, gqa: int = 8) -> int:
    """The reference's split table (mlx_qsdpa.py:534-569): 32 below 16k, then 64 at gqa 8
    and 128 at gqa 4. Apple-tuned; kept so callers porting split counts get the same
    numbers. The B200 kernel sizes its split from the SM count unless given one."""
    if n >= 16384:
        return 128 if gqa == 4 else 64
    return 32


def qsdpa(q: torch.Tensor, k_quant: tuple, v_quant: tuple, scale: float, n: int,
          mask: Any = None, bits: Optional[int] = None, splits: int = 0) -> torch.Tensor:
    """Fused attention over full padded QuantizedKVCache buffers.

    q: (B, HQ, S, D); k_quant/v_quant: (w, scales, biases) with seq length NP >= n;
    n: valid positions. `bits` defaults to what the packed width implies.
    """
    d = q.shape[-1]
    if bits is None:
        bits = k_quant[0].shape[-1] * 32 // d
    return ops.attention(q.contiguous(), tuple(t.contiguous() for t in k_quant),
                         tuple(t.contiguous() for t in v_quant), scale, n, bits, mask=mask,
                         splits=splits)


def _eligible(q: Any, cache: Any, mask: Any) -> bool:
    """True iff this call is one the fused kernels handle."""
    if mask is not None and not isinstance(mask, (str, torch.Tensor)):
        return False
    if isinstance(mask, str) and mask != "causal":
        return False
    if not isinstance(q, torch.Tensor) or q.ndim != 4 or q.shape[2] < 1:
        return False
    if q.dtype not in (torch.float16, torch.bfloat16) or not q.is_cuda:
        return False
    if getattr(cache, "bits", None) not in _BITS or getattr(cache, "group_size", None) != 64:
        return False
    keys = getattr(cache, "keys", None)
    if keys is None or cache.offset <= 0:
        return False
    kw, ks, _ = keys
    if kw.ndim != 4 or kw.shape[1] == 0 or q.shape[1] % kw.shape[1]:
        return False
    if q.shape[3] not in _DIMS or kw.shape[3] != q.shape[3] * cache.bits // 32:
        return False
    if ks.dtype != q.dtype:
        return False
    if cache.offset > kw.shape[2] or kw.shape[2] % 8:
        return False
    return True


_KERNEL_HEALTHY: Optional[bool] = None


def _reference_gpu(q, kq, vq, scale, n, bits):
    """dequantize -> fp32 reference on the GPU (the check kernel_healthy compares with)."""
    kd = ops.dequantize(*kq, bits)[..., :n, :].float()
    vd = ops.dequantize(*vq, bits)[..., :n, :].float()
    b, hq, s, d = q.shape
    hkv = kd.shape[1]
    qf = (q.float() * scale).reshape(b, hkv, hq // hkv, s, d)
    sc = qf @ kd.unsqueeze(2).transpose(-1, -2)
    p = torch.softmax(sc, dim=-1)
    return (p @ vd.unsqueeze(2)).reshape(b, hq, s, d)


def kernel_healthy() -> bool:
    """One-time numeric self-check of the fused kernel on the probe shapes of
    mlx_qsdpa.py:689-692 (hkv, n, dtype, tol), at head_dim 256 and 128, 8- and 4-bit.
    Cached per process; NaN fails the `err < tol` test by construction."""
    global _KERNEL_HEALTHY
    if _KERNEL_HEALTHY is not None:
        return _KERNEL_HEALTHY
    if not torch.cuda.is_available():
        _KERNEL_HEALTHY = False
        return False
    from .cache import QuantizedKVCache

    cases = ((2, 3, torch.float16, 4e-3), (2, 3, torch.bfloat16, 1.6e-2),
             (4, 3, torch.float16, 4e-3), (2, 100, torch.float16, 4e-3),
             (2, 2570, torch.float16, 4e-3), (2, 2570, torch.bfloat16, 1.6e-2))
    try:
        for d, bits in ((256, 8), (128, 4)):
            for hkv, n, dtype, tol in cases:
                g = torch.Generator(device="cuda").manual_seed(7)
                q = torch.randn((1, 16, 1, d), generator=g, device="cuda").to(dtype)
                k = (0.7 * torch.randn((1, hkv, n, d), generator=g, device="cuda")).to(dtype)
                v = (0.7 * torch.randn((1, hkv, n, d), generator=g, device="cuda")).to(dtype)
                c = QuantizedKVCache(group_size=64, bits=bits)
                c.update_and_fetch(k, v)
                out = qsdpa(q, c.keys, c.values, d ** -0.5, n)
                ref = _reference_gpu(q, c.keys, c.values, d ** -0.5, n, bits)
                err = (out.float() - ref).abs().max().item()
                if not err < tol * (2 if bits == 4 else 1):
                    log.warning("QSDPA self-check FAILED (d=%d bits=%d hkv=%d n=%d %s: err=%s, "
                                "tol=%s); refusing to install", d, bits, hkv, n, dtype, err, tol)
                    _KERNEL_HEALTHY = False
                    return False
    except Exception as e:  # noqa: BLE001 — a broken probe means an unusable kernel
        log.warning("QSDPA self-check errored (%s); refusing to install", e)
        _KERNEL_HEALTHY = False
        return False
    _KERNEL_HEALTHY = True
    return True


def install() -> bool:
    """Route eligible quantized-cache attention calls through the fused kernels."""
    if _flag("CHAD_NO_QSDPA"):
        return False
    if getattr(_attention.scaled_dot_product_attention, "_chad_qsdpa", False):
        return True  # already installed
    try:
        from . import _lib
        _lib.load()
    except Exception as e:  # noqa: BLE001
        log.warning("QSDPA unavailable: %s", e)
        return False
    if not kernel_healthy():
        log.warning("QSDPA disabled: numeric self-check failed; stock attention stays")
        return False

    stock = _attention.scaled_dot_product_attention
    from .cache import QuantizedKVCache

    def patched(queries, keys, values, cache=None, scale=1.0, mask=None, sinks=None):
        if sinks is None and type(cache) is QuantizedKVCache and _eligible(queries, cache, mask):
            # the cache's FULL padded buffers with a runtime valid length: the sliced
            # views in keys/values would force a contiguity copy per call
            return qsdpa(queries, cache.keys, cache.values, scale, cache.offset, mask=mask,
                         bits=cache.bits)
        return stock(queries, keys, values, cache=cache, scale=scale, mask=mask, sinks=sinks)

    patched._chad_qsdpa = True  # type: ignore[attr-defined]
    patched._stock = stock  # type: ignore[attr-defined]
    _attention.scaled_dot_product_attention = patched
    for mod_name, mod in list(sys.modules.items()):
        if (mod_name.startswith("chad_b200.")
                and getattr(mod, "scaled_dot_product_attention", None) is stock):
            setattr(mod, "scaled_dot_product_attention", patched)
    log.info("QSDPA installed: fused quantized-KV attention (sm_100a)")
    return True


def uninstall() -> None:
    """Undo install() (test helper)."""
    cur = _attention.scaled_dot_product_attention
    stock = getattr(cur, "_stock", None)
    if stock is None:
        return
    _attention.scaled_dot_product_attention = stock
    for mod_name, mod in list(sys.modules.items()):
        if mod_name.startswith("chad_b200.") and getattr(mod, "scaled_dot_product_attention",
                                                          None) is cur:
            setattr(mod, "scaled_dot_product_attention", stock)
