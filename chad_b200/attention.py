"""The attention seam: ``scaled_dot_product_attention(queries, keys, values, cache, scale,
mask=None, sinks=None)``.

This is the B200 counterpart of mlx-lm's ``mlx_lm.models.base.scaled_dot_product_attention``,
the function the reference monkeypatches (src/chad/mlx_qsdpa.py:741-780). The function
defined here is the *stock* behaviour; ``chad_b200.qsdpa.install()`` replaces it (and every
module-level binding of it under ``chad_b200.``) with the fused-kernel router.

Stock behaviour, on the GPU with torch:
* plain caches / raw tensors: torch SDPA over (B, HQ, S, D) x (B, HKV, N, D) with GQA;
* quantized caches: dequantize the valid keys/values, then the same SDPA — the unfused
  route mlx-lm takes for quantized caches the reference's kernel does not cover.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import ops


def _sdpa(q, k, v, scale, mask):
    hq, hkv = q.shape[1], k.shape[1]
    if hq != hkv:
        k = k.repeat_interleave(hq // hkv, dim=1)
        v = v.repeat_interleave(hq // hkv, dim=1)
    s, n = q.shape[2], k.shape[2]
    attn_mask = None
    if isinstance(mask, str):
        if mask != "causal":
            raise ValueError(mask)
        qi = torch.arange(n - s, n, device=q.device)[:, None]
        ki = torch.arange(n, device=q.device)[None, :]
        attn_mask = ki <= qi
    elif mask is not None:
        attn_mask = mask[..., :n] if mask.dtype == torch.bool else mask[..., :n].to(q.dtype)
    return F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, scale=scale)


def scaled_dot_product_attention(queries, keys, values, cache=None, scale=1.0, mask=None,
                                 sinks=None):
    if sinks is not None:
        raise NotImplementedError("attention sinks are not supported by this seam")
    bits = getattr(cache, "bits", None)
    if isinstance(keys, (tuple, list)):
        if bits is None:
            raise ValueError("quantized keys need a cache carrying .bits")
        gs = getattr(cache, "group_size", ops.GROUP_SIZE)
        kd = ops.dequantize(*(t.contiguous() for t in keys), bits, gs)
        vd = ops.dequantize(*(t.contiguous() for t in values), bits, gs)
        return _sdpa(queries, kd, vd, scale, mask)
    return _sdpa(queries, keys, values, scale, mask)
