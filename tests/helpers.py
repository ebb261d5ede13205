"""Shared helpers for the test-suite: seeded inputs and numpy <-> torch bit transfers."""

from __future__ import annotations

import numpy as np

from oracle import qkv_oracle as orc

DT = {"bf16": "bfloat16", "f16": "float16"}


def torch_from_f32(x: np.ndarray, dtype: str, device="cuda"):
    """float32 numpy values (already representable in `dtype`) -> torch tensor of dtype."""
    import torch

    if dtype == "f32":
        return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(device)
    bits = orc.to_bits(x, dtype)
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(getattr(torch, DT[dtype])).to(device)


def torch_from_bits(bits: np.ndarray, dtype: str, device="cuda"):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(getattr(torch, DT[dtype])).to(device)


def bits_of(t) -> np.ndarray:
    """torch 16-bit float tensor -> uint16 bit patterns."""
    import torch

    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def u32_of(t) -> np.ndarray:
    return t.detach().cpu().contiguous().numpy().view(np.uint32)


def f32_of(t) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def make_case(seed, B, HQ, HKV, S, D, n, dtype="bf16", kv_scale=1.0, outliers=False,
              kv_dtype=None):
    """q (B,HQ,S,D) and k, v (B,HKV,n,D) as float32 arrays holding `dtype` values."""
    rng = np.random.default_rng(seed)
    q = orc.round_to(rng.standard_normal((B, HQ, S, D), dtype=np.float32), dtype)
    kd = kv_dtype or dtype
    k = orc.make_kv(rng, (B, HKV, n, D), outliers=outliers, dtype="f32") * np.float32(kv_scale)
    v = orc.make_kv(rng, (B, HKV, n, D), outliers=False, dtype="f32") * np.float32(kv_scale)
    if kd != "f32":
        k = orc.round_to(k, kd)
        v = orc.round_to(v, kd)
    return q, k, v
