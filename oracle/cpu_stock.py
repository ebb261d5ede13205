"""torch-CPU restatement of the reference's attention path over a quantized cache — TEST /
CPU BASELINE INFRASTRUCTURE ONLY (timed by bench.py's cpu_baseline and --impl reference legs;
checked against qkv_oracle in tests; never imported by the product).

It follows the stock route the reference takes where its fused kernel declines
(src/chad/mlx_qsdpa.py:3-8, 751-771; tests/test_mlx_qsdpa.py:52-65): dequantize the
cache (scale*code+bias per group of 64, rounded to the storage dtype), then
softmax((q*scale) K^T) V in float32, on the host cores with all available threads.
PARITY UNPINNED (see qkv_oracle): MLX itself cannot run here.
"""

from __future__ import annotations

import torch


def dequantize(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, bits: int,
               group_size: int = 64) -> torch.Tensor:
    """(…, W) int32 codes + (…, G) scales/biases -> (…, D) in the scale dtype (CPU)."""
    per = 32 // bits
    shifts = torch.arange(per, dtype=torch.int32) * bits
    c = (w.to(torch.int32).unsqueeze(-1) >> shifts) & ((1 << bits) - 1)
    c = c.reshape(*w.shape[:-1], -1).to(torch.float32)
    d = c.shape[-1]
    c = c.view(*w.shape[:-1], d // group_size, group_size)
    v = c * scales.to(torch.float32).unsqueeze(-1) + biases.to(torch.float32).unsqueeze(-1)
    return v.view(*w.shape[:-1], d).to(scales.dtype)


def attention(q: torch.Tensor, kq, vq, scale: float, n: int, bits: int,
              group_size: int = 64, causal: bool = False, q_pos0=None) -> torch.Tensor:
    """q (B, HQ, S, D) CPU; kq/vq (w, scales, biases) CPU with >= n positions.

    causal: query s sits at key position q_pos0 + s (default n - S, the cache tail) and sees
    the keys up to it, as in the reference's causal multi-token branch."""
    k = dequantize(*(t[:, :, :n] for t in kq), bits, group_size).float()
    v = dequantize(*(t[:, :, :n] for t in vq), bits, group_size).float()
    b, hq, s, d = q.shape
    hkv = k.shape[1]
    qf = (q.float() * scale).view(b, hkv, hq // hkv, s, d)
    sc = qf @ k.unsqueeze(2).transpose(-1, -2)
    if causal:
        pos = torch.arange(s).unsqueeze(1) + (n - s if q_pos0 is None else q_pos0)
        sc = sc.masked_fill(torch.arange(n).unsqueeze(0) > pos, float("-inf"))
    p = torch.softmax(sc, dim=-1)
    return (p @ v.unsqueeze(2)).view(b, hq, s, d).to(q.dtype)
