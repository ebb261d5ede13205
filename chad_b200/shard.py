"""Sequence-sharded split-KV decode across the GPUs of one node.

Each rank holds a contiguous range of every sequence's keys in its own HBM. A decode step
computes, per rank, one (max, sum, un-normalised out) partial row per query row over the
local range (qkv_attention with QKV_OUT_PARTIAL), gathers every rank's rows with ONE
collective (``all_gather_into_tensor`` over NCCL/NVLink, or gloo on CPU for tests), and
merges them with the log-sum-exp combine — the reference's pass 2
(src/chad/mlx_qsdpa.py:233-258) applied across GPUs instead of across blocks. Several
layers can share the one gather when their inputs are independent (`layers` axis).

The compute functions are injectable so the host protocol (ranges, gather layout, merge
order) is testable with CPU ranks.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch


def shard_ranges(lens: Sequence[int], world: int, rank: int) -> Tuple[List[int], List[int]]:
    """(pos_base, local_len) per batch row: rank r owns keys [L*r/world, L*(r+1)/world)."""
    base, loc = [], []
    for L in lens:
        lo = (int(L) * rank) // world
        hi = (int(L) * (rank + 1)) // world
        base.append(lo)
        loc.append(hi - lo)
    return base, loc


class ShardedDecoder:
    """One rank's side of the sharded decode.

    partial_fn(layer, q) -> (B, HQ, S, D+4) float partial rows of this rank's keys;
    combine_fn(parts (world, L, B, HQ, S, D+4)) -> merged output (L, B, HQ, S, D).
    """

    def __init__(self, group=None, partial_fn: Optional[Callable] = None,
                 combine_fn: Optional[Callable] = None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.partial_fn = partial_fn
        self.combine_fn = combine_fn or self._gpu_combine

    @staticmethod
    def _gpu_combine(parts: torch.Tensor) -> torch.Tensor:
        from . import ops

        return ops.combine(parts.contiguous(), torch.bfloat16)

    def step(self, qs: Sequence[torch.Tensor]) -> torch.Tensor:
        """qs: one query tensor (B, HQ, S, D) per layer. Returns (L, B, HQ, S, D)."""
        local = torch.stack([self.partial_fn(l, q) for l, q in enumerate(qs)])
        return self.merge(local)

    def gather(self, local: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Every rank's partial rows: (world, *local.shape), one all_gather_into_tensor.
        `out` (optional) is a preallocated buffer of that shape, reused across steps."""
        if self.world == 1:
            return local.unsqueeze(0)
        if out is None:
            out = torch.empty((self.world, *local.shape), dtype=local.dtype,
                              device=local.device)
        self.dist.all_gather_into_tensor(out.view(-1), local.contiguous().view(-1),
                                        group=self.group)
        return out

    def merge(self, local: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Gather this rank's partial rows (any leading layer axes) with every other rank's
        and merge them: the cross-GPU pass 2. Several layers may share the one gather."""
        return self.combine_fn(self.gather(local, out))


def gpu_partial_fn(caches, lens_local: torch.Tensor, pos_base: torch.Tensor,
                   total_lens: torch.Tensor, n_max: int, bits: int, scale: float,
                   mask=None):
    """partial_fn over this rank's per-layer QuantizedKVCache shards."""
    from . import ops

    def fn(layer: int, q: torch.Tensor) -> torch.Tensor:
        c = caches[layer]
        return ops.attention(q, c.keys, c.values, scale, n_max, bits, lens=lens_local,
                             pos_base=pos_base, total_lens=total_lens, mask=mask, out_kind=1)

    return fn
