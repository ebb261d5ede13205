"""Sequence-sharded split-KV decode across the GPUs of one node.

Each rank holds a contiguous range of every sequence's keys in its own HBM. A decode step
computes, per rank, one (max, sum, un-normalised out) partial row per query row over the
local range (qkv_attention with QKV_OUT_PARTIAL) and merges every rank's rows with the
log-sum-exp combine — the reference's pass 2 (src/chad/mlx_qsdpa.py:233-258) applied
across GPUs instead of across blocks. Two transports move the rows:

  "nccl"  ONE collective (``all_gather_into_tensor`` over NCCL/NVLink, or gloo on CPU for
          tests) followed by the combine kernel;
  "peer"  ONE kernel per rank (qkv_gather_combine): it writes the rank's rows straight into
          every rank's receive buffer over NVLink (buffers mapped into every process with
          CUDA IPC), waits for the other ranks' rows and merges them. No collective, no
          second launch, and it captures in a CUDA graph.

Several layers can share the one exchange when their inputs are independent (`layers` axis).

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


class PeerGather:
    """Receive buffers of qkv_gather_combine for one row shape, one per rank, each mapped
    into every rank's process. Built collectively (every rank, same order); `close` too."""

    def __init__(self, rows: int, D: int, group=None, device=None, lib=None):
        """`lib`: the library to call (the loaded libqkv.so; a stand-in in host tests)."""
        import ctypes

        import torch.distributed as dist

        from . import _lib

        self.dist, self.group = dist, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows, self.D = int(rows), int(D)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.lib = lib = lib if lib is not None else _lib.load()
        self.nbytes = lib.qkv_gather_buffer_size(self.rows, self.D, self.world)
        if self.nbytes == 0:
            raise ValueError(f"qkv_gather_buffer_size: unsupported shape rows={rows} D={D}")
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(_lib.QKV_IPC_HANDLE_BYTES)
        with self._on_device():
            _lib.check(lib.qkv_peer_alloc(self.nbytes, ctypes.byref(own), handle))
        self._own = own.value
        handles: List[Optional[bytes]] = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._opened: List[int] = []
        ptrs = []
        try:
            with self._on_device():
                for p, h in enumerate(handles):
                    if p == self.rank:
                        ptrs.append(self._own)
                        continue
                    mapped = ctypes.c_void_p()
                    _lib.check(lib.qkv_peer_open(h, ctypes.byref(mapped)))
                    self._opened.append(mapped.value)
                    ptrs.append(mapped.value)
        except Exception:
            self._release(barrier=False)
            raise
        self.peer_ptrs = torch.tensor(ptrs, dtype=torch.int64, device=self.device)

    def combine(self, local: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16,
                out_kind: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Merge this rank's partial rows (..., D+4) fp32 with every rank's: (..., D) in
        out_dtype (out_kind 0) or one merged partial row each (out_kind 1)."""
        from . import _lib, ops

        if local.dtype != torch.float32 or not local.is_contiguous() \
                or local.shape[-1] != self.D + 4 or local.numel() != self.rows * (self.D + 4):
            raise ValueError(f"PeerGather({self.rows} rows, D={self.D}): got "
                             f"{tuple(local.shape)} {local.dtype}")
        if out is None:
            shape = (*local.shape[:-1], self.D) if out_kind == _lib.QKV_OUT_NORMALIZED \
                else local.shape
            out = torch.empty(shape, dtype=out_dtype if out_kind == 0 else torch.float32,
                              device=local.device)
        code = ops.dtype_code(out_dtype)
        with ops._on(local.device):
            _lib.check(_lib.fn("qkv_gather_combine")(
                local.data_ptr(), self.rows, self.D, self.peer_ptrs.data_ptr(), self._own,
                self.world, self.rank, out.data_ptr(), code, out_kind,
                ops._stream(local.device)))
        return out

    def _on_device(self):
        import contextlib

        return torch.cuda.device(self.device) if self.device.type == "cuda" \
            else contextlib.nullcontext()

    def _release(self, barrier: bool) -> None:
        lib = self.lib
        with self._on_device():
            if self.device.type == "cuda":
                torch.cuda.synchronize()
            for p in self._opened:
                lib.qkv_peer_free(p, 1)
            self._opened = []
            if barrier:  # every mapping of this rank's buffer is closed before it is freed
                self.dist.barrier(group=self.group)
            if self._own:
                lib.qkv_peer_free(self._own, 0)
                self._own = None

    def close(self) -> None:
        if self._own is not None:
            self._release(barrier=True)


class ShardedDecoder:
    """One rank's side of the sharded decode.

    partial_fn(layer, q) -> (B, HQ, S, D+4) float partial rows of this rank's keys;
    combine_fn(parts (world, L, B, HQ, S, D+4)) -> merged output (L, B, HQ, S, D).
    """

    def __init__(self, group=None, partial_fn: Optional[Callable] = None,
                 combine_fn: Optional[Callable] = None, transport: str = "nccl"):
        import torch.distributed as dist

        if transport not in ("nccl", "peer"):
            raise ValueError(f"transport must be 'nccl' or 'peer', not {transport!r}")
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.partial_fn = partial_fn
        self.combine_fn = combine_fn or self._gpu_combine
        self.transport = transport
        self._peer: dict = {}  # (rows, D) -> PeerGather

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
        and merge them: the cross-GPU pass 2. Several layers may share the one gather.
        `out` is the gather buffer for the "nccl" transport, the merged output for "peer"."""
        if self.world > 1 and self.transport == "peer":
            D = local.shape[-1] - 4
            key = (local.numel() // (D + 4), D)
            pg = self._peer.get(key)
            if pg is None:  # collective: every rank meets the same shapes in the same order
                pg = self._peer[key] = PeerGather(key[0], D, self.group, local.device)
            return pg.combine(local, out=out)
        return self.combine_fn(self.gather(local, out))

    def close(self) -> None:
        """Release the peer transport's buffers (collective)."""
        for pg in self._peer.values():
            pg.close()
        self._peer = {}


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
