"""Quantized KV cache in HBM, with the contract of mlx-lm's QuantizedKVCache.

The reference builds one `QuantizedKVCache(group_size=64, bits=kv_bits)` per attention
layer (src/chad/engine.py:537-555) and its attention reads `cache.keys`, `cache.values`,
`cache.offset`, `cache.bits`, `cache.group_size` (src/chad/mlx_qsdpa.py:633-658, 743-748).
This class keeps that surface on torch CUDA tensors:

* `keys` / `values` are tuples ``(w, scales, biases)``: ``w`` int32 (uint32 bit patterns)
  (B, H, NP, D*bits/32), scales/biases (B, H, NP, D/64) in the K/V dtype;
* NP is a multiple of `step` (256) — the padded tail past `offset` is never read as keys;
* `update_and_fetch` quantizes the new rows on the GPU (qkv_quantize_append) straight into
  the padded buffers, growing them by whole steps (copying the valid prefix only);
* `trim(n)` rewinds by offset only (rows below the write point are never mutated), which is
  what the reference's rewind relies on (src/chad/engine.py:670-718);
* `state` / `meta_state` round-trip through `save_prompt_cache` / `load_prompt_cache`
  (safetensors), keyed by bit width so a cache of one mode never loads into another.
"""

from __future__ import annotations

import json
from typing import List, Optional, Sequence, Tuple

import torch

from . import ops

QuantTuple = Tuple[torch.Tensor, torch.Tensor, torch.Tensor]


class KVCache:
    """Plain (non-quantized) KV cache: the fp16/bf16 path the seam leaves on stock SDPA."""

    step = 256

    def __init__(self):
        self.keys: Optional[torch.Tensor] = None
        self.values: Optional[torch.Tensor] = None
        self.offset = 0

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor):
        b, h, s, d = keys.shape
        prev = self.offset
        if self.keys is None or prev + s > self.keys.shape[2]:
            cap = (prev + s + self.step - 1) // self.step * self.step
            nk = keys.new_zeros((b, h, cap, d))
            nv = values.new_zeros((b, h, cap, values.shape[-1]))
            if self.keys is not None:
                nk[:, :, :prev] = self.keys[:, :, :prev]
                nv[:, :, :prev] = self.values[:, :, :prev]
            self.keys, self.values = nk, nv
        self.keys[:, :, prev:prev + s] = keys
        self.values[:, :, prev:prev + s] = values
        self.offset += s
        return self.keys[:, :, : self.offset], self.values[:, :, : self.offset]

    def is_trimmable(self) -> bool:
        return True

    def trim(self, n: int) -> int:
        n = min(self.offset, n)
        self.offset -= n
        return n

    @property
    def nbytes(self) -> int:
        if self.keys is None:
            return 0
        return self.keys.numel() * self.keys.element_size() * 2


class QuantizedKVCache:
    step = 256

    def __init__(self, group_size: int = 64, bits: int = 8):
        if bits not in (4, 8):
            raise ValueError("bits must be 4 or 8")
        if group_size != 64:
            raise ValueError("group_size must be 64")
        self.group_size = group_size
        self.bits = bits
        self.keys: Optional[QuantTuple] = None
        self.values: Optional[QuantTuple] = None
        self.offset = 0

    # -- growth ------------------------------------------------------------------------
    def _alloc(self, b, h, cap, d, dtype, device) -> QuantTuple:
        return (
            torch.zeros((b, h, cap, d * self.bits // 32), dtype=torch.int32, device=device),
            torch.zeros((b, h, cap, d // self.group_size), dtype=dtype, device=device),
            torch.zeros((b, h, cap, d // self.group_size), dtype=dtype, device=device),
        )

    def _grow(self, need: int, b, h, dk, dv, dtype, device) -> None:
        cap = (need + self.step - 1) // self.step * self.step
        nk = self._alloc(b, h, cap, dk, dtype, device)
        nv = self._alloc(b, h, cap, dv, dtype, device)
        if self.keys is not None and self.offset:
            for dst, src in zip(nk + nv, self.keys + self.values):
                dst[:, :, : self.offset].copy_(src[:, :, : self.offset])
        self.keys, self.values = nk, nv

    def reserve(self, n: int, b: int, h: int, d: int, dtype: torch.dtype,
                device: torch.device) -> None:
        """Pre-size the buffers for n positions (rounded up to whole steps) so that appends
        up to n never grow them. mlx-lm grows by one step per crossing, copying the valid
        prefix each time; a decode loop that knows its budget avoids those copies."""
        if n > self.capacity:
            self._grow(n, b, h, d, d, dtype, device)

    @property
    def capacity(self) -> int:
        return 0 if self.keys is None else self.keys[0].shape[2]

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor):
        """Quantize keys/values (B, H, S, D) into positions [offset, offset+S).

        Returns the valid views ``(w, scales, biases)[..., :offset, :]`` like mlx-lm.
        """
        b, h, s, dk = keys.shape
        dv = values.shape[-1]
        prev = self.offset
        if self.keys is None or prev + s > self.capacity:
            self._grow(prev + s, b, h, dk, dv, keys.dtype, keys.device)
        k, v = keys.contiguous(), values.contiguous()
        if k.shape == v.shape and k.dtype == v.dtype:
            ops.quantize_append_kv(k, v, self.keys, self.values, prev, self.bits, self.group_size)
        else:  # (different K and V head dims)
            ops.quantize_append(k, *self.keys, prev, self.bits, self.group_size)
            ops.quantize_append(v, *self.values, prev, self.bits, self.group_size)
        self.offset = prev + s
        return self.fetch()

    def fetch(self):
        n = self.offset
        return (tuple(x[:, :, :n] for x in self.keys), tuple(x[:, :, :n] for x in self.values))

    # -- trim / rewind -----------------------------------------------------------------
    def is_trimmable(self) -> bool:
        return True

    def trim(self, n: int) -> int:
        n = min(self.offset, n)
        self.offset -= n
        return n

    # -- accounting --------------------------------------------------------------------
    @property
    def nbytes(self) -> int:
        if self.keys is None:
            return 0
        return sum(t.numel() * t.element_size() for t in self.keys + self.values)

    def bytes_per_token(self) -> float:
        """Exact per-position stride of the allocation (padding cancels out)."""
        if self.keys is None:
            return 0.0
        return self.nbytes / self.capacity

    # -- persistence -------------------------------------------------------------------
    @property
    def state(self):
        if self.keys is None:
            return None
        return self.fetch() if self.offset < self.capacity else (self.keys, self.values)

    @property
    def meta_state(self) -> Tuple[str, ...]:
        return (str(self.step), str(self.offset), str(self.group_size), str(self.bits))

    def restore(self, keys: QuantTuple, values: QuantTuple, meta: Sequence[str]) -> None:
        step, offset, group_size, bits = (int(x) for x in meta)
        if (group_size, bits) != (self.group_size, self.bits):
            raise ValueError(f"cache mode mismatch: file has gs{group_size}/{bits}-bit, "
                             f"cache is gs{self.group_size}/{self.bits}-bit")
        b, h, n, wk = keys[0].shape
        dk = wk * 32 // self.bits
        dv = values[0].shape[-1] * 32 // self.bits
        self.keys = None
        self.offset = 0
        self._grow(max(n, 1), b, h, dk, dv, keys[1].dtype, keys[0].device)
        for dst, src in zip(self.keys + self.values, tuple(keys) + tuple(values)):
            dst[:, :, :n].copy_(src)
        self.offset = offset


def trim_prompt_cache(caches: List, n: int) -> int:
    """Trim every layer by n positions; returns the count actually trimmed."""
    if not caches or not all(c.is_trimmable() for c in caches):
        return 0
    return [c.trim(n) for c in caches][0]


_FORMAT = "chad_b200.qkv-cache/1"


def save_prompt_cache(path: str, caches: List, metadata: Optional[dict] = None) -> None:
    """Persist a list of per-layer caches (safetensors + JSON metadata)."""
    from safetensors.torch import save_file

    tensors = {}
    layers = []
    for i, c in enumerate(caches):
        if isinstance(c, QuantizedKVCache):
            kind = "quantized"
            st = c.state
            if st is not None:
                for j, t in enumerate(st[0]):
                    tensors[f"{i}.k{j}"] = t.contiguous()
                for j, t in enumerate(st[1]):
                    tensors[f"{i}.v{j}"] = t.contiguous()
            layers.append({"kind": kind, "meta": list(c.meta_state), "empty": st is None})
        elif isinstance(c, KVCache):
            if c.keys is not None:
                tensors[f"{i}.k"] = c.keys[:, :, : c.offset].contiguous()
                tensors[f"{i}.v"] = c.values[:, :, : c.offset].contiguous()
            layers.append({"kind": "plain", "offset": c.offset, "empty": c.keys is None})
        else:
            raise TypeError(f"cannot persist {type(c).__name__}")
    meta = {"format": _FORMAT, "layers": json.dumps(layers),
            "user": json.dumps(metadata or {})}
    save_file(tensors, path, metadata=meta)


def load_prompt_cache(path: str, device="cuda", return_metadata: bool = False):
    from safetensors import safe_open

    with safe_open(path, framework="pt", device=str(device)) as f:
        meta = f.metadata() or {}
        if meta.get("format") != _FORMAT:
            raise ValueError(f"{path}: not a {_FORMAT} file")
        layers = json.loads(meta["layers"])
        out = []
        for i, spec in enumerate(layers):
            if spec["kind"] == "quantized":
                _, _, gs, bits = (int(x) for x in spec["meta"])
                c = QuantizedKVCache(group_size=gs, bits=bits)
                if not spec["empty"]:
                    k = tuple(f.get_tensor(f"{i}.k{j}") for j in range(3))
                    v = tuple(f.get_tensor(f"{i}.v{j}") for j in range(3))
                    c.restore(k, v, spec["meta"])
                out.append(c)
            else:
                c = KVCache()
                if not spec["empty"]:
                    c.update_and_fetch(f.get_tensor(f"{i}.k"), f.get_tensor(f"{i}.v"))
                out.append(c)
    if return_metadata:
        return out, json.loads(meta.get("user", "{}"))
    return out
