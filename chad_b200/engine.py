"""KV-cache glue around the fused kernels: kv_bits policy, per-layer cache build, byte
accounting, trim / rewind by offset and the mode-keyed on-disk prefix cache.

These mirror the reference's Engine pieces that touch the quantized cache:
  * ``resolve_kv_bits``  — Engine._resolve_kv_bits (src/chad/engine.py:444-470)
  * ``make_caches``      — Engine._reset_cache (src/chad/engine.py:537-555)
  * ``kv_bytes_per_token`` — Engine._measure_kv_bytes_per_token (src/chad/engine.py:491-522)
  * ``ckpt_path``        — Engine._ckpt_path (src/chad/engine.py:596-612)
  * ``KVSession.warm_prefix`` — Engine.warm_prefix (src/chad/engine.py:614-650)
  * ``KVSession.rewind_to`` — the attention-cache part of Engine._rewind_to
    (src/chad/engine.py:686-718): trim back by offset, then re-feed.
The model forward itself is out of scope; callers pass a ``prefill`` callable that feeds
token ids through their layers and appends to the caches.
"""

from __future__ import annotations

import hashlib
import logging
import os
from typing import Callable, List, Optional, Sequence

import numpy as np

from .cache import KVCache, QuantizedKVCache, load_prompt_cache, save_prompt_cache

log = logging.getLogger("chad")

CKPT_WARM = "warm"
CKPT_PUSH = "push"


def resolve_kv_bits(kv_bits: Optional[int], head_dim: int, n_heads: int, n_kv_heads: int,
                    qsdpa_ok: bool) -> Optional[int]:
    """None = auto: 8-bit exactly when the fused kernels cover the shape and installed;
    0/falsy forces the plain cache; an explicit width is honoured (with a warning when
    the shape is not covered)."""
    from .qsdpa import covers

    gqa = n_heads // n_kv_heads if n_kv_heads else 0
    covered = bool(qsdpa_ok and gqa and covers(head_dim, gqa))
    if kv_bits is None:
        return 8 if covered else None
    if not kv_bits:
        return None
    if not covered:
        log.warning("KV cache: kv_bits=%s forced on an uncovered shape (head_dim=%s gqa=%s)",
                    kv_bits, head_dim, gqa or "?")
    return int(kv_bits)


def make_caches(attention_layers: Sequence[bool], kv_bits: Optional[int]) -> List:
    """One cache per layer: quantized for attention layers when kv_bits is set, a plain
    KVCache otherwise; None for layers without an attention cache (e.g. recurrent ones)."""
    out = []
    for is_attn in attention_layers:
        if not is_attn:
            out.append(None)
        elif kv_bits:
            out.append(QuantizedKVCache(group_size=64, bits=kv_bits))
        else:
            out.append(KVCache())
    return out


def kv_bytes_per_token(caches: Sequence) -> float:
    """Per-token bytes of the growing attention caches, read from the allocations'
    per-position stride (exact regardless of the step padding)."""
    total = 0.0
    for c in caches:
        if isinstance(c, QuantizedKVCache):
            total += c.bytes_per_token()
        elif isinstance(c, KVCache) and c.keys is not None:
            total += c.nbytes / c.keys.shape[2]
    return total


def ckpt_path(cache_dir: str, model_id: str, kv_bits: Optional[int], ids: Sequence[int],
              tag: str = "") -> str:
    """Checkpoint file for exactly these token ids; the cache MODE (kv bits) is part of
    the key so a file of one mode is never loaded by a session of another."""
    h = hashlib.sha1()
    h.update(model_id.encode("utf-8", "ignore"))
    h.update(b"\x00")
    h.update(f"kv{kv_bits or 0}".encode())
    h.update(b"\x00")
    if tag:
        h.update(tag.encode("utf-8", "ignore"))
        h.update(b"\x00")
    h.update(np.asarray(ids, dtype=np.uint32).tobytes())
    kind = CKPT_PUSH if tag == CKPT_PUSH else CKPT_WARM
    return os.path.join(cache_dir, f"{kind}-{h.hexdigest()}.safetensors")


class KVSession:
    """The live per-layer caches of one session plus the token ids they hold."""

    def __init__(self, attention_layers: Sequence[bool], kv_bits: Optional[int],
                 model_id: str = "model", cache_dir: Optional[str] = None):
        self.attention_layers = list(attention_layers)
        self.kv_bits = kv_bits
        self.model_id = model_id
        self.cache_dir = cache_dir
        self.reset()

    def reset(self) -> None:
        self.caches = make_caches(self.attention_layers, self.kv_bits)
        self.cached_ids: List[int] = []

    @property
    def kv_caches(self) -> List:
        return [c for c in self.caches if c is not None]

    def offsets(self) -> List[int]:
        return [c.offset for c in self.kv_caches]

    def trim(self, n: int) -> int:
        """Drop the last n positions of every attention layer (offset only)."""
        got = [c.trim(n) for c in self.kv_caches]
        k = got[0] if got else 0
        if k:
            self.cached_ids = self.cached_ids[: len(self.cached_ids) - k]
        return k

    def rewind_to(self, target_ids: Sequence[int], upto: int,
                  prefill: Callable[["KVSession", List[int]], int]) -> Optional[int]:
        """Land the caches at exactly target_ids[:upto]: trim back to the longest common
        prefix with what is cached, then re-feed the rest."""
        common = 0
        for a, b in zip(self.cached_ids, target_ids[:upto]):
            if a != b:
                break
            common += 1
        peel = len(self.cached_ids) - common
        if peel:
            self.trim(peel)
        refeed = list(target_ids[common:upto])
        if refeed:
            prefill(self, refeed)
            self.cached_ids = list(target_ids[:upto])
        return upto

    def warm_prefix(self, prefix_ids: Sequence[int],
                    prefill: Callable[["KVSession", List[int]], int]):
        """('hit'|'miss'|'skip', n): load a checkpoint of exactly these ids (zero prefill)
        or prefill once and persist."""
        if not self.cache_dir or not prefix_ids:
            return ("skip", 0)
        if self.cached_ids:
            return ("skip", 0)
        path = ckpt_path(self.cache_dir, self.model_id, self.kv_bits, prefix_ids)
        if os.path.isfile(path):
            try:
                loaded, meta = load_prompt_cache(path, return_metadata=True)
                if len(loaded) == len(self.kv_caches) and meta.get("kv_bits") == (self.kv_bits or 0):
                    it = iter(loaded)
                    self.caches = [next(it) if c is not None else None for c in self.caches]
                    self.cached_ids = list(prefix_ids)
                    return ("hit", len(prefix_ids))
            except Exception:  # noqa: BLE001 — corrupt/incompatible -> recompute
                pass
        self.reset()
        fed = prefill(self, list(prefix_ids))
        if fed < len(prefix_ids):
            self.cached_ids = list(prefix_ids[:fed])
            return ("miss", fed)
        self.cached_ids = list(prefix_ids)
        try:
            os.makedirs(self.cache_dir, exist_ok=True)
            save_prompt_cache(path, self.kv_caches, metadata={"kv_bits": self.kv_bits or 0,
                                                              "model_id": self.model_id})
        except Exception:  # noqa: BLE001 — disk full / read-only -> skip persist
            pass
        return ("miss", len(prefix_ids))
