"""CPU oracle for the quantized-KV attention path — TEST INFRASTRUCTURE ONLY.

This module is test infrastructure, never the product: only `tests/`, `__graft_entry__.smoke()`
and the `cpu_baseline` / `--impl reference` legs of `bench.py` may import it. The
product path (`chad_b200`) never calls into it and fails loudly when its CUDA library is
missing.

PARITY UNPINNED. The reference (nathansutton/chad, `src/chad/mlx_qsdpa.py`) computes this
path with mlx 0.32.0 / mlx-lm 0.31.3 (pinned at `uv.lock:672-712`, macOS-arm64 wheels
only). Neither package is present in this environment and the reference stores no golden
vectors (every expected value in `tests/test_mlx_qsdpa.py` is computed at run time from
MLX's RNG). This file therefore restates the published algorithms; it is checked against
hand-derived known answers and against the reference tests' relations (tolerance classes,
padded-tail invariance, split/LSE associativity), not against MLX output.

What is restated, and from where:

* ``affine_quantize`` — MLX affine quantization (mlx 0.32.0 ``mx.quantize``, CPU kernel),
  as called by mlx-lm's ``QuantizedKVCache.update_and_fetch`` (call sites:
  ``tests/test_mlx_qsdpa.py:45-49``, ``src/chad/engine.py:546-548``). Per group of
  ``group_size`` values along the last axis, in float32:
  ``scale = max((max-min)/(2^bits-1), 1e-7)``; the sign of ``scale`` and the ``edge``
  (min or max) follow whichever end has the larger magnitude; ``q0 = rint(edge/scale)``;
  if ``q0 != 0`` then ``scale = edge/q0, bias = edge`` else ``bias = 0``; codes are
  ``clip(rint((x-bias)/scale), 0, 2^bits-1)`` from the float32 scale/bias; scale and bias
  are then stored rounded (RNE) to the storage dtype. Codes pack LSB-first into uint32
  (element i of a word at bits ``[i*bits, (i+1)*bits)``; ``mlx_qsdpa.py:131-134`` reads
  8-bit words as ``uchar4`` in exactly this order).
* ``dequantize`` — ``mx.dequantize`` (``mlx_qsdpa.py:701-702``, ``761-764``):
  ``scale*code + bias`` per group. ``round_mode="fused"`` (the default) evaluates in
  float32 and rounds once to the storage dtype; ``round_mode="per_op"`` rounds after the
  multiply and again after the add (the behaviour of an implementation that does the
  arithmetic in the storage dtype). Which of the two mlx 0.32.0 uses is not pinned here.
* ``attention_fp32`` — the tests' dequantize→fp32 reference, ``tests/test_mlx_qsdpa.py:52-65``
  (q pre-scaled in fp32, precise softmax, optional causal mask aligned to the cache tail:
  query i of S sits at position ``n-S+i``), generalised to per-batch lengths, additive and
  boolean masks, and any GQA.
* ``attention_stock`` — mlx-lm's unfused quantized SDPA that the reference falls through to
  for shapes its kernel declines (``mlx_qsdpa.py:3-8``, ``770-771``): q*scale rounded to the
  input dtype, scores = q @ dequant(K)^T accumulated in fp32 and rounded to the input dtype,
  mask, precise softmax (fp32, rounded to the input dtype), then p @ dequant(V) rounded to
  the input dtype.
* ``lse_combine`` — pass 2 of the reference (``mlx_qsdpa.py:233-258``): global max over
  the partial blocks, rescaled sum, rescaled output sum, divide (0 stays 0 for empty rows).
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# storage-dtype helpers (bit patterns held in uint16)
# ---------------------------------------------------------------------------


def f32_to_bf16_bits(x) -> np.ndarray:
    """float32 -> bfloat16 bit pattern, round to nearest even (NaN -> canonical qNaN)."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = x.view(np.uint32)
    # finite values and infinities cannot carry out of 32 bits (at most 0xFF807FFF); NaN
    # patterns may wrap, and are replaced below
    with np.errstate(over="ignore"):
        r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1)))
             >> np.uint32(16)).astype(np.uint16)
    r[np.isnan(x)] = 0x7FC0
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(np.asarray(b, dtype=np.uint16))
    return (b.astype(np.uint32) << 16).view(np.float32)


def f32_to_f16_bits(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def f16_bits_to_f32(b) -> np.ndarray:
    return np.asarray(b, dtype=np.uint16).view(np.float16).astype(np.float32)


def to_bits(x, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    if dtype == "f16":
        return f32_to_f16_bits(x)
    raise ValueError(dtype)


def from_bits(b, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_bits_to_f32(b)
    if dtype == "f16":
        return f16_bits_to_f32(b)
    raise ValueError(dtype)


def round_to(x, dtype: str) -> np.ndarray:
    """Round float32 values to `dtype` ('bf16', 'f16' or 'f32') and return them as float32."""
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    return from_bits(to_bits(x, dtype), dtype)


# ---------------------------------------------------------------------------
# affine quantization (mx.quantize restated)
# ---------------------------------------------------------------------------


def affine_quantize(x, bits: int, group_size: int = 64, scale_dtype: str = "bf16"):
    """Quantize `x` (..., D) along the last axis.

    Returns ``(w, scales, biases)``: ``w`` uint32 (..., D*bits/32) packed LSB-first,
    ``scales``/``biases`` uint16 bit patterns of `scale_dtype` with shape (..., D/group_size).
    `x` holds the values exactly as stored (e.g. bf16 values upcast to float32).
    """
    if bits not in (4, 8):
        raise ValueError("bits must be 4 or 8")
    x = np.asarray(x, dtype=np.float32)
    *lead, d = x.shape
    if d % group_size or (d * bits) % 32:
        raise ValueError("last axis must be a multiple of group_size and of 32/bits")
    g = x.reshape(*lead, d // group_size, group_size)
    n_bins = np.float32((1 << bits) - 1)
    eps = np.float32(1e-7)
    w_max = g.max(axis=-1)
    w_min = g.min(axis=-1)
    with np.errstate(divide="ignore", invalid="ignore"):
        scale = np.maximum((w_max - w_min) / n_bins, eps).astype(np.float32)
        side = np.abs(w_min) > np.abs(w_max)
        scale = np.where(side, scale, -scale).astype(np.float32)
        edge = np.where(side, w_min, w_max).astype(np.float32)
        q0 = np.rint(edge / scale).astype(np.float32)
        at_zero = q0 == 0
        scale = np.where(at_zero, scale, edge / q0).astype(np.float32)
        bias = np.where(at_zero, np.float32(0.0), edge).astype(np.float32)
        codes = np.rint((g - bias[..., None]) / scale[..., None])
    codes = np.clip(codes, 0, n_bins).astype(np.uint32).reshape(*lead, d)
    per_word = 32 // bits
    cw = codes.reshape(*lead, d // per_word, per_word)
    shifts = (np.arange(per_word, dtype=np.uint32) * bits).astype(np.uint32)
    w = np.bitwise_or.reduce(cw << shifts, axis=-1).astype(np.uint32)
    return w, to_bits(scale, scale_dtype), to_bits(bias, scale_dtype)


def unpack_codes(w, bits: int) -> np.ndarray:
    """uint32 (..., W) -> integer codes (..., W*32/bits), LSB-first."""
    w = np.ascontiguousarray(np.asarray(w, dtype=np.uint32))
    per_word = 32 // bits
    # little-endian bytes of a word are its elements in order (LSB-first packing)
    by = w.astype("<u4", copy=False).view(np.uint8).reshape(*w.shape[:-1], w.shape[-1] * 4)
    if bits == 8:
        return by.astype(np.uint32)
    c = np.empty((*w.shape[:-1], w.shape[-1] * per_word), dtype=np.uint32)
    c[..., 0::2] = by & np.uint8(0xF)
    c[..., 1::2] = by >> np.uint8(4)
    return c


def dequantize(w, scales, biases, bits: int, group_size: int = 64,
               scale_dtype: str = "bf16", round_mode: str = "fused") -> np.ndarray:
    """Dequantize to the storage dtype; returns uint16 bit patterns of `scale_dtype`."""
    c = unpack_codes(w, bits).astype(np.float32)
    *lead, d = c.shape
    s = from_bits(scales, scale_dtype)[..., :, None]
    b = from_bits(biases, scale_dtype)[..., :, None]
    cg = c.reshape(*lead, d // group_size, group_size)
    if round_mode == "fused":
        # scale*code is exact in float32 (<= 11 + 8 significant bits), so this is a
        # single rounding of the exact value scale*code+bias.
        v = (s * cg + b).astype(np.float32)
    elif round_mode == "per_op":
        v = round_to(s * cg, scale_dtype) + b
    else:
        raise ValueError(round_mode)
    return to_bits(v.reshape(*lead, d), scale_dtype)


def dequantize_f32(w, scales, biases, bits, group_size=64, scale_dtype="bf16",
                   round_mode="fused") -> np.ndarray:
    return from_bits(dequantize(w, scales, biases, bits, group_size, scale_dtype, round_mode),
                     scale_dtype)


# ---------------------------------------------------------------------------
# attention references
# ---------------------------------------------------------------------------


def _visible(n_b: int, s_len: int, mask, b: int, hq: int, n_keys: int):
    """(S, n_keys) bool/additive handling. Returns (keep bool array, additive float array)."""
    keep = np.zeros((s_len, n_keys), dtype=bool)
    keep[:, :n_b] = True
    add = np.zeros((s_len, n_keys), dtype=np.float32)
    if mask is None:
        return keep, add
    if isinstance(mask, str):
        if mask != "causal":
            raise ValueError(mask)
        qi = np.arange(n_b - s_len, n_b)[:, None]
        ki = np.arange(n_keys)[None, :]
        return keep & (ki <= qi), add
    m = np.asarray(mask)
    while m.ndim < 4:
        m = m[None]
    mb = m[b if m.shape[0] > 1 else 0, hq if m.shape[1] > 1 else 0]
    mb = np.broadcast_to(mb, (s_len, mb.shape[-1]))[:, :n_keys]
    if mb.dtype == bool:
        keep[:, : mb.shape[1]] &= mb
    else:
        add[:, : mb.shape[1]] += mb.astype(np.float32)
    return keep, add


def attention_fp32(q, k, v, scale: float, lens, mask=None) -> np.ndarray:
    """Reference attention in float32 over already-dequantized K/V.

    q (B, HQ, S, D) float32; k, v (B, HKV, N, D) float32 (dequantized values);
    lens: int or per-batch sequence of valid key counts; mask None | 'causal' |
    array broadcastable to (B, HQ, S, N) (bool keep-mask or additive float).
    Follows tests/test_mlx_qsdpa.py:52-65. Returns float32 (B, HQ, S, D);
    rows with no visible key are 0 (pass-2 convention, mlx_qsdpa.py:256).
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    b_, hq_, s_, d_ = q.shape
    hkv = k.shape[1]
    gqa = hq_ // hkv
    lens = [lens] * b_ if np.isscalar(lens) else list(lens)
    out = np.zeros((b_, hq_, s_, d_), np.float32)
    for b in range(b_):
        n = int(lens[b])
        for h in range(hq_):
            kh = k[b, h // gqa, :n]
            vh = v[b, h // gqa, :n]
            qs = q[b, h] * np.float32(scale)
            sc = (qs @ kh.T).astype(np.float32)
            keep, add = _visible(n, s_, mask, b, h, n)
            sc = np.where(keep, sc + add, -np.inf)
            mx = sc.max(axis=-1, keepdims=True)
            ok = np.isfinite(mx)
            e = np.where(ok, np.exp(sc - np.where(ok, mx, 0)), 0.0)
            den = e.sum(axis=-1, keepdims=True)
            p = np.where(den > 0, e / np.where(den > 0, den, 1), 0.0)
            out[b, h] = (p @ vh).astype(np.float32)
    return out


def attention_quantized_fp32(q, kq, vq, scale, lens, bits, group_size=64, mask=None,
                             scale_dtype="bf16", round_mode="fused"):
    """Dequantize (w, scales, biases) tuples, then `attention_fp32`."""
    k = dequantize_f32(*kq, bits, group_size, scale_dtype, round_mode)
    v = dequantize_f32(*vq, bits, group_size, scale_dtype, round_mode)
    return attention_fp32(q, k, v, scale, lens, mask)


def attention_quantized_rows(q, kq, vq, scale, lens, bits, group_size=64,
                             scale_dtype="bf16", q_pos=None, round_mode="fused",
                             key_base=0):
    """`attention_quantized_fp32` for long caches, one (batch, kv head) at a time.

    Same arithmetic as ``attention_quantized_fp32`` (dequantize to the storage dtype, then
    float32 attention, tests/test_mlx_qsdpa.py:52-65) but it dequantizes only the
    ``lens[b]`` valid positions of one kv head at a time, so a 128K-key batch fits in a few
    hundred MB. ``q_pos`` (B, S) int, optional: absolute position of each query row; row s
    of batch b sees only keys at positions ``key_base + j <= q_pos[b, s]`` (the causal rule
    of mlx_qsdpa.py:751-766 evaluated for an arbitrary subset of the new chunk's rows).
    """
    import concurrent.futures as cf
    import os

    q = np.asarray(q, np.float32)
    b_, hq_, s_, d_ = q.shape
    hkv = kq[0].shape[1]
    gqa = hq_ // hkv
    lens = [lens] * b_ if np.isscalar(lens) else list(lens)
    out = np.zeros((b_, hq_, s_, d_), np.float32)

    def one(bh):
        b, h = bh
        n = int(lens[b])
        if n > 0:
            k = dequantize_f32(kq[0][b, h, :n], kq[1][b, h, :n], kq[2][b, h, :n], bits,
                               group_size, scale_dtype, round_mode)
            v = dequantize_f32(vq[0][b, h, :n], vq[1][b, h, :n], vq[2][b, h, :n], bits,
                               group_size, scale_dtype, round_mode)
            qs = q[b, h * gqa:(h + 1) * gqa].reshape(gqa * s_, d_) * np.float32(scale)
            sc = qs @ k.T  # (gqa*S, n)
            if q_pos is not None:
                pos = np.tile(np.asarray(q_pos[b]), gqa)[:, None]
                sc = np.where(key_base + np.arange(n)[None, :] <= pos, sc, -np.inf)
            mx = sc.max(axis=-1, keepdims=True)
            ok = np.isfinite(mx)
            e = np.where(ok, np.exp(sc - np.where(ok, mx, 0)), 0.0).astype(np.float32)
            den = e.sum(axis=-1, keepdims=True)
            p = np.where(den > 0, e / np.where(den > 0, den, 1), 0.0).astype(np.float32)
            out[b, h * gqa:(h + 1) * gqa] = (p @ v).reshape(gqa, s_, d_)

    # (numpy releases the GIL in the heavy array operations: threads share the work)
    pairs = [(b, h) for b in range(b_) for h in range(hkv)]
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(pairs), os.cpu_count() or 1, 16))) as ex:
        list(ex.map(one, pairs))
    return out


def attention_stock(q, kq, vq, scale, lens, bits, group_size=64, mask=None,
                    dtype="bf16", round_mode="fused"):
    """mlx-lm's unfused quantized path, with storage-dtype rounding at op boundaries."""
    k = dequantize_f32(*kq, bits, group_size, dtype, round_mode)
    v = dequantize_f32(*vq, bits, group_size, dtype, round_mode)
    q = np.asarray(q, np.float32)
    qs = round_to(q * np.float32(scale), dtype)
    b_, hq_, s_, d_ = q.shape
    gqa = hq_ // k.shape[1]
    lens = [lens] * b_ if np.isscalar(lens) else list(lens)
    out = np.zeros_like(q)
    for b in range(b_):
        n = int(lens[b])
        for h in range(hq_):
            sc = round_to(qs[b, h] @ k[b, h // gqa, :n].T, dtype)
            keep, add = _visible(n, s_, mask, b, h, n)
            sc = np.where(keep, round_to(sc + add, dtype), -np.inf)
            mx = sc.max(axis=-1, keepdims=True)
            ok = np.isfinite(mx)
            e = np.where(ok, np.exp(sc - np.where(ok, mx, 0)), 0.0)
            den = e.sum(axis=-1, keepdims=True)
            p = round_to(np.where(den > 0, e / np.where(den > 0, den, 1), 0.0), dtype)
            out[b, h] = round_to(p @ v[b, h // gqa, :n], dtype)
    return out


def lse_combine(maxs, sums, partials):
    """Pass-2 combine (mlx_qsdpa.py:233-258).

    maxs, sums: (..., P) float32 (max of scaled logits, sum of exp relative to that max);
    partials: (..., P, D) un-normalised outputs. Natural-log domain.
    """
    maxs = np.asarray(maxs, np.float32)
    sums = np.asarray(sums, np.float32)
    partials = np.asarray(partials, np.float32)
    gmax = maxs.max(axis=-1, keepdims=True)
    ok = np.isfinite(gmax)
    f = np.where(ok, np.exp(np.where(np.isfinite(maxs), maxs, -np.inf) - np.where(ok, gmax, 0)),
                 0.0)
    den = (f * sums).sum(axis=-1)
    num = (f[..., None] * partials).sum(axis=-2)
    return np.where(den[..., None] == 0, num, num / np.where(den == 0, 1, den)[..., None])


def split_partials_fp32(q, k, v, scale, n, splits):
    """Split-KV pass 1 restated (mlx_qsdpa.py:73-209): per contiguous block of keys, the
    (max, sum, un-normalised output) triple per query row. q (HQ, D), k/v (HKV, N, D)."""
    q = np.asarray(q, np.float32)
    hq, d = q.shape
    gqa = hq // k.shape[0]
    edges = np.linspace(0, n, splits + 1).astype(int)
    maxs = np.full((hq, splits), -np.inf, np.float32)
    sums = np.zeros((hq, splits), np.float32)
    parts = np.zeros((hq, splits, d), np.float32)
    for h in range(hq):
        sc = (q[h] * np.float32(scale)) @ k[h // gqa, :n].T
        for i in range(splits):
            a, b = edges[i], edges[i + 1]
            if b <= a:
                continue
            m = sc[a:b].max()
            e = np.exp(sc[a:b] - m)
            maxs[h, i], sums[h, i] = m, e.sum()
            parts[h, i] = e @ v[h // gqa, a:b]
    return maxs, sums, parts


# ---------------------------------------------------------------------------
# seeded synthetic inputs (the benchmark configurations' value distributions)
# ---------------------------------------------------------------------------

OUTLIER_CHANNELS = (3, 37, 70, 101)


def make_kv(rng: np.random.Generator, shape, outliers=True, dtype="bf16"):
    """K or V ~ N(0,1) rounded to `dtype` ('bf16' or 'f32'); key outlier channels x8."""
    x = rng.standard_normal(shape, dtype=np.float32)
    if outliers:
        d = shape[-1]
        for c in OUTLIER_CHANNELS:
            if c < d:
                x[..., c] *= 8.0
    return round_to(x, dtype) if dtype != "f32" else x
