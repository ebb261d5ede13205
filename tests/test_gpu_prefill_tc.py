"""Tensor-core multi-token path (tcgen05) vs the CPU oracle, through the C ABI.

Calls with head_dim 128, a GQA group dividing 128, at least 64 query rows per kv head and
no mask or a causal mask take the tcgen05 kernel (qkv_prefill_tc.cu). Like the reference's
multi-token branch (src/chad/mlx_qsdpa.py:751-766) it attends over K/V dequantized to the
query dtype, so it is held to the configurations' tolerance (max-abs 2e-2, mean-abs 2e-3)
against the fp32 dequantize -> fp32 attention reference.
"""

import numpy as np
import pytest

from oracle import qkv_oracle as orc
from tests.helpers import f32_of, make_case, torch_from_f32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _cache(k, v, bits, dtype):
    from chad_b200.cache import QuantizedKVCache

    c = QuantizedKVCache(group_size=64, bits=bits)
    c.update_and_fetch(torch_from_f32(k, dtype), torch_from_f32(v, dtype))
    return c


def _ref(q, k, v, bits, dtype, n, mask):
    kq = orc.affine_quantize(k, bits, 64, dtype)
    vq = orc.affine_quantize(v, bits, 64, dtype)
    return orc.attention_quantized_fp32(q, kq, vq, q.shape[-1] ** -0.5, n, bits, 64, mask, dtype)


def _run(q, c, n, bits, dtype, mask, splits=0):
    from chad_b200 import ops

    tq = torch_from_f32(q, dtype)
    return ops.attention(tq, c.keys, c.values, q.shape[-1] ** -0.5, n, bits, mask=mask,
                         splits=splits)


def _check(got, ref, tol_max=2e-2, tol_mean=2e-3):
    g = f32_of(got)
    assert np.isfinite(g).all()
    err = np.abs(g - ref)
    assert err.max() < tol_max, f"max err {err.max()}"
    assert err.mean() < tol_mean, f"mean err {err.mean()}"


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("prefix,S", [(700, 64), (1000, 37), (0, 128), (2000, 200)])
def test_causal_chunk_over_prefix(bits, dtype, prefix, S):
    n = prefix + S
    q, k, v = make_case(100 + S, 1, 32, 4, S, 128, n, dtype, outliers=True)
    c = _cache(k, v, bits, dtype)
    _check(_run(q, c, n, bits, dtype, "causal"), _ref(q, k, v, bits, dtype, n, "causal"))


@pytest.mark.parametrize("hq,hkv,S", [(16, 4, 40), (32, 2, 20), (8, 8, 130), (64, 4, 9)])
def test_gqa_groups(hq, hkv, S):
    """GQA 4 (32 tokens per tile), 16 (8), 1 (128) and 16 with one partial tile."""
    n = 900 + S
    q, k, v = make_case(7 + hq + S, 1, hq, hkv, S, 128, n, "bf16", outliers=True)
    c = _cache(k, v, 4, "bf16")
    _check(_run(q, c, n, 4, "bf16", "causal"), _ref(q, k, v, 4, "bf16", n, "causal"))


def test_no_mask_and_batch():
    B, S, n = 2, 48, 1500
    q, k, v = make_case(31, B, 32, 4, S, 128, n, "bf16", outliers=True)
    c = _cache(k, v, 4, "bf16")
    _check(_run(q, c, n, 4, "bf16", None), _ref(q, k, v, 4, "bf16", n, None))


@pytest.mark.parametrize("splits", [1, 2, 5])
def test_key_splits_agree(splits):
    S, n = 64, 3000 + 64
    q, k, v = make_case(5, 1, 32, 4, S, 128, n, "bf16", outliers=True)
    c = _cache(k, v, 4, "bf16")
    ref = _ref(q, k, v, 4, "bf16", n, "causal")
    _check(_run(q, c, n, 4, "bf16", "causal", splits=splits), ref)


def test_partials_then_combine():
    from chad_b200 import ops

    S, n = 32, 2000 + 32
    q, k, v = make_case(6, 1, 32, 4, S, 128, n, "bf16", outliers=True)
    c = _cache(k, v, 8, "bf16")
    tq = torch_from_f32(q, "bf16")
    parts = ops.partials(tq, c.keys, c.values, 128 ** -0.5, n, 8, mask="causal", splits=3)
    assert parts.shape[0] == 3
    _check(ops.combine(parts.contiguous(), torch.bfloat16),
           _ref(q, k, v, 8, "bf16", n, "causal"))


def test_padded_tail_poison_is_ignored():
    """Codes, scales and biases past n are never used: the output is bit-identical."""
    S, n = 64, 777
    q, k, v = make_case(12, 1, 32, 4, S, 128, n, "bf16")
    c = _cache(k, v, 4, "bf16")
    clean = _run(q, c, n, 4, "bf16", "causal")
    NP = c.keys[0].shape[2]
    assert NP > n
    for t in (c.keys[1], c.keys[2], c.values[1], c.values[2]):
        t[:, :, n:] = float("nan")
    for t in (c.keys[0], c.values[0]):
        t[:, :, n:] = -1
    poisoned = _run(q, c, n, 4, "bf16", "causal")
    assert torch.equal(clean, poisoned)


def test_prefill_entry_point_uses_cache_append():
    """qkv_prefill: quantize-append the chunk, then the causal tensor-core attention."""
    from chad_b200 import ops
    from chad_b200.cache import QuantizedKVCache

    prefix, S, D = 1300, 96, 128
    q, k, v = make_case(8, 1, 32, 4, S, D, prefix + S, "bf16", outliers=True)
    c = QuantizedKVCache(group_size=64, bits=4)
    c.update_and_fetch(torch_from_f32(k[:, :, :prefix], "bf16"),
                       torch_from_f32(v[:, :, :prefix], "bf16"))
    c._grow(prefix + S, 1, 4, D, D, torch.bfloat16, torch.device("cuda"))
    out = ops.prefill(torch_from_f32(q, "bf16"), torch_from_f32(k[:, :, prefix:], "bf16"),
                      torch_from_f32(v[:, :, prefix:], "bf16"), c.keys, c.values, prefix, 4,
                      D ** -0.5)
    _check(out, _ref(q, k, v, 4, "bf16", prefix + S, "causal"))
    assert ops.device_status() == 0


def test_repeated_calls_are_bit_identical():
    """The pipeline's barriers order every tensor-memory read after the MMA writing it, so
    repeated calls give identical bits (a missed wait shows up as run-to-run noise)."""
    S, n = 256, 4000 + 256
    q, k, v = make_case(44, 1, 32, 4, S, 128, n, "bf16", outliers=True)
    c = _cache(k, v, 4, "bf16")
    first = _run(q, c, n, 4, "bf16", "causal", splits=1)
    for _ in range(6):
        assert torch.equal(first, _run(q, c, n, 4, "bf16", "causal", splits=1))


@pytest.mark.parametrize("bits", [4, 8])
def test_verify_block_shape(bits):
    """A speculative-verify block (8 draft tokens at the cache tail, GQA 8: 64 query rows per
    kv head, half a tile) split over many key ranges."""
    S, n = 8, 6000 + 8
    q, k, v = make_case(70 + bits, 1, 32, 4, S, 128, n, "bf16", outliers=True)
    c = _cache(k, v, bits, "bf16")
    _check(_run(q, c, n, bits, "bf16", "causal"), _ref(q, k, v, bits, "bf16", n, "causal"))


def test_key_split_tiles_partials():
    """A block that fits one 128-row tile runs its keys on both tensor-memory tiles
    alternately and the epilogue folds tile 1 into tile 0: one partial row per query row
    per split, and the normalized output directly when there is one split."""
    from chad_b200 import ops

    S, n = 8, 2500 + 8
    q, k, v = make_case(91, 1, 32, 4, S, 128, n, "bf16", outliers=True)
    c = _cache(k, v, 4, "bf16")
    tq = torch_from_f32(q, "bf16")
    parts = ops.partials(tq, c.keys, c.values, 128 ** -0.5, n, 4, mask="causal", splits=3)
    assert parts.shape[0] == 3
    ref = _ref(q, k, v, 4, "bf16", n, "causal")
    _check(ops.combine(parts.contiguous(), torch.bfloat16), ref)
    _check(_run(q, c, n, 4, "bf16", "causal", splits=1), ref)


@pytest.mark.parametrize("n", [8, 100, 128 + 8, 256 + 8, 300])
def test_key_split_tiles_with_one_or_two_key_tiles(n):
    """Key ranges of one tile (tile 1 has no keys and is left out of the fold) and of two or
    three tiles, 8- and 4-bit, one split (direct output)."""
    S = 8
    for bits in (4, 8):
        q, k, v = make_case(93 + n, 1, 32, 4, S, 128, n, "bf16", outliers=True)
        c = _cache(k, v, bits, "bf16")
        _check(_run(q, c, n, bits, "bf16", "causal", splits=1),
               _ref(q, k, v, bits, "bf16", n, "causal"))
