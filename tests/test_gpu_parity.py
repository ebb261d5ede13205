"""CUDA path vs the CPU oracle, through the C ABI (libqkv.so).

Bit-exact for the integer/byte work (codes, scales, biases, dequantized K/V); within the
reference's tolerance classes for attention output (tests/test_mlx_qsdpa.py:68-79:
max-abs 2e-3 fp16 / 8e-3 bf16 against the dequantize->fp32 reference at head_dim 256,
8-bit) and max-abs 2e-2 / mean-abs 2e-3 at the head_dim-128 decode, verify and prefill
shapes.
"""

import numpy as np
import pytest

from oracle import qkv_oracle as orc
from tests.helpers import bits_of, f32_of, make_case, torch_from_f32, u32_of

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _cache(k, v, bits, dtype):
    from chad_b200.cache import QuantizedKVCache

    c = QuantizedKVCache(group_size=64, bits=bits)
    c.update_and_fetch(torch_from_f32(k, dtype), torch_from_f32(v, dtype))
    return c


def _oracle_quant(x, bits, dtype):
    return orc.affine_quantize(x, bits, 64, dtype)


# ------------------------------------------------------------------ quantize / dequantize
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_quantize_append_bit_exact(bits, D, dtype):
    _, k, v = make_case(11 + D + bits, 2, 4, 2, 1, D, 300, dtype, outliers=True)
    c = _cache(k, v, bits, dtype)
    assert c.keys[0].shape[2] == 512  # step 256 pads 300 -> 512
    w, s, b = _oracle_quant(k, bits, dtype)
    n = 300
    np.testing.assert_array_equal(u32_of(c.keys[0])[:, :, :n], w)
    np.testing.assert_array_equal(bits_of(c.keys[1])[:, :, :n], s)
    np.testing.assert_array_equal(bits_of(c.keys[2])[:, :, :n], b)
    w, s, b = _oracle_quant(v, bits, dtype)
    np.testing.assert_array_equal(u32_of(c.values[0])[:, :, :n], w)
    np.testing.assert_array_equal(bits_of(c.values[1])[:, :, :n], s)


def test_quantize_fp32_input_bf16_scales():
    """Single-layer 4K decode inputs: K,V fp32 N(0,1) with key outliers, scales/biases in bf16."""
    from chad_b200 import ops

    rng = np.random.default_rng(5)
    x = orc.make_kv(rng, (1, 2, 256, 128), outliers=True, dtype="f32")
    w, s, b = ops.quantize(torch.from_numpy(x).cuda(), 4, scale_dtype=torch.bfloat16)
    ow, os_, ob = orc.affine_quantize(x, 4, 64, "bf16")
    np.testing.assert_array_equal(u32_of(w), ow)
    np.testing.assert_array_equal(bits_of(s), os_)
    np.testing.assert_array_equal(bits_of(b), ob)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("round_mode", [0, 1])
def test_dequantize_bit_exact(bits, dtype, round_mode):
    from chad_b200 import ops

    _, k, _ = make_case(3, 1, 2, 2, 1, 128, 1000, dtype, outliers=True)
    w, s, b = _oracle_quant(k, bits, dtype)
    tw = torch.from_numpy(w.view(np.int32)).cuda()
    from tests.helpers import torch_from_bits

    ts, tb = torch_from_bits(s, dtype), torch_from_bits(b, dtype)
    got = ops.dequantize(tw, ts, tb, bits, round_mode=round_mode)
    want = orc.dequantize(w, s, b, bits, 64, dtype, "fused" if round_mode == 0 else "per_op")
    np.testing.assert_array_equal(bits_of(got), want)


# ------------------------------------------------------------------ attention parity
def _np_mask(mask):
    if not isinstance(mask, torch.Tensor):
        return mask
    return mask.cpu().numpy() if mask.dtype == torch.bool else mask.float().cpu().numpy()


def _attn_check(q, k, v, bits, dtype, n, tol_max, tol_mean=None, mask=None, lens=None,
                splits=0):
    from chad_b200 import qsdpa

    c = _cache(k, v, bits, dtype)
    tq = torch_from_f32(q, dtype)
    scale = q.shape[-1] ** -0.5
    out = qsdpa.qsdpa(tq, c.keys, c.values, scale, n, mask=mask, splits=splits)
    kq = _oracle_quant(k, bits, dtype)
    vq = _oracle_quant(v, bits, dtype)
    ref = orc.attention_quantized_fp32(q, kq, vq, scale, n if lens is None else lens, bits, 64,
                                       _np_mask(mask), dtype)
    got = f32_of(out)
    assert np.isfinite(got).all()
    err = np.abs(got - ref)
    assert err.max() < tol_max, f"max err {err.max()}"
    if tol_mean is not None:
        assert err.mean() < tol_mean, f"mean err {err.mean()}"
    return out


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("hkv", [2, 4])
@pytest.mark.parametrize("n", [3, 100, 1024, 5000])
def test_reference_shape_matches_dequant_reference(dtype, hkv, n):
    """The reference's own kernel shape: D=256, 8-bit, HQ=16, K/V scaled x0.7."""
    q, k, v = make_case(3, 1, 16, hkv, 1, 256, n, dtype, kv_scale=0.7)
    tol = 2e-3 if dtype == "f16" else 8e-3
    _attn_check(q, k, v, 8, dtype, n, tol)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("n", [1, 7, 64, 65, 4095, 12345])
@pytest.mark.parametrize("hkv,hq", [(2, 16), (4, 32), (4, 16), (8, 8), (2, 32)])
def test_d128_decode(bits, n, hkv, hq):
    q, k, v = make_case(n + bits, 1, hq, hkv, 1, 128, n, "bf16", outliers=True)
    _attn_check(q, k, v, bits, "bf16", n, 2e-2, 2e-3)


@pytest.mark.parametrize("D", [64, 256])
@pytest.mark.parametrize("bits", [4, 8])
def test_other_head_dims(D, bits):
    q, k, v = make_case(D, 1, 8, 2, 1, D, 777, "f16", outliers=True)
    _attn_check(q, k, v, bits, "f16", 777, 2e-2, 2e-3)


def test_padded_tail_poison_is_ignored():
    """tests/test_mlx_qsdpa.py:82-95: positions past n must not change the output."""
    from chad_b200 import qsdpa

    n = 300
    q, k, v = make_case(3, 1, 16, 2, 1, 256, n, "f16")
    c = _cache(k, v, 8, "f16")
    tq = torch_from_f32(q, "f16")
    out1 = qsdpa.qsdpa(tq, c.keys, c.values, 256 ** -0.5, n)
    kw, ks, kb = c.keys
    vw, vs, vb = c.values
    kw[:, :, n:] = -1  # 0xFFFFFFFF
    ks[:, :, n:] = 100.0
    vw[:, :, n:] = -1
    vs[:, :, n:] = float("nan")
    vb[:, :, n:] = float("inf")
    out2 = qsdpa.qsdpa(tq, c.keys, c.values, 256 ** -0.5, n)
    assert torch.equal(out1, out2)


@pytest.mark.parametrize("splits", [1, 2, 3, 17, 64])
def test_split_count_does_not_change_result(splits):
    q, k, v = make_case(9, 1, 32, 4, 1, 128, 3000, "bf16", outliers=True)
    _attn_check(q, k, v, 4, "bf16", 3000, 2e-2, 2e-3, splits=splits)


@pytest.mark.parametrize("S", [2, 8, 16])
@pytest.mark.parametrize("bits", [4, 8])
def test_multi_token_causal(S, bits):
    """Verify block: S draft tokens at the cache tail, causal within the block."""
    n = 1000 + S
    q, k, v = make_case(S, 1, 32, 4, S, 128, n, "bf16", outliers=True)
    _attn_check(q, k, v, bits, "bf16", n, 2e-2, 2e-3, mask="causal")


@pytest.mark.parametrize("S,n", [(8, 1000), (5, 3000), (16, 130)])
def test_multi_token_causal_row_groups(S, n):
    """GQA 4: 4*S query rows per kv head stay on the split-KV kernel, whose causal mask is
    only evaluated on tiles past the first draft position."""
    q, k, v = make_case(40 + S, 1, 16, 4, S, 128, n, "bf16", outliers=True)
    _attn_check(q, k, v, 4, "bf16", n, 2e-2, 2e-3, mask="causal")


def test_bool_and_additive_masks():
    n = 500
    q, k, v = make_case(21, 1, 16, 2, 2, 128, n, "bf16")
    rng = np.random.default_rng(0)
    keep = rng.random((1, 16, 2, n)) > 0.3
    keep[..., 0] = True
    _attn_check(q, k, v, 8, "bf16", n, 2e-2, 2e-3, mask=torch.from_numpy(keep).cuda())
    add = orc.round_to(rng.standard_normal((1, 1, 2, n)).astype(np.float32), "bf16")
    _attn_check(q, k, v, 8, "bf16", n, 2e-2, 2e-3,
                mask=torch_from_f32(add, "bf16"))


def test_ragged_lengths_and_partials_combine():
    """Per-batch lengths, then a sequence split into two shards merged by qkv_combine."""
    from chad_b200 import ops

    B, HQ, HKV, D, NP = 3, 32, 4, 128, 2048
    lens = np.array([1500, 37, 2048], np.int32)
    q, k, v = make_case(4, B, HQ, HKV, 1, D, NP, "bf16", outliers=True)
    c = _cache(k, v, 4, "bf16")
    tq = torch_from_f32(q, "bf16")
    tl = torch.from_numpy(lens).cuda()
    out = ops.attention(tq, c.keys, c.values, D ** -0.5, NP, 4, lens=tl)
    kq, vq = _oracle_quant(k, 4, "bf16"), _oracle_quant(v, 4, "bf16")
    ref = orc.attention_quantized_fp32(q, kq, vq, D ** -0.5, lens, 4)
    assert np.abs(f32_of(out) - ref).max() < 2e-2

    # two shards: [0, cut) and [cut, len) of every row, each its own padded cache
    cut = 800
    parts = []
    for lo, hi in ((0, cut), (cut, NP)):
        sub = _cache(k[:, :, lo:hi], v[:, :, lo:hi], 4, "bf16")
        sl = torch.from_numpy(np.clip(lens - lo, 0, hi - lo).astype(np.int32)).cuda()
        parts.append(ops.attention(tq, sub.keys, sub.values, D ** -0.5, hi - lo, 4, lens=sl,
                                   out_kind=1))
    merged = ops.combine(torch.stack(parts), torch.bfloat16)
    assert np.abs(f32_of(merged) - ref).max() < 2e-2


@pytest.mark.parametrize("lens,bits,S", [
    ([5000, 0, 1, 4096], 4, 1),       # an empty batch and a one-key batch
    ([3000, 3000, 3000, 3000, 3000, 3000], 8, 1),
    ([64, 8191, 200, 7000, 1, 4500, 33, 128], 4, 1),
    ([2500, 700, 4100], 8, 3),        # multi-token rows (causal) over ragged lengths
])
def test_ragged_lengths_balanced_against_oracle(lens, bits, S):
    """Ragged batches share the CTAs by key count (the in-kernel merge's balanced mode):
    every batch, including empty and one-key ones, against the oracle, and against the
    per-batch split mode (forced split count) on the same inputs."""
    from chad_b200 import ops

    B, HQ, HKV, D = len(lens), 16, 2, 128
    NP = (max(lens) + 255) // 256 * 256
    lens = np.array(lens, np.int32)
    q, k, v = make_case(77 + B + bits, B, HQ, HKV, S, D, NP, "bf16", outliers=True)
    c = _cache(k, v, bits, "bf16")
    tq = torch_from_f32(q, "bf16")
    tl = torch.from_numpy(lens).cuda()
    mask = "causal" if S > 1 else None
    out = ops.attention(tq, c.keys, c.values, D ** -0.5, NP, bits, lens=tl, mask=mask)
    kq, vq = _oracle_quant(k, bits, "bf16"), _oracle_quant(v, bits, "bf16")
    live = lens > 0  # a batch with no keys has no softmax: its rows come out zero

    def sel(t):
        return tuple(x[live] for x in t)

    ref = orc.attention_quantized_fp32(q[live], sel(kq), sel(vq), D ** -0.5, lens[live], bits,
                                       64, _np_mask(mask), "bf16")
    got = f32_of(out)
    assert np.isfinite(got).all()
    assert (got[~live] == 0).all()
    err = np.abs(got[live] - ref)
    assert err.max() < 2e-2 and err.mean() < 2e-3
    dense = ops.attention(tq, c.keys, c.values, D ** -0.5, NP, bits, lens=tl, mask=mask,
                          splits=5)
    assert np.abs(f32_of(dense)[live] - got[live]).max() < 2e-2


def test_prefill_chunk_over_prefix():
    """Prefix cache + new chunk quantized on append, causal within the chunk."""
    from chad_b200 import ops
    from chad_b200.cache import QuantizedKVCache

    prefix, S, D = 700, 64, 128
    q, k, v = make_case(8, 1, 32, 4, S, D, prefix + S, "bf16", outliers=True)
    c = QuantizedKVCache(group_size=64, bits=4)
    c.update_and_fetch(torch_from_f32(k[:, :, :prefix], "bf16"),
                       torch_from_f32(v[:, :, :prefix], "bf16"))
    c._grow(prefix + S, 1, 4, D, D, torch.bfloat16, torch.device("cuda"))
    out = ops.prefill(torch_from_f32(q, "bf16"), torch_from_f32(k[:, :, prefix:], "bf16"),
                      torch_from_f32(v[:, :, prefix:], "bf16"), c.keys, c.values, prefix, 4,
                      D ** -0.5)
    kq, vq = _oracle_quant(k, 4, "bf16"), _oracle_quant(v, 4, "bf16")
    ref = orc.attention_quantized_fp32(q, kq, vq, D ** -0.5, prefix + S, 4, mask="causal")
    err = np.abs(f32_of(out) - ref)
    assert err.max() < 2e-2 and err.mean() < 2e-3


@pytest.mark.parametrize("HQ,HKV,S,bits,n0", [
    (32, 4, 1, 4, 4095),   # decode step, last position of the padded buffer
    (32, 4, 1, 8, 777),
    (16, 4, 2, 4, 1000),   # short draft block, one 8-row group per kv head
    (32, 4, 2, 8, 2999),   # 16-row group
    (8, 8, 4, 4, 3000),
    (32, 2, 2, 4, 500),    # two row groups per kv head: the separate append launch
])
def test_prefill_decode_step_appends(HQ, HKV, S, bits, n0):
    """qkv_prefill on the decode path: when one query-row group covers a kv head, the
    attention kernel quantizes the new tokens into the cache itself (no append launch).
    The rows it writes are bit-exact with the oracle's quantization, the older rows are
    untouched, and the output over the whole cache matches the oracle."""
    from chad_b200 import ops

    n = n0 + S
    D = 128
    q, k, v = make_case(500 + n0 + S + bits, 1, HQ, HKV, S, D, n, "bf16", outliers=True)
    c = _cache(k[:, :, :n0], v[:, :, :n0], bits, "bf16")
    assert c.keys[0].shape[2] >= n
    tq = torch_from_f32(q, "bf16")
    kn = torch_from_f32(np.ascontiguousarray(k[:, :, n0:n]), "bf16")
    vn = torch_from_f32(np.ascontiguousarray(v[:, :, n0:n]), "bf16")
    out = ops.prefill(tq, kn, vn, c.keys, c.values, n0, bits, D ** -0.5)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    for cache_t, x in ((c.keys, k), (c.values, v)):
        w, s, b = _oracle_quant(x, bits, "bf16")
        np.testing.assert_array_equal(u32_of(cache_t[0])[:, :, :n], w)
        np.testing.assert_array_equal(bits_of(cache_t[1])[:, :, :n], s)
        np.testing.assert_array_equal(bits_of(cache_t[2])[:, :, :n], b)
    kq, vq = _oracle_quant(k, bits, "bf16"), _oracle_quant(v, bits, "bf16")
    ref = orc.attention_quantized_fp32(q, kq, vq, D ** -0.5, n, bits, 64,
                                       "causal" if S > 1 else None, "bf16")
    err = np.abs(f32_of(out) - ref)
    assert err.max() < 2e-2 and err.mean() < 2e-3
