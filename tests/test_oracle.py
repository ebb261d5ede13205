"""The CPU oracle pinned on hand-derived known answers, the reference tests' relations and
the committed golden fixtures. No GPU needed."""

import os

import numpy as np
import pytest

from oracle import qkv_oracle as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "qkv_golden.npz")


# ---------------------------------------------------------------- packing / quantize KATs
def test_codes_pack_lsb_first():
    codes4 = np.arange(8, dtype=np.float32)
    # a group whose min is 0 and max 7 at 4 bits: scale 7/15 -> codes are not identity,
    # so check the packer directly through unpack_codes round trip instead
    w = np.array([[0x76543210]], dtype=np.uint32)
    np.testing.assert_array_equal(orc.unpack_codes(w, 4)[0], np.arange(8))
    w8 = np.array([[0x04030201]], dtype=np.uint32)
    np.testing.assert_array_equal(orc.unpack_codes(w8, 8)[0], [1, 2, 3, 4])
    assert codes4.size == 8


def test_quantize_known_answer_linear_ramp():
    # 64 values from -1 to 2: max=2 dominates, so scale is negative and the edge is 2
    x = np.linspace(-1.0, 2.0, 64, dtype=np.float32)[None, :]
    w, s, b = orc.affine_quantize(x, 4, 64, "bf16")
    scale = orc.bf16_bits_to_f32(s)[0, 0]
    bias = orc.bf16_bits_to_f32(b)[0, 0]
    assert bias == 2.0
    assert scale == pytest.approx(-0.2, rel=1e-2)
    c = orc.unpack_codes(w, 4)[0]
    assert c[-1] == 0 and c[0] == 15           # x=2 -> code 0, x=-1 -> code 15
    assert np.all(np.diff(c.astype(int)) <= 0)  # monotone in x (negative scale)


def test_quantize_degenerate_groups():
    zeros = np.zeros((1, 64), np.float32)
    w, s, b = orc.affine_quantize(zeros, 8, 64, "bf16")
    assert np.all(orc.unpack_codes(w, 8) == 0)
    assert orc.bf16_bits_to_f32(b)[0, 0] == 0.0
    np.testing.assert_array_equal(orc.dequantize_f32(w, s, b, 8), zeros)
    const = np.full((1, 64), 3.0, np.float32)
    w, s, b = orc.affine_quantize(const, 4, 64, "bf16")
    np.testing.assert_array_equal(orc.dequantize_f32(w, s, b, 4), const)


@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_round_trip_error_bound(bits):
    rng = np.random.default_rng(bits)
    x = orc.make_kv(rng, (3, 5, 128), outliers=True)
    w, s, b = orc.affine_quantize(x, bits, 64, "f16")
    deq = orc.dequantize_f32(w, s, b, bits, 64, "f16")
    step = np.abs(orc.f16_bits_to_f32(s)).repeat(64, axis=-1)
    # half a step inside the range; the far end may clip by up to one step because the
    # scale is re-fitted so that the dominant edge is exact (edge / rint(edge / scale))
    err = np.abs(deq - x)
    assert np.all(err <= step + 1e-2 * np.abs(x) + 1e-3)
    assert np.mean(err <= 0.5 * step + 1e-2 * np.abs(x) + 1e-3) > 0.97


def test_dequantize_modes_differ_but_fused_is_single_rounding():
    rng = np.random.default_rng(0)
    x = orc.make_kv(rng, (4, 256), outliers=True)
    kq = orc.affine_quantize(x, 4, 64, "bf16")
    fused = orc.dequantize(*kq, 4, 64, "bf16", "fused")
    per_op = orc.dequantize(*kq, 4, 64, "bf16", "per_op")
    assert (fused != per_op).any()           # the two rounding conventions are distinct
    c = orc.unpack_codes(kq[0], 4).astype(np.float64)
    s = orc.bf16_bits_to_f32(kq[1]).astype(np.float64).repeat(64, -1)
    bb = orc.bf16_bits_to_f32(kq[2]).astype(np.float64).repeat(64, -1)
    exact = (s * c + bb).astype(np.float32)  # exact in f64, then one fp32 rounding
    np.testing.assert_array_equal(fused, orc.f32_to_bf16_bits(exact))


# ---------------------------------------------------------------- attention relations
def _naive(q, k, v, scale, causal=False):
    out = np.zeros_like(q)
    gqa = q.shape[1] // k.shape[1]
    n = k.shape[2]
    for b in range(q.shape[0]):
        for h in range(q.shape[1]):
            for s in range(q.shape[2]):
                sc = [float(np.dot(q[b, h, s] * scale, k[b, h // gqa, j])) for j in range(n)]
                lim = n - q.shape[2] + s if causal else n - 1
                sc = np.array([x if j <= lim else -np.inf for j, x in enumerate(sc)])
                p = np.exp(sc - sc.max())
                p /= p.sum()
                out[b, h, s] = p @ v[b, h // gqa]
    return out


def test_attention_matches_naive_and_causal_alignment():
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 4, 3, 16), dtype=np.float32)
    k = rng.standard_normal((1, 2, 9, 16), dtype=np.float32)
    v = rng.standard_normal((1, 2, 9, 16), dtype=np.float32)
    np.testing.assert_allclose(orc.attention_fp32(q, k, v, 0.25, 9), _naive(q, k, v, 0.25),
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(orc.attention_fp32(q, k, v, 0.25, 9, "causal"),
                               _naive(q, k, v, 0.25, causal=True), rtol=1e-5, atol=1e-6)


def test_masks_bool_additive_equivalent_and_empty_rows():
    rng = np.random.default_rng(2)
    q = rng.standard_normal((1, 2, 2, 16), dtype=np.float32)
    k = rng.standard_normal((1, 1, 7, 16), dtype=np.float32)
    v = rng.standard_normal((1, 1, 7, 16), dtype=np.float32)
    keep = rng.random((1, 2, 2, 7)) > 0.4
    keep[0, 0, 1, :] = False  # one fully masked row -> zeros
    add = np.where(keep, 0.0, -np.inf).astype(np.float32)
    a = orc.attention_fp32(q, k, v, 0.3, 7, keep)
    b = orc.attention_fp32(q, k, v, 0.3, 7, add)
    np.testing.assert_allclose(a, b, rtol=1e-6, atol=1e-7)
    assert np.all(a[0, 0, 1] == 0)


def test_split_partials_combine_is_associative():
    """Pass 1 per block + pass-2 LSE combine equals one softmax (mlx_qsdpa.py:73-265)."""
    rng = np.random.default_rng(4)
    q = rng.standard_normal((8, 32), dtype=np.float32)
    k = rng.standard_normal((2, 200, 32), dtype=np.float32)
    v = rng.standard_normal((2, 200, 32), dtype=np.float32)
    full = orc.attention_fp32(q[None, :, None], k[None], v[None], 0.2, 170)[0, :, 0]
    for splits in (1, 3, 32, 200):
        m, s, p = orc.split_partials_fp32(q, k, v, 0.2, 170, splits)
        np.testing.assert_allclose(orc.lse_combine(m, s, p), full, rtol=2e-5, atol=2e-6)


def test_padded_tail_is_ignored_by_the_oracle():
    rng = np.random.default_rng(5)
    q = orc.round_to(rng.standard_normal((1, 16, 1, 128), dtype=np.float32), "bf16")
    k = orc.make_kv(rng, (1, 2, 512, 128))
    v = orc.make_kv(rng, (1, 2, 512, 128))
    kq = orc.affine_quantize(k, 8, 64, "bf16")
    vq = orc.affine_quantize(v, 8, 64, "bf16")
    a = orc.attention_quantized_fp32(q, kq, vq, 0.1, 300, 8)
    kq[0][:, :, 300:] = 0xFFFFFFFF
    kq[1][:, :, 300:] = orc.f32_to_bf16_bits(np.float32(100.0))
    b = orc.attention_quantized_fp32(q, kq, vq, 0.1, 300, 8)
    np.testing.assert_array_equal(a, b)


def test_stock_path_distance_from_fp32_reference():
    """mlx-lm's unfused path rounds the scores and the softmax to bf16, so it sits up to
    ~5e-2 (max-abs) from the dequantize->fp32 reference on key-outlier data while staying
    close on average; the fused kernels are held to the fp32 reference instead."""
    rng = np.random.default_rng(6)
    q = orc.round_to(rng.standard_normal((1, 8, 1, 128), dtype=np.float32), "bf16")
    k = orc.make_kv(rng, (1, 2, 300, 128), outliers=True)
    v = orc.make_kv(rng, (1, 2, 300, 128))
    kq, vq = orc.affine_quantize(k, 4, 64), orc.affine_quantize(v, 4, 64)
    a = orc.attention_stock(q, kq, vq, 128 ** -0.5, 300, 4)
    b = orc.attention_quantized_fp32(q, kq, vq, 128 ** -0.5, 300, 4)
    err = np.abs(a - b)
    assert err.max() < 1e-1 and err.mean() < 2e-3


def test_cpu_stock_torch_matches_numpy_oracle():
    torch = pytest.importorskip("torch")
    from oracle import cpu_stock

    rng = np.random.default_rng(7)
    q = orc.round_to(rng.standard_normal((1, 8, 1, 128), dtype=np.float32), "bf16")
    k = orc.make_kv(rng, (1, 2, 257, 128), outliers=True)
    v = orc.make_kv(rng, (1, 2, 257, 128))
    for bits in (4, 8):
        kq, vq = orc.affine_quantize(k, bits, 64), orc.affine_quantize(v, bits, 64)

        def t(qt):
            return (torch.from_numpy(qt[0].view(np.int32)),
                    torch.from_numpy(qt[1].view(np.int16)).view(torch.bfloat16),
                    torch.from_numpy(qt[2].view(np.int16)).view(torch.bfloat16))

        kd = cpu_stock.dequantize(*t(kq), bits).view(torch.int16).numpy().view(np.uint16)
        np.testing.assert_array_equal(kd, orc.dequantize(*kq, bits))
        tq = torch.from_numpy(orc.f32_to_bf16_bits(q).view(np.int16)).view(torch.bfloat16)
        got = cpu_stock.attention(tq, t(kq), t(vq), 128 ** -0.5, 257, bits).float().numpy()
        ref = orc.attention_quantized_fp32(q, kq, vq, 128 ** -0.5, 257, bits)
        assert np.abs(got - ref).max() < 2e-2  # output rounded to bf16


# ---------------------------------------------------------------- golden fixtures
def test_golden_fixtures_reproduce():
    g = np.load(GOLDEN)
    from tests.golden.make_golden import build

    fresh = build()
    assert set(fresh) == set(g.files)
    for name in g.files:
        np.testing.assert_array_equal(fresh[name], g[name], err_msg=name)
