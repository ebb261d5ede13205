"""The CUDA path against the oracle at every benchmark configuration, at its stated size.

Each configuration the benchmark measures is checked here at the size it is measured at,
against the oracle's dequantize -> fp32 attention (tests/test_mlx_qsdpa.py:52-65) with the
configurations' tolerance (max-abs 2e-2, mean-abs 2e-3), or the reference's own tolerance
classes where its test shape is used (2e-3 fp16 / 8e-3 bf16, test_mlx_qsdpa.py:133-144):

* single-layer 4-bit decode over 4096 keys, HQ16/HKV2, K/V quantized from fp32 with bf16
  scales (codes checked bit-exact too);
* decode over 32768 keys, HQ32/HKV4, 8-bit and 4-bit, through qkv_attention and through the
  one-launch decode step (qkv_prefill appends the new token itself);
* an 8-token speculative-verify block over 16384 4-bit keys, causal in the block;
* a 2048-token prefill chunk after a 30720-token 4-bit prefix (a strided sample of 129 query
  rows, first and last included, is compared; every appended row's codes are bit-exact);
* batch 4 with ragged 64K-128K key counts on the balanced plan, and the same sequences
  split in two shards (pos_base / total_lens) merged by qkv_combine;
* the reference's wide-split case (D256, 8-bit, HQ16/HKV4, n=16500), automatic and 128
  forced splits;
* large-magnitude data: V at 1e4-1e5, q at 1e2 (K scaled down so scores stay moderate),
  held to the oracle relative to the data's scale.

Big caches are generated and quantized on the GPU and read back for the oracle; a sample of
their rows is re-quantized by the oracle and must match bit for bit, so the oracle's input
is pinned independently of the kernel under test. The distance to the restated stock path
(mlx-lm's unfused route, which the reference takes at head_dim 128) is printed and loosely
bounded.
"""

import numpy as np
import pytest

from oracle import qkv_oracle as orc
from tests.helpers import bits_of, f32_of, make_case, torch_from_f32, u32_of

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL_MAX, TOL_MEAN = 2e-2, 2e-3
OUTLIERS = list(orc.OUTLIER_CHANNELS)


def _gpu_kv(seed, B, HKV, n, D, k_scale=1.0, v_scale=1.0, dtype=torch.bfloat16):
    """K (key outlier channels x8) and V ~ N(0,1), generated on the GPU."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn((B, HKV, n, D), generator=g, device="cuda")
    k[..., OUTLIERS] *= 8.0
    v = torch.randn((B, HKV, n, D), generator=g, device="cuda")
    return (k * k_scale).to(dtype), (v * v_scale).to(dtype)


def _cache_of(k, v, bits):
    from chad_b200.cache import QuantizedKVCache

    c = QuantizedKVCache(group_size=64, bits=bits)
    c.update_and_fetch(k, v)
    return c


def _readback(tup, n, dtype="bf16"):
    """A cache tuple on the GPU -> (uint32 codes, uint16 scale bits, uint16 bias bits)."""
    w, s, b = (t[:, :, :n] for t in tup)
    return u32_of(w), bits_of(s), bits_of(b)


def _check_quant_sample(x_gpu, tup_np, bits, dtype="bf16", rows=2048, seed=0):
    """Re-quantize a random sample of rows with the oracle: must equal the cache bit for bit."""
    B, H, n, D = x_gpu.shape
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, n, size=min(rows, n))
    xs = x_gpu[:, :, torch.as_tensor(idx, device=x_gpu.device)].float().cpu().numpy()
    w, s, b = orc.affine_quantize(xs, bits, 64, dtype)
    np.testing.assert_array_equal(tup_np[0][:, :, idx], w)
    np.testing.assert_array_equal(tup_np[1][:, :, idx], s)
    np.testing.assert_array_equal(tup_np[2][:, :, idx], b)


def _err(got, ref, tol_max=TOL_MAX, tol_mean=TOL_MEAN, what=""):
    g = f32_of(got) if not isinstance(got, np.ndarray) else got
    assert np.isfinite(g).all(), what
    e = np.abs(g - ref)
    assert e.max() < tol_max and e.mean() < tol_mean, (what, float(e.max()), float(e.mean()))
    return float(e.max()), float(e.mean())


def _stock_distance(out, q, kq, vq, n, bits, dtype="bf16"):
    stock = orc.attention_stock(q, kq, vq, q.shape[-1] ** -0.5, n, bits, 64, None, dtype)
    d = np.abs(f32_of(out) - stock)
    print(f"distance to the stock path: max {d.max():.3e} mean {d.mean():.3e}")
    assert d.max() < 0.15 and d.mean() < 1e-2
    return d


def _q(seed, B, HQ, S, D, scale=1.0, dtype="bf16"):
    rng = np.random.default_rng(seed)
    return orc.round_to(rng.standard_normal((B, HQ, S, D), dtype=np.float32) * np.float32(scale),
                        dtype)


# ---------------------------------------------------------------------------------------
def test_decode4k_fp32_kv_bf16_scales():
    """Single-layer 4-bit decode: B1 S1 HQ16 HKV2 D128 N4096; K,V fp32 N(0,1) (key
    outliers) quantized with bf16 scales and biases; q bf16; scale 1/sqrt(128)."""
    from chad_b200 import ops, qsdpa
    from chad_b200.cache import QuantizedKVCache

    rng = np.random.default_rng(1)
    n, D = 4096, 128
    q = orc.round_to(rng.standard_normal((1, 16, 1, D), dtype=np.float32), "bf16")
    k = orc.make_kv(rng, (1, 2, n, D), outliers=True, dtype="f32")
    v = orc.make_kv(rng, (1, 2, n, D), outliers=False, dtype="f32")
    c = QuantizedKVCache(group_size=64, bits=4)
    c.reserve(n, 1, 2, D, torch.bfloat16, torch.device("cuda"))
    ops.quantize_append_kv(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), c.keys,
                           c.values, 0, 4)
    c.offset = n
    kq = orc.affine_quantize(k, 4, 64, "bf16")
    vq = orc.affine_quantize(v, 4, 64, "bf16")
    for got, want in zip(_readback(c.keys, n) + _readback(c.values, n), kq + vq):
        np.testing.assert_array_equal(got, want)
    out = qsdpa.qsdpa(torch_from_f32(q, "bf16"), c.keys, c.values, D ** -0.5, n)
    ref = orc.attention_quantized_fp32(q, kq, vq, D ** -0.5, n, 4)
    _err(out, ref)
    _stock_distance(out, q, kq, vq, n, 4)


@pytest.mark.parametrize("bits", [8, 4])
def test_decode32k(bits):
    """B1 S1 HQ32 HKV4 D128 over 32768 keys (8-bit: the headline workload; 4-bit: the
    north-star decode), q ~ N(0,1) bf16, K/V bf16 with key outliers."""
    from chad_b200 import ops

    n, D = 32768, 128
    k, v = _gpu_kv(100 + bits, 1, 4, n, D)
    c = _cache_of(k, v, bits)
    kq, vq = _readback(c.keys, n), _readback(c.values, n)
    _check_quant_sample(k, kq, bits)
    _check_quant_sample(v, vq, bits, seed=1)
    q = _q(200 + bits, 1, 32, 1, D)
    out = ops.attention(torch_from_f32(q, "bf16"), c.keys, c.values, D ** -0.5, n, bits)
    ref = orc.attention_quantized_rows(q, kq, vq, D ** -0.5, n, bits)
    _err(out, ref, what="attention")
    _stock_distance(out, q, kq, vq, n, bits)


@pytest.mark.parametrize("bits", [8, 4])
def test_decode32k_step_appends_its_token(bits):
    """The one-launch decode step at 32K keys: the cache holds 32767 keys, qkv_prefill
    quantizes the 32768th into it inside the attention kernel and attends over all."""
    from chad_b200 import ops

    n, D = 32768, 128
    k, v = _gpu_kv(300 + bits, 1, 4, n, D)
    c = _cache_of(k[:, :, : n - 1].contiguous(), v[:, :, : n - 1].contiguous(), bits)
    q = _q(400 + bits, 1, 32, 1, D)
    out = ops.prefill(torch_from_f32(q, "bf16"), k[:, :, n - 1:].contiguous(),
                      v[:, :, n - 1:].contiguous(), c.keys, c.values, n - 1, bits, D ** -0.5)
    kq, vq = _readback(c.keys, n), _readback(c.values, n)
    last_k = orc.affine_quantize(k[:, :, n - 1:].float().cpu().numpy(), bits, 64, "bf16")
    last_v = orc.affine_quantize(v[:, :, n - 1:].float().cpu().numpy(), bits, 64, "bf16")
    for got, want in zip(kq + vq, last_k + last_v):
        np.testing.assert_array_equal(got[:, :, n - 1:], want)
    ref = orc.attention_quantized_rows(q, kq, vq, D ** -0.5, n, bits)
    _err(out, ref)


def test_verify_block_16k():
    """Speculative verify: 8 draft tokens at the tail of a 16384-key 4-bit cache, causal in
    the block, HQ32 HKV4 D128 — through qkv_attention (drafts already in the cache) and
    through qkv_prefill (the drafts appended by the call)."""
    from chad_b200 import ops

    n, S, D = 16384, 8, 128
    k, v = _gpu_kv(500, 1, 4, n, D)
    q = _q(501, 1, 32, S, D)
    tq = torch_from_f32(q, "bf16")
    c = _cache_of(k, v, 4)
    kq, vq = _readback(c.keys, n), _readback(c.values, n)
    _check_quant_sample(k, kq, 4)
    pos = np.arange(n - S, n)[None, :]
    ref = orc.attention_quantized_rows(q, kq, vq, D ** -0.5, n, 4, q_pos=pos)
    out = ops.attention(tq, c.keys, c.values, D ** -0.5, n, 4, mask="causal")
    _err(out, ref, what="attention")
    from chad_b200.cache import QuantizedKVCache

    c2 = QuantizedKVCache(group_size=64, bits=4)
    c2.reserve(n, 1, 4, D, torch.bfloat16, torch.device("cuda"))
    c2.update_and_fetch(k[:, :, : n - S].contiguous(), v[:, :, : n - S].contiguous())
    out2 = ops.prefill(tq, k[:, :, n - S:].contiguous(), v[:, :, n - S:].contiguous(), c2.keys,
                       c2.values, n - S, 4, D ** -0.5)
    for got, want in zip(_readback(c2.keys, n) + _readback(c2.values, n), kq + vq):
        np.testing.assert_array_equal(got, want)
    _err(out2, ref, what="prefill")


def test_prefill_2048_over_30720_prefix():
    """Prefix-cache prefill: 2048 new tokens after a 30720-token 4-bit prefix, causal over
    the new chunk, full visibility of the prefix, HQ32 HKV4 D128 (the tensor-core path)."""
    from chad_b200 import ops

    from chad_b200.cache import QuantizedKVCache

    P, S, D = 30720, 2048, 128
    n = P + S
    k, v = _gpu_kv(600, 1, 4, n, D)
    c = QuantizedKVCache(group_size=64, bits=4)
    c.reserve(n, 1, 4, D, torch.bfloat16, torch.device("cuda"))  # room for the new chunk
    c.update_and_fetch(k[:, :, :P].contiguous(), v[:, :, :P].contiguous())
    q = _q(601, 1, 32, S, D)
    out = ops.prefill(torch_from_f32(q, "bf16"), k[:, :, P:].contiguous(),
                      v[:, :, P:].contiguous(), c.keys, c.values, P, 4, D ** -0.5)
    kq, vq = _readback(c.keys, n), _readback(c.values, n)
    # every appended row, bit for bit
    nk = orc.affine_quantize(k[:, :, P:].float().cpu().numpy(), 4, 64, "bf16")
    nv = orc.affine_quantize(v[:, :, P:].float().cpu().numpy(), 4, 64, "bf16")
    for got, want in zip(kq + vq, nk + nv):
        np.testing.assert_array_equal(got[:, :, P:], want)
    _check_quant_sample(k[:, :, :P], tuple(t[:, :, :P] for t in kq), 4)
    rows = sorted(set(range(0, S, 16)) | {S - 1})
    assert len(rows) >= 128
    ref = orc.attention_quantized_rows(q[:, :, rows], kq, vq, D ** -0.5, n, 4,
                                       q_pos=(P + np.asarray(rows))[None, :])
    _err(f32_of(out)[:, :, rows], ref)


def _ragged_lens(B=4, seed=1234):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(65536, 131072 + 1, (B,), generator=g).tolist()


def test_long_context_ragged_batch_and_two_shards():
    """Batch 4, ragged key counts in [65536, 131072], 4-bit, HQ32 HKV4 D128, one decode
    token: the balanced plan on one GPU, and the same sequences split into two contiguous
    shards (pos_base / total_lens) whose partial rows qkv_combine merges."""
    from chad_b200 import ops

    B, D, bits = 4, 128, 4
    lens = _ragged_lens(B)
    nmax = max(lens)
    k, v = _gpu_kv(700, B, 4, nmax, D)
    c = _cache_of(k, v, bits)
    del k, v
    kq, vq = _readback(c.keys, nmax), _readback(c.values, nmax)
    q = _q(701, B, 32, 1, D)
    tq = torch_from_f32(q, "bf16")
    lens_t = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = ops.attention(tq, c.keys, c.values, D ** -0.5, nmax, bits, lens=lens_t)
    ref = orc.attention_quantized_rows(q, kq, vq, D ** -0.5, lens, bits)
    _err(out, ref, what="balanced")

    parts = []
    for r in range(2):
        base = [L * r // 2 for L in lens]
        loc = [L * (r + 1) // 2 - L * r // 2 for L in lens]
        npad = (max(loc) + 255) // 256 * 256
        sk, sv = [], []
        for src, dst in ((c.keys, sk), (c.values, sv)):
            for t in src:
                s = torch.zeros((B, 4, npad, t.shape[-1]), dtype=t.dtype, device="cuda")
                for b in range(B):
                    s[b, :, : loc[b]] = t[b, :, base[b]: base[b] + loc[b]]
                dst.append(s)
        p = ops.attention(tq, tuple(sk), tuple(sv), D ** -0.5, max(loc), bits,
                          lens=torch.tensor(loc, dtype=torch.int32, device="cuda"),
                          pos_base=torch.tensor(base, dtype=torch.int32, device="cuda"),
                          total_lens=lens_t, out_kind=1)
        parts.append(p)
    merged = ops.combine(torch.stack(parts).contiguous(), torch.bfloat16)
    _err(merged, ref, what="two shards")


@pytest.mark.parametrize("dtype,tol", [("f16", 2e-3), ("bf16", 8e-3)])
@pytest.mark.parametrize("splits", [0, 128])
def test_reference_wide_split_case(dtype, tol, splits):
    """tests/test_mlx_qsdpa.py:133-144: D256, 8-bit, HQ16 HKV4 (GQA 4), n=16500, K/V
    0.7 N(0,1): the reference's blocks=128 tier; here automatic and 128 forced splits (the
    forced grid is larger than one wave, so it takes the two-launch merge)."""
    from chad_b200 import qsdpa

    n, D = 16500, 256
    q, k, v = make_case(3, 1, 16, 4, 1, D, n, dtype, kv_scale=0.7)
    c = _cache_of(torch_from_f32(k, dtype), torch_from_f32(v, dtype), 8)
    kq = orc.affine_quantize(k, 8, 64, dtype)
    vq = orc.affine_quantize(v, 8, 64, dtype)
    out = qsdpa.qsdpa(torch_from_f32(q, dtype), c.keys, c.values, D ** -0.5, n, splits=splits)
    ref = orc.attention_quantized_fp32(q, kq, vq, D ** -0.5, n, 8, 64, None, dtype)
    _err(out, ref, tol_max=tol, tol_mean=tol)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("v_scale", [1e4, 1e5])
def test_large_magnitude_values(bits, dtype, v_scale):
    """V at 1e4-1e5 (group scales far above what a 16-bit P*scale product holds unscaled),
    q at 1e2 with K scaled down by 1e-2 so the scores stay moderate. Held to the oracle
    relative to the data's scale. (f16 caches hold values below 65504 only.)"""
    from chad_b200 import ops

    if dtype == "f16" and v_scale > 1e4:
        v_scale = 6e3  # N(0,1) * 6e3 stays inside f16's range
    n, D = 5000, 128
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    k, v = _gpu_kv(800 + bits, 1, 4, n, D, k_scale=1e-2, v_scale=v_scale, dtype=tdt)
    c = _cache_of(k, v, bits)
    kq, vq = _readback(c.keys, n), _readback(c.values, n)
    q = _q(801, 1, 32, 1, D, scale=100.0, dtype=dtype)
    out = ops.attention(torch_from_f32(q, dtype), c.keys, c.values, D ** -0.5, n, bits)
    ref = orc.attention_quantized_rows(q, kq, vq, D ** -0.5, n, bits, scale_dtype=dtype)
    _err(out, ref, tol_max=TOL_MAX * v_scale, tol_mean=TOL_MEAN * v_scale)
    # and through the tensor-core path (a verify block), which stages dequantized tiles
    q8 = _q(802, 1, 32, 8, D, scale=100.0, dtype=dtype)
    out8 = ops.attention(torch_from_f32(q8, dtype), c.keys, c.values, D ** -0.5, n, bits,
                         mask="causal")
    ref8 = orc.attention_quantized_rows(q8, kq, vq, D ** -0.5, n, bits, scale_dtype=dtype,
                                        q_pos=np.arange(n - 8, n)[None, :])
    _err(out8, ref8, tol_max=TOL_MAX * v_scale, tol_mean=TOL_MEAN * v_scale)
