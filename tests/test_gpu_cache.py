"""Cache glue, the attention seam and the self-check on the GPU (ported from
tests/test_mlx_qsdpa.py:147-247 and tests/test_engine_kvquant.py:89-180)."""

import numpy as np
import pytest

from oracle import qkv_oracle as orc
from tests.helpers import f32_of, make_case, torch_from_f32, u32_of

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _kv(seed, n, D=128, hkv=4, dtype="bf16"):
    _, k, v = make_case(seed, 1, hkv * 8, hkv, 1, D, n, dtype, outliers=True)
    return k, v


def test_update_and_fetch_grows_by_steps_and_keeps_rows():
    from chad_b200.cache import QuantizedKVCache

    c = QuantizedKVCache(group_size=64, bits=4)
    k, v = _kv(1, 700)
    for lo, hi in ((0, 100), (100, 256), (256, 300), (300, 700)):
        kk, vv = c.update_and_fetch(torch_from_f32(k[:, :, lo:hi], "bf16"),
                                    torch_from_f32(v[:, :, lo:hi], "bf16"))
        assert kk[0].shape[2] == hi and c.offset == hi
        assert c.capacity % 256 == 0 and c.capacity >= hi
    w, s, b = orc.affine_quantize(k, 4, 64, "bf16")
    np.testing.assert_array_equal(u32_of(c.keys[0])[:, :, :700], w)


def test_kv_bytes_per_token_ratio():
    from chad_b200 import engine
    from chad_b200.cache import KVCache, QuantizedKVCache

    k, v = _kv(2, 64)
    q8, q4, fp = QuantizedKVCache(64, 8), QuantizedKVCache(64, 4), KVCache()
    for c in (q8, q4, fp):
        c.update_and_fetch(torch_from_f32(k, "bf16"), torch_from_f32(v, "bf16"))
    b8 = engine.kv_bytes_per_token([q8])
    b4 = engine.kv_bytes_per_token([q4])
    bf = engine.kv_bytes_per_token([fp])
    assert 0.2 * bf < b8 < 0.7 * bf        # tests/test_engine_kvquant.py:114
    assert b4 < b8


def test_trim_then_refeed_rewrites_identically():
    from chad_b200.cache import QuantizedKVCache

    k, v = _kv(3, 300)
    c = QuantizedKVCache(64, 8)
    c.update_and_fetch(torch_from_f32(k, "bf16"), torch_from_f32(v, "bf16"))
    ref = [t.clone() for t in c.keys]
    assert c.trim(44) == 44 and c.offset == 256
    c.update_and_fetch(torch_from_f32(k[:, :, 256:], "bf16"), torch_from_f32(v[:, :, 256:], "bf16"))
    for a, b in zip(c.keys, ref):
        assert torch.equal(a[:, :, :300], b[:, :, :300])


def test_warm_prefix_roundtrip_and_mode_isolation(tmp_path):
    """tests/test_engine_kvquant.py:155-180 on the HBM layout."""
    from chad_b200 import engine
    from chad_b200.cache import KVCache, QuantizedKVCache

    def prefill(sess, ids):
        g = torch.Generator(device="cuda").manual_seed(sum(ids))
        for c in sess.kv_caches:
            k = torch.randn((1, 2, len(ids), 128), generator=g, device="cuda").to(torch.bfloat16)
            v = torch.randn((1, 2, len(ids), 128), generator=g, device="cuda").to(torch.bfloat16)
            c.update_and_fetch(k, v)
        return len(ids)

    ids = [5, 9, 3, 7, 12, 44, 2, 8]
    mk = lambda bits: engine.KVSession([True, False, True], bits, "tiny", str(tmp_path))  # noqa
    a = mk(8)
    assert a.warm_prefix(ids, prefill) == ("miss", len(ids))
    hit = mk(8)
    assert hit.warm_prefix(ids, prefill) == ("hit", len(ids))
    assert [type(c) for c in hit.caches] == [QuantizedKVCache, type(None), QuantizedKVCache]
    for c0, c1 in zip(a.kv_caches, hit.kv_caches):
        assert c1.offset == len(ids)
        for t0, t1 in zip(c0.keys + c0.values, c1.keys + c1.values):
            assert torch.equal(t0[:, :, :8], t1[:, :, :8])
    fp = mk(None)
    assert fp.warm_prefix(ids, prefill)[0] == "miss"  # never cross-loads the kv8 file
    assert all(isinstance(c, KVCache) for c in fp.kv_caches)
    q4 = mk(4)
    assert q4.warm_prefix(ids, prefill)[0] == "miss"


def test_rewind_trims_and_refeeds():
    from chad_b200 import engine

    fed = []

    def prefill(sess, ids):
        fed.append(list(ids))
        for c in sess.kv_caches:
            k = torch.randn((1, 2, len(ids), 128), device="cuda").to(torch.bfloat16)
            c.update_and_fetch(k, k)
        return len(ids)

    s = engine.KVSession([True, True], 8)
    base = [7, 12, 33, 8, 91, 40, 55, 2, 19, 77, 30, 4]
    prefill(s, base)
    s.cached_ids = list(base)
    prefill(s, [64, 25, 3, 88])
    s.cached_ids = base + [64, 25, 3, 88]
    assert s.offsets() == [16, 16]
    assert s.rewind_to(base + [5, 6], len(base), prefill) == len(base)
    assert s.offsets() == [12, 12] and s.cached_ids == base
    s.rewind_to(base + [5, 6], len(base) + 2, prefill)
    assert s.offsets() == [14, 14] and fed[-1] == [5, 6]


# ---------------------------------------------------------------- seam + self-check
def test_install_patches_seam_and_matches():
    from chad_b200 import attention, qsdpa
    from chad_b200.cache import QuantizedKVCache

    assert qsdpa.install()
    assert getattr(attention.scaled_dot_product_attention, "_chad_qsdpa", False)
    assert qsdpa.install()  # idempotent
    n = 700
    q, k, v = make_case(5, 1, 16, 2, 1, 256, n, "f16")
    c = QuantizedKVCache(64, 8)
    keys, values = c.update_and_fetch(torch_from_f32(k, "f16"), torch_from_f32(v, "f16"))
    out = attention.scaled_dot_product_attention(torch_from_f32(q, "f16"), keys, values,
                                                 cache=c, scale=256 ** -0.5, mask=None)
    kq, vq = orc.affine_quantize(k, 8, 64, "f16"), orc.affine_quantize(v, 8, 64, "f16")
    ref = orc.attention_quantized_fp32(q, kq, vq, 256 ** -0.5, n, 8, scale_dtype="f16")
    assert np.abs(f32_of(out) - ref).max() < 2e-3


def test_install_leaves_plain_cache_on_stock():
    from chad_b200 import attention, qsdpa
    from chad_b200.cache import KVCache

    qsdpa.install()
    q, k, v = make_case(6, 1, 16, 2, 1, 128, 128, "f16")
    c = KVCache()
    keys, values = c.update_and_fetch(torch_from_f32(k, "f16"), torch_from_f32(v, "f16"))
    tq = torch_from_f32(q, "f16")
    out = attention.scaled_dot_product_attention(tq, keys, values, cache=c, scale=0.1)
    stock = attention.scaled_dot_product_attention._stock(tq, keys, values, cache=c, scale=0.1)
    assert torch.equal(out, stock)


def test_prefill_route_through_seam_causal():
    from chad_b200 import attention, qsdpa
    from chad_b200.cache import QuantizedKVCache

    qsdpa.install()
    n_prev, s_new = 512, 64
    q, k, v = make_case(7, 1, 16, 2, s_new, 128, n_prev + s_new, "bf16")
    c = QuantizedKVCache(64, 4)
    keys, values = c.update_and_fetch(torch_from_f32(k, "bf16"), torch_from_f32(v, "bf16"))
    out = attention.scaled_dot_product_attention(torch_from_f32(q, "bf16"), keys, values,
                                                 cache=c, scale=128 ** -0.5, mask="causal")
    kq, vq = orc.affine_quantize(k, 4, 64), orc.affine_quantize(v, 4, 64)
    ref = orc.attention_quantized_fp32(q, kq, vq, 128 ** -0.5, n_prev + s_new, 4, mask="causal")
    err = np.abs(f32_of(out) - ref)
    assert err.max() < 2e-2 and err.mean() < 2e-3


def test_self_check_passes_and_catches_poisoned_kernel(monkeypatch):
    from chad_b200 import qsdpa

    monkeypatch.setattr(qsdpa, "_KERNEL_HEALTHY", None)
    assert qsdpa.kernel_healthy() is True

    def nan_kernel(q, keys, values, scale, n, **kw):
        return torch.full_like(q, float("nan"))

    monkeypatch.setattr(qsdpa, "qsdpa", nan_kernel)
    monkeypatch.setattr(qsdpa, "_KERNEL_HEALTHY", None)
    assert qsdpa.kernel_healthy() is False
    calls = []
    monkeypatch.setattr(qsdpa, "qsdpa", lambda *a, **k: calls.append(1))
    assert qsdpa.kernel_healthy() is False and not calls  # cached verdict


# ---------------------------------------------------------------- shards on one GPU
def test_causal_shards_with_pos_base_merge_to_full_attention():
    from chad_b200 import ops
    from chad_b200.cache import QuantizedKVCache

    S, n, D = 4, 1500, 128
    q, k, v = make_case(8, 2, 32, 4, S, D, n, "bf16", outliers=True)
    tq = torch_from_f32(q, "bf16")
    cuts = [0, 400, 1111, n]
    parts = []
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        c = QuantizedKVCache(64, 4)
        c.update_and_fetch(torch_from_f32(k[:, :, lo:hi], "bf16"),
                           torch_from_f32(v[:, :, lo:hi], "bf16"))
        dev = torch.device("cuda")
        pb = torch.full((2,), lo, dtype=torch.int32, device=dev)
        tot = torch.full((2,), n, dtype=torch.int32, device=dev)
        ln = torch.full((2,), hi - lo, dtype=torch.int32, device=dev)
        parts.append(ops.attention(tq, c.keys, c.values, D ** -0.5, hi - lo, 4, lens=ln,
                                   pos_base=pb, total_lens=tot, mask="causal", out_kind=1))
    out = ops.combine(torch.stack(parts), torch.bfloat16)
    kq, vq = orc.affine_quantize(k, 4, 64), orc.affine_quantize(v, 4, 64)
    ref = orc.attention_quantized_fp32(q, kq, vq, D ** -0.5, n, 4, mask="causal")
    err = np.abs(f32_of(out) - ref)
    assert err.max() < 2e-2 and err.mean() < 2e-3


def test_device_status_clean_after_runs():
    from chad_b200 import ops

    assert ops.device_status(reset=True) == 0
