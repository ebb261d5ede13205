"""Host-side logic that mirrors the reference's mlx_qsdpa / Engine glue (CPU only).

Ported from tests/test_mlx_qsdpa.py (split table, covers, flag, eligibility) and
tests/test_engine_kvquant.py (kv_bits auto-gate, ckpt key by kv mode), adjusted where the
B200 kernels deliberately cover more (head_dim 64/128/256, 4- and 8-bit, any GQA).
"""

import numpy as np
import pytest
import torch

from chad_b200 import engine, qsdpa
from chad_b200.cache import KVCache, QuantizedKVCache


def test_pick_blocks_table():
    for gqa in (4, 8):
        for n in (100, 8192, 16000):
            assert qsdpa._pick_blocks(n, gqa=gqa) == 32
    for n in (16384, 32000, 98304):
        assert qsdpa._pick_blocks(n, gqa=8) == 64
        assert qsdpa._pick_blocks(n, gqa=4) == 128
    for n in (100, 16384, 99999):
        for gqa in (4, 8):
            assert qsdpa._pick_blocks(n, gqa) % 32 == 0


def test_covers_b200_surface():
    assert qsdpa.covers(256, 8)      # the reference's 35B shape
    assert qsdpa.covers(256, 4)      # its 9B shape
    assert qsdpa.covers(128, 8)      # head_dim 128: covered here (not in the reference)
    assert qsdpa.covers(64, 2)
    assert not qsdpa.covers(96, 8)
    assert not qsdpa.covers(128, 8, bits=3)


def test_no_qsdpa_flag_blocks_install(monkeypatch):
    monkeypatch.setenv("CHAD_NO_QSDPA", "1")
    assert qsdpa.install() is False


def test_eligibility_declines_host_tensors_and_bad_modes():
    q = torch.zeros((1, 16, 1, 128), dtype=torch.bfloat16)
    c = QuantizedKVCache(group_size=64, bits=4)
    assert not qsdpa._eligible(q, c, None)          # empty cache
    c.keys = (torch.zeros((1, 2, 256, 16), dtype=torch.int32),
              torch.zeros((1, 2, 256, 2), dtype=torch.bfloat16),
              torch.zeros((1, 2, 256, 2), dtype=torch.bfloat16))
    c.offset = 10
    assert not qsdpa._eligible(q, c, None)          # host tensor: the kernels are CUDA only
    assert not qsdpa._eligible(q, c, "sliding")     # unknown mask string
    assert not qsdpa._eligible(q, c, 3.0)           # not a mask
    with pytest.raises(ValueError):
        QuantizedKVCache(group_size=64, bits=3)
    with pytest.raises(ValueError):
        QuantizedKVCache(group_size=32, bits=4)


# ---- kv_bits policy (tests/test_engine_kvquant.py:52-75) -----------------------------------
def test_kv_bits_auto_defaults_on_for_covered_shapes():
    r = engine.resolve_kv_bits
    assert r(None, 256, 16, 2, True) == 8     # 35B: gqa 8
    assert r(None, 256, 16, 4, True) == 8     # 9B: gqa 4
    assert r(None, 128, 32, 4, True) == 8     # head_dim 128, GQA 8: covered on B200
    assert r(None, 96, 16, 2, True) is None   # head_dim not covered
    assert r(None, 256, 16, 0, True) is None  # shape unknown
    assert r(None, 256, 16, 2, False) is None  # kernel absent


def test_kv_bits_explicit_wins():
    assert engine.resolve_kv_bits(0, 256, 16, 2, True) is None
    assert engine.resolve_kv_bits(8, 96, 16, 2, True) == 8
    assert engine.resolve_kv_bits(4, 128, 32, 4, True) == 4


def test_make_caches_quantizes_attention_layers_only():
    cs = engine.make_caches([True, False, True, False], 8)
    assert [type(c) for c in cs] == [QuantizedKVCache, type(None), QuantizedKVCache, type(None)]
    cs = engine.make_caches([True, False], None)
    assert isinstance(cs[0], KVCache) and cs[1] is None


def test_ckpt_path_keyed_by_kv_mode(tmp_path):
    a = engine.ckpt_path(str(tmp_path), "m", 8, [1, 2, 3])
    b = engine.ckpt_path(str(tmp_path), "m", None, [1, 2, 3])
    c = engine.ckpt_path(str(tmp_path), "m", 4, [1, 2, 3])
    assert len({a, b, c}) == 3
    assert engine.ckpt_path(str(tmp_path), "m", 8, [1, 2, 3]) == a
    assert engine.ckpt_path(str(tmp_path), "m", 8, [1, 2, 4]) != a
    assert "push-" in engine.ckpt_path(str(tmp_path), "m", 8, [1], tag=engine.CKPT_PUSH)


def test_trim_by_offset_bookkeeping():
    c = QuantizedKVCache(group_size=64, bits=8)
    c.offset = 12
    assert c.trim(5) == 5 and c.offset == 7
    assert c.trim(50) == 7 and c.offset == 0
    s = engine.KVSession([True, True], 8)
    for cc in s.kv_caches:
        cc.offset = 16
    s.cached_ids = list(range(16))
    assert s.trim(4) == 4
    assert s.offsets() == [12, 12] and s.cached_ids == list(range(12))


def test_warm_prefix_skips_without_cache_dir():
    s = engine.KVSession([True], 8, cache_dir=None)
    assert s.warm_prefix([1, 2, 3], lambda sess, ids: len(ids)) == ("skip", 0)
    s2 = engine.KVSession([True], 8, cache_dir="/tmp/x")
    s2.cached_ids = [9]
    assert s2.warm_prefix([1, 2], lambda sess, ids: len(ids)) == ("skip", 0)


def test_shard_ranges_cover_every_key():
    from chad_b200.shard import shard_ranges

    lens = [70000, 131072, 65536, 99999]
    for world in (1, 2, 4, 8):
        rng = [shard_ranges(lens, world, r) for r in range(world)]
        for b, L in enumerate(lens):
            got = []
            for r in range(world):
                lo, n = rng[r][0][b], rng[r][1][b]
                got.extend(range(lo, lo + n))
            assert got == list(range(L))
    assert np.all(np.array(shard_ranges([10], 4, 3)[1]) >= 0)


def test_bench_clock_sampler_parses_nvidia_smi_lines():
    """bench.py's clock record: SM MHz median, max clock and the throttle reasons named
    from the bit mask (gpu_idle dropped); malformed lines are skipped."""
    import bench

    c = bench.ClockSampler(0, 0.05)
    for line in ("1965, 1965, 0x0000000000000000", "1950, 1965, 0x0000000000000004",
                 "1900, 1965, 0x0000000000000001", "not a sample", "1965, 1965, 0x48"):
        c._parse(line)
    sm = c.summary()
    assert sm["samples"] == 4 and sm["sm_max_mhz"] == 1965 and sm["sm_mhz"] == 1957.5
    assert sm["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_power_cap"]
