"""The attention workspace contract: zero before the first call, zero after every call.

The decode kernel's in-kernel merge reads a partial-row word as "not yet written" while it
is zero and clears every word it reads; the tensor-core path's combine clears the partials
it reads. So one zeroed workspace serves any sequence of shapes and paths, and a call's
result never depends on what ran before it.
"""

import numpy as np
import pytest

from tests.helpers import make_case, torch_from_f32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _cache(k, v, bits, dtype):
    from chad_b200.cache import QuantizedKVCache

    c = QuantizedKVCache(group_size=64, bits=bits)
    c.update_and_fetch(torch_from_f32(k, dtype), torch_from_f32(v, dtype))
    return c


# (HQ, HKV, S, n, bits, splits, mask): decode, multi-token decode, verify on the
# tensor-core path with one and several key splits, prefill-sized chunk
CASES = [
    (32, 4, 1, 32768, 4, 0, None),
    (32, 4, 1, 5000, 8, 0, None),
    (16, 2, 1, 4096, 4, 200, None),
    (8, 8, 4, 3000, 8, 0, "causal"),
    (32, 4, 8, 16384, 4, 0, "causal"),
    (32, 4, 8, 2000, 4, 1, "causal"),
    (32, 4, 64, 3000, 8, 0, "causal"),
]


def _run(case, ws, seed=0):
    from chad_b200 import ops

    HQ, HKV, S, n, bits, splits, mask = case
    q, k, v = make_case(seed + n + S, 1, HQ, HKV, S, 128, n, "bf16", outliers=True)
    c = _cache(k, v, bits, "bf16")
    tq = torch_from_f32(q, "bf16")
    return ops.attention(tq, c.keys, c.values, 128 ** -0.5, n, bits, mask=mask,
                         splits=splits, workspace=ws)


@pytest.mark.parametrize("case", CASES)
def test_workspace_left_zero(case):
    from chad_b200 import ops

    ws = torch.zeros(256 << 20, dtype=torch.uint8, device="cuda")
    first = _run(case, ws)
    torch.cuda.synchronize()
    assert int(torch.count_nonzero(ws)) == 0
    for _ in range(3):
        again = _run(case, ws)
        assert torch.equal(first, again)
    torch.cuda.synchronize()
    assert int(torch.count_nonzero(ws)) == 0
    assert ops.device_status() == 0


def test_workspace_shared_across_shapes_and_paths():
    """Interleave every case on one workspace: each result equals its fresh-workspace one."""
    ws = torch.zeros(256 << 20, dtype=torch.uint8, device="cuda")
    fresh = [_run(c, torch.zeros(256 << 20, dtype=torch.uint8, device="cuda")) for c in CASES]
    for rnd in range(2):
        order = CASES if rnd == 0 else CASES[::-1]
        for c in order:
            got = _run(c, ws)
            assert torch.equal(got, fresh[CASES.index(c)]), c
    torch.cuda.synchronize()
    assert int(torch.count_nonzero(ws)) == 0


def test_more_splits_than_one_wave():
    """Splits beyond the resident-CTA count: the merging splits come last in dispatch
    order, so every split they wait for has already been given a slot."""
    from chad_b200 import ops

    case = (32, 4, 1, 65536, 8, 256, None)
    ws = torch.zeros(256 << 20, dtype=torch.uint8, device="cuda")
    a = _run(case, ws)
    b = _run((32, 4, 1, 65536, 8, 7, None), ws)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    diff = (a.float() - b.float()).abs()
    assert float(diff.max()) < 2e-2
    assert int(torch.count_nonzero(ws)) == 0
    assert np.isfinite(a.float().cpu().numpy()).all()
