"""qkv_gather_combine: the cross-GPU merge of sequence shards over peer memory.

Parity target: the pass-2 log-sum-exp merge (src/chad/mlx_qsdpa.py:233-258), here as a
torch fp32 restatement in the kernel's log2 domain.

On one GPU the ranks are emulated one after another, every rank's receive buffer in this
process. No launch waits on another launch: before rank r's kernel runs, the words of the
ranks that have not run yet are written into r's buffer by the host (the same flagged words
their kernels push later), so each wait is met before the kernel starts or by the kernel's
own push. Three calls in a row cover both buffer parities and the counters' growth. A
two-process run on two GPUs (skipped with fewer) covers the IPC mapping and real
concurrent waits; the bounded wait is driven with a row that nothing ever pushes.
"""

import os
import socket

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def make_parts(W, rows, D, seed, empty_rows=()):
    """Partial rows (W, rows, D+4) as a split-KV kernel writes them: out = sum p*v,
    sum = sum p with p relative to max (log2 units); rank w's range of row i is empty
    for (w, i) in empty_rows (max -inf, sum 0, out 0)."""
    g = torch.Generator().manual_seed(seed)
    m = torch.rand((W, rows), generator=g) * 10 - 5
    l = torch.rand((W, rows), generator=g) * 99 + 1
    v = torch.randn((W, rows, D), generator=g)
    parts = torch.zeros((W, rows, D + 4))
    parts[..., :D] = v * l[..., None]
    parts[..., D] = m
    parts[..., D + 1] = l
    for w, i in empty_rows:
        parts[w, i] = 0
        parts[w, i, D] = float("-inf")
    return parts


def ref_merge(parts):
    D = parts.shape[-1] - 4
    m, l, o = parts[..., D], parts[..., D + 1], parts[..., :D]
    mx = m.max(0).values
    mu = torch.where(torch.isinf(mx), torch.zeros_like(mx), mx)
    f = torch.exp2(m - mu)
    L = (f * l).sum(0)
    O = (f[..., None] * o).sum(0)
    return O / torch.where(L == 0, torch.ones_like(L), L)[..., None], mx, L, O


class Emulated:
    """W ranks' receive buffers in one process, ranks launched in order."""

    def __init__(self, W, rows, D):
        from chad_b200 import _lib

        self.lib = _lib.load()
        self.W, self.rows, self.D = W, rows, D
        nbytes = self.lib.qkv_gather_buffer_size(rows, D, W)
        assert nbytes > 0
        self.bufs = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(W)]
        self.ptrs = torch.tensor([b.data_ptr() for b in self.bufs], dtype=torch.int64,
                                 device="cuda")
        self.calls = 0

    def words(self, r):
        n = 2 * self.W * self.rows * (self.D + 4)
        return self.bufs[r].view(torch.int64)[:n].view(2, self.W, self.rows, self.D + 4)

    def run(self, parts, out_dtype=torch.bfloat16, out_kind=0, preseed=True, ranks=None):
        from chad_b200 import _lib, ops

        c = self.calls
        parts = parts.cuda().contiguous()
        outs = []
        for r in (range(self.W) if ranks is None else ranks):
            if preseed:  # the words the later ranks' kernels will push: (flag << 32) | bits
                for q in range(r + 1, self.W):
                    bits = parts[q].view(torch.int32).to(torch.int64) & 0xFFFFFFFF
                    self.words(r)[c % 2, q] = bits | ((c + 1) << 32)
            if out_kind == 0:
                out = torch.empty((self.rows, self.D), dtype=out_dtype, device="cuda")
            else:
                out = torch.empty((self.rows, self.D + 4), dtype=torch.float32, device="cuda")
            _lib.check(self.lib.qkv_gather_combine(
                parts[r].data_ptr(), self.rows, self.D, self.ptrs.data_ptr(),
                self.bufs[r].data_ptr(), self.W, r, out.data_ptr(), ops.dtype_code(out_dtype),
                out_kind, ops._stream(out.device)))
            outs.append(out)
        torch.cuda.synchronize()
        self.calls += 1
        return outs


@pytest.mark.parametrize("W,D", [(2, 128), (4, 128), (8, 64), (3, 256)])
def test_emulated_ranks_match_the_lse_merge(W, D):
    from chad_b200 import ops

    rows = 96
    em = Emulated(W, rows, D)
    for call in range(3):  # parity 0, 1, 0
        empty = [(w, i) for i in range(0, rows, 7) for w in range(W) if (w + i) % 3 == 0]
        empty += [(w, 5) for w in range(W)]  # a row with no keys on any rank
        parts = make_parts(W, rows, D, seed=100 * W + call, empty_rows=empty)
        ref, _, _, _ = ref_merge(parts)
        outs = em.run(parts)
        for r, o in enumerate(outs):
            got = o.float().cpu()
            # bf16 output of an fp32 merge: within one bf16 rounding of the fp32 value
            torch.testing.assert_close(got, ref.to(torch.bfloat16).float(), rtol=8e-3,
                                       atol=1e-5)
            assert torch.equal(o, outs[0]), f"rank {r} differs from rank 0"
        assert torch.count_nonzero(outs[0][5]) == 0
    assert ops.device_status() == 0


def test_partial_output_and_f16():
    from chad_b200 import _lib, ops

    W, rows, D = 4, 64, 128
    em = Emulated(W, rows, D)
    parts = make_parts(W, rows, D, seed=9, empty_rows=[(0, 1), (1, 1), (2, 1), (3, 1)])
    _, mx, L, O = ref_merge(parts)
    outs = em.run(parts, out_kind=_lib.QKV_OUT_PARTIAL)
    got = outs[2].cpu()
    torch.testing.assert_close(got[:, :D], O, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(got[:, D], mx)
    torch.testing.assert_close(got[:, D + 1], L, rtol=1e-5, atol=1e-6)
    parts = make_parts(W, rows, D, seed=10)
    ref, _, _, _ = ref_merge(parts)
    outs = em.run(parts, out_dtype=torch.float16)
    torch.testing.assert_close(outs[3].float().cpu(), ref.to(torch.float16).float(),
                               rtol=2e-3, atol=1e-5)
    assert ops.device_status() == 0


def test_wait_for_a_row_nobody_pushes_gives_up_and_reports():
    """Rank 0 of two, launched alone and without rank 1's rows: its wait must end after the
    shortened bound and the status word must say so; a fresh buffer set then works."""
    from chad_b200 import _lib, ops

    lib = _lib.load()
    W, rows, D = 2, 8, 128
    em = Emulated(W, rows, D)
    assert ops.device_status() == 0
    assert lib.qkv_test_hooks(0, 200_000) == _lib.QKV_OK
    try:
        em.run(make_parts(W, rows, D, seed=3), preseed=False, ranks=[0])
    finally:
        assert lib.qkv_test_hooks(0, 0) == _lib.QKV_OK
    st = ops.device_status()
    assert st == _lib.QKV_EDEVICE * 1000 - 60, st
    assert ops.device_status() == 0
    em = Emulated(W, rows, D)
    parts = make_parts(W, rows, D, seed=4)
    ref, _, _, _ = ref_merge(parts)
    outs = em.run(parts)
    torch.testing.assert_close(outs[1].float().cpu(), ref.to(torch.bfloat16).float(),
                               rtol=8e-3, atol=1e-5)
    assert ops.device_status() == 0


def _two_gpu_worker(rank, world, port, D, rows, results):
    import torch.distributed as dist

    from chad_b200 import ops
    from chad_b200.shard import PeerGather

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        pg = PeerGather(rows, D)
        worst = 0.0
        for call in range(5):
            parts = make_parts(world, rows, D, seed=700 + call,
                               empty_rows=[(0, 3), (1, 4), (0, 6), (1, 6)])
            ref, _, _, _ = ref_merge(parts)
            out = pg.combine(parts[rank].cuda().contiguous())
            torch.cuda.synchronize()
            err = (out.float().cpu() - ref.to(torch.bfloat16).float()).abs()
            tol = 8e-3 * ref.abs() + 1e-5
            worst = max(worst, float((err / tol).max()))
        status = ops.device_status()
        pg.close()
        results.put((rank, worst, status))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_processes_over_nvlink():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    results = ctx.Queue()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, 2, port, 128, 256, results))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = sorted(results.get(timeout=5) for _ in range(2))
    for rank, worst, status in got:
        assert status == 0, (rank, status)
        assert worst <= 1.0, (rank, worst)
