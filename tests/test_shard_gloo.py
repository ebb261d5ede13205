"""Sequence-sharded decode protocol on two CPU ranks (gloo): each rank computes the partial
rows of its key range with the oracle, ShardedDecoder gathers them with one collective and
the LSE merge reproduces single-device attention. Failure handling: a rank that raises
before the collective ends the other rank's step with an error (short timeout), no hang."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

LOG2E = 1.4426950408889634


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs():
    rng = np.random.default_rng(11)
    B, HQ, HKV, D, L = 2, 8, 2, 64, 3
    lens = [77, 130]
    q = rng.standard_normal((L, B, HQ, 1, D)).astype(np.float32)
    k = rng.standard_normal((L, B, HKV, max(lens), D)).astype(np.float32)
    v = rng.standard_normal((L, B, HKV, max(lens), D)).astype(np.float32)
    return q, k, v, lens


def _partial_rows(q, k, v, lo, n, scale):
    """Oracle partial rows [O(D), m (log2 units), l, 0, 0] of keys [lo, lo+n)."""
    from oracle import qkv_oracle as orc

    B, HQ, _, D = q.shape
    out = np.zeros((B, HQ, 1, D + 4), np.float32)
    for b in range(B):
        if n[b] == 0:
            out[b, :, 0, D] = -np.inf
            continue
        kk = k[b, :, lo[b]:lo[b] + n[b]]
        vv = v[b, :, lo[b]:lo[b] + n[b]]
        m, s, p = orc.split_partials_fp32(q[b, :, 0], kk, vv, scale, n[b], 1)
        out[b, :, 0, :D] = p[:, 0]
        out[b, :, 0, D] = m[:, 0] * LOG2E
        out[b, :, 0, D + 1] = s[:, 0]
    return out


def _cpu_combine(parts):
    from oracle import qkv_oracle as orc

    D = parts.shape[-1] - 4
    p = parts.numpy()
    m = np.moveaxis(p[..., D] / LOG2E, 0, -1)
    s = np.moveaxis(p[..., D + 1], 0, -1)
    o = np.moveaxis(p[..., :D], 0, -2)
    return torch.from_numpy(orc.lse_combine(m, s, o).astype(np.float32))


def _worker(rank, world, port, fail_rank, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    from chad_b200.shard import ShardedDecoder, shard_ranges

    q, k, v, lens = _inputs()
    lo, n = shard_ranges(lens, world, rank)

    def partial_fn(layer, ql):
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        return torch.from_numpy(_partial_rows(ql.numpy(), k[layer], v[layer], lo, n, 0.125))

    dec = ShardedDecoder(partial_fn=partial_fn, combine_fn=_cpu_combine)
    try:
        out = dec.step([torch.from_numpy(q[l]) for l in range(q.shape[0])])
        result[rank] = out.numpy().tobytes()
    except Exception as e:  # noqa: BLE001
        result[rank] = f"error: {type(e).__name__}: {e}"
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, result))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        assert not p.is_alive(), "rank hung"
    return dict(result)


def test_two_rank_sharded_decode_matches_single_device():
    from oracle import qkv_oracle as orc

    res = _run(2)
    q, k, v, lens = _inputs()
    L, B, HQ, _, D = q.shape
    want = np.stack([orc.attention_fp32(q[l], k[l], v[l], 0.125, lens) for l in range(L)])
    for r in range(2):
        got = np.frombuffer(res[r], np.float32).reshape(want.shape)
        np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-6)


def test_failed_rank_surfaces_as_error_not_hang():
    res = _run(2, fail_rank=1)
    assert res[1].startswith("error")
    assert res[0].startswith("error")  # the peer's collective errors out (timeout / abort)


def test_transport_choice_is_checked():
    from chad_b200.shard import ShardedDecoder

    with pytest.raises(ValueError):
        ShardedDecoder(transport="shm")
    dec = ShardedDecoder(transport="peer")  # no process group: one rank, nothing to merge
    assert dec.world == 1 and dec.transport == "peer"
    local = torch.zeros((2, 1, 4, 1, 68))
    assert dec.gather(local).shape == (1, 2, 1, 4, 1, 68)
    dec.close()



class _FakePeerLib:
    """Stand-in for libqkv's peer-buffer entry points: buffer pointers and IPC handles are
    made up per rank, opened mappings recorded, frees logged in order."""

    def __init__(self, rank):
        self.rank, self.log = rank, []

    def qkv_gather_buffer_size(self, rows, D, world):
        return rows * (D + 4) * world * 16 + rows * 4

    def qkv_peer_alloc(self, nbytes, own_ref, handle):
        import ctypes

        own_ref._obj.value = 0x100000 * (self.rank + 1)
        tag = b"rank%d" % self.rank
        ctypes.memmove(handle, tag, len(tag))
        self.log.append(("alloc", nbytes))
        return 0

    def qkv_peer_open(self, h, mapped_ref):
        r = int(bytes(h).split(b"\0")[0][4:])
        mapped_ref._obj.value = 0x7000000 + 0x100000 * (r + 1)
        self.log.append(("open", r))
        return 0

    def qkv_peer_free(self, ptr, opened):
        self.log.append(("free", ptr, opened))
        return 0


def _peer_setup_worker(rank, world, port, q):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from chad_b200.shard import PeerGather

        lib = _FakePeerLib(rank)
        pg = PeerGather(4, 128, device="cpu", lib=lib)
        ptrs = pg.peer_ptrs.tolist()
        pg.close()
        pg.close()  # a second close is a no-op
        q.put((rank, ptrs, lib.log))
    finally:
        dist.destroy_process_group()


def test_peer_transport_setup_exchanges_handles_and_frees_in_order():
    """The host side of the peer transport on two gloo ranks: every rank's pointer table
    holds its own buffer at its rank and the other rank's buffer as opened from that rank's
    handle; teardown closes the mappings before the own buffer is freed."""
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_peer_setup_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = sorted(q.get(timeout=5) for _ in range(world))
    for rank, ptrs, log in got:
        other = 1 - rank
        assert ptrs[rank] == 0x100000 * (rank + 1)
        assert ptrs[other] == 0x7000000 + 0x100000 * (other + 1)
        assert ("open", other) in log and ("open", rank) not in log
        frees = [e for e in log if e[0] == "free"]
        assert frees == [("free", ptrs[other], 1), ("free", ptrs[rank], 0)]
