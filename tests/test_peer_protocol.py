"""Model check of qkv_gather_combine's exchange protocol on the CPU.

Each simulated rank runs the kernel's steps as separate atomic actions: for every row, one
write of its flagged word into every rank's buffer, slot (call parity, this rank); then,
for every row, one read per source rank that succeeds only when the word carries the call's
flag (seen + 1). A rank starts call k+1 only after its call k finished reading (stream order
through the kernel's dependency wait). A random scheduler interleaves single actions of all
ranks. Every read must return the value of its own call, and every run must finish: that
is the argument that two parity slots suffice (src/chad/mlx_qsdpa.py:233-258 is the merge
the values feed; the merge itself is checked on the GPU).
"""

import random

import pytest


def value(call, rank, row):
    return (call * 1000 + rank) * 100 + row


def rank_program(r, world, rows, calls, bufs, seen, log):
    """Generator of rank r's actions; yields after every write and every read attempt."""
    for k in range(calls):
        # push: the rank's rows of call k to every rank (flag = seen + 1, slot = seen & 1)
        for row in range(rows):
            s = seen[r][row]
            for p in range(world):
                bufs[p][s & 1][r][row] = (s + 1, value(k, r, row))
                yield
        # read: every source rank's word of this call, as it lands
        for row in range(rows):
            s = seen[r][row]
            for q in range(world):
                while True:
                    flag, v = bufs[r][s & 1][q][row]
                    if flag == s + 1:
                        break
                    yield  # not landed yet: try again later
                log.append((r, k, q, row, v))
                yield
            seen[r][row] = s + 1


@pytest.mark.parametrize("world,rows,calls", [(2, 3, 6), (3, 2, 5), (4, 2, 4), (8, 1, 3)])
def test_random_interleavings_read_their_own_call(world, rows, calls):
    for seed in range(60):
        rng = random.Random(seed * 7919 + world)
        bufs = [[[[(0, None) for _ in range(rows)] for _ in range(world)] for _ in range(2)]
                for _ in range(world)]
        seen = [[0] * rows for _ in range(world)]
        log = []
        progs = {r: rank_program(r, world, rows, calls, bufs, seen, log) for r in range(world)}
        steps = 0
        while progs:
            r = rng.choice(sorted(progs))
            # a rank may run ahead in bursts, as a fast GPU would
            for _ in range(rng.randint(1, 6)):
                try:
                    next(progs[r])
                except StopIteration:
                    del progs[r]
                    break
            steps += 1
            assert steps < 2_000_000, "no progress: the protocol deadlocked"
        assert len(log) == world * calls * rows * world
        for r, k, q, row, v in log:
            assert v == value(k, q, row), (seed, r, k, q, row, v)


def test_one_parity_slot_would_not_suffice():
    """With a single slot a fast rank overwrites words of call k before a slow rank read
    them: the checker must catch that (it guards the two-slot argument above)."""
    world, rows, calls = 2, 1, 3
    bufs = [[[[(0, None) for _ in range(rows)] for _ in range(world)] for _ in range(2)]
            for _ in range(world)]
    seen = [[0] * rows for _ in range(world)]

    def single_slot_program(r, log):
        for k in range(calls):
            s = seen[r][0]
            for p in range(world):
                bufs[p][0][r][0] = (s + 1, value(k, r, 0))
                yield
            for q in range(world):
                while bufs[r][0][q][0][0] < s + 1:
                    yield
                log.append((r, k, q, bufs[r][0][q][0][1]))
                yield
            seen[r][0] = s + 1

    log = []
    fast, slow = single_slot_program(0, log), single_slot_program(1, log)
    # rank 1 pushes call 0 and stalls; rank 0 reads call 0, then pushes call 1 into rank 1's
    # only slot before rank 1 read rank 0's call-0 word
    for _ in range(2):
        next(slow)
    for _ in range(6):
        next(fast)
    for _ in range(10):
        try:
            next(slow)
        except StopIteration:
            break
    bad = [(r, k, q, v) for r, k, q, v in log if v != value(k, q, 0)]
    assert bad, "a single slot should have let a later call overwrite an unread word"
