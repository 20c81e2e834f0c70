"""The output-buffer rule of the fused tensor-parallel exchange, checked on a
happens-before model of the two kernels per step (CPU only).

Per rank and step n the stream runs the decode kernel D(n), which stores this
rank's output rows into buffer n % nbuf of EVERY rank, then the barrier kernel,
whose signal half S(n) runs after D(n) and whose end E(n) waits for S(n) of every
rank.  A consumer's read R(n) of its own buffer n % nbuf is enqueued on the same
stream.  A read races with a decode of another step m (same buffer) when neither
happens before the other.

The rule that ``TPDecode.step`` and ``gdn_decode_tp`` document: with two buffers,
the output of step n must be consumed before step n+1 is enqueued on that rank.
The model shows that the rule is enough, that reading one step later races, and
that a third buffer would be the price of the looser promise.
"""

import itertools

import pytest


def _schedule(world, steps, read_lag, nbuf):
    """Per-rank op lists: ('D', n), ('S', n), ('E', n), ('R', n); the read of step n
    is enqueued after the barrier of step n + read_lag."""
    ops = {}
    for r in range(world):
        seq = []
        pending = []
        for n in range(steps):
            seq += [("D", n), ("S", n), ("E", n)]
            pending.append(n)
            while pending and pending[0] + read_lag <= n:
                seq.append(("R", pending.pop(0)))
        seq += [("R", n) for n in pending]
        ops[r] = seq
    return ops


def _happens_before(world, ops):
    nodes = [(r, op) for r in range(world) for op in ops[r]]
    succ = {x: set() for x in nodes}
    for r in range(world):                      # stream order
        for a, b in zip(ops[r], ops[r][1:]):
            succ[(r, a)].add((r, b))
    steps = {op[1] for r in ops for op in ops[r] if op[0] == "S"}
    for n in steps:                             # the barrier waits for every signal
        for r, j in itertools.product(range(world), repeat=2):
            succ[(j, ("S", n))].add((r, ("E", n)))
    reach = {}
    for x in nodes:                             # transitive closure (small graphs)
        seen, stack = set(), [x]
        while stack:
            y = stack.pop()
            for z in succ[y]:
                if z not in seen:
                    seen.add(z)
                    stack.append(z)
        reach[x] = seen
    return reach


def _races(world, steps, read_lag, nbuf):
    ops = _schedule(world, steps, read_lag, nbuf)
    hb = _happens_before(world, ops)
    found = []
    for r in range(world):
        for op in ops[r]:
            if op[0] != "R":
                continue
            n = op[1]
            for a in range(world):
                for m in range(steps):
                    if m == n or m % nbuf != n % nbuf:
                        continue
                    d, rd = (a, ("D", m)), (r, op)
                    if rd not in hb[d] and d not in hb[rd]:
                        found.append((r, n, a, m))
    return found


@pytest.mark.parametrize("world", [2, 4])
def test_consuming_before_the_next_step_is_race_free_with_two_buffers(world):
    assert _races(world, steps=6, read_lag=0, nbuf=2) == []


@pytest.mark.parametrize("world", [2, 4])
def test_reading_after_the_next_step_races_with_two_buffers(world):
    races = _races(world, steps=6, read_lag=1, nbuf=2)
    # the read of step n races with another rank's decode of step n + 2
    assert races
    assert all(m == n + 2 and a != r for r, n, a, m in races)


def test_a_third_buffer_would_cover_a_read_one_step_late():
    assert _races(2, steps=6, read_lag=1, nbuf=3) == []
    assert _races(2, steps=6, read_lag=2, nbuf=3)
