"""Exhaustive interleaving model of the two peer-memory exchanges of a row-parallel layer (csrc/ex_tp_fused.cuh):
k_tp_digitize (row maxima sent to every rank as (epoch, value) words into one of two slot halves chosen by the call
epoch's parity) and k_tp_allreduce_epilogue (a "partial ready" flag to every rank, loads of every rank's partial,
finished values sent to every rank as (epoch, value) words). Every rank runs the same calls in order; the model
enumerates every interleaving of the ranks' single-word steps and checks that

* every value a rank reads is the one written for the same call (no slot or partial overwritten before it is read),
* no rank can be left waiting for a word that will never carry its epoch (the kernels' waits are bounded; here a
  wait that can never succeed is reported as a deadlock).

The model executes steps one at a time (sequentially consistent). The kernels give less: each 64-bit word store is
single-copy atomic and the stores to one location are seen in order, and only the flags' release/acquire orders
one location (the partial) before another (its flag). Nothing else in these protocols depends on the order in which
two different words become visible, so the model loses nothing by it. The steps inside a kernel phase run in every
order, as its threads and blocks may. The model covers calls of one kernel back to back and whole layers
(exchange + digitize, the partial GEMM writing this rank's partial buffer, reduce + epilogue). A planted variant with
one slot half instead of two must fail, since that is the race that back-to-back ex_tp_digitize calls had, and so
must one where two calls of a rank take the same epoch.
No GPU: this checks the protocol, the GPU tests check the kernels."""
from collections import deque

import pytest


def program(r, world, calls, kind, halves=2, same_epoch_twice=False):
    """The phases of rank r, each a list of steps that different threads or blocks run in any order; a phase starts
    when the previous one has finished. Steps: ("w", loc, (epoch, value)), ("wait_eq" | "wait_ge", loc, epoch,
    expected value or None), ("read", loc, expected value). Values are (writer rank, epoch) so every check is exact.
    same_epoch_twice: rank 0's first two calls take the same epoch, as two calls overlapping on one rank's GPU would
    (both read ctl before either advanced it)."""
    phases = []
    for c in range(calls):
        e = c + 1  # ctl starts at 0; call c reads ctl + 1
        if same_epoch_twice and r == 0 and c >= 1:
            e = c
        if kind in ("digitize", "layer"):
            h = e % halves
            # maxima of this rank's slice -> slot [half][rank] of every rank p (thread p)
            phases.append([("w", ("x", p, h, r), (e, (r, e))) for p in range(world)])
            # every rank's word of this call in this rank's buffer (thread p)
            phases.append([("wait_eq", ("x", r, h, p), e, (p, e)) for p in range(world)])
        if kind in ("reduce", "layer"):
            phases.append([("w", ("part", r), (e, (r, e)))])  # the partial GEMM of this call (previous kernel)
            # "partial ready" flag of this rank, in every rank p's flags; then every rank's flag in this rank's
            phases.append([("w", ("flag", p, r), (e, None)) for p in range(world)])
            phases.append([("wait_ge", ("flag", r, p), e, None) for p in range(world)])
            # peer loads of every rank's partial (this rank's columns), then the finished values to every rank
            phases.append([("read", ("part", p), (p, e)) for p in range(world)])
            phases.append([("w", ("out", p, r), (e, (r, e))) for p in range(world)])
            # every rank's finished columns in this rank's buffer
            phases.append([("wait_eq", ("out", r, q), e, (q, e)) for q in range(world)])
    return phases


def explore(world, calls, kind, halves=2, same_epoch_twice=False):
    """Breadth-first over all interleavings of all ranks' steps, the steps of a phase in every order. A rank's state
    is (phase, set of its steps done); memory is a function of the states (every location has one writer, which
    writes it once per call, calls in order), so a global state is the tuple of rank states."""
    progs = [program(r, world, calls, kind, halves, same_epoch_twice) for r in range(world)]
    start = tuple((0, 0) for _ in range(world))  # (phase index, bit mask of the phase's steps done)
    mem_of = {start: {}}
    seen = {start}
    todo = deque([start])
    violations, deadlocks = [], []
    while todo:
        st = todo.popleft()
        mem = mem_of.pop(st)
        moved = False
        for r in range(world):
            ph, done = st[r]
            if ph == len(progs[r]):
                continue
            steps = progs[r][ph]
            for i, act in enumerate(steps):
                if done >> i & 1:
                    continue
                new_mem = mem
                if act[0] == "w":
                    new_mem = dict(mem)
                    new_mem[act[1]] = act[2]
                else:
                    ep, val = mem.get(act[1], (0, None))
                    if act[0] == "wait_eq" and ep != act[2]:
                        continue
                    if act[0] == "wait_ge" and ep < act[2]:
                        continue
                    want = act[3] if act[0] != "read" else act[2]
                    if want is not None and val != want:
                        violations.append((r, ph, act, (ep, val)))
                        continue
                moved = True
                nd = done | (1 << i)
                rs = (ph + 1, 0) if nd == (1 << len(steps)) - 1 else (ph, nd)
                nxt = st[:r] + (rs,) + st[r + 1:]
                if nxt not in seen:
                    seen.add(nxt)
                    mem_of[nxt] = new_mem
                    todo.append(nxt)
        if not moved and any(st[r][0] < len(progs[r]) for r in range(world)):
            deadlocks.append(st)
    return len(seen), violations, deadlocks


# Up to 3 ranks here (under a second each). 4 ranks with 2-3 calls (4.4 M to 20 M states, one to nine minutes in
# this interpreter) also came out safe, which is too slow for the CPU suite.
@pytest.mark.parametrize("world,calls,kind", [(2, 8, "digitize"), (3, 4, "digitize"), (2, 4, "reduce"),
                                              (3, 3, "reduce"), (2, 4, "layer"), (3, 3, "layer")])
def test_peer_protocol_safe_in_every_interleaving(world, calls, kind):
    states, violations, deadlocks = explore(world, calls, kind)
    assert states > calls * world  # the model did branch
    assert not violations, violations[:3]
    assert not deadlocks, deadlocks[:3]


def test_planted_single_slot_half_is_caught():
    """One slot half for back-to-back exchange calls: a fast rank's next-call word overwrites a word a slower rank
    has not read yet."""
    _, violations, deadlocks = explore(2, 3, "digitize", halves=1)
    assert violations or deadlocks


@pytest.mark.parametrize("kind", ["digitize", "reduce", "layer"])
def test_planted_overlapping_calls_on_one_rank_are_caught(kind):
    """Two calls of one rank that overlap on its GPU take the same epoch; the ranks then never agree again (which is
    why PeerRowParallel orders a call issued on another stream after the previous one)."""
    _, violations, deadlocks = explore(2, 3, kind, same_epoch_twice=True)
    assert violations or deadlocks
