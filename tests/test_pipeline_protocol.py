"""Model check of the mbarrier hand-offs of the 8-panel tensor-memory kernel (CPU only).

`spmm_tmem8.cuh` (2 producer warps that also gather the X rows, 4 consumer warps) orders its
roles with mbarriers waited on by phase parity
(`mbarrier.try_wait.parity`). A parity wait cannot tell a phase from the one two ahead, so the
phase a role waits for must be the barrier's current phase or the one just completed. This test
restates, per role, the sequence of waits and arrivals the kernels perform for one CTA's stream
of chunks, and runs the roles under many random interleavings:

* no interleaving deadlocks (every wait is eventually satisfied);
* every wait finds the barrier at the awaited phase or one past it, never a phase short of it
  (the wait would return at once) nor two past it (the wait would never end).

A copy with one `sFree` barrier shared by all chunks and two producers (the first form of the
8-panel kernel, which returned wrong Y for multi-chunk windows) must fail the second check: a
producer then waits for chunk c - 1's commit while chunk c - 2's is still pending.
Copies and MMAs complete at once in the model; the property is about the order of the waits,
which the delays do not change.
"""
from __future__ import annotations

import random
from dataclasses import dataclass

import pytest


@dataclass(frozen=True)
class Shape:
    producers: int
    consumers: int
    sfree: int        # number of sFree barriers (chunk c commits to sFree[c % sfree])
    a_ring: int
    a_lead: int
    v_ring: int
    v_lead: int
    x_ring: int       # X ring slots (the V step of chunk s waits until chunk s - x_ring is released)


TMEM8 = Shape(producers=2, consumers=4, sfree=2, a_ring=8, a_lead=5, v_ring=4, v_lead=2, x_ring=3)
SINGLE_SFREE = Shape(producers=2, consumers=4, sfree=1, a_ring=8, a_lead=5, v_ring=4, v_lead=2, x_ring=3)
SHALLOW_X = Shape(producers=2, consumers=4, sfree=2, a_ring=8, a_lead=5, v_ring=4, v_lead=2, x_ring=1)


class Aliased(AssertionError):
    pass


class Barrier:
    def __init__(self, name: str, count: int):
        self.name, self.count, self.arrived, self.phase = name, count, 0, 0

    def arrive(self):
        self.arrived += 1
        assert self.arrived <= self.count, self.name
        if self.arrived == self.count:
            self.arrived, self.phase = 0, self.phase + 1

    def done(self, n: int) -> bool:
        """Phase n has completed, as a parity wait on phase n sees it. The parity wait is right
        only while the barrier's current phase is n or n + 1: at n - 1 it has the other parity
        and the wait returns at once, at n + 2 it has the same parity and the wait never ends."""
        if self.phase < n or self.phase >= n + 2:
            raise Aliased(f"{self.name}: waiting on phase {n} while phase {self.phase} is current")
        return self.phase == n + 1


def producer(pw, s: Shape, total, bars):
    seq_a = seq_v = pw
    for seq_f in range(pw, total, s.producers):
        while seq_a < total and seq_a <= seq_f + s.a_lead:             # A steps (IDs, metadata)
            bars["aLand"][seq_a % s.a_ring].arrive()
            seq_a += s.producers
        while seq_v < seq_a and seq_v <= seq_f + s.v_lead:             # V steps (values, scales, X)
            yield bars["aLand"][seq_v % s.a_ring], seq_v // s.a_ring
            if seq_v >= s.x_ring:
                yield bars["xFree"][seq_v % s.x_ring], seq_v // s.x_ring - 1
            bars["vFull"][seq_v % s.v_ring].arrive()
            bars["xFull"][seq_v % s.x_ring].arrive()
            seq_v += s.producers
        yield bars["vFull"][seq_f % s.v_ring], seq_f // s.v_ring        # B step
        if seq_f >= 1:
            yield bars["sFree"][(seq_f - 1) % s.sfree], (seq_f - 1) // s.sfree
        bars["bFull"].arrive()


def consumer(s: Shape, tasks, total, bars):
    seq = windows = 0
    for chunks in tasks:
        for _ in range(chunks):
            yield bars["xFull"][seq % s.x_ring], seq // s.x_ring
            if seq >= 1:
                yield bars["sFree"][(seq - 1) % s.sfree], (seq - 1) // s.sfree
            bars["aFull"].arrive()
            bars["xFree"][seq % s.x_ring].arrive()
            seq += 1
        if chunks:
            yield bars["dFull"], windows
            windows += 1
            bars["dFree"].arrive()


def mma(s: Shape, tasks, bars):
    seq = windows = 0
    for chunks in tasks:
        if not chunks:
            continue
        if windows >= 1:
            yield bars["dFree"], windows - 1
        windows += 1
        for _ in range(chunks):
            yield bars["aFull"], seq
            yield bars["bFull"], seq
            bars["sFree"][seq % s.sfree].arrive()
            seq += 1
        bars["dFull"].arrive()


def run(s: Shape, tasks, rng: random.Random) -> None:
    total = sum(tasks)
    bars = {
        "bFull": Barrier("bFull", 1), "aFull": Barrier("aFull", s.consumers),
        "sFree": [Barrier(f"sFree{i}", 1) for i in range(s.sfree)],
        "dFull": Barrier("dFull", 1), "dFree": Barrier("dFree", s.consumers),
        "aLand": [Barrier(f"aLand{i}", 1) for i in range(s.a_ring)],
        "vFull": [Barrier(f"vFull{i}", 1) for i in range(s.v_ring)],
        "xFull": [Barrier(f"xFull{i}", 1) for i in range(s.x_ring)],
        "xFree": [Barrier(f"xFree{i}", s.consumers) for i in range(s.x_ring)],
    }
    roles = [producer(p, s, total, bars) for p in range(s.producers)]
    roles += [consumer(s, tasks, total, bars) for _ in range(s.consumers)]
    roles.append(mma(s, tasks, bars))
    waiting = {}
    for i, r in enumerate(roles):                  # run every role to its first wait
        waiting[i] = next(r, None)
    live = {i for i, w in waiting.items() if w is not None}
    while live:
        ready = [i for i in live if waiting[i][0].done(waiting[i][1])]
        for i in live:                             # every blocked waiter checks its parity too
            waiting[i][0].done(waiting[i][1])
        assert ready, "deadlock: " + ", ".join(f"{waiting[i][0].name}@{waiting[i][1]}" for i in sorted(live))
        i = rng.choice(ready)
        waiting[i] = next(roles[i], None)
        if waiting[i] is None:
            live.discard(i)
    for b in [bars["bFull"], bars["aFull"], bars["dFull"], bars["dFree"], *bars["sFree"]]:
        assert b.arrived == 0, b.name


def task_lists(seed: int):
    rng = random.Random(seed)
    yield [1]
    yield [48]
    yield [1, 1, 1, 1, 1, 1, 1]
    yield [0, 3, 0, 0, 2]
    for _ in range(6):
        yield [rng.choice([0, 1, 1, 2, 3, 5, 8, 13, 48]) for _ in range(rng.randint(1, 12))]


def test_handoffs_never_alias_or_deadlock():
    shape = TMEM8
    for k, tasks in enumerate(task_lists(7)):
        for trial in range(40):
            run(shape, tasks, random.Random(1000 * k + trial))


def test_single_sfree_barrier_aliases():
    hit = False
    for k, tasks in enumerate(task_lists(7)):
        for trial in range(40):
            try:
                run(SINGLE_SFREE, tasks, random.Random(1000 * k + trial))
            except Aliased:
                hit = True
    assert hit, "a single sFree barrier with two producers must be caught"


def test_x_ring_must_outlast_the_v_lead():
    """With one X slot, the V step of chunk s (issued kVLead chunks ahead of the B step) waits for
    the consumers to release chunk s - 1, which needs the B tiles of chunk s - 1: the roles
    deadlock or alias. The kernel's static_assert requires kXDepth > kVLead."""
    caught = False
    for k, tasks in enumerate(task_lists(5)):
        for trial in range(10):
            try:
                run(SHALLOW_X, tasks, random.Random(100 * k + trial))
            except (Aliased, AssertionError):
                caught = True
    assert caught
