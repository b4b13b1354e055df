"""Discrete-event model of the barrier protocol of ``hc_mix_tc_kernel``
(``mosaic_b200/csrc/hc_tc.cu``), for CPU tests of its ordering.

The model follows the kernel's roles and waits one for one:

- the producer waits ``empty[s]`` (parity of the previous use) and issues a
  stage fill that lands after a random delay (TMA complete_tx on ``full[s]``);
- issuer ``i`` takes slices ``i, i + I, ...``; it waits ``full[s]`` and its
  accumulator buffer's ``acc_empty``, issues, and its MMAs complete after a
  random delay, arriving on ``empty[s]`` and ``acc_full`` (tcgen05.commit);
- each summing warp waits ``full[s]`` for every slice in order, reads the
  staged x tile, arrives on ``empty[s]`` (32 arrivals), waits the slice's
  ``acc_full``, reads it and arrives on ``acc_empty``.

An mbarrier is a pending count and a phase counter; a parity wait for P
succeeds when ``phase & 1 != P``, as ``mbarrier.try_wait.parity`` does.  The
checks: every read of a stage (by the summing warps, or by an MMA from issue
to completion) sees the fill of the slice it belongs to.
"""
from __future__ import annotations

import random


class Barrier:
    def __init__(self, count: int):
        self.count = count
        self.pending = count
        self.phase = 0
        self.tx = 0

    def arrive(self, n: int = 1):
        self.pending -= n
        self._advance()

    def expect_tx(self, units: int):
        self.tx += units
        self.arrive()

    def complete_tx(self, units: int):
        self.tx -= units
        self._advance()

    def _advance(self):
        if self.pending <= 0 and self.tx == 0:
            extra = -self.pending  # arrivals beyond the count fall into the next phase
            self.phase += 1
            self.pending = self.count - extra

    def passed(self, parity: int) -> bool:
        return (self.phase & 1) != parity


def run(stages: int, issuers: int, nit: int, seed: int, warps: int = 4, max_steps: int = 200_000) -> list:
    """One randomised execution; returns the list of violations (empty = clean)."""
    rnd = random.Random(seed)
    full = [Barrier(1) for _ in range(stages)]
    empty = [Barrier(1 + 32 * warps) for _ in range(stages)]
    acc_full = [[Barrier(1) for _ in range(2)] for _ in range(issuers)]
    acc_empty = [[Barrier(32 * warps) for _ in range(2)] for _ in range(issuers)]
    content: list = [None] * stages
    events: list = []
    clock = [0]
    errors: list = []

    def later(delay, fn):
        events.append((clock[0] + delay, rnd.random(), fn))

    def producer():
        for j in range(nit):
            s = j % stages
            while not empty[s].passed(((j // stages) & 1) ^ 1):
                yield
            full[s].expect_tx(1)
            content[s] = ("landing", j)

            def land(s=s, j=j):
                content[s] = j
                full[s].complete_tx(1)

            later(rnd.randint(1, 40), land)
            yield

    def issuer(i):
        for j in range(i, nit, issuers):
            s = j % stages
            b = (j // issuers) & 1
            while not full[s].passed((j // stages) & 1):
                yield
            while not acc_empty[i][b].passed(((j // (2 * issuers)) & 1) ^ 1):
                yield
            if content[s] != j:
                errors.append(("MMA issued on another fill", j, s, content[s]))

            def complete(s=s, j=j, i=i, b=b):
                if content[s] != j:
                    errors.append(("MMA operand replaced before completion", j, s, content[s]))
                empty[s].arrive()
                acc_full[i][b].arrive()

            later(rnd.randint(1, 30), complete)
            yield

    def summing_warp(w):
        for j in range(nit):
            s = j % stages
            while not full[s].passed((j // stages) & 1):
                yield
            if content[s] != j:
                errors.append(("x tile of another fill", w, j, s, content[s]))
            yield  # the read takes time
            if content[s] != j:
                errors.append(("x tile replaced during the read", w, j, s, content[s]))
            empty[s].arrive(32)
            i, b = j % issuers, (j // issuers) & 1
            while not acc_full[i][b].passed((j // (2 * issuers)) & 1):
                yield
            acc_empty[i][b].arrive(32)
            yield

    alive = [producer()] + [issuer(i) for i in range(issuers)] + [summing_warp(w) for w in range(warps)]
    steps = 0
    while alive or events:
        steps += 1
        if steps > max_steps:
            errors.append(("no progress",))
            break
        clock[0] += 1
        for e in sorted(e for e in events if e[0] <= clock[0]):
            events.remove(e)
            e[2]()
        rnd.shuffle(alive)
        for a in list(alive):
            if rnd.random() < 0.5:
                continue
            try:
                next(a)
            except StopIteration:
                alive.remove(a)
    return errors
