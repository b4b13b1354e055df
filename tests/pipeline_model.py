"""Discrete-event models of the mbarrier protocols of the tensor-core kernels,
for CPU tests of their ordering: ``run`` models ``hc_mix_tc_kernel``
(``mosaic_b200/csrc/hc_tc.cu``), ``run_gemm`` the grouped GEMM.

``run`` follows the mixing kernel's roles and waits one for one:

- the producer waits ``empty[s]`` (parity of the previous use) and issues a
  stage fill that lands after a random delay (TMA complete_tx on ``full[s]``);
- the slices form groups of ``group`` consecutive slices, one accumulation
  chain each; issuer ``i`` takes groups ``i, i + I, ...``, using accumulator
  buffer ``n & 1`` for its n-th group.  Per group it waits that buffer's
  ``acc_empty``, then per slice ``full[s]``; its MMAs complete in issue order
  after random delays, each arriving on ``empty[s]``, and the group's last
  one on ``acc_full`` (tcgen05.commit);
- each summing warp waits ``full[s]`` for every slice in order, reads the
  staged x tile, arrives on ``empty[s]`` (32 arrivals); after a group's last
  slice it waits the group's ``acc_full``, reads it and arrives on
  ``acc_empty``.

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


def run(stages: int, issuers: int, nit: int, seed: int, warps: int = 4, group: int = 1,
        max_steps: int = 200_000) -> list:
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

    n_groups = (nit + group - 1) // group
    completed = set()  # slices whose MMAs completed
    last_done = [0] * issuers

    def issuer(i):
        for n, g in enumerate(range(i, n_groups, issuers)):
            b = n & 1
            while not acc_empty[i][b].passed(((n >> 1) & 1) ^ 1):
                yield
            j1 = min((g + 1) * group, nit)
            for j in range(g * group, j1):
                s = j % stages
                while not full[s].passed((j // stages) & 1):
                    yield
                if content[s] != j:
                    errors.append(("MMA issued on another fill", j, s, content[s]))
                last_done[i] = max(clock[0], last_done[i]) + rnd.randint(1, 30)

                def complete(s=s, j=j, i=i, b=b, last=(j == j1 - 1)):
                    if content[s] != j:
                        errors.append(("MMA operand replaced before completion", j, s, content[s]))
                    completed.add(j)
                    empty[s].arrive()
                    if last:
                        acc_full[i][b].arrive()

                events.append((last_done[i], rnd.random(), complete))
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
            if j % group != group - 1 and j != nit - 1:
                continue
            g = j // group
            i, n = g % issuers, g // issuers
            b = n & 1
            while not acc_full[i][b].passed((n >> 1) & 1):
                yield
            if any(jj not in completed for jj in range(g * group, j + 1)):
                errors.append(("group read before its MMAs completed", w, g))
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


def run_gemm(stages: int, parities: int, nbuf: int, copier: bool, n_items: int, kt: int, seed: int,
             observe_all: bool = True, max_steps: int = 400_000) -> list:
    """The barrier protocol of ``moe_gemm_kernel`` (``mosaic_b200/csrc/gemm_bs.cu``).

    - Two producers (weights, activations + scale chunks) arm ``full[s]`` (count
      2); their copies land after random delays.
    - With ``copier`` one warp waits ``full[s]`` for every fill, copies the
      stage's scale chunks into TMEM slot s and commits ``sf_ready[s]``; the
      issuers then wait ``sf_ready[s]`` instead of ``full[s]``.
    - 2P issuers: issuer i takes the stages with kt % P == i // 2 (both blocks
      of a pair).  With ``observe_all`` (the kernel) it also waits on every
      other stage and arrives on its ``empty`` (count 2P).  Without it, an
      issuer skips the other parities' stages and ``empty`` counts only the
      two consumers (an earlier scheme of the kernel).
    - Per item an issuer waits its accumulator buffer's ``acc_empty``, issues,
      and commits ``acc_full`` (count 2P) after its last stage; a commit
      arrives when the issuer's MMAs so far have completed (in issue order).
    - The epilogue (128 threads) waits ``acc_full``, reads the buffer and
      arrives on ``acc_empty``.

    Checks: the stage's data and TMEM scale slot belong to the fill an MMA is
    for, at issue and at completion; an item's MMAs start on a buffer only
    after the epilogue released the buffer's previous item; the epilogue reads
    a buffer only when every chain of its item is complete and no later item
    has started on it.
    """
    rnd = random.Random(seed)
    P = parities
    n_iss = 2 * P
    full = [Barrier(2) for _ in range(stages)]
    empty = [Barrier(n_iss if observe_all else 2) for _ in range(stages)]
    sf_ready = [Barrier(1) for _ in range(stages)]
    acc_full = [Barrier(n_iss) for _ in range(nbuf)]
    acc_empty = [Barrier(128) for _ in range(nbuf)]
    sf_slot: list = [None] * stages  # fill whose scales sit in TMEM slot s
    owner: list = [None] * nbuf      # latest item that issued into buffer b
    done: dict = {}                  # item -> issuers whose chains completed
    released = [-1] * nbuf           # latest item the epilogue released from buffer b
    events: list = []
    clock = [0]
    errors: list = []
    last_done = [0] * n_iss          # completion time of each issuer's latest MMA

    def at(time, fn):
        events.append((time, rnd.random(), fn))

    def holds(s, it):  # full[s] has completed the phase of fill it and no later one
        return full[s].phase == it // stages + 1

    def producer():
        it = 0
        for _ in range(n_items * kt):
            s = it % stages
            while not empty[s].passed(((it // stages) & 1) ^ 1):
                yield
            full[s].expect_tx(1)
            at(clock[0] + rnd.randint(1, 40), lambda s=s: full[s].complete_tx(1))
            it += 1
            yield

    def copier_warp():
        for it in range(n_items * kt):
            s = it % stages
            while not full[s].passed((it // stages) & 1):
                yield
            if not holds(s, it):
                errors.append(("copier reads another fill", it, s))

            def copied(s=s, it=it):
                sf_slot[s] = it
                sf_ready[s].arrive()

            at(clock[0] + rnd.randint(1, 10), copied)
            yield

    def issuer(i):
        ip = i >> 1
        it = 0
        for li in range(n_items):
            b = li % nbuf
            while not acc_empty[b].passed(((li // nbuf) & 1) ^ 1):
                yield
            for k in range(kt):
                s = it % stages
                mine = (k % P) == ip
                if not observe_all and not mine:
                    it += 1
                    continue
                bar = sf_ready[s] if copier else full[s]
                while not bar.passed((it // stages) & 1):
                    yield
                if not mine:
                    empty[s].arrive()
                    it += 1
                    yield
                    continue
                if not holds(s, it):
                    errors.append(("MMA issued on another fill", i, it, s))
                if copier and sf_slot[s] != it:
                    errors.append(("MMA issued with another fill's scales", i, it, s, sf_slot[s]))
                if li >= nbuf and released[b] < li - nbuf:
                    errors.append(("accumulator written before the epilogue released it", i, li, b))
                owner[b] = li if owner[b] is None else max(owner[b], li)
                last_done[i] = max(clock[0], last_done[i]) + rnd.randint(1, 25)

                def complete(s=s, it=it, i=i):
                    if not holds(s, it):
                        errors.append(("stage refilled under an MMA", i, it, s))
                    if copier and sf_slot[s] != it:
                        errors.append(("scale slot rewritten under an MMA", i, it, s))
                    empty[s].arrive()

                at(last_done[i], complete)
                it += 1
                yield

            def chains_done(b=b, li=li, i=i):
                done.setdefault(li, set()).add(i)
                acc_full[b].arrive()

            at(max(clock[0], last_done[i]) + 1, chains_done)
            yield

    def epilogue():
        for li in range(n_items):
            b = li % nbuf
            while not acc_full[b].passed((li // nbuf) & 1):
                yield
            if len(done.get(li, ())) != n_iss or owner[b] != li:
                errors.append(("epilogue reads an unfinished accumulator", li, b, owner[b]))
            yield  # reading takes time
            if owner[b] != li:
                errors.append(("accumulator overwritten during the epilogue", li, b, owner[b]))
            released[b] = li
            acc_empty[b].arrive(128)
            yield

    alive = [producer(), producer()] + [issuer(i) for i in range(n_iss)] + [epilogue()]
    if copier:
        alive.append(copier_warp())
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


def run_router(stages: int, nit: int, convert: bool, seed: int, wait_conv: bool = True,
               max_steps: int = 200_000) -> list:
    """The barrier protocol of ``router_logits_tc_kernel`` (``mosaic_b200/csrc/router_tc.cu``).

    - The producer waits ``empty[s]`` and fills stage s (x and W, as parts or
      as the fp32 tile), landing after a random delay.
    - With ``convert`` warps 2-5 wait ``full[s]`` for every slice, write the
      stage's part tiles from its fp32 tile and arrive on ``conv[s]`` (32 each).
    - One issuer waits ``full[s]`` (and ``conv[s]``) and the slice's
      accumulator buffer (j % 2), issues, and its commits arrive on ``empty[s]``
      and ``acc_full`` when the MMAs complete.
    - Warps 2-5 add slice j - 1's buffer after converting slice j (and the last
      one after the loop), then arrive on ``acc_empty`` (128).
    Checks: the converters read the fp32 tile of their fill and write parts
    the MMAs of the stage's previous fill no longer read; every MMA sees the
    x tile and parts of its fill from issue to completion; a buffer is added
    only after its slice's MMAs and rewritten only after it was added.
    ``wait_conv=False`` drops the issuer's wait on ``conv`` (a planted fault).
    """
    rnd = random.Random(seed)
    full = [Barrier(1) for _ in range(stages)]
    empty = [Barrier(1) for _ in range(stages)]
    conv = [Barrier(128) for _ in range(stages)]
    acc_full = [Barrier(1) for _ in range(2)]
    acc_empty = [Barrier(128) for _ in range(2)]
    parts: list = [None] * stages    # fill whose parts the stage holds
    reading: list = [set() for _ in range(stages)]  # fills whose MMAs are in flight on stage s
    acc: list = [None] * 2           # slice whose MMAs wrote buffer b
    acc_complete: list = [None] * 2  # slice whose MMAs into buffer b completed
    added = [-1]                     # slices added so far (in order)
    events: list = []
    clock = [0]
    errors: list = []
    last = [0]

    def at(time, fn):
        events.append((time, rnd.random(), fn))

    def holds(s, j):
        return full[s].phase == j // stages + 1

    def producer():
        for j in range(nit):
            s = j % stages
            while not empty[s].passed(((j // stages) & 1) ^ 1):
                yield
            full[s].expect_tx(1)
            if not convert:
                def land(s=s, j=j):
                    parts[s] = j
                    full[s].complete_tx(1)
            else:
                def land(s=s):
                    full[s].complete_tx(1)
            at(clock[0] + rnd.randint(1, 40), land)
            yield

    def issuer():
        for j in range(nit):
            s, b = j % stages, j & 1
            while not full[s].passed((j // stages) & 1):
                yield
            if convert and wait_conv:
                while not conv[s].passed((j // stages) & 1):
                    yield
            while not acc_empty[b].passed(((j >> 1) & 1) ^ 1):
                yield
            if not holds(s, j) or parts[s] != j:
                errors.append(("MMA issued on another fill", j, s, parts[s]))
            if j >= 2 and added[0] < j - 2:
                errors.append(("buffer rewritten before it was added", j, b))
            acc[b] = j
            reading[s].add(j)
            last[0] = max(clock[0], last[0]) + rnd.randint(1, 25)

            def complete(s=s, j=j, b=b):
                if not holds(s, j) or parts[s] != j:
                    errors.append(("stage changed under an MMA", j, s, parts[s]))
                reading[s].discard(j)
                acc_complete[b] = j
                empty[s].arrive()
                acc_full[b].arrive()

            at(last[0], complete)
            yield

    def warps():
        def add(j):
            b = j & 1
            while not acc_full[b].passed((j >> 1) & 1):
                yield
            if acc_complete[b] != j or acc[b] != j:
                errors.append(("buffer added before its MMAs", j, b, acc_complete[b]))
            added[0] = j
            acc_empty[b].arrive(128)

        for j in range(nit):
            if convert:
                s = j % stages
                while not full[s].passed((j // stages) & 1):
                    yield
                if not holds(s, j):
                    errors.append(("converters read another fill", j, s))
                if reading[s]:
                    errors.append(("parts written under the previous fill's MMAs", j, s, sorted(reading[s])))
                yield  # the split takes time
                parts[s] = j
                conv[s].arrive(128)
            if j > 0:
                yield from add(j - 1)
            yield
        if nit > 0:
            yield from add(nit - 1)

    alive = [producer(), issuer(), warps()]
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
    if added[0] != nit - 1:
        errors.append(("not every slice was added", added[0], nit))
    return errors
