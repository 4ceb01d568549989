"""A discrete model of the mbarrier protocol of the tcgen05 attention kernels with a
persistent item loop (csrc/attn_prefill_tc.cu; the decode kernel csrc/attn_decode_tc.cu uses
the same S / P / PV hand-over within one item), checked for deadlocks over random
schedules on the CPU.

Roles, as in the kernel: one TMA producer filling a ring of slots in the order the MMAs
consume them (K0 .. K(SBUF-1), then V(j), K(j+SBUF)); one MMA-issuing thread (S(j) into
score buffer j % SBUF, PV(j) after the softmax's p_full, S(j+SBUF) after PV(j)); four
softmax warps (q_full per item, s_full wait, an occasional O rescale that waits for PV(j-1)
before arriving on p_full(j), otherwise the wait after the arrival, and the epilogue's wait
for the item's last PV). The tensor pipe completes MMAs in issue order; a commit arrives
when everything issued before it has completed. Barriers follow the hardware's phase
semantics: a wait for parity p returns once the current phase's parity differs from p, so
a barrier two phases ahead of a waiter looks not yet complete.

With PV completions on a single barrier, a warp that arrives on p_full(j) and is delayed
past PV(j)'s completion waits forever for PV(j-1) (the model finds such schedules); with
two alternating barriers, which the kernels use, no schedule deadlocks.

The d = 64 prefill form with two query tiles per item (ring K0 V0 K1 V1 ... with a slot
released after its second reader, one score buffer per tile, MMA order S_0(0) S_1(0) |
PV_0(j) S_0(j+1) PV_1(j) S_1(j+1) ..., a softmax group per tile) is modelled the same way
(run_paired) and checked over the same random schedules at 2, 3 and 6 ring slots."""
import random

import pytest


class Bar:
    def __init__(self, count):
        self.count = count
        self.pending = count
        self.phase = 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def done(self, parity):
        return (self.phase & 1) != parity


def run(sbuf, nslot, items, seed, pv_bars, steps=200000):
    rnd = random.Random(seed)
    full = [Bar(1) for _ in range(nslot)]
    empty = [Bar(1) for _ in range(nslot)]
    q_full = Bar(4)
    s_full = [Bar(1) for _ in range(sbuf)]
    p_full = [Bar(4) for _ in range(sbuf)]
    pv_done = [Bar(1) for _ in range(pv_bars)]
    pipe, tma = [], []

    def pv_wait(gj):
        b = gj % pv_bars
        return pv_done[b], (gj // pv_bars) & 1

    def producer():
        n = 0
        for n_t in items:
            seq = [j for j in range(min(sbuf, n_t))]
            for j in range(n_t):
                seq.append(-1)
                if j + sbuf < n_t:
                    seq.append(j + sbuf)
            for _ in seq:
                slot = n % nslot
                if n >= nslot:
                    while not empty[slot].done(((n // nslot) - 1) & 1):
                        yield
                tma.append([rnd.randint(1, 30), slot])
                n += 1
                yield

    def mma():
        n, g = 0, 0
        for it, n_t in enumerate(items):
            while not q_full.done(it & 1):
                yield

            def issue_s(j):
                nonlocal n
                s, slot = (g + j) % sbuf, n % nslot
                while not full[slot].done((n // nslot) & 1):
                    yield
                pipe.append([rnd.randint(1, 10), [empty[slot]]])
                pipe.append([0, [s_full[s]]])
                n += 1

            for j in range(min(sbuf, n_t)):
                yield from issue_s(j)
            for j in range(n_t):
                gj = g + j
                s = gj % sbuf
                while not p_full[s].done((gj // sbuf) & 1):
                    yield
                slot = n % nslot
                while not full[slot].done((n // nslot) & 1):
                    yield
                pipe.append([rnd.randint(1, 10), [empty[slot]]])
                n += 1
                pipe.append([0, [pv_done[gj % pv_bars]]])
                if j + sbuf < n_t:
                    yield from issue_s(j + sbuf)
                yield
            g += n_t

    def softmax():
        g = 0
        for n_t in items:
            for _ in range(rnd.randint(0, 3)):
                yield
            q_full.arrive()
            for j in range(n_t):
                gj = g + j
                s = gj % sbuf
                while not s_full[s].done((gj // sbuf) & 1):
                    yield
                for _ in range(rnd.randint(0, 20)):
                    yield
                rescale = j > 0 and rnd.random() < 0.1
                if rescale:
                    bar, par = pv_wait(gj - 1)
                    while not bar.done(par):
                        yield
                p_full[s].arrive()
                for _ in range(rnd.randint(0, 2)):
                    yield
                if j > 0 and not rescale:
                    bar, par = pv_wait(gj - 1)
                    while not bar.done(par):
                        yield
            bar, par = pv_wait(g + n_t - 1)
            while not bar.done(par):
                yield
            for _ in range(rnd.randint(0, 5)):
                yield
            g += n_t

    alive = {"producer": producer(), "mma": mma()}
    for w in range(4):
        alive[f"softmax{w}"] = softmax()
    for _ in range(steps):
        if not alive:
            return True
        if pipe:
            pipe[0][0] -= 1
            if pipe[0][0] <= 0:
                for b in pipe.pop(0)[1]:
                    b.arrive()
        for t in tma:
            t[0] -= 1
        for t in [t for t in tma if t[0] <= 0]:
            tma.remove(t)
            full[t[1]].arrive()
        for k in list(alive):
            if rnd.random() < 0.5:
                continue
            try:
                next(alive[k])
            except StopIteration:
                del alive[k]
    return False


def schedules(n):
    for seed in range(n):
        rnd = random.Random(seed)
        yield seed, [rnd.randint(1, 6) for _ in range(rnd.randint(1, 4))]


@pytest.mark.parametrize("sbuf,nslot", [(2, 3), (2, 6), (1, 3)])
def test_two_pv_barriers_never_deadlock(sbuf, nslot):
    for seed, items in schedules(120):
        assert run(sbuf, nslot, items, seed, pv_bars=2), (seed, items)


def test_one_pv_barrier_can_miss_a_phase():
    """The form the kernels had before: some schedule deadlocks."""
    assert not all(run(2, 3, items, seed, pv_bars=1) for seed, items in schedules(60))


def run_paired(nslot, items, seed, steps=400000):
    """The d = 64 form with two query tiles per item: ring K0 V0 K1 V1 ... (a slot released
    by the commit after its second reader), one score buffer per tile, MMA order
    S_0(0) S_1(0) | PV_0(j) S_0(j+1) PV_1(j) S_1(j+1) ..., a softmax group of four warps per
    tile with the same waits as the one-tile form at one score buffer."""
    rnd = random.Random(seed)
    full = [Bar(1) for _ in range(nslot)]
    empty = [Bar(1) for _ in range(nslot)]
    q_full = [Bar(4) for _ in range(2)]
    s_full = [Bar(1) for _ in range(2)]
    p_full = [Bar(4) for _ in range(2)]
    pv_done = [[Bar(1) for _ in range(2)] for _ in range(2)]
    pipe, tma = [], []

    def producer():
        n = 0
        for n_t in items:
            for _ in range(2 * n_t):
                slot = n % nslot
                if n >= nslot:
                    while not empty[slot].done(((n // nslot) - 1) & 1):
                        yield
                tma.append([rnd.randint(1, 30), slot])
                n += 1
                yield

    def mma():
        n, g = 0, 0
        for it, n_t in enumerate(items):
            for t in range(2):
                while not q_full[t].done(it & 1):
                    yield
            n0 = n

            def issue_s(t, j):
                ln = n0 + 2 * j
                slot = ln % nslot
                if t == 0:
                    while not full[slot].done((ln // nslot) & 1):
                        yield
                arrive = [s_full[t]] if t == 0 else [empty[slot], s_full[t]]
                pipe.append([rnd.randint(1, 10), arrive])

            for t in range(2):
                yield from issue_s(t, 0)
            for j in range(n_t):
                gj = g + j
                for t in range(2):
                    while not p_full[t].done(gj & 1):
                        yield
                    ln = n0 + 2 * j + 1
                    slot = ln % nslot
                    if t == 0:
                        while not full[slot].done((ln // nslot) & 1):
                            yield
                    arrive = [pv_done[t][gj & 1]] if t == 0 else [empty[slot], pv_done[t][gj & 1]]
                    pipe.append([rnd.randint(1, 10), arrive])
                    if j + 1 < n_t:
                        yield from issue_s(t, j + 1)
                    yield
            n = n0 + 2 * n_t
            g += n_t

    def softmax(t):
        g = 0
        for n_t in items:
            for _ in range(rnd.randint(0, 3)):
                yield
            q_full[t].arrive()
            for j in range(n_t):
                gj = g + j
                while not s_full[t].done(gj & 1):
                    yield
                for _ in range(rnd.randint(0, 20)):
                    yield
                rescale = j > 0 and rnd.random() < 0.1
                bar, par = pv_done[t][(gj - 1) & 1], ((gj - 1) >> 1) & 1
                if rescale:
                    while not bar.done(par):
                        yield
                p_full[t].arrive()
                for _ in range(rnd.randint(0, 2)):
                    yield
                if j > 0 and not rescale:
                    while not bar.done(par):
                        yield
            last = g + n_t - 1
            while not pv_done[t][last & 1].done((last >> 1) & 1):
                yield
            for _ in range(rnd.randint(0, 5)):
                yield
            g += n_t

    alive = {"producer": producer(), "mma": mma()}
    for t in range(2):
        for w in range(4):
            alive[f"softmax{t}.{w}"] = softmax(t)
    for _ in range(steps):
        if not alive:
            return True
        if pipe:
            pipe[0][0] -= 1
            if pipe[0][0] <= 0:
                for b in pipe.pop(0)[1]:
                    b.arrive()
        for x in tma:
            x[0] -= 1
        for x in [x for x in tma if x[0] <= 0]:
            tma.remove(x)
            full[x[1]].arrive()
        for k in list(alive):
            if rnd.random() < 0.5:
                continue
            try:
                next(alive[k])
            except StopIteration:
                del alive[k]
    return False


@pytest.mark.parametrize("nslot", [2, 3, 6])
def test_two_tiles_per_item_never_deadlock(nslot):
    for seed, items in schedules(120):
        assert run_paired(nslot, items, seed), (seed, items)
