"""CPU model of the persistent tcgen05 GEMM's pipeline protocol
(mbr-cuda-tile_b200/csrc/gemm_tc.cu), for single CTAs and CTA pairs: the TMA
producer of each CTA, the leader's MMA thread, the epilogue warps of each CTA,
the in-order tensor pipe and the asynchronous loads, stepped in random orders.

The kernel's rules, as modelled:
  * operand ring of STAGES stages: the producer waits empty[s] with parity
    (r & 1) ^ 1 (use r of stage s needs the release of use r - 1), the MMA
    thread waits full[s] with parity r & 1 and releases the stage with a
    commit (a pair's commit arrives on both CTAs' empty[s]); a pair's full[s]
    completes on the leader's barrier once the leader has armed it and both
    CTAs' bytes have landed;
  * double-buffered accumulator: tile n uses buffer n % 2; the MMA thread waits
    acc_empty[buf] with parity ((n / 2) & 1) ^ 1 and commits acc_full[buf] after
    the tile's MMAs; every epilogue warp of every CTA of the pair waits
    acc_full[buf] with parity (n / 2) & 1, reads the accumulator and arrives on
    the leader's acc_empty[buf] (count: warps x CTAs);
  * tiles carry different k-block counts (grouped GEMMs).
Every run checks for deadlock, exact parity waits (c == n + 1 when a wait for
the n-th completion succeeds), that a stage is reloaded only after the MMAs
that read it completed, and that an accumulator buffer is overwritten only
after every epilogue warp read its previous tile.
"""
import random

import pytest


class Bar:
    def __init__(self, name, count=1):
        self.name, self.count, self.pending, self.done = name, count, 0, 0

    def arrive(self):
        self.pending += 1
        if self.pending == self.count:
            self.pending = 0
            self.done += 1


class Model:
    def __init__(self, cg, stages, nkbs, epi_warps, seed):
        self.cg, self.stages, self.nkbs, self.ew = cg, stages, nkbs, epi_warps
        self.rng = random.Random(seed)
        self.full = [Bar(f"full{s}") for s in range(stages)]  # the leader's
        self.full_tx = [[0] * cg for _ in range(stages)]  # bytes landed per CTA for the armed use
        self.full_armed = [False] * stages
        self.empty = [[Bar(f"empty{c}.{s}") for s in range(stages)] for c in range(cg)]
        self.acc_full = [[Bar(f"accfull{c}.{b}") for b in range(2)] for c in range(cg)]
        self.acc_empty = [Bar(f"accempty{b}", epi_warps * cg) for b in range(2)]
        self.loads, self.tensor = [], []
        self.mma_done = set()  # k-block iterations whose MMAs completed
        self.epi_read = {}  # tile -> number of epilogue warps that read its accumulator
        self.tile_mma_done = set()

    def ok_wait(self, bar, n):
        c = bar.done
        assert c <= n + 1, f"{bar.name}: waiter for completion {n} is behind ({c} completions): parity alias"
        return c == n + 1

    def producer(self, cta):
        it = 0
        for nkb in self.nkbs:
            for _ in range(nkb):
                s, r = it % self.stages, it // self.stages
                if r >= 1:
                    yield ("wait", self.empty[cta][s], r - 1)
                assert it < self.stages or (it - self.stages) in self.mma_done, \
                    f"CTA {cta} reloads stage {s} before the MMAs of iteration {it - self.stages} completed"
                if cta == 0:
                    self.arm(s)
                self.loads.append((cta, s, it))
                it += 1
                yield None

    def arm(self, s):
        assert not self.full_armed[s]
        self.full_armed[s] = True
        self.check_full(s)

    def land(self, cta, s):
        self.full_tx[s][cta] += 1
        self.check_full(s)

    def check_full(self, s):
        if self.full_armed[s] and all(x >= 1 for x in self.full_tx[s]):
            self.full_armed[s] = False
            for c in range(self.cg):
                self.full_tx[s][c] -= 1
            self.full[s].done += 1

    def mma(self):
        it = 0
        for n, nkb in enumerate(self.nkbs):
            buf, use = n & 1, n >> 1
            if use >= 1:
                yield ("wait", self.acc_empty[buf], use - 1)
            for _ in range(nkb):
                s, r = it % self.stages, it // self.stages
                yield ("wait", self.full[s], r)
                self.tensor.append(("mma", it, n))
                self.tensor.append(("commit", [self.empty[c][s] for c in range(self.cg)], None))
                it += 1
                yield None
            self.tensor.append(("commit", [self.acc_full[c][buf] for c in range(self.cg)], n))

    def epilogue(self, cta, warp):
        for n in range(len(self.nkbs)):
            buf, use = n & 1, n >> 1
            yield ("wait", self.acc_full[cta][buf], use)
            assert n in self.tile_mma_done, f"tile {n} read before its MMAs completed"
            self.epi_read[n] = self.epi_read.get(n, 0) + 1
            self.acc_empty[buf].arrive()
            yield None

    def complete_tensor(self):
        op, arg, n = self.tensor.pop(0)
        if op == "mma":
            if n >= 2 and n not in self.started:
                assert self.epi_read.get(n - 2, 0) == self.ew * self.cg, \
                    f"tile {n} overwrites an accumulator tile {n - 2} is still being read from"
            self.started.add(n)
            self.mma_done.add(arg)
        else:
            if n is not None:
                self.tile_mma_done.add(n)
            for b in arg:
                b.done += 1  # a commit arrives once every earlier MMA has completed (in-order pipe)

    def run(self):
        self.started = set()
        procs = {("prod", c): self.producer(c) for c in range(self.cg)}
        procs["mma"] = self.mma()
        for c in range(self.cg):
            for w in range(self.ew):
                procs[("epi", c, w)] = self.epilogue(c, w)
        blocked = {k: None for k in procs}
        while procs:
            runnable = [k for k in procs if blocked[k] is None or self.ok_wait(*blocked[k][1:])]
            choices = [("p", k) for k in runnable]
            if self.loads:
                choices.append(("load", None))
            if self.tensor:
                choices.append(("tensor", None))
            assert choices, f"deadlock: {({str(k): (v[1].name, v[2]) if v else None for k, v in blocked.items()})}"
            kind, k = self.rng.choice(choices)
            if kind == "load":
                cta, s, _ = self.loads.pop(self.rng.randrange(len(self.loads)))
                self.land(cta, s)
                continue
            if kind == "tensor":
                self.complete_tensor()
                continue
            try:
                blocked[k] = None
                while True:
                    step = next(procs[k])
                    if step is None:
                        break
                    if not self.ok_wait(step[1], step[2]):
                        blocked[k] = step
                        break
            except StopIteration:
                del procs[k]
                del blocked[k]
        while self.tensor:
            self.complete_tensor()
        assert all(self.epi_read.get(n, 0) == self.ew * self.cg for n in range(len(self.nkbs)))


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("stages", [3, 4, 8])
def test_gemm_pipeline_protocol(cg, stages):
    for seed in range(40):
        rng = random.Random(seed)
        nkbs = [rng.randint(1, 6) for _ in range(rng.randint(1, 7))]
        Model(cg, stages, nkbs, 2, seed).run()


class NoEmptyWait(Model):
    def producer(self, cta):
        for step in super().producer(cta):
            if step is not None and step[0] == "wait":
                continue  # refills a stage without waiting for its release
            yield step


class NoAccEmptyWait(Model):
    def mma(self):
        for step in super().mma():
            if step is not None and step[1] in self.acc_empty:
                continue  # starts a tile in a buffer whose previous tile may still be read
            yield step


@pytest.mark.parametrize("variant,cg", [(NoEmptyWait, 1), (NoEmptyWait, 2), (NoAccEmptyWait, 1), (NoAccEmptyWait, 2)])
def test_gemm_model_catches_planted_mistakes(variant, cg):
    failures = 0
    for seed in range(60):
        try:
            variant(cg, 3, [3, 2, 4, 1, 3, 2], 2, seed).run()
        except AssertionError:
            failures += 1
    assert failures > 0, f"{variant.__name__} was never caught"
