"""CPU model of the tcgen05 attention kernel's pipeline protocol
(mbr-cuda-tile_b200/csrc/attention_tc.cu): the TMA producer warp, the MMA warp,
the softmax warps, the in-order tensor pipe and the asynchronous loads, as
processes stepped in a random order with random completion times.

The processes wait on mbarriers the way the kernel does (a wait for the n-th
completion passes the parity n & 1 and succeeds while the barrier's completion
count c has c & 1 != n & 1).  Every run checks:
  * no deadlock: some process or async operation can always advance until all
    processes finish;
  * parity waits are exact: whenever a wait succeeds, c == n + 1 (a waiter two
    phases behind would alias and wait for the wrong phase);
  * no stage or TMEM buffer is overwritten before its last reader completed:
    a K / V / Q stage is reloaded only after the MMAs that read it completed;
    S(g) is written only after the softmax read S(g-2); P(g) is written only
    after P.V(g-2) completed; a tile's first P.V (which restarts O) runs only
    after the softmax read that O buffer's previous tile.
Both instantiations are modelled: the time axis (13 key blocks per tile,
separate P buffers, one O buffer, output written at the tile's end) and the
band axis (2 key blocks per tile, P over its own S, O double buffered by tile
parity, output written after the next tile's first block).
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
    def __init__(self, pack, tiles, seed):
        self.pack = pack
        self.rng = random.Random(seed)
        self.NSK, self.NSV, self.NQ = (3, 5, 3) if pack else (4, 6, 2)
        self.nkv = 2 if pack else 13
        self.tiles = tiles
        self.total = tiles * self.nkv
        B = Bar
        self.bar_q = [B(f"q{i}") for i in range(self.NQ)]
        self.bar_k = [B(f"k{i}") for i in range(self.NSK)]
        self.bar_v = [B(f"v{i}") for i in range(self.NSV)]
        self.bar_s = [B(f"s{i}") for i in range(2)]
        self.bar_p = [B(f"p{i}") for i in range(2)]  # the four softmax warps act as one process
        self.bar_o = [B(f"o{i}") for i in range(2)]
        self.kv_free = [B(f"f{i}") for i in range(self.NSK)]
        self.o_free = [B(f"of{i}") for i in range(2)]
        self.loads = []  # in-flight TMA loads: (kind, block or tile)
        self.tensor = []  # in-order tensor pipe: ("S"|"PV"|"commit", block, barrier)
        self.s_done, self.pv_done, self.s_read = set(), set(), set()
        self.o_read_tiles = set()  # tiles whose output the softmax has read

    # ---- helpers ----
    def tile_of(self, g):
        return g // self.nkv, g % self.nkv

    def ok_wait(self, bar, n):
        c = bar.done
        assert c <= n + 1, f"{bar.name}: waiter for completion {n} is behind ({c} completions): parity alias"
        return c == n + 1

    # ---- processes (generators yielding ("wait", bar, n) or None) ----
    def producer(self):
        NSK, NSV, NQ, total, nkv = self.NSK, self.NSV, self.NQ, self.total, self.nkv
        for tl in range(min(NQ, self.tiles)):
            self.issue_load("Q", tl)
        for g in range(min(NSV, total)):
            if g < NSK:
                self.issue_load("K", g)
            self.issue_load("V", g)
        ck, cv = min(NSK, total), min(NSV, total)
        for g in range(total):
            yield ("wait", self.kv_free[g % NSK], g // NSK)
            if ck < total:
                self.issue_load("K", ck)
                ck += 1
            if g >= 2 and cv < total:
                self.issue_load("V", cv)
                cv += 1
            tl, j = self.tile_of(g)
            if j == nkv - 1 and tl + NQ < self.tiles:
                self.issue_load("Q", tl + NQ)
            yield None

    def issue_load(self, kind, idx):
        # the stage being overwritten must have no pending reader
        if kind == "K" and idx >= self.NSK:
            assert idx - self.NSK in self.s_done, f"K({idx}) overwrites a stage S({idx - self.NSK}) still reads"
        if kind == "V" and idx >= self.NSV:
            assert idx - self.NSV in self.pv_done, f"V({idx}) overwrites a stage P.V({idx - self.NSV}) still reads"
        if kind == "Q" and idx >= self.NQ:
            last = (idx - self.NQ) * self.nkv + self.nkv - 1
            assert last in self.s_done, f"Q({idx}) overwrites a tile whose last S has not completed"
        self.loads.append((kind, idx))

    def mma(self):
        total, NSK, NSV, NQ, nkv = self.total, self.NSK, self.NSV, self.NQ, self.nkv

        def s_ready(g):
            tl, j = self.tile_of(g)
            if j == 0:
                yield ("wait", self.bar_q[tl % NQ], tl // NQ)
            yield ("wait", self.bar_k[g % NSK], g // NSK)
            yield ("wait", self.bar_v[g % NSV], g // NSV)

        cs = 0
        for _ in range(min(2, total)):
            yield from s_ready(cs)
            self.tensor.append(("S", cs, None))
            self.tensor.append(("commit", cs, self.bar_s[cs & 1]))
            cs += 1
            yield None
        for g in range(total):
            yield ("wait", self.bar_p[g & 1], g >> 1)
            self.kv_free[g % NSK].arrive()
            tl, j = self.tile_of(g)
            if self.pack and j == 0 and tl >= 2:
                yield ("wait", self.o_free[tl & 1], (tl >> 1) - 1)
            self.tensor.append(("PV", g, None))
            if g + 2 >= total:
                self.tensor.append(("commit", g, self.bar_o[g & 1]))
            if cs < total:
                yield from s_ready(cs)
                self.tensor.append(("S", cs, None))
                self.tensor.append(("commit", cs, self.bar_s[cs & 1]))
                cs += 1
            yield None

    def wait_pv(self, x):
        """P.V(x) complete: through the commit of S(x+2), issued right behind
        it, or, for the last two blocks, the block's own commit."""
        if x + 2 < self.total:
            yield ("wait", self.bar_s[x & 1], (x + 2) >> 1)
        else:
            yield ("wait", self.bar_o[x & 1], 0)
        assert x in self.pv_done, f"P.V({x}) not complete when its completion was observed"

    def softmax(self):
        total, nkv = self.total, self.nkv
        wait_pv = self.wait_pv
        pending = None
        for tl in range(self.tiles):
            for j in range(nkv):
                g = tl * nkv + j
                yield ("wait", self.bar_s[g & 1], g >> 1)
                assert g in self.s_done
                self.s_read.add(g)
                # P(g): its own buffer (time) or over S(g) (band); last reader P.V(g-2)
                assert g < 2 or (g - 2) in self.pv_done, f"P({g}) written before P.V({g - 2}) completed"
                self.bar_p[g & 1].arrive()
                yield None
                if self.pack and j == 0 and pending is not None:
                    yield from wait_pv(pending)
                    self.o_read_tiles.add(self.tile_of(pending)[0])
                    self.o_free[self.tile_of(pending)[0] & 1].arrive()
                    pending = None
            g_last = tl * nkv + nkv - 1
            if self.pack:
                pending = g_last
            else:
                yield from wait_pv(g_last)
                self.o_read_tiles.add(tl)
                self.o_free[0].arrive()
        if pending is not None:
            yield from wait_pv(pending)
            self.o_read_tiles.add(self.tile_of(pending)[0])

    # ---- async completions ----
    def complete_load(self):
        i = self.rng.randrange(len(self.loads))
        kind, idx = self.loads.pop(i)
        if kind == "Q":
            self.bar_q[idx % self.NQ].done += 1
        elif kind == "K":
            self.bar_k[idx % self.NSK].done += 1
        else:
            self.bar_v[idx % self.NSV].done += 1

    def complete_tensor(self):
        op, g, bar = self.tensor.pop(0)
        if op == "S":
            assert g < 2 or (g - 2) in self.s_read, f"S({g}) overwrites S({g - 2}) before the softmax read it"
            self.s_done.add(g)
        elif op == "PV":
            tl, j = self.tile_of(g)
            if j == 0 and tl >= (2 if self.pack else 1):
                prev = tl - (2 if self.pack else 1)
                assert prev in self.o_read_tiles, f"P.V({g}) restarts O before tile {prev}'s output was read"
            self.pv_done.add(g)
        else:
            bar.done += 1  # a commit arrives once every earlier MMA has completed (in-order pipe)

    def run(self):
        procs = {"producer": self.producer(), "mma": self.mma(), "softmax": self.softmax()}
        blocked = {k: None for k in procs}
        while procs:
            runnable = [k for k in procs if blocked[k] is None or self.ok_wait(*blocked[k][1:])]
            choices = [("p", k) for k in runnable]
            if self.loads:
                choices.append(("load", None))
            if self.tensor:
                choices.append(("tensor", None))
            assert choices, f"deadlock: {({k: (v[1].name, v[2]) if v else None for k, v in blocked.items()})}"
            kind, k = self.rng.choice(choices)
            if kind == "load":
                self.complete_load()
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
        assert self.s_done == set(range(self.total)) and self.pv_done == set(range(self.total))
        assert self.o_read_tiles == set(range(self.tiles))


@pytest.mark.parametrize("pack", [False, True])
@pytest.mark.parametrize("tiles", [1, 2, 3, 5])
def test_attention_pipeline_protocol(pack, tiles):
    for seed in range(60):
        Model(pack, tiles, seed * 7919 + tiles).run()


# The model must catch protocol mistakes: each variant below breaks one rule of
# the kernel's protocol and is expected to fail an invariant on some schedule.
# (Dropping the band axis's o_free wait is not among them: the softmax reads a
# tile's O before it signals the P that lets the MMA warp restart that buffer,
# so program order alone already orders the two; the model confirms it.)
class NoKvFreeWait(Model):
    def producer(self):
        for step in super().producer():
            if step is not None and step[1] in self.kv_free:
                continue  # refills a stage without waiting for its release
            yield step


class WaitPvTooEarly(Model):
    def wait_pv(self, x):
        # reads P.V(x)'s completion from S(x+1), issued before it
        if x + 1 < self.total:
            yield ("wait", self.bar_s[(x + 1) & 1], (x + 1) >> 1)
        else:
            yield ("wait", self.bar_o[x & 1], 0)
        assert x in self.pv_done, f"P.V({x}) not complete when its completion was observed"


class OneStageKRing(Model):
    def __init__(self, pack, tiles, seed):
        super().__init__(pack, tiles, seed)
        self.NSK = 1  # S(g+2) needs K(g+2), loaded only after P(g+1): the MMA warp waits for itself
        self.bar_k = [Bar("k0")]
        self.kv_free = [Bar("f0")]


@pytest.mark.parametrize("variant,pack", [(NoKvFreeWait, False), (NoKvFreeWait, True), (WaitPvTooEarly, False),
                                          (WaitPvTooEarly, True), (OneStageKRing, False)])
def test_protocol_model_catches_planted_mistakes(variant, pack):
    failures = 0
    for seed in range(60):
        try:
            variant(pack, 3, seed).run()
        except AssertionError:
            failures += 1
    assert failures > 0, f"{variant.__name__} was never caught"
