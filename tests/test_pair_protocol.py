"""A model of the barrier protocol of the fused depthwise + pointwise pair in
the row-streaming kernel (csrc/dwrs_tc.cu, NPW > 0), run under random
schedules on the CPU.

Actors of one slot, each a generator that yields the barrier phase it waits
for (the kernel's parity waits; a wait is meaningful only if the barrier has
completed at least `target` and never more than `target + 1` phases while
it waits), mirroring the kernel's loops:

* the MMA thread: per input row it waits for the freed ring block of every
  output row the row starts, issues the depthwise MMAs, commits the rows it
  completes to dw_full[g % RS][r % R], and issues the pointwise MMAs of row
  y - 2 (waiting for that row's A tile, apw_full, and the pointwise
  accumulator, pw_empty; committing pw_full);
* epilogue set 0: per row waits dw_full, reads and frees the ring block
  (dw_free), waits for the pointwise MMAs of row g - RS that read A buffer
  g % RS (pw_full), writes the A tile and arrives on apw_full;
* epilogue set 1: per row waits pw_full, reads the accumulator and arrives
  on pw_empty;
* the tensor pipe: commits complete in issue order, at random times.

The checks: every actor finishes (no deadlock), every wait starts no more
than one phase ahead and is never overtaken by two completions, a ring block
is written only while free and read only for its row, an A buffer is never
rewritten while a pointwise MMA that reads it is in flight, and the
pointwise accumulator holds the row set 1 expects.  A second model covers
the depthwise (or dense) conv alone: stride 1 with a 4-block ring, stride 2
with a 2-block ring, sets taking rows in turn or row pairs with the fused
2x2 max pool.
"""
import random

import pytest

R = 3   # depthwise ring blocks of the fused pair
RS = 2  # epilogue sets / A buffers


class Barrier:
    def __init__(self, name, count):
        self.name, self.count, self.arrived, self.done = name, count, 0, 0
        self.waiters = []  # targets of waits in progress

    def arrive(self, n=1):
        self.arrived += n
        assert self.arrived <= self.count, f"{self.name}: too many arrivals"
        if self.arrived == self.count:
            self.arrived = 0
            self.done += 1
            for t in self.waiters:
                assert self.done <= t + 1, f"{self.name}: a wait for phase {t} was overtaken"


class Model:
    def __init__(self, ho, strips, rng):
        self.ho, self.strips, self.rng = ho, strips, rng
        self.dw_full = [[Barrier(f"dw_full[{b}][{j}]", 1) for j in range(R)] for b in range(RS)]
        self.dw_free = [Barrier(f"dw_free[{j}]", 4) for j in range(R)]
        self.apw_full = [Barrier(f"apw_full[{b}]", 4) for b in range(RS)]
        self.pw_full = [Barrier(f"pw_full[{b}]", 1) for b in range(RS)]
        self.pw_empty = Barrier("pw_empty", 4)
        self.pipe = []            # committed completions, in issue order
        self.block = [None] * R   # ring block -> (row, complete?) or None when free
        self.abuf = [None] * RS   # A buffer -> row written there
        self.abuf_busy = [0] * RS  # pointwise MMAs in flight reading the buffer
        self.acc = None           # pointwise accumulator: ("busy"/"full", row)

    def wait(self, bar, target):
        assert bar.done >= target, f"{bar.name}: wait for phase {target} at {bar.done} (two ahead)"
        return bar, target

    # The MMA thread (the loops of k_dwrs_s8's issuer for S = 1, pad 1).
    def mma(self):
        ho, hin, pt = self.ho, self.ho, 1
        free_cnt = [0] * R
        gp = 0
        gbase = 0
        for _ in range(self.strips):
            pw_next = 0
            nn = nc = nn_blk = nc_blk = 0
            for y in range(hin):
                while nn < ho and nn - pt <= y:
                    yield self.wait(self.dw_free[nn_blk], free_cnt[nn_blk])
                    free_cnt[nn_blk] += 1
                    assert self.block[nn_blk] is None, "ring block taken while in use"
                    self.block[nn_blk] = (gbase + nn, False)
                    nn += 1
                    nn_blk = (nn_blk + 1) % R
                while nc < ho and (nc - pt + 2 <= y or y == hin - 1):
                    g = gbase + nc
                    self.pipe.append(("dw", g, nc_blk))
                    nc += 1
                    nc_blk = (nc_blk + 1) % R
                while pw_next <= y - 2:
                    yield from self.pointwise(gp)
                    gp += 1
                    pw_next += 1
            while pw_next < ho:
                yield from self.pointwise(gp)
                gp += 1
                pw_next += 1
            gbase += ho

    def pointwise(self, gp):
        b = gp % RS
        yield self.wait(self.apw_full[b], gp // RS)
        if gp > 0:
            yield self.wait(self.pw_empty, gp - 1)
        assert self.abuf[b] == gp, f"A buffer {b} holds row {self.abuf[b]}, not {gp}"
        assert self.acc is None, "pointwise accumulator still full"
        self.abuf_busy[b] += 1
        self.acc = ("busy", gp)
        self.pipe.append(("pw", gp, b))

    # Epilogue set 0: every row's depthwise half.
    def set0(self):
        for j in range(R):
            self.dw_free[j].arrive(4)
        full_cnt = [[0] * R for _ in range(RS)]
        g = 0
        for _ in range(self.strips):
            for r in range(self.ho):
                b, rb = g % RS, r % R
                yield self.wait(self.dw_full[b][rb], full_cnt[b][rb])
                full_cnt[b][rb] += 1
                assert self.block[rb] == (g, True), f"block {rb} holds {self.block[rb]}, not row {g}"
                self.block[rb] = None
                self.dw_free[rb].arrive(4)
                if g >= RS:
                    yield self.wait(self.pw_full[b], g // RS - 1)
                assert self.abuf_busy[b] == 0, "A buffer rewritten under a pointwise MMA"
                self.abuf[b] = g
                self.apw_full[b].arrive(4)
                g += 1

    # Epilogue set 1: every row's pointwise half.
    def set1(self):
        g = 0
        for _ in range(self.strips):
            for _ in range(self.ho):
                b = g % RS
                yield self.wait(self.pw_full[b], g // RS)
                assert self.acc == ("full", g), f"accumulator {self.acc}, expected row {g}"
                self.acc = None
                self.pw_empty.arrive(4)
                g += 1

    def complete_one(self):
        kind, g, x = self.pipe.pop(0)
        if kind == "dw":
            assert self.block[x] == (g, False)
            self.block[x] = (g, True)
            self.dw_full[g % RS][x].arrive()
        else:
            self.abuf_busy[x] -= 1
            assert self.acc == ("busy", g)
            self.acc = ("full", g)
            self.pw_full[x].arrive()

    def actors(self):
        return {"mma": self.mma(), "set0": self.set0(), "set1": self.set1()}

    def run(self):
        actors = self.actors()
        pending = {k: None for k in actors}
        live = set(actors)
        for k in list(actors):
            self._advance(k, actors, pending, live)
        while live or self.pipe:
            ready = [k for k in live if pending[k] is None or pending[k][0].done > pending[k][1]]
            choices = ready + (["pipe"] if self.pipe else [])
            assert choices, f"deadlock: {[(k, pending[k][0].name, pending[k][1]) for k in live]}"
            k = self.rng.choice(choices)
            if k == "pipe":
                self.complete_one()
                continue
            bar, target = pending[k]
            bar.waiters.remove(target)
            pending[k] = None
            self._advance(k, actors, pending, live)

    @staticmethod
    def _advance(k, actors, pending, live):
        try:
            bar, target = next(actors[k])
            bar.waiters.append(target)
            pending[k] = (bar, target)
        except StopIteration:
            live.discard(k)


@pytest.mark.parametrize("ho", [1, 2, 3, 4, 5, 8, 48])
@pytest.mark.parametrize("strips", [1, 2, 3])
def test_pair_protocol_random_schedules(ho, strips):
    for seed in range(40 if ho < 48 else 4):
        Model(ho, strips, random.Random(1000 * ho + 10 * strips + seed)).run()


class RowModel(Model):
    """The depthwise (or dense) conv alone: stride S, an R-block ring, two
    epilogue sets taking rows in turn (row pairs with the fused 2x2 pool),
    dw_full per (set, block) and dw_free per block, as in k_dwrs_s8 with
    NPW = 0."""

    def __init__(self, s, r, pt, ho, hin, pool, strips, rng):
        self.s, self.r, self.pt, self.hin, self.pool = s, r, pt, hin, pool
        super().__init__(ho, strips, rng)
        self.dw_full = [[Barrier(f"dw_full[{b}][{j}]", 1) for j in range(r)] for b in range(RS)]
        self.dw_free = [Barrier(f"dw_free[{j}]", 4) for j in range(r)]
        self.block = [None] * r

    def owner(self, g):
        return ((g >> 1) if self.pool else g) % RS

    def mma(self):
        s, r, pt, ho, hin = self.s, self.r, self.pt, self.ho, self.hin
        free_cnt = [0] * r
        gbase = 0
        for _ in range(self.strips):
            nn = nc = nn_blk = nc_blk = 0
            for y in range(hin):
                while nn < ho and s * nn - pt <= y:
                    yield self.wait(self.dw_free[nn_blk], free_cnt[nn_blk])
                    free_cnt[nn_blk] += 1
                    assert self.block[nn_blk] is None, "ring block taken while in use"
                    self.block[nn_blk] = (gbase + nn, False)
                    nn += 1
                    nn_blk = (nn_blk + 1) % r
                while nc < ho and (s * nc - pt + 2 <= y or y == hin - 1):
                    self.pipe.append(("dw", gbase + nc, nc_blk))
                    nc += 1
                    nc_blk = (nc_blk + 1) % r
            assert nc == ho and nn == ho
            gbase += ho

    def epilogue(self, st):
        if st == 0:
            for j in range(self.r):
                self.dw_free[j].arrive(4)
        full_cnt = [0] * self.r
        g = 0
        for _ in range(self.strips):
            for row in range(self.ho):
                if self.owner(g) == st:
                    rb = row % self.r
                    yield self.wait(self.dw_full[st][rb], full_cnt[rb])
                    full_cnt[rb] += 1
                    assert self.block[rb] == (g, True), f"block {rb}: {self.block[rb]}, row {g}"
                    self.block[rb] = None
                    self.dw_free[rb].arrive(4)
                g += 1

    def complete_one(self):
        kind, g, x = self.pipe.pop(0)
        assert self.block[x] == (g, False)
        self.block[x] = (g, True)
        self.dw_full[self.owner(g)][x].arrive()

    def actors(self):
        return {"mma": self.mma(), "set0": self.epilogue(0), "set1": self.epilogue(1)}

# (stride, ring blocks, pad top, output rows, input rows, pooled row pairs)
ROW_CASES = [
    (1, 4, 1, 1, 1, False), (1, 4, 1, 2, 2, False), (1, 4, 1, 5, 5, False),
    (1, 4, 1, 6, 6, False), (1, 4, 1, 24, 24, False),
    (1, 4, 0, 4, 6, False),                      # valid padding
    (1, 4, 1, 4, 4, True), (1, 4, 1, 8, 8, True),  # dense conv with the 2x2 pool
    (2, 2, 0, 3, 6, False), (2, 2, 0, 12, 24, False),  # stride 2, even input
    (2, 2, 1, 3, 5, False), (2, 2, 1, 6, 11, False),   # stride 2, odd input
    (2, 2, 0, 1, 2, False),
]


@pytest.mark.parametrize("s,r,pt,ho,hin,pool", ROW_CASES)
@pytest.mark.parametrize("strips", [1, 2, 3])
def test_row_streaming_protocol_random_schedules(s, r, pt, ho, hin, pool, strips):
    for seed in range(30):
        RowModel(s, r, pt, ho, hin, pool, strips,
                 random.Random(7919 * ho + 31 * hin + 3 * strips + seed)).run()
