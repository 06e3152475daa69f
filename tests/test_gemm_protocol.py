"""A model of the barrier protocol of the tensor-core GEMM (csrc/gemm_tc.cuh,
k_gemm_s8), run under random schedules on the CPU for every shape of its
epilogue (EpiShape: accumulator buffers, epilogue groups, and the column
split that lets two groups drain one 256-column tile).

Actors of one CTA, mirroring the kernel's loops: the TMA producer (per tile
and k-iteration it waits for a free stage, empty[s], and issues a load that
completes full[s] at a random later time, loads completing in any order);
the MMA thread (per tile it waits for its accumulator buffer, tempty[b],
then per k-iteration for full[s], committing empty[s], and finally commits
tfull[b]; its commits complete in issue order); and the epilogue groups
(group grp drains columns [c_lo, c_lo + W) of the tiles of its tile slot
grp / SPL: it waits for tfull[b] and arrives on tempty[b], which expects
4 * SPL warp arrivals).  The checks: no deadlock, no parity wait more than
one phase off, every buffer drained by exactly its SPL groups before the
MMA thread reuses it, every column of every tile drained once.
"""
import random

import pytest

from test_pair_protocol import Barrier


def epi_shape(bn, mt, split_mode):
    """(buffers, groups, split) as EpiShape<BN, MT, MODE> computes them."""
    cols = bn * mt
    bufs = min(8, 512 // cols)
    split = 2 if (bn == 256 and mt == 1 and split_mode) else 1
    groups = (3 if mt == 2 else (4 if bufs >= 4 else bufs)) * split
    return bufs, groups, split


class GemmModel:
    def __init__(self, nb, g, spl, stages, kiters, tiles, rng):
        self.nb, self.g, self.spl = nb, g, spl
        self.stages, self.kiters, self.tiles, self.rng = stages, kiters, tiles, rng
        self.full = [Barrier(f"full[{s}]", 1) for s in range(stages)]
        self.empty = [Barrier(f"empty[{s}]", 1) for s in range(stages)]
        self.tfull = [Barrier(f"tfull[{b}]", 1) for b in range(nb)]
        self.tempty = [Barrier(f"tempty[{b}]", 4 * spl) for b in range(nb)]
        self.tma = []    # loads in flight: stage indices (complete in any order)
        self.pipe = []   # MMA commits, in issue order
        self.stage = [None] * stages  # stage -> ("loading"/"ready"/"reading", tile, it) or "used"
        self.buf = [None] * nb        # buffer -> (tile, {drained column parts})
        self.drained = {}             # tile -> set of column parts

    @staticmethod
    def wait(bar, target):
        assert bar.done >= target, f"{bar.name}: wait for phase {target} at {bar.done} (two ahead)"
        return bar, target

    def producer(self):
        s = 0
        n = 0  # loads issued so far
        for j in range(self.tiles):
            for it in range(self.kiters):
                # The k-th use of stage s waits for the (k-1)-th release.
                if n >= self.stages:
                    yield self.wait(self.empty[s], n // self.stages - 1)
                assert self.stage[s] in (None, "used"), f"stage {s} overwritten: {self.stage[s]}"
                self.stage[s] = ("loading", j, it)
                self.tma.append(s)
                n += 1
                s = (s + 1) % self.stages

    def mma(self):
        s = 0
        n = 0
        for j in range(self.tiles):
            b = j % self.nb
            if j >= self.nb:
                yield self.wait(self.tempty[b], j // self.nb - 1)
            assert self.buf[b] is None, f"buffer {b} reused before it was drained"
            self.buf[b] = (j, set())
            for it in range(self.kiters):
                yield self.wait(self.full[s], n // self.stages)
                assert self.stage[s] == ("ready", j, it), f"stage {s}: {self.stage[s]}"
                self.stage[s] = ("reading", j, it)
                self.pipe.append(("empty", s))
                n += 1
                s = (s + 1) % self.stages
            self.pipe.append(("tfull", b))

    def epilogue(self, grp):
        slots = self.g // self.spl
        gt, part = grp // self.spl, grp % self.spl
        for i in range(gt, self.tiles, slots):
            b = i % self.nb
            yield self.wait(self.tfull[b], i // self.nb)
            tile, parts = self.buf[b]
            assert tile == i, f"group {grp} expected tile {i} in buffer {b}, found {tile}"
            assert part not in parts, "a column part drained twice"
            parts.add(part)
            self.drained.setdefault(i, set()).add(part)
            if len(parts) == self.spl:
                self.buf[b] = None  # freed by the last of its groups (the kernel's count 4 * SPL)
            self.tempty[b].arrive(4)

    def run(self):
        actors = {"prod": self.producer(), "mma": self.mma()}
        for grp in range(self.g):
            actors[f"epi{grp}"] = self.epilogue(grp)
        pending = {}
        live = set(actors)

        def advance(k):
            try:
                bar, target = next(actors[k])
                bar.waiters.append(target)
                pending[k] = (bar, target)
            except StopIteration:
                live.discard(k)

        for k in list(actors):
            advance(k)
        while live or self.tma or self.pipe:
            ready = [k for k in live if pending[k][0].done > pending[k][1]]
            choices = ready + (["load"] if self.tma else []) + (["pipe"] if self.pipe else [])
            assert choices, f"deadlock: {[(k, pending[k][0].name, pending[k][1]) for k in live]}"
            k = self.rng.choice(choices)
            if k == "load":
                s = self.tma.pop(self.rng.randrange(len(self.tma)))
                _, j, it = self.stage[s]
                self.stage[s] = ("ready", j, it)
                self.full[s].arrive()
            elif k == "pipe":
                kind, x = self.pipe.pop(0)
                if kind == "empty":
                    self.stage[x] = "used"  # the MMAs that read the stage have run
                (self.empty if kind == "empty" else self.tfull)[x].arrive()
            else:
                bar, target = pending.pop(k)
                bar.waiters.remove(target)
                advance(k)
        assert all(len(p) == self.spl for p in self.drained.values())
        assert len(self.drained) == self.tiles


SHAPES = sorted({epi_shape(bn, mt, sm) for bn in (32, 64, 128, 256) for mt in (1, 2)
                 for sm in (False, True) if not (mt == 2 and bn > 64)})


@pytest.mark.parametrize("nb,g,spl", SHAPES)
@pytest.mark.parametrize("stages,kiters", [(2, 1), (4, 3), (8, 4), (3, 9)])
@pytest.mark.parametrize("tiles", [1, 5, 23])
def test_gemm_protocol_random_schedules(nb, g, spl, stages, kiters, tiles):
    for seed in range(12):
        GemmModel(nb, g, spl, stages, kiters, tiles,
                  random.Random(97 * nb + 13 * g + 7 * stages + kiters + 1000 * tiles + seed)).run()


def test_epi_shape_mirror_matches_the_kernel(tmp_path):
    """The model's epi_shape agrees with EpiShape<BN, MT, MODE> in
    csrc/gemm_tc.cuh (compiled here as host code; no GPU needed)."""
    import shutil
    import subprocess
    from pathlib import Path

    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc not available")
    csrc = Path(__file__).resolve().parents[1] / "psp-ml_b200" / "csrc"
    combos = [(bn, mt, mode) for bn in (32, 64, 128, 256) for mt in (1, 2) for mode in range(4)
              if not (mt == 2 and bn > 64)]
    calls = "".join(f"show<{bn}, {mt}, {mode}>();" for bn, mt, mode in combos)
    src = tmp_path / "shape.cu"
    src.write_text(
        '#include <cstdio>\n#include "gemm_tc.cuh"\nusing namespace pspml::tcg;\n'
        "template <int BN, int MT, int MODE> void show() {\n"
        "  using S = EpiShape<BN, MT, MODE>;\n"
        '  std::printf("%d %d %d %d %d %d\\n", BN, MT, MODE, S::kBufs, S::kGroups, S::kSplit);\n'
        "}\nint main() { " + calls + " return 0; }\n")
    exe = tmp_path / "shape"
    subprocess.run([nvcc, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-I", str(csrc), str(src), "-o", str(exe)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    for line in out.split("\n"):
        if not line:
            continue
        bn, mt, mode, bufs, groups, split = map(int, line.split())
        assert (bufs, groups, split) == epi_shape(bn, mt, mode in (1, 2)), line
