"""The device requantisation uses a closed form of TFLite's
MultiplyByQuantizedMultiplier (see psp-ml_b200/csrc/requant.cuh).  This
restates that closed form in Python integers and checks it against the
oracle's literal gemmlowp arithmetic over edge and random inputs."""
import random

from oracle import oracle as orc

U64 = (1 << 64) - 1


def closed_form(a: int, m: int, r: int, zp: int) -> int:
    """(hi + ((a & ~lo) >> 31)) >> (r - 1) with t = a*m + C split in halves."""
    c = (1 << 30) + (1 << (30 + r)) + zp * (1 << (31 + r))
    t = (a * m + c) & U64                      # 64-bit wrap (never needed for r <= 23)
    lo = t & 0xFFFFFFFF
    hi = t >> 32
    if hi >= 1 << 31:
        hi -= 1 << 32
    adj = -1 if ((a & 0xFFFFFFFF) & (~lo & 0xFFFFFFFF)) >> 31 else 0
    return (hi + adj) >> (r - 1)


def test_closed_form_matches_tflite_definition():
    rng = random.Random(1)
    edges = [0, 1, -1, 2, -2, (1 << 31) - 1, -(1 << 31), 1 << 30, -(1 << 30), 12345, -12345]
    for it in range(60000):
        m = rng.choice([1 << 30, (1 << 31) - 1, rng.randint(1 << 30, (1 << 31) - 1)])
        r = rng.randint(1, 23)
        zp = rng.randint(-128, 127)
        if it % 5 == 0:
            a = rng.choice(edges)
        elif it % 3 == 0:
            a = rng.randint(-(1 << 31), (1 << 31) - 1)
        else:
            a = rng.randint(-(1 << 26), 1 << 26)
        assert closed_form(a, m, r, zp) == orc.mbqm(a, m, -r) + zp, (a, m, r, zp)


def test_closed_form_exact_halves():
    # values whose first rounding lands exactly on a tie of the second
    for r in range(1, 24):
        for a in (-(3 << r), -(1 << r), -1, 0, 1, 1 << r, 3 << r):
            for m in (1 << 30, (1 << 30) + 1, (1 << 31) - 1):
                for zp in (-128, 0, 127):
                    assert closed_form(a, m, r, zp) == orc.mbqm(a, m, -r) + zp


def closed_form_predecremented(a: int, m: int, r: int, zp: int) -> int:
    """The form the device evaluates: C - 2^32 in the table and
    hi' + ((~a | lo) >>> 31)."""
    c = (1 << 30) + (1 << (30 + r)) + zp * (1 << (31 + r)) - (1 << 32)
    t = (a * m + c) & U64
    lo = t & 0xFFFFFFFF
    hi = t >> 32
    if hi >= 1 << 31:
        hi -= 1 << 32
    bit = ((~a & 0xFFFFFFFF) | lo) >> 31
    return (hi + bit) >> (r - 1)


def test_predecremented_form_matches_tflite_definition():
    rng = random.Random(5)
    edges = [0, 1, -1, 2, -2, (1 << 31) - 1, -(1 << 31), 1 << 30, -(1 << 30)]
    for it in range(60000):
        m = rng.choice([1 << 30, (1 << 31) - 1, rng.randint(1 << 30, (1 << 31) - 1)])
        r = rng.randint(1, 23)
        zp = rng.randint(-128, 127)
        a = rng.choice(edges) if it % 4 == 0 else rng.randint(-(1 << 31), (1 << 31) - 1)
        assert closed_form_predecremented(a, m, r, zp) == orc.mbqm(a, m, -r) + zp, (a, m, r, zp)


def _clamp(v: int, lo: int, hi: int) -> int:
    return max(lo, min(hi, v))


def floor_form_folded(acc: int, bias: int, m: int, r: int, zp: int) -> int:
    """The floor form with the bias folded into the 64-bit addend, as the
    constant tables hold it (floor_entry in kernels.h): D = bias*M + C,
    out + zp = hi(acc*M + D) >> (r - 1)."""
    c = (1 << 30) + (1 << (30 + r)) + zp * (1 << (31 + r))
    d = bias * m + c
    t = acc * m + d
    return (t >> 32) >> (r - 1)


def test_floor_form_matches_tflite_after_the_clamp():
    """For ops clamped at or above their output zero point the sign term of
    the fast form can be dropped: both results clamp to the same byte."""
    rng = random.Random(3)
    for it in range(80000):
        m = rng.choice([1 << 30, (1 << 31) - 1, rng.randint(1 << 30, (1 << 31) - 1)])
        r = rng.randint(2, 23)
        zp = rng.randint(-128, 127)
        act_min = rng.randint(zp, 127)            # act_min >= zp_out (ReLU-like)
        act_max = rng.randint(act_min, 127)
        bias = rng.randint(-(1 << 21), 1 << 21)
        if it % 4 == 0:
            acc = -bias + rng.randint(-4, 4)       # a = acc + bias near zero
        else:
            acc = rng.randint(-(1 << 22), 1 << 22)
        a = acc + bias
        want = _clamp(_clamp(orc.mbqm(a, m, -r) + zp, -128, 127), act_min, act_max)
        got = _clamp(_clamp(floor_form_folded(acc, bias, m, r, zp), -128, 127), act_min, act_max)
        assert got == want, (acc, bias, m, r, zp, act_min, act_max)


def test_floor_form_differs_without_the_clamp():
    """Without a clamp at the zero point the floor form is not TFLite's (the
    sign term matters for negative accumulators): the kernels use it only
    when act_min >= zp_out."""
    rng = random.Random(4)
    diffs = 0
    for _ in range(20000):
        m = rng.randint(1 << 30, (1 << 31) - 1)
        r = rng.randint(2, 12)
        zp = rng.randint(-20, 20)
        a = rng.randint(-(1 << 22), -1)
        if floor_form_folded(a, 0, m, r, zp) != orc.mbqm(a, m, -r) + zp:
            diffs += 1
    assert diffs > 0
