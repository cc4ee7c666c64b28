"""Division by a launch constant (FastDiv in
flodl_b200/csrc/kernels/sm100_ptx.cuh), restated with Python integers: the
quotient must be exact for every dividend below 2^31."""
import random


def _fastdiv(d):
    s = 0
    while (1 << s) < d:
        s += 1
    m = ((((1 << s) - d) << 32) // d + 1) & 0xFFFFFFFF
    return m, s


def _div(n, m, s):
    t = (n * m) >> 32
    assert t + n < 1 << 32
    return (t + n) >> s


def test_fastdiv_is_exact_below_2_31():
    rng = random.Random(0)
    divisors = list(range(1, 300)) + [2**k for k in range(31)] + [2**k + 1 for k in range(1, 31)] \
        + [2**k - 1 for k in range(2, 32)] + [rng.randrange(1, 2**31) for _ in range(200)] + [2**31]
    edge = [0, 1, 2**31 - 1, 2**31 - 2, 2**30, 2**30 - 1]
    for d in divisors:
        m, s = _fastdiv(d)
        ns = edge + [rng.randrange(0, 2**31) for _ in range(300)] + \
            [q * d + r for q in (1, 7, 2**31 // d - 1) for r in (0, d - 1) if q * d + r < 2**31]
        for n in ns:
            assert _div(n, m, s) == n // d, (n, d)
