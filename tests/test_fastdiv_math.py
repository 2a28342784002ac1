"""The glue kernels' division by a run-time constant (FastDiv in
dragonwing_edge_rs_b200/csrc/elementwise.cu): for n < 2^31 and 1 <= d < 2^31,
n // d == (n * m) >> (32 + l) with l = floor(log2 d), m = ceil(2^(32+l) / d)
when d is not a power of two (a shift when it is).  Checked here on the
boundaries where an off-by-one would show (n = k*d - 1, k*d, near 2^31) and on
random operands."""
import numpy as np


def fastdiv(n, d):
    l = d.bit_length() - 1
    if d & (d - 1) == 0:
        return n >> l
    m = -(-(1 << (32 + l)) // d)
    assert m < (1 << 32)
    return ((n * m) >> 32) >> l


def test_fastdiv_exact():
    rng = np.random.default_rng(0)
    ds = list(range(1, 300)) + [2 ** k + e for k in range(2, 31) for e in (-1, 1) if 2 ** k + e < 2 ** 31] + \
        [int(x) for x in rng.integers(1, 2 ** 31, 300)] + [2 ** 31 - 1, 3, 7, 80, 84, 8400, 12800]
    for d in ds:
        ns = {0, 1, d - 1, d, d + 1, 2 ** 31 - 1, 2 ** 31 - 2, (2 ** 31 - 1) // d * d, (2 ** 31 - 1) // d * d - 1}
        ns |= {int(x) for x in rng.integers(0, 2 ** 31, 40)}
        for k in (1, 2, 3, 1000, 12345):
            if k * d < 2 ** 31:
                ns |= {k * d - 1, k * d}
        for n in ns:
            if 0 <= n < 2 ** 31:
                assert fastdiv(n, d) == n // d, (n, d)
