"""The multiply-and-shift division of the kernel's work-item decode (FastDiv in
csrc/fa_internal.h), restated in Python with the same integer steps and checked against exact
division for every divisor the decode can meet and boundary numerators."""

import random


def fastdiv(d: int):
    l = 0
    while (1 << l) < d:
        l += 1
    m = ((1 << (31 + l)) + d - 1) // d
    assert m < (1 << 32), (d, m)  # fits the 32-bit field
    return lambda n: (n * m) >> (31 + l)


def test_fastdiv_exact_small_divisors_all_numerators_to_2_17():
    for d in range(1, 300):
        f = fastdiv(d)
        for n in range(0, 1 << 17):
            assert f(n) == n // d


def test_fastdiv_random_and_boundaries():
    rng = random.Random(5)
    divisors = [1, 2, 3, 7, 64, 65, 127, 128, 129, 4096, 65535, 65536, 65537, (1 << 30) + 1, (1 << 31) - 1]
    divisors += [rng.randrange(1, 1 << 31) for _ in range(2000)]
    for d in divisors:
        f = fastdiv(d)
        ns = [0, 1, d - 1, d, d + 1, (1 << 31) - 1, (1 << 31) - 2]
        ns += [k * d + r for k in (1, 2, 1000) for r in (-1, 0, 1) if 0 <= k * d + r < (1 << 31)]
        ns += [rng.randrange(0, 1 << 31) for _ in range(200)]
        for n in ns:
            if 0 <= n < (1 << 31):
                assert f(n) == n // d, (n, d)
