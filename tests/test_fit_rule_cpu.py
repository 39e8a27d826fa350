"""CPU: the arithmetic of the partition kernel's fitted partition size.

`fit_partition_size` (decodekernels_b200/csrc/decode_params.cuh) picks the
smallest multiple of the kernel's tile, between the workspace's floor and the
planned size, whose live items fit the resident CTAs -- else the planned
size.  It counts only the candidates in [ceil(T / c), ceil(T / (c - N))]
(T the total tile count, N the sequences, c the slots per KV head), capped
at the planned size, and divides with a multiply-high by ceil(2^32 / m).
These tests restate those steps in Python and hold them to a brute-force
search over every candidate, on random batches and on the edge where even
the planned size does not fit; and check the multiply-high division against
exact division over the ranges the planner allows.  The GPU tests
(tests/test_gpu_fit_partition.py) tie the kernel to the same rule.
"""

import random

import pytest


def _items(tiles, m):
    return sum(max(1, -(-t // m)) for t in tiles)


def brute_force(tiles, lo, hi, cap):
    for m in range(lo, hi + 1):
        if _items(tiles, m) <= cap:
            return m
    return hi


def ceil_div_mulhi(t, m):
    magic = 0xFFFFFFFF // m + 1  # ceil(2^32 / m)
    return ((t + m - 1) * magic) >> 32


def device_rule(tiles, lo_ws, hi, cap, k=4, warps=3):
    """The kernel's steps: the narrowed range, candidates counted k per warp
    and round, the smallest fitting one kept; the planned size otherwise."""
    n = len(tiles)
    total = sum(tiles)
    lo = max(lo_ws, -(-total // cap)) if cap > 0 else hi + 1
    top = hi
    if cap > n:
        top = min(hi, max(lo, -(-total // (cap - n))))
    best = None
    for w in range(warps):
        m0 = lo + k * w
        while m0 <= top:
            for j in range(k):
                m = min(m0 + j, top)
                count = sum(max(1, ceil_div_mulhi(t, m)) for t in tiles)
                if m0 + j <= top and count <= cap:
                    best = m0 + j if best is None else min(best, m0 + j)
                    break
            m0 += k * warps
    return hi if best is None else best


@pytest.mark.parametrize("seed", range(40))
def test_device_rule_equals_brute_force(seed):
    rng = random.Random(seed)
    n = rng.choice([2, 5, 24, 37, 64, 96, 128, 148])
    gran = rng.choice([32, 64, 128])
    max_len = rng.choice([4096, 32768, 131072])
    spread = rng.choice(["lognormal", "uniform", "near_max", "short"])
    lens = []
    for _ in range(n):
        if spread == "lognormal":
            length = int(min(max_len, max(1, rng.lognormvariate(7.6, 1.0))))
        elif spread == "uniform":
            length = rng.randint(0, max_len)
        elif spread == "near_max":
            length = max_len - rng.randint(0, 64)
        else:
            length = rng.randint(0, 600)
        lens.append(length)
    tiles = [-(-length // gran) for length in lens]
    hi = max(2, rng.randint(512, 8192) // gran)
    lo_ws = min(hi, max(2, 512 // gran))
    cap = rng.choice([222, 296, 444, 592, 888]) // rng.choice([1, 2, 8])
    assert device_rule(tiles, lo_ws, hi, cap) == brute_force(tiles, lo_ws, hi, cap)


def test_device_rule_keeps_the_planned_size_when_nothing_fits_below_it():
    # 37 sequences of 256 tiles, the planned size 8 tiles, 222 slots per KV
    # head: ceil(T / c) = 43 lies above the planned size -- where 43 tiles
    # would fit exactly (37 x 6 = 222 items) -- and the rule must keep 8.
    tiles = [256] * 37
    assert _items(tiles, 43) == 222
    assert device_rule(tiles, 4, 8, 222) == 8 == brute_force(tiles, 4, 8, 222)


def test_item_bounds_behind_the_narrowed_range():
    rng = random.Random(7)
    for _ in range(2000):
        tiles = [rng.randint(0, 4096) for _ in range(rng.randint(1, 64))]
        m = rng.randint(2, 256)
        items, total = _items(tiles, m), sum(tiles)
        assert total / m <= items <= total / m + len(tiles)


def test_multiply_high_division_is_exact_in_range():
    rng = random.Random(3)
    # t <= 2^17 (max_seq_len <= 2^22 in tiles of at least 32 tokens), 4 <= m <= 2^8
    for m in range(4, 257):
        for t in [0, 1, m - 1, m, m + 1, 2 * m, (1 << 17) - 1, 1 << 17] + [rng.randint(0, 1 << 17) for _ in range(64)]:
            assert ceil_div_mulhi(t, m) == -(-t // m), (t, m)
