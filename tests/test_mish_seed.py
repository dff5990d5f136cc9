"""The reciprocal in the CTA-pair GEMM's mish epilogue (gemm_pair.cuh mish2): 1 / d for d = e^2 + 2e + 2 in
[2, 2.4e17] from an integer-subtraction seed on the IEEE-754 bit pattern (J. Blinn, "Floating-Point Tricks", IEEE
Computer Graphics and Applications 17(4), 1997: the bit pattern of a float is a scaled, offset piecewise-linear
log2, so subtracting it from a constant approximates the bit pattern of the reciprocal), refined by two
Newton-Raphson steps r <- r (2 - d r) in float32.

Checked here on the CPU, in float32 arithmetic as the kernel does it:
* the seed constant is the one that minimises the largest relative error of the seed over a binade (exhaustive
  over the 2^23 significands), about 5.05%;
* after the two Newton steps the relative error is below 7e-6 over the whole range of d the epilogue sees, below
  the 2^-11 rounding of its f16 / bf16 outputs.
"""

import os
import re

import numpy as np

_SRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "katago-rs_b200", "csrc",
                    "gemm_pair.cuh")
SEED = int(re.search(r"kRcpSeed = (0x[0-9A-Fa-f]+);", open(_SRC).read()).group(1), 16)  # the kernel's constant


def seed(bits):
    return (np.int64(SEED) - bits.astype(np.int64)).astype(np.uint32).view(np.float32)


def seed_error(constant, bits, d):
    r = (np.int64(constant) - bits.astype(np.int64)).astype(np.uint32).view(np.float32).astype(np.float64)
    return float(np.abs(r * d - 1.0).max())


def test_seed_constant_is_the_minimax_one():
    bits = (np.uint32(127 << 23) | np.arange(0, 1 << 23, dtype=np.uint32))  # d in [1, 2)
    d = bits.view(np.float32).astype(np.float64)
    e = seed_error(SEED, bits, d)
    assert 0.0505 < e < 0.0506
    for delta in (-0x40, -1, 1, 0x40, 0x1000):
        assert seed_error(SEED + delta, bits, d) >= e, hex(SEED + delta)


def f32_fma(a, b, c):
    # a * b is exact in float64 (24-bit x 24-bit significands); one float32 rounding at the end
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def test_two_newton_steps_reach_7e_6_over_the_epilogue_range():
    rng = np.random.default_rng(5)
    ds = []
    for e in range(1, 58):  # binades [2^e, 2^(e+1)) covering [2, 2.4e17]
        sig = rng.integers(0, 1 << 23, size=4096, dtype=np.uint32)
        ds.append(((np.uint32(127 + e) << 23) | sig).view(np.float32))
    d = np.concatenate(ds + [np.array([2.0, 2.4e17], np.float32)])
    d = d[(d >= 2.0) & (d <= 2.4e17)]
    two = np.float32(2.0)
    r = seed(d.view(np.uint32))
    for _ in range(2):
        r = (r * f32_fma(-d, r, np.full_like(d, two))).astype(np.float32)
    rel = np.abs(r.astype(np.float64) * d.astype(np.float64) - 1.0)
    assert rel.max() < 7e-6, rel.max()
