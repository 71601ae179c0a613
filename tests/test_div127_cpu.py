"""The quantise-on-write kernel computes scale = absmax / 127 without a division
(multiply by RN(1/127), one FMA correction: Brisebarre, Muller and Raina,
IEEE Trans. Computers 2004).  This test restates that float32 sequence with an
exact float32-FMA emulation (float64 products, TwoSum for the last sum) and
checks it against IEEE float32 division: on 1M random non-negative floats
plus every float of [1, 1.5), where unit-scale K/V row maxima lie (every
significand from 1.0 to 1.5 once; the check depends on the significand only,
away from the subnormal and overflow ends).  With PIE_B200_EXHAUSTIVE=1 it
checks every non-negative finite float32 (minutes).
"""
import os

import numpy as np

C32 = np.float32(1.0) / np.float32(127.0)
C64 = np.float64(C32)


def _rn32_exact(s, err):
    """RN to float32 of the exact value s + err (s = RN64 of it)."""
    f = s.astype(np.float32)
    up = np.nextafter(f, np.float32(np.inf))
    dn = np.nextafter(f, np.float32(-np.inf))
    fd = f.astype(np.float64)
    mid_up = (fd + up.astype(np.float64)) / 2
    mid_dn = (fd + dn.astype(np.float64)) / 2
    res = np.where((s == mid_up) & (err > 0), up, f)
    res = np.where((s == mid_dn) & (err < 0), dn, res)
    return res


def div127_emulated(a: np.ndarray) -> np.ndarray:
    a64 = a.astype(np.float64)
    y = (a64 * C64).astype(np.float32)
    y64 = y.astype(np.float64)
    r = (a64 - y64 * 127.0).astype(np.float32)
    rc = r.astype(np.float64) * C64
    s = y64 + rc
    bb = s - y64
    err = (y64 - (s - bb)) + (rc - bb)
    return _rn32_exact(s, err)


def _check_bits(bits: np.ndarray) -> int:
    a = bits.view(np.float32)
    return int(np.count_nonzero(div127_emulated(a).view(np.uint32) != (a / np.float32(127.0)).view(np.uint32)))


def test_div127_random_and_common_binades():
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 0x7F800000, size=1 << 20, dtype=np.uint32)
    assert _check_bits(bits) == 0
    # every float in [1, 1.5)
    lo = np.float32(1.0).view(np.uint32)
    hi = np.float32(1.5).view(np.uint32)
    for start in range(int(lo), int(hi), 1 << 24):
        assert _check_bits(np.arange(start, min(start + (1 << 24), int(hi)), dtype=np.uint32)) == 0


def test_div127_exhaustive():
    if not os.environ.get("PIE_B200_EXHAUSTIVE"):
        return
    for start in range(0, 0x7F800000, 1 << 24):
        assert _check_bits(np.arange(start, min(start + (1 << 24), 0x7F800000), dtype=np.uint32)) == 0
