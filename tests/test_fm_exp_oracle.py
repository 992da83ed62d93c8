"""CPU checks of fm_exp as the C oracle states it (oracle/accept_oracle.c),
the exponential the CUDA sampling and acceptance kernels evaluate bit for bit
(tests/test_gpu_ops.py holds the GPU side to it): accuracy against the exact
exponential over the whole finite range, the limits, and the paired
formulation the kernels run on element pairs (the 1.5 * 2^23 shifter, one
unsigned range test on its bits, the scale built from them) equal to fm_exp
wherever that formulation applies."""

import math
import random
import struct

import numpy as np
import pytest

from oracle import accept as A

FLT_MAX = 3.4028234663852886e38
TINY = 2.0 ** -149  # the smallest subnormal float


def f32(x: float) -> float:
    return struct.unpack("f", struct.pack("f", x))[0]


def f32_bits(x: float) -> int:
    return struct.unpack("I", struct.pack("f", x))[0]


def test_fm_exp_within_one_ulp_for_normal_results():
    rng = random.Random(3)
    xs = [f32(rng.uniform(-87.33, 88.7228)) for _ in range(100000)]
    xs += [0.0, -0.0, 1.0, -1.0, 0.5, f32(math.log(2.0)), f32(-87.33), f32(88.376), f32(88.38), f32(88.5),
           f32(88.7), f32(88.72283), 1e-30, -1e-30]
    worst = 0.0
    for x in xs:
        ref = math.exp(x)
        got = A.fm_exp(x)
        if ref > FLT_MAX:
            assert got == math.inf, x
            continue
        assert math.isfinite(got), x
        worst = max(worst, abs(got - ref) / float(np.spacing(np.float32(ref))))
    assert worst <= 1.0, f"worst error {worst} ulp"


def test_fm_exp_subnormal_results_and_limits():
    rng = random.Random(4)
    for _ in range(50000):
        x = f32(rng.uniform(-103.97, -87.34))
        assert abs(A.fm_exp(x) - math.exp(x)) <= TINY, x
    assert A.fm_exp(-104.0) == 0.0 and A.fm_exp(-math.inf) == 0.0
    assert A.fm_exp(89.0) == math.inf and A.fm_exp(math.inf) == math.inf
    assert math.isnan(A.fm_exp(math.nan))
    # e^x is finite up to ln(FLT_MAX) = 88.7228391...: the 2^128 scale goes in two steps
    assert A.fm_exp(f32(88.72283)) < math.inf


@pytest.mark.parametrize("start,stride,count", [
    (0x9E3779B9, 4099, 1 << 22),                 # a spread over every exponent and sign
    (f32_bits(-87.0), 1, 1 << 18),              # the subnormal threshold (e = -126 / -127)
    (f32_bits(88.0), 1, 1 << 18),               # the top of the range (e = 127 / 128)
    (f32_bits(0.0), 1, 1 << 16),                # tiny positive inputs
    (f32_bits(-0.0), 1, 1 << 16),               # tiny negative inputs
    (0x7F7F0000, 1, 1 << 18),                   # the largest finite, infinity and NaNs
])
def test_paired_formulation_equals_fm_exp(start, stride, count):
    fast, bad = A.fm_exp_shifter_sweep(start, stride, count)
    assert bad == 0, f"{bad} of {fast} fast-path inputs differ from fm_exp"


def test_paired_formulation_fast_path_bounds():
    # fast exactly for e in [-126, 127], fm_exp's one-multiply scales (e = -126 may give a
    # subnormal, rounded once either way); NaN, infinities and the two-step scales never
    for x, want in [(0.0, True), (-87.0, True), (-87.5, True), (-88.0, False), (88.0, True), (88.5, False),
                    (math.inf, False), (-math.inf, False), (math.nan, False), (-100.0, False)]:
        v, fast = A.fm_exp_shifter(x)
        assert fast == want, x
        r = A.fm_exp(x)
        assert (math.isnan(v) and math.isnan(r)) or f32_bits(v) == f32_bits(r), x
