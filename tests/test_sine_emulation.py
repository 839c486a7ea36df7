"""The time-encoding backward's sine (fast_b200/csrc/gather.cu, sin_big), its
arithmetic restated on the CPU with every fp32 / fp64 operation rounded
exactly (rational arithmetic, round to nearest even), against math.sin of
the same float.  This pins the accuracy argument of the kernel's comments
(Cody & Waite reductions, Taylor series on |r| <= 0.96) without a GPU; the GPU
test tests/test_gemm_gather_gpu.py::test_time_encode_bwd_sine_accuracy runs
the kernel itself on a larger set.  Constants are the kernel's: fp32 pi/2 in
three floats, fp32 2/pi, the 30-bit + 53-bit double split of pi/2."""
import math
import struct
from fractions import Fraction as F

import numpy as np

f32 = np.float32


def _rf(fr):
    """Fraction -> nearest float32 (ties to even)."""
    x = np.float32(float(fr))
    best = x
    for c in (np.nextafter(x, np.float32(-np.inf)), np.nextafter(x, np.float32(np.inf))):
        d, db = abs(F(float(c)) - fr), abs(F(float(best)) - fr)
        if d < db or (d == db and (struct.unpack('<I', struct.pack('<f', c))[0] & 1) == 0):
            best = c
    return best


def _fma(a, b, c):
    return _rf(F(float(a)) * F(float(b)) + F(float(c)))


def _mul(a, b):
    return _rf(F(float(a)) * F(float(b)))


TWO_OVER_PI = f32(float.fromhex('0x1.45f306p-1'))
C1, C2, C3 = (f32(float.fromhex(h)) for h in ('0x1.921fb6p+0', '-0x1.777a5cp-25', '-0x1.ee59dap-50'))
MAGIC = f32(12582912.0)                                   # 1.5 * 2^23
HEAD, TAIL = float.fromhex('0x1.921fb548p+0'), float.fromhex('-0x1.de973dcb3b39ap-31')
TWO_OVER_PI_D = float.fromhex('0x1.45f306dc9c883p-1')
SIN_C = [f32(-1 / 39916800), f32(1 / 362880), f32(-1 / 5040), f32(1 / 120), f32(-1 / 6)]
COS_C = [f32(-1 / 3628800), f32(1 / 40320), f32(-1 / 720), f32(1 / 24), f32(-0.5)]


def _quadrant(r, q):
    r2 = _mul(r, r)
    p = SIN_C[0]
    for c in SIN_C[1:]:
        p = _fma(r2, p, c)
    sr = _fma(_mul(r2, r), p, r)
    p = COS_C[0]
    for c in COS_C[1:]:
        p = _fma(r2, p, c)
    cr = _fma(r2, p, f32(1))
    v = cr if q & 1 else sr
    return -v if q & 2 else v


def sin_big(x):
    ax = abs(float(x))
    if ax < 4194304.0:                                   # fp32 three-float reduction
        s = _fma(x, TWO_OVER_PI, MAGIC)
        k = _rf(F(float(s)) - F(float(MAGIC)))
        r = _fma(-k, C1, x)
        r = _fma(-k, C2, r)
        r = _fma(-k, C3, r)
        assert abs(float(r)) <= 0.96
        return _quadrant(r, struct.unpack('<i', struct.pack('<f', s))[0])
    if ax < 268435456.0:                                 # double two-part reduction
        xd = float(x)
        kd = float(round(F(xd) * F(TWO_OVER_PI_D)))
        r1 = F(xd) - F(kd) * F(HEAD)
        assert F(float(r1)) == r1                        # the first fma is exact
        r = _rf(F(float(r1 - F(kd) * F(TAIL))))
        return _quadrant(r, int(kd) & 3)
    return f32(math.sin(float(x)))


def _ulp_err(x):
    ref = math.sin(float(x))
    ulp = float(np.spacing(np.float32(abs(ref))))
    return abs(float(sin_big(x)) - ref) / ulp if ulp else 0.0


def test_sine_emulation_within_one_and_a_half_ulp():
    rng = np.random.default_rng(11)
    mags = 10.0 ** rng.uniform(-6, 8.4, 800)
    args = [(mags * rng.choice([-1.0, 1.0], mags.size)).astype(np.float32)]
    # the floats nearest to k pi/2 (smallest reduced arguments) and to (k + 1/2) pi/2
    # just below 2^22 (largest reduced arguments of the fp32 path)
    ks = np.concatenate([np.arange(1, 300), rng.integers(300, 10 ** 8, 400)])
    near = (ks.astype(np.float64) * (np.pi / 2)).astype(np.float32)
    args += [near, np.nextafter(near, np.float32(0))]
    args.append(((np.arange(2660000, 2670000, 37) + 0.5) * (np.pi / 2)).astype(np.float32))
    args.append(np.array([0.0, 1e-30, 0.7853982, 4194303.5, 4194304.0, 268435440.0], dtype=np.float32))
    x = np.concatenate(args)
    worst = max(_ulp_err(v) for v in x)
    assert worst <= 1.5, worst
