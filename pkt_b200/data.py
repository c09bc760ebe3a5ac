"""Seeded synthetic data of the single-Linear train_linear benchmark configuration.

The recipe: std::mt19937(seed); x ~ N(0, 1) [batch, in]; W ~ U(-1/sqrt(in),
1/sqrt(in)) [out, in]; b = 0; W*, b* ~ N(0, 1); target = x W*^T + b* + N(0, noise^2).
Values follow the C++ standard library's definitions as libstdc++ implements them
(the same stream a host program using <random> draws): 32-bit Mersenne Twister
outputs, std::generate_canonical<float> (one output / 2^32), uniform_real_distribution
as a + u (b - a), and normal_distribution by Marsaglia's polar method, which caches
the second value of each pair.
"""
import ctypes
import ctypes.util
import math

import numpy as np

# the C library's single-precision log / sqrt, as <random> calls them for float
_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.logf.argtypes = [ctypes.c_float]
_libm.logf.restype = ctypes.c_float
_libm.sqrtf.argtypes = [ctypes.c_float]
_libm.sqrtf.restype = ctypes.c_float


class _Stream:
    """std::mt19937(seed) outputs, drawn in blocks."""

    def __init__(self, seed):
        self.bg = np.random.MT19937()
        self.bg._legacy_seeding(int(seed) & 0xFFFFFFFF)  # init_genrand: std::mt19937's seeding
        self.buf = np.empty(0, np.uint64)
        self.pos = 0

    def next(self):
        if self.pos == len(self.buf):
            self.buf = self.bg.random_raw(65536)
            self.pos = 0
        v = int(self.buf[self.pos])
        self.pos += 1
        return v

    def canonical(self):
        # std::generate_canonical<float, 24>: float(u32) / 2^32 in float arithmetic
        r = np.float32(self.next()) / np.float32(4294967296.0)
        return np.float32(0.99999994) if r >= 1 else r


class _Normal:
    """std::normal_distribution<float> (polar method, one cached value)."""

    def __init__(self, mean=0.0, std=1.0):
        self.mean, self.std = np.float32(mean), np.float32(std)
        self.saved = None

    def __call__(self, s):
        if self.saved is not None:
            r, self.saved = self.saved, None
        else:
            while True:
                x = np.float32(np.float64(np.float32(2.0) * s.canonical()) - 1.0)
                y = np.float32(np.float64(np.float32(2.0) * s.canonical()) - 1.0)
                r2 = np.float32(x * x + y * y)
                if not (r2 > 1.0 or r2 == 0.0):
                    break
            lg = np.float32(_libm.logf(float(r2)))
            mult = np.float32(_libm.sqrtf(float(np.float32(np.float32(-2.0) * lg) / r2)))
            self.saved = np.float32(x * mult)
            r = np.float32(y * mult)
        return np.float32(r * self.std + self.mean)


def make_linear_task(inp, out, batch, seed=0, noise=0.01):
    """Returns x [batch, inp], W [out, inp], b [out], target [batch, out] (float32)."""
    s = _Stream(seed)
    nd = _Normal()
    x = np.array([nd(s) for _ in range(batch * inp)], np.float32).reshape(batch, inp)
    bound = np.float32(1.0) / np.float32(math.sqrt(float(inp)))
    lo, hi = -bound, bound
    W = np.array([np.float32(s.canonical() * (hi - lo)) + lo for _ in range(out * inp)],
                 np.float32).reshape(out, inp)
    b = np.zeros(out, np.float32)
    Ws = np.array([nd(s) for _ in range(out * inp)], np.float32).reshape(out, inp)
    bs = np.array([nd(s) for _ in range(out)], np.float32)
    nz = _Normal(0.0, noise)
    clean = (x.astype(np.float64) @ Ws.astype(np.float64).T).astype(np.float32)
    t = np.empty((batch, out), np.float32)
    for r in range(batch):
        for j in range(out):
            t[r, j] = np.float32(np.float32(clean[r, j] + bs[j]) + nz(s))
    return x, W, b, t
