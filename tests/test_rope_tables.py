"""RoPE tables built with the fdlibm method of Math.pow / Math.cos / Math.sin.

public/infer.js:71-81 fills its rotary tables with V8's Math.pow, Math.cos and
Math.sin, which follow fdlibm (Sun Microsystems, 1993).  The oracle and the
library (dc_fdlibm.cuh) restate that method instead of calling the C library.
No JavaScript runtime exists on either machine, so the restatements are held
to the C library's results within 1 ulp (fdlibm's own error bound), and the
f32 tables are compared with tables built from the C library: they differ in
no entry at the positions the benchmark models use (one entry differs at
theta 500000, position 3531, from a 1-ulp difference in pow).
"""
import math
import struct

import numpy as np
import pytest


def ulps(a: float, b: float) -> int:
    ia = struct.unpack("<q", struct.pack("<d", a))[0]
    ib = struct.unpack("<q", struct.pack("<d", b))[0]
    if ia < 0:
        ia = -(ia & 0x7FFFFFFFFFFFFFFF)
    if ib < 0:
        ib = -(ib & 0x7FFFFFFFFFFFFFFF)
    return abs(ia - ib)


def test_sin_cos_within_one_ulp(O):
    rng = np.random.default_rng(5)
    xs = np.concatenate([rng.uniform(-3e3, 3e3, 20000), rng.uniform(-1, 1, 5000), rng.uniform(-8e5, 8e5, 5000),
                         np.arange(0, 64) * (math.pi / 2), [0.0, -0.0, 1e-300, 2.0 ** -27, math.pi / 4]])
    worst = 0
    for x in xs:
        x = float(x)
        worst = max(worst, ulps(O.fdl_sin(x), math.sin(x)), ulps(O.fdl_cos(x), math.cos(x)))
    assert worst <= 1


def test_pow_within_one_ulp(O):
    rng = np.random.default_rng(6)
    worst = 0
    for theta in (10000.0, 500000.0, 1e6, 2.0, 1.5, 0.3):
        for hd in (32, 64, 96, 128, 256):
            for i in range(hd // 2):
                e = (2.0 * i) / hd
                worst = max(worst, ulps(O.fdl_pow(theta, e), math.pow(theta, e)))
    for x, y in zip(np.exp(rng.uniform(-30, 30, 20000)), rng.uniform(-8, 8, 20000)):
        worst = max(worst, ulps(O.fdl_pow(float(x), float(y)), math.pow(float(x), float(y))))
    assert worst <= 1
    assert O.fdl_pow(1.0, 123.4) == 1.0 and O.fdl_pow(7.0, 0.0) == 1.0


def libc_tables(hd, theta, max_pos):
    half = hd // 2
    c = np.empty(max_pos * half, np.float32)
    s = np.empty(max_pos * half, np.float32)
    for i in range(half):
        den = math.pow(theta, (2.0 * i) / hd)
        for p in range(max_pos):
            f = p / den
            c[p * half + i] = math.cos(f)
            s[p * half + i] = math.sin(f)
    return c, s


@pytest.mark.parametrize("hd,theta,max_pos", [(64, 10000.0, 2305), (128, 500000.0, 2305)],
                         ids=["hd64-theta1e4", "hd128-theta5e5"])
def test_tables_equal_the_c_library_ones_at_the_benchmark_positions(O, hd, theta, max_pos):
    c, s = O.rope_tables(hd, theta, max_pos)
    lc, ls = libc_tables(hd, theta, max_pos)
    assert c.tobytes() == lc.tobytes() and s.tobytes() == ls.tobytes()


def test_one_known_table_difference(O):
    """theta 500000, head_dim 128, position 3531, i = 6: pow differs by 1 ulp
    and the f32 cosine by one step."""
    hd, theta, p, i = 128, 500000.0, 3531, 6
    e = (2.0 * i) / hd
    assert ulps(O.fdl_pow(theta, e), math.pow(theta, e)) == 1
    c, _ = O.rope_tables(hd, theta, p + 1)
    lc = np.float32(math.cos(p / math.pow(theta, e)))
    assert c[p * (hd // 2) + i] != lc
