"""The interval the device kernels put around the reference's serial f64 sums.

RMSNorm's sum of squares (infer.js:73-76) and the softmax denominator
(infer.js:100-104) are left-to-right sums of non-negative doubles.  The
kernels (dc_stage.cu: k_rmsnorm_quant, softmax_z, k_attention_dcl) first sum
the terms in block order and take the exact serial order only when the
interval s -/+ serial_sum_radius(s, w, depth) cannot decide an output.  This
restates that radius and the block-reduction order in numpy and checks that
the interval holds the serial sum on random and adversarial rows (large terms
first or last, many binades, float squares).
"""
import numpy as np
import pytest

U = 2.0 ** -53


def serial_sum_radius(s, w, depth):  # dc_stage.cu serial_sum_radius
    return 1.1102230246251565e-16 * (1.001 * w + (depth + 8) * s)


def block_order_sum(t, threads=256):
    """Per-thread strided sums, a butterfly over each warp, then over the warp
    totals (block_sum_d2's order)."""
    n = len(t)
    part = np.array([sum_left(t[i:n:threads]) for i in range(threads)])
    w = part.reshape(threads // 32, 32)
    for o in (16, 8, 4, 2, 1):
        w = w + w[:, np.arange(32) ^ o]
    red = np.zeros(32)
    red[: threads // 32] = w[:, 0]
    for o in (16, 8, 4, 2, 1):
        red = red + red[np.arange(32) ^ o]
    return red[0]


def sum_left(v):
    s = 0.0
    for x in v:
        s = s + float(x)
    return s


def rows():
    rng = np.random.default_rng(2024)
    for n in (1, 31, 257, 2048, 4096):
        yield rng.random(n)
        yield np.sort(rng.random(n))[::-1].copy()                       # large terms first
        yield np.sort(np.exp(rng.standard_normal(n) * 12))[::-1].copy()  # many binades, large first
        yield np.sort(np.exp(rng.standard_normal(n) * 12))               # large last
        yield rng.standard_normal(n).astype(np.float32).astype(np.float64) ** 2
        yield np.exp(-rng.random(n) * 40.0)


@pytest.mark.parametrize("t", list(rows()), ids=lambda t: f"n{len(t)}")
def test_interval_holds_the_serial_sum(t):
    n = len(t)
    s = block_order_sum(t)
    w = block_order_sum(np.array([(n - j) * t[j] for j in range(n)]))
    r = serial_sum_radius(s, w, (n + 255) // 256 + 10)
    serial = sum_left(t)
    assert s - r <= serial <= s + r
    # and, for rows of a few hundred terms or more, much narrower than the
    # a-priori bound 2 gamma_n s
    if n >= 256:
        assert r <= 0.35 * 4 * (n + 4) * U * s
