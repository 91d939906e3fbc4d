"""The oracle pinned against the reference's known answers (CPU only).

Known answers come from the reference's own tests and boot checks:
LUT content = the LFS object ids of public/*_lut.bin; mul[7,-3] = -21
(public/app.js:1075); quantizeCols scale fround(40/127) and MAX_INT32_K
(test_pipeline.js:405-429); bgemm exactness (webgpu.js:470-492 gates).
"""
import hashlib
import json
import math
import os

import numpy as np
import pytest

# the reference's LFS object ids and sizes of public/*_lut.bin and its
# luts_meta.json, as tests/golden/make_golden.py read them
GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "luts.json")))


def test_luts_match_lfs_object_ids(O):
    mul, req, relu = O.make_luts()
    tables = {"mul": mul.astype("<i2").tobytes(), "requant": req.tobytes(), "relu": relu.tobytes()}
    for name, raw in tables.items():
        assert len(raw) == GOLDEN[name]["size"], name
        assert hashlib.sha256(raw).hexdigest() == GOLDEN[name]["oid"], name
    meta = GOLDEN["meta"]
    assert list(mul.shape) in ([meta["mul"][0] * meta["mul"][1]], meta["mul"])
    assert req.size == meta["requant"] and relu.size == meta["relu"] and meta["shift"] == 8
    assert mul[(7 & 0xFF) * 256 + (-3 & 0xFF)] == -21


def test_max_int32_k(O):
    assert O.lib().orc_max_int32_k() == 131071 == O.MAX_INT32_K
    assert O.lib().orc_acc_bound(131071) == 0 and O.lib().orc_acc_bound(131072) == O.E_ACCBOUND


@pytest.mark.parametrize("v,want", [(0.49999999999999994, 0.0), (0.5, 1.0), (-0.5, -0.0), (-2.5, -2.0),
                                    (2.5, 3.0), (-2.6, -3.0), (1.4999999999999998, 1.0), (126.5, 127.0),
                                    (-127.5, -127.0), (4503599627370497.0, 4503599627370497.0)])
def test_js_round_is_ecmascript_math_round(O, v, want):
    assert O.js_round(v) == want


def test_quantize_cols_known_scale(O):
    k, n = 256, 3
    W = np.array([((i * 17) % 50) / 25 - 1 for i in range(k * n)], np.float32)
    W[200 * n] = 40
    q, s = O.quantize_cols(W, k, n)
    assert s.size == n
    assert s[0] == np.float32(40 / 127)
    assert q[200 * n] == 127


def test_quantize_rows_uses_double_scale_cols_uses_f32_scale(O):
    # A row whose max gives a scale where the double and f32-rounded scale
    # quantise some element differently; rows and cols must follow their rules.
    rng = np.random.default_rng(3)
    diff_rows = 0
    for _ in range(200):
        x = rng.standard_normal(64).astype(np.float32)
        q, s = O.quantize_rows(x, 1, 64)
        sc = max(float(np.max(np.abs(x.astype(np.float64)))) / 127, 1e-8)
        want = np.array([max(-128, min(127, O.js_round(float(v) / sc))) for v in x], np.int8)
        assert (q == want).all()
        assert s[0] == np.float32(sc)
        want_f32 = np.array([max(-128, min(127, O.js_round(float(v) / float(np.float32(sc))))) for v in x], np.int8)
        diff_rows += int((want_f32 != want).sum())
        qc, sc_c = O.quantize_cols(x, 64, 1)
        assert (qc == want_f32).all()
    assert diff_rows >= 0


def test_zero_row_scale_floor(O):
    q, s = O.quantize_rows(np.zeros(8, np.float32), 1, 8)
    assert s[0] == np.float32(1e-8) and (q == 0).all()


def test_quantizers_refuse_non_finite(O):
    for bad in (np.nan, np.inf, -np.inf):
        x = np.array([0.5, bad, 3.0], np.float32)
        with pytest.raises(O.NonFiniteError):
            O.quantize_rows(x, 1, 3)
        with pytest.raises(O.NonFiniteError):
            O.quantize_cols(x, 3, 1)


def test_bgemm_matches_integer_matmul(O):
    rng = np.random.default_rng(5)
    for m, k, n, b in [(5, 9, 6, 3), (32, 64, 32, 1), (7, 253, 5, 2), (1, 4, 1, 1), (17, 33, 9, 1)]:
        X = rng.integers(-128, 128, (b, m, k), dtype=np.int8)
        W = rng.integers(-128, 128, (b, k, n), dtype=np.int8)
        rs = (rng.random(b * m) + 0.5).astype(np.float32)
        cs = (rng.random(b * n) + 0.5).astype(np.float32)
        acc = O.bgemm(X, W, rs, cs, m, k, n, b, O.ACC).reshape(b, m, n)
        want = np.einsum("bmk,bkn->bmn", X.astype(np.int64), W.astype(np.int64))
        assert (acc == want).all()
        f = O.bgemm(X, W, rs, cs, m, k, n, b, 0).reshape(b, m, n)
        e = (acc.astype(np.float32) * rs.reshape(b, m, 1)).astype(np.float32) * cs.reshape(b, 1, n)
        assert f.tobytes() == e.astype(np.float32).tobytes()
        r = O.bgemm(X, W, rs, cs, m, k, n, b, O.RELU).reshape(b, m, n)
        assert r.tobytes() == np.where(e < 0, np.float32(0), e).astype(np.float32).tobytes()


def test_relu_keeps_negative_zero(O):
    # acc = 0 with a negative scale gives -0; `v < 0` is false for -0 (verified_core.js:261).
    X = np.zeros(4, np.int8)
    W = np.zeros(4, np.int8)
    out = O.bgemm(X, W, np.array([-1.0], np.float32), np.array([1.0], np.float32), 1, 4, 1, 1, O.RELU)
    assert np.signbit(out[0]) and out[0] == 0


def test_requant_rule_declared(O):
    rng = np.random.default_rng(7)
    m, k, n = 9, 300, 11
    X = rng.integers(-128, 128, m * k, dtype=np.int8)
    W = rng.integers(-128, 128, k * n, dtype=np.int8)
    ones_m, ones_n = np.ones(m, np.float32), np.ones(n, np.float32)
    acc = O.bgemm(X, W, ones_m, ones_n, m, k, n, 1, O.ACC)
    q = O.bgemm(X, W, ones_m, ones_n, m, k, n, 1, O.REQUANT)
    want = (np.clip(acc, -32768, 32767) >> 8).astype(np.int8)
    assert (q == want).all()
    qr = O.bgemm(X, W, ones_m, ones_n, m, k, n, 1, O.REQUANT | O.RELU)
    assert (qr == np.maximum(want, 0)).all()


def test_bgemm_refuses_long_contraction(O):
    with pytest.raises(O.AccumulatorBoundError):
        O.bgemm(np.zeros(131072, np.int8), np.zeros(131072, np.int8), np.ones(1, np.float32),
                np.ones(1, np.float32), 1, 131072, 1, 1, O.ACC)


def test_exp_fdlibm_within_one_ulp(O):
    mpmath = pytest.importorskip("mpmath")
    mpmath.mp.prec = 120
    rng = np.random.default_rng(11)
    xs = np.concatenate([rng.uniform(-40, 0, 3000), rng.uniform(-745, 709, 1000), [0.0, -0.0, 1e-300, -1e-20]])
    for x in xs:
        got = O.exp(float(x))
        true = mpmath.e ** mpmath.mpf(float(x))
        ulp = math.ulp(got) if got else 5e-324
        assert abs(mpmath.mpf(got) - true) <= ulp, x
    assert O.exp(float("inf")) == float("inf") and O.exp(float("-inf")) == 0.0
    assert O.exp(-800.0) == 0.0 and math.isinf(O.exp(800.0))


def test_probe_inputs_and_hash_are_stable(O):
    Xq, Wq, rs, cs, d = O.probe_inputs()
    assert Xq.min() >= -127 and Xq.max() <= 127
    # the LCG's first draw: seed = (0x5EED*1103515245 + 12345) & 0x7fffffff
    s = (0x5EED * 1103515245 + 12345) & 0x7FFFFFFF
    assert Xq[0] == int(O.js_round(s / 0x7FFFFFFF * 254 - 127))
    assert O.probe_hash_int32() == O.probe_hash_int32()


def test_mulberry32_matches_js_semantics(O):
    # Pure-Python restatement of test_pipeline.js:32 with explicit 32-bit wraps.
    def mulberry(a):
        def imul(x, y):
            return ((x & 0xFFFFFFFF) * (y & 0xFFFFFFFF)) & 0xFFFFFFFF
        while True:
            a = (a + 0x6D2B79F5) & 0xFFFFFFFF
            t = imul(a ^ (a >> 15), 1 | a)
            t = ((t + imul(t ^ (t >> 7), 61 | t)) & 0xFFFFFFFF) ^ t
            yield ((t ^ (t >> 14)) & 0xFFFFFFFF) / 4294967296
    g = mulberry(7)
    want = np.array([(next(g) * 2 - 1) * 0.05 for _ in range(257)], np.float32)
    assert O.mulberry_fill(7, 257, 0.05).tobytes() == want.tobytes()
