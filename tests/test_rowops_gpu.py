"""Row operations of the layer forward on the B200, bit for bit.

The serial double chains of infer.js (rmsnorm's sum of squares, :73-76; the
softmax denominator, :100-104) are computed on the device by a whole block; the
result must equal the one-add-at-a-time loop for every input -- including the
inputs built to defeat the parallel path: ties that depend on the running
sum's last bit, sums landing exactly on powers of two, subnormal terms, sums
that change binade at every term, and terms that are negative or not finite.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def serial(row):
    s = 0.0
    for v in row:
        s += float(v)
    return s


def run_sum(comp, rows):
    import torch
    n = len(rows[0])
    t = torch.tensor(np.array(rows, np.float64).reshape(-1), dtype=torch.float64, device="cuda")
    out = torch.empty(len(rows), dtype=torch.float64, device="cuda")
    comp.ordered_sum_dev(t, len(rows), n, out)
    comp.sync()
    return out.cpu().numpy()


def check(comp, rows):
    got = run_sum(comp, rows)
    for r, g in zip(rows, got):
        want = serial(r)
        if np.isnan(want):
            assert np.isnan(g)
        else:
            assert np.float64(g).tobytes() == np.float64(want).tobytes(), (len(r), g, want)


@pytest.mark.parametrize("n", [0, 1, 2, 3, 31, 32, 33, 255, 256, 257, 1000, 4096, 5000, 8192, 20000])
def test_random_terms(comp, n):
    rng = np.random.default_rng(n)
    rows = [rng.random(n), rng.random(n) ** 8, rng.standard_normal(n).astype(np.float32).astype(np.float64) ** 2,
            np.exp(-rng.random(n) * 40.0), np.exp(-rng.random(n) * 800.0)]
    check(comp, [list(r) for r in rows])


def test_ties_follow_the_running_sum(comp):
    h = 2.0 ** -53
    rows = [
        [1.0] + [h] * 999,                                   # every add ties and rounds back to 1
        [1.0, 2.0 ** -52] + [h] * 998,                       # odd last bit: the first tie rounds up
        [1.0] + [h, 2.0 ** -52] * 500,
        [1.5] + [3 * h] * 999,                               # 1.5 ulp: ties at every step
        [4.0] + [2.0 ** -51, 2.0 ** -50, 2.0 ** -51] * 333,
        [1.0] + ([2.0 ** -40] * 24 + [h]) * 20,              # a few ties: handled as explicit terms
        [1.0, 2.0 ** -52] + ([2.0 ** -40] * 30 + [h, h]) * 15,
    ]
    n = max(len(r) for r in rows)
    check(comp, [r + [0.0] * (n - len(r)) for r in rows])


def test_sums_on_binade_edges(comp):
    rows = [[1.0] * 4096, [0.5] * 4096, [0.25, 0.75] * 2048, [2.0 ** -1074] * 4096, [0.0] * 4096,
            [2.0 ** -1022 - 2.0 ** -1074] + [2.0 ** -1074] * 4095,
            [1.0 - 2.0 ** -53] * 4096]
    check(comp, rows)


def test_binade_at_every_term_falls_back_exactly(comp):
    rows = [[2.0 ** j for j in range(300)] + [1e-3] * 212,
            [2.0 ** (j - 800) * (1 + 2.0 ** -40) for j in range(512)],
            list(np.random.default_rng(5).random(512) * 2.0 ** np.arange(512) / 2.0 ** 400)]
    check(comp, rows)


def test_negative_and_non_finite_terms_take_the_serial_loop(comp):
    rng = np.random.default_rng(9)
    a = list(rng.standard_normal(3000))
    b = list(rng.random(3000)); b[1234] = float("inf")
    c = list(rng.random(3000)); c[17] = float("nan")
    d = list(rng.random(3000)); d[2999] = -0.0
    check(comp, [a, b, c, d])


@pytest.mark.parametrize("cols", [64, 1000, 4096, 5120, 8192, 14336])
def test_rmsnorm_matches_oracle(comp, O, cols):
    import torch
    rng = np.random.default_rng(cols)
    rows = 5
    x = (rng.standard_normal((rows, cols)) * np.array([1e-3, 1.0, 30.0, 1e4, 1e-20])[:, None]).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    want = O.rmsnorm(x, rows, cols, w, 1e-5).reshape(rows, cols)
    xd = torch.tensor(x, device="cuda")
    wd = torch.tensor(w, device="cuda")
    for exact_sum in (False, True):  # bracketed sum, and the serial-order sum on the device
        y = torch.empty_like(xd)
        comp.rmsnorm_dev(xd, rows, cols, wd, 1e-5, y, exact_sum=exact_sum)
        comp.sync()
        assert y.cpu().numpy().tobytes() == want.tobytes(), exact_sum


def test_rmsnorm_many_rows_matches_oracle(comp, O):
    """Many rows, so that the bracket of the serial sum is ambiguous for some
    (an output within ~1e-12 of an f32 rounding boundary) and those rows take
    the serial-order sum: every row must still equal the oracle's."""
    import torch
    rng = np.random.default_rng(11)
    rows, cols = 4096, 256
    x = (rng.standard_normal((rows, cols)) * rng.random((rows, 1)) * 10).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    want = O.rmsnorm(x, rows, cols, w, 1e-6).reshape(rows, cols)
    xd, wd = torch.tensor(x, device="cuda"), torch.tensor(w, device="cuda")
    y = torch.empty_like(xd)
    comp.rmsnorm_dev(xd, rows, cols, wd, 1e-6, y)
    comp.sync()
    assert y.cpu().numpy().tobytes() == want.tobytes()


def exp_inputs():
    """Arguments across every branch of the fdlibm method, both signs: tiny,
    the k = 0 and k = +-1 ranges and their high-word bounds (0x3fd62e42,
    0x3ff0a2b2) from both sides, the general reduction, subnormal results
    (k < -1021), the underflow and overflow thresholds, and non-finite
    values; plus the ranges the softmax (x <= 0) and SiLU (exp(-v)) take."""
    import struct
    rng = np.random.default_rng(5)

    def hw(h, lo=0):
        return struct.unpack("<d", struct.pack("<Q", (h << 32) | lo))[0]

    mag = [1e-300, 2.0 ** -30, 2.0 ** -28, hw(0x3e300000), hw(0x3e2fffff, 0xffffffff), hw(0x3fd62e42),
           hw(0x3fd62e42, 0xffffffff), hw(0x3fd62e43), hw(0x3fd62e42, 0xfefa39ef), hw(0x3ff0a2b1, 0xffffffff),
           hw(0x3ff0a2b2), hw(0x3ff0a2b2, 0x3f3bab73), 0.5 * np.log(2), 1.5 * np.log(2), np.log(2), 700.0,
           707.7, 708.39, 708.4, 709.78, hw(0x40862E42, 0xFEFA39EF), 709.79, 730.0, 745.13,
           745.1332191019411, 745.1332191019412, 745.14, 800.0, 1e300]
    edges = [0.0, -0.0] + [m * s for m in mag for s in (1.0, -1.0)]
    near = []
    for e in edges[2:]:
        for d in range(1, 4):
            near += [e + d * np.spacing(e), e - d * np.spacing(e)]
    special = [np.inf, -np.inf, np.nan]
    xs = np.concatenate([np.array(edges + near + special, np.float64), -rng.exponential(3.0, 20000),
                         rng.uniform(-750, 750, 20000), rng.uniform(-1.1, 1.1, 10000),
                         rng.standard_normal(10000) * 1e-9, rng.standard_normal(10000) * 4])
    return xs


def test_exp_table_driven_within_bound_and_settles_f32(comp):
    """The table-driven exp of the chunk softmax stays within 2^-51 relative of
    the fdlibm value on -700 <= x <= 0, and the f32 value the softmax settles
    from it is f32 of the fdlibm value for every argument (including those it
    hands back to the fdlibm path: x < -700, x > 0, non-finite)."""
    import torch
    rng = np.random.default_rng(11)
    xs = np.concatenate([exp_inputs(), -rng.exponential(2.0, 200000), rng.uniform(-700, 0, 100000),
                         -np.abs(rng.standard_normal(50000)) * 1e-3, np.array([-700.0, -699.999, -0.0])])
    x = torch.tensor(xs, dtype=torch.float64, device="cuda")
    ys = {}
    for sel in (1, 2, 3):
        y = torch.empty_like(x)
        comp.exp_dev(x, xs.size, y, sel=sel)
        ys[sel] = y
    comp.sync()
    fd, tg, st = (ys[k].cpu().numpy() for k in (1, 2, 3))
    dom = (xs >= -700.0) & (xs <= 0.0)
    rel = np.abs(tg[dom] - fd[dom]) / fd[dom]
    assert rel.max() <= 2.0 ** -51, (rel.max(), xs[dom][np.argmax(rel)])
    with np.errstate(over="ignore"):  # (results above the float range round to infinity)
        want = fd.astype(np.float32).astype(np.float64)
    bad = np.nonzero((want.view(np.uint64) != st.view(np.uint64)) & ~(np.isnan(want) & np.isnan(st)))[0]
    assert bad.size == 0, [(xs[i], want[i], st[i]) for i in bad[:5]]


def test_swiglu_settled_equals_exact(comp):
    """The SwiGLU value settled from the table-driven exp is the exact chain's
    f32 (infer.js:59, :212) for every argument: g = f32(x), u = f32(x/2 + 1/4)
    over the fast range, its edges (-80, 700), zeros, tiny, huge and
    non-finite values."""
    import torch
    rng = np.random.default_rng(13)
    edges = np.array([-80.0, -80.00001, -79.99999, 700.0, 700.001, 699.999, 0.0, -0.0, 1e-30, -1e-30, 1e-8,
                      88.7, -88.7, 1e30, -1e30, 3e38, -3e38, np.inf, -np.inf, np.nan])
    xs = np.concatenate([edges, rng.standard_normal(200000) * 3, rng.uniform(-90, 720, 100000),
                         rng.standard_normal(50000) * 1e-3]).astype(np.float32).astype(np.float64)
    x = torch.tensor(xs, dtype=torch.float64, device="cuda")
    fast, exact = torch.empty_like(x), torch.empty_like(x)
    comp.exp_dev(x, xs.size, fast, sel=4)
    comp.exp_dev(x, xs.size, exact, sel=5)
    comp.sync()
    a, b = fast.cpu().numpy(), exact.cpu().numpy()
    bad = np.nonzero((a.view(np.uint64) != b.view(np.uint64)) & ~(np.isnan(a) & np.isnan(b)))[0]
    assert bad.size == 0, [(xs[i], a[i], b[i]) for i in bad[:5]]


def test_exp_branch_free_equals_fdlibm_and_oracle(comp, O):
    """The kernels' branch-free exp gives the bits of the branching fdlibm
    method on the device for every argument, and both the oracle's exp."""
    import torch
    xs = exp_inputs()
    x = torch.tensor(xs, dtype=torch.float64, device="cuda")
    y0 = torch.empty_like(x)
    y1 = torch.empty_like(x)
    comp.exp_dev(x, xs.size, y0, sel=False)
    comp.exp_dev(x, xs.size, y1, sel=True)
    comp.sync()
    a, b = y0.cpu().numpy(), y1.cpu().numpy()
    bad = np.nonzero((a.view(np.uint64) != b.view(np.uint64)) & ~(np.isnan(a) & np.isnan(b)))[0]
    assert bad.size == 0, [(xs[i], a[i], b[i]) for i in bad[:5]]
    want = np.array([O.exp(float(v)) for v in xs])
    bad = np.nonzero((a.view(np.uint64) != want.view(np.uint64)) & ~(np.isnan(a) & np.isnan(want)))[0]
    assert bad.size == 0, [(xs[i], a[i], want[i]) for i in bad[:5]]
