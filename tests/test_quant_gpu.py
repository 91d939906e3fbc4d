"""Quantiser parity on the B200 (verified_core.js:108-136), bit for bit."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def edge_rows():
    rows = []
    r = np.zeros(64, np.float32); r[0] = 127.0; r[1:9] = [2.5, -2.5, 0.5, -0.5, 126.5, -126.5, 1.5, -1.5]
    rows.append(r)                                           # scale exactly 1: ties go toward +inf
    r = np.zeros(64, np.float32); r[0] = 127.0; r[1] = np.float32(0.49999997); r[2] = np.float32(-0.49999997)
    rows.append(r)                                           # just below a tie
    rows.append(np.zeros(64, np.float32))                    # all zero: scale floor 1e-8
    r = np.full(64, 1e-7, np.float32); r[3] = -1.2e-6
    rows.append(r)                                           # tiny: scale floor, values clamp
    r = np.linspace(-3e38, 3e38, 64).astype(np.float32)
    rows.append(r)                                           # huge magnitudes
    r = np.zeros(64, np.float32); r[5] = -0.0; r[6] = 5e-45  # -0 and a subnormal
    rows.append(r)
    return np.stack(rows)


def test_quantize_rows_matches_oracle(comp, O):
    import torch
    rng = np.random.default_rng(1)
    for rows, cols in [(1, 576), (16, 2048), (3, 14336), (64, 64), (5, 17)]:
        X = (rng.standard_normal((rows, cols)) * rng.uniform(0.01, 100, (rows, 1))).astype(np.float32)
        ld = (cols + 15) // 16 * 16
        q = torch.full((rows, ld), 99, dtype=torch.int8, device="cuda")
        s = torch.empty(rows, dtype=torch.float32, device="cuda")
        comp.quantize_rows_dev(torch.from_numpy(X).cuda(), rows, cols, q, ld, s)
        comp.sync()
        wq, ws = O.quantize_rows(X, rows, cols)
        qh = q.cpu().numpy()
        assert (qh[:, cols:] == 0).all()
        assert qh[:, :cols].tobytes() == wq.tobytes() and s.cpu().numpy().tobytes() == ws.tobytes()


def test_quantize_rows_edge_values(comp, O):
    import torch
    X = edge_rows()
    rows, cols = X.shape
    q = torch.empty((rows, cols), dtype=torch.int8, device="cuda")
    s = torch.empty(rows, dtype=torch.float32, device="cuda")
    comp.quantize_rows_dev(torch.from_numpy(X).cuda(), rows, cols, q, cols, s)
    comp.sync()
    wq, ws = O.quantize_rows(X, rows, cols)
    assert q.cpu().numpy().tobytes() == wq.tobytes() and s.cpu().numpy().tobytes() == ws.tobytes()
    assert list(wq[1:9]) == [3, -2, 1, 0, 127, -126, 2, -1]


def test_quantize_cols_transposed_matches_oracle(comp, O):
    import torch
    rng = np.random.default_rng(2)
    for k, n in [(576, 960), (64, 33), (253, 5), (1536, 576)]:
        W = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
        W[rng.integers(0, k), rng.integers(0, n)] = 40.0
        ld = (k + 15) // 16 * 16
        qt = torch.full((n, ld), 99, dtype=torch.int8, device="cuda")
        s = torch.empty(n, dtype=torch.float32, device="cuda")
        comp.quantize_cols_t_dev(torch.from_numpy(W).cuda(), k, n, qt, ld, s)
        comp.sync()
        wq, ws = O.quantize_cols(W, k, n)
        qh = qt.cpu().numpy()
        assert (qh[:, k:] == 0).all()
        assert qh[:, :k].T.copy().tobytes() == wq.tobytes() and s.cpu().numpy().tobytes() == ws.tobytes()
    E = edge_rows().T.copy()  # columns carry the edge values
    k, n = E.shape
    qt = torch.empty((n, k), dtype=torch.int8, device="cuda")
    s = torch.empty(n, dtype=torch.float32, device="cuda")
    comp.quantize_cols_t_dev(torch.from_numpy(E).cuda(), k, n, qt, k, s)
    comp.sync()
    wq, ws = O.quantize_cols(E, k, n)
    assert qt.cpu().numpy().T.copy().tobytes() == wq.tobytes() and s.cpu().numpy().tobytes() == ws.tobytes()


def test_non_finite_is_refused(comp, P):
    import torch
    for bad in (float("nan"), float("inf")):
        X = torch.zeros(2, 32, device="cuda")
        X[1, 7] = bad
        q = torch.empty(2, 32, dtype=torch.int8, device="cuda")
        s = torch.empty(2, device="cuda")
        comp.quantize_rows_dev(X, 2, 32, q, 32, s)
        with pytest.raises(P.NonFiniteError):
            comp.sync()
    comp.sync()  # the status word was cleared


def test_registered_weight_vgemm_matches_oracle(comp, O):
    import torch
    rng = np.random.default_rng(4)
    for m, k, n in [(1, 576, 1536), (16, 2048, 256), (64, 960, 320)]:
        X = rng.standard_normal((m, k)).astype(np.float32)
        W = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
        w = comp.register_weight(W, k, n)
        out = torch.empty(m * n, dtype=torch.float32, device="cuda")
        comp.vgemm_dev(torch.from_numpy(X).cuda(), m, w, 0, out)
        comp.sync()
        want = O.vgemm(X, W, m, k, n)
        assert out.cpu().numpy().tobytes() == want.tobytes(), (m, k, n)
