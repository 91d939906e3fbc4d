"""GEMM unit parity on the B200: every kernel against the CPU oracle, bit for bit.

Covers the reference's gate shapes (webgpu.js:471-475) in every output mode,
ragged and empty shapes, the k bound, the kernel probe, and the standalone
INT8 GEMM sweep: M in {1,16,128,512} x (K,N) in {(576,1536), (1536,576),
(2048,5632), (4096,14336)}, int32 and int8 outputs bit-exact.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GATE_SHAPES = [(5, 9, 6, 3, True), (32, 64, 32, 1, False), (7, 253, 5, 2, True), (1, 4, 1, 1, False),
               (17, 33, 9, 1, True)]
SWEEP_KN = [(576, 1536), (1536, 576), (2048, 5632), (4096, 14336)]


def modes(relu):
    return [dict(acc=True), dict(relu=relu), dict(requant=True), dict(requant=True, relu=True)]


def rand_case(rng, m, k, n, b):
    X = rng.integers(-128, 128, b * m * k, dtype=np.int8)
    W = rng.integers(-128, 128, b * k * n, dtype=np.int8)
    rs = (rng.random(b * m) + 0.5).astype(np.float32)
    cs = (rng.random(b * n) + 0.5).astype(np.float32)
    return X, W, rs, cs


def test_init_label_and_luts(comp, O):
    assert "sm_100a" in comp.label
    L = comp.luts()
    mul, req, relu = O.make_luts()
    assert L["mul"].tobytes() == mul.tobytes() and L["requant"].tobytes() == req.tobytes()
    assert L["relu"].tobytes() == relu.tobytes() and L["shift"] == 8


@pytest.mark.parametrize("shape", GATE_SHAPES)
def test_bgemm_host_gate_shapes(comp, O, P, shape):
    m, k, n, b, relu = shape
    X, W, rs, cs = rand_case(np.random.default_rng(m * 1000 + k), m, k, n, b)
    for d in modes(relu):
        d.update(m=m, k=k, n=n, batch=b)
        got = comp.bgemm(X, W, rs, cs, d)
        want = O.bgemm(X, W, rs, cs, m, k, n, b, P.compute.flags_of(d))
        assert got.tobytes() == want.tobytes(), d


def test_bgemm_empty_and_refusals(comp, P):
    out = comp.bgemm(np.zeros(0, np.int8), np.zeros(0, np.int8), np.zeros(0, np.float32), np.zeros(3, np.float32),
                     dict(m=0, k=0, n=3))
    assert out.size == 0
    with pytest.raises(P.AccumulatorBoundError):
        comp.bgemm(np.zeros(131072, np.int8), np.zeros(131072, np.int8), np.ones(1, np.float32),
                   np.ones(1, np.float32), dict(m=1, k=131072, n=1, acc=True))
    # k = 0: every accumulator is 0
    out = comp.bgemm(np.zeros(0, np.int8), np.zeros(0, np.int8), np.ones(2, np.float32), np.ones(3, np.float32),
                     dict(m=2, k=0, n=3, acc=True))
    assert (out == 0).all() and out.size == 6


def test_tensor_core_paths_passed_their_gates(comp):
    """dc_init gates the one-SM tcgen05 kernel and its 2-SM variant (M > 128)
    against the LUT kernel; both must be in use on a B200."""
    assert comp.tc_enabled
    assert "gate failed" not in comp.label, comp.label


def test_kernel_probe_matches_oracle(comp, O):
    assert comp.kernel_probe() == O.probe_hash_int32()


def _dev_case(torch, X, W, m, k, n, b):
    ld = (k + 15) // 16 * 16
    xq = torch.zeros(b * m, ld, dtype=torch.int8, device="cuda")
    xq[:, :k] = torch.from_numpy(X.reshape(b * m, k)).cuda()
    wt = torch.zeros(b, n, ld, dtype=torch.int8, device="cuda")
    wt[:, :, :k] = torch.from_numpy(W.reshape(b, k, n)).cuda().transpose(1, 2)
    return xq, wt, ld


@pytest.mark.parametrize("kind", [1, 2, 3], ids=["gemv", "simt", "tc"])
@pytest.mark.parametrize("m,k,n,b", [(1, 576, 200, 1), (5, 1536, 96, 2), (8, 64, 333, 1), (16, 576, 160, 1),
                                     (33, 960, 130, 1), (128, 2048, 256, 1), (200, 320, 72, 2), (64, 14336, 64, 1)])
def test_bgemm_dev_each_kernel(comp, O, P, kind, m, k, n, b):
    import torch
    if kind == 1 and m > 8:
        pytest.skip("GEMV kernel takes M <= 8")
    if kind == 3 and not comp.tc_enabled:
        pytest.fail("tcgen05 path is off: it failed its init gate")
    rng = np.random.default_rng(m * 7 + k + n)
    X, W, rs, cs = rand_case(rng, m, k, n, b)
    xq, wt, ld = _dev_case(torch, X, W, m, k, n, b)
    drs, dcs = torch.from_numpy(rs).cuda(), torch.from_numpy(cs).cuda()
    for d in modes(True):
        f = P.compute.flags_of(d)
        dt = torch.int32 if f & 2 else (torch.int8 if f & 4 else torch.float32)
        out = torch.empty(b * m * n, dtype=dt, device="cuda")
        out.view(torch.uint8).fill_(0x7F)  # poisoned, like the reference's dirty-buffer gate
        comp.bgemm_dev(xq, ld, wt, ld, drs, dcs, m, k, n, b, f, out, kind=kind)
        torch.cuda.synchronize()
        want = O.bgemm(X, W, rs, cs, m, k, n, b, f)
        assert out.cpu().numpy().tobytes() == want.tobytes(), (kind, d)


@pytest.mark.parametrize("M", [1, 16, 128, 512])
@pytest.mark.parametrize("K,N", SWEEP_KN)
def test_gemm_sweep_full_size(comp, O, P, M, K, N):
    """The standalone GEMM sweep as configured: A f32 ~N(0,1) quantised per row
    on the device (quantizeRows), B int8 uniform in [-127, 127] with column
    scales uniform in [1e-3, 1e-2]; every output cell of the live dispatch, as
    int32 accumulators, f32 and requant int8, equals the oracle's (its
    exact-product path, equal to bgemmJS by tests/test_oracle_fast.py) and the
    LUT kernel's.  The int8 output follows the declared requant rule."""
    import torch
    rng = np.random.default_rng(M + K + N)
    A = rng.standard_normal(M * K).astype(np.float32)
    W = rng.integers(-127, 128, K * N, dtype=np.int8)
    cs = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    ld = (K + 15) // 16 * 16
    xq = torch.zeros(M, ld, dtype=torch.int8, device="cuda")
    drs = torch.empty(M, dtype=torch.float32, device="cuda")
    comp.quantize_rows_dev(torch.from_numpy(A).cuda(), M, K, xq, ld, drs)
    X, rs = O.quantize_rows(A, M, K)
    torch.cuda.synchronize()
    assert xq[:, :K].cpu().numpy().tobytes() == X.tobytes()
    assert drs.cpu().numpy().tobytes() == rs.tobytes()
    wt = torch.zeros(N, ld, dtype=torch.int8, device="cuda")
    wt[:, :K] = torch.from_numpy(np.ascontiguousarray(W.reshape(K, N).T)).cuda()
    wq = torch.from_numpy(W).cuda()
    xr = torch.from_numpy(X).cuda()
    dcs = torch.from_numpy(cs).cuda()
    Wt = np.ascontiguousarray(W.reshape(K, N).T)
    for f in (2, 0, 4):
        dt = torch.int32 if f & 2 else (torch.int8 if f & 4 else torch.float32)
        out = torch.empty(M * N, dtype=dt, device="cuda")
        ref = torch.empty(M * N, dtype=dt, device="cuda")
        comp.bgemm_dev(xq, ld, wt, ld, drs, dcs, M, K, N, 1, f, out)
        comp.bgemm_lut_dev(xr, wq, drs, dcs, M, K, N, 1, f, ref)
        torch.cuda.synchronize()
        want = O.bgemm_t(X, Wt, rs, cs, M, K, N, f)
        assert out.cpu().numpy().tobytes() == want.tobytes(), (M, K, N, f)
        assert ref.cpu().numpy().tobytes() == want.tobytes(), (M, K, N, f, "lut")


def test_capacity_probe_and_real_shapes(comp, P):
    """measureCapacity (app.js:508-519) in the reference's unit, and at a model's
    real shapes; the planner apportions layers by these numbers."""
    unit = comp.measure_capacity(seconds=0.05)
    spec = P.infer.Spec(hidden=512, layers=4, heads=8, kvHeads=4, inter=1536, vocab=1000)
    real = comp.measure_capacity(spec, T=16, seconds=0.05)
    assert unit > 100 and real > unit  # a waited-for 32x64x64 call vs streamed layer GEMMs
    plan = P.shard.plan_stages(spec.layers, [dict(id="gpu", capacity=real), dict(id="peer", capacity=unit)])
    assert plan[0]["hi"] - plan[0]["lo"] >= plan[-1]["hi"] - plan[-1]["lo"]
