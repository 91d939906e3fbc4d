"""dc_bgemm_dev_noalloc: the GEMM for callers that must not allocate device memory.

Some hosts plan every byte of HBM before they start, or own all device
allocation themselves, and cannot let the library cudaMalloc a split-K buffer
(or cudaFree an old one, which stalls every stream on the device).  This entry
point keeps that scratch in a fixed array inside the library instead.  The
tests call it through the C ABI, twice in a row with different inputs (so a
result cannot lean on what the previous call left in the shared array), and
check each output bit for bit against the oracle's bgemmJS and against
dc_bgemm_dev, the entry point that allocates; one test checks on a fresh
context that the calls leave the device's free memory unchanged.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr())


def _case(torch, rng, m, k, n, b):
    """Device operands in the library's layout plus the same in the reference's
    (X (b*m) x k, W b x (k x n)) for the oracle."""
    ld = max(16, (k + 15) // 16 * 16)
    X = rng.integers(-128, 128, (b * m, k), dtype=np.int8)
    W = rng.integers(-128, 128, (b, k, n), dtype=np.int8)
    rs = (rng.random(b * m) + 0.5).astype(np.float32)
    cs = rng.uniform(1e-3, 1e-2, b * n).astype(np.float32)
    xq = torch.zeros(b * m, ld, dtype=torch.int8, device="cuda")
    xq[:, :k] = torch.from_numpy(X).cuda()
    wt = torch.zeros(b, n, ld, dtype=torch.int8, device="cuda")
    wt[:, :, :k] = torch.from_numpy(np.ascontiguousarray(W.transpose(0, 2, 1))).cuda()
    return dict(X=X, W=W, rs=rs, cs=cs, xq=xq, wt=wt, drs=torch.from_numpy(rs).cuda(),
                dcs=torch.from_numpy(cs).cuda(), ld=ld)


def _call(L, h, fn, c, m, k, n, b, flags, out):
    return getattr(L, fn)(h, _p(c["xq"]), c["ld"], _p(c["wt"]), c["ld"], _p(c["drs"]), _p(c["dcs"]), m, k, n, b,
                          flags, _p(out))


# split-K tensor-core shapes (few output tiles, long K; one with batch 2), a
# one-row and a k = 0 shape
SHAPES = [(16, 4096, 1536, 1), (64, 2048, 4096, 1), (24, 3000, 200, 2), (1, 576, 960, 1), (12, 0, 40, 1)]


@pytest.mark.parametrize("flags", [2, 0, 1, 4], ids=["int32", "f32", "f32-relu", "requant"])
def test_noalloc_matches_oracle_and_allocating_entry_point_twice(comp, O, flags):
    import torch
    L = comp.L
    rng = np.random.default_rng(flags + 1)
    dt = torch.int32 if flags & 2 else (torch.int8 if flags & 4 else torch.float32)
    for m, k, n, b in SHAPES:
        for rep in range(2):
            c = _case(torch, rng, m, k, n, b)
            got = torch.empty(b * m * n, dtype=dt, device="cuda")
            want = torch.empty(b * m * n, dtype=dt, device="cuda")
            got.view(torch.uint8).fill_(0x7F)
            rc = _call(L, comp.h, "dc_bgemm_dev_noalloc", c, m, k, n, b, flags, got)
            assert rc == 0, L.dc_last_error(comp.h)
            rc = _call(L, comp.h, "dc_bgemm_dev", c, m, k, n, b, flags, want)
            assert rc == 0, L.dc_last_error(comp.h)
            comp.sync()
            ref = O.bgemm(c["X"], c["W"], c["rs"], c["cs"], m, k, n, b, flags)
            assert got.cpu().numpy().tobytes() == ref.tobytes(), (m, k, n, b, rep)
            assert torch.equal(got.view(torch.uint8), want.view(torch.uint8)), (m, k, n, b, rep)


def test_noalloc_leaves_device_memory_unchanged(P):
    """On a fresh context the no-allocation calls (split-K shapes, batch 1 and
    2) leave the device's free memory exactly as it was."""
    import torch
    rng = np.random.default_rng(7)
    cases = [(16, 4096, 1536, 1), (24, 3000, 200, 2)]
    cs = [_case(torch, rng, *sh) for sh in cases]
    outs = [torch.empty(b * m * n, dtype=torch.int32, device="cuda") for m, k, n, b in cases]
    fresh = P.init_compute(0)
    try:
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for _ in range(3):
            for (m, k, n, b), c, out in zip(cases, cs, outs):
                assert _call(fresh.L, fresh.h, "dc_bgemm_dev_noalloc", c, m, k, n, b, 2, out) == 0
        fresh.sync()
        assert torch.cuda.mem_get_info()[0] == free0
    finally:
        fresh.close()


def test_noalloc_refuses_outputs_beyond_its_fixed_scratch(comp):
    import torch
    L = comp.L
    m, k, n = 256, 64, 8192          # 2M outputs > DC_NOALLOC_MAX_OUT = 1M
    xq = torch.zeros(m, k, dtype=torch.int8, device="cuda")
    wt = torch.zeros(n, k, dtype=torch.int8, device="cuda")
    rs = torch.ones(m, device="cuda")
    cs = torch.ones(n, device="cuda")
    out = torch.empty(m * n, dtype=torch.int32, device="cuda")
    rc = L.dc_bgemm_dev_noalloc(comp.h, _p(xq), k, _p(wt), k, _p(rs), _p(cs), m, k, n, 1, 2, _p(out))
    assert rc == 3  # DC_E_INVAL
    assert b"fixed scratch" in L.dc_last_error(comp.h)
    rc = L.dc_bgemm_dev_noalloc(comp.h, None, k, _p(wt), k, _p(rs), _p(cs), 4, k, 8, 1, 2, _p(out))
    assert rc == 3 and b"null" in L.dc_last_error(comp.h)
