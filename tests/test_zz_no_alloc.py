"""dc_bgemm_dev_noalloc: the GEMM for callers that must not allocate device memory.

Some hosts plan every byte of HBM before they start, or own all device
allocation themselves, and cannot let the library cudaMalloc a split-K buffer
(or cudaFree an old one, which stalls every stream on the device).  This entry
point keeps that scratch in a fixed array inside the library instead.  The test
calls it through the C ABI, twice in a row with different inputs (so a result
cannot lean on what the previous call left in the shared array), and checks
each output bit for bit against dc_bgemm_dev, the entry point that allocates.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr())


def _case(torch, rng, m, k, n):
    ld = (k + 15) // 16 * 16
    xq = torch.zeros(m, ld, dtype=torch.int8, device="cuda")
    xq[:, :k] = torch.from_numpy(rng.integers(-128, 128, (m, k), dtype=np.int8)).cuda()
    wt = torch.zeros(n, ld, dtype=torch.int8, device="cuda")
    wt[:, :k] = torch.from_numpy(rng.integers(-128, 128, (n, k), dtype=np.int8)).cuda()
    rs = torch.from_numpy((rng.random(m) + 0.5).astype(np.float32)).cuda()
    cs = torch.from_numpy(rng.uniform(1e-3, 1e-2, n).astype(np.float32)).cuda()
    return xq, wt, rs, cs, ld


@pytest.mark.parametrize("flags", [2, 0, 4], ids=["int32", "f32", "requant"])
def test_noalloc_matches_allocating_entry_point_twice(comp, flags):
    import torch
    L = comp.L
    rng = np.random.default_rng(flags + 1)
    dt = torch.int32 if flags & 2 else (torch.int8 if flags & 4 else torch.float32)
    # split-K shapes (few output tiles, long K) and a one-row shape
    for m, k, n in [(16, 4096, 1536), (64, 2048, 4096), (1, 576, 960)]:
        xq, wt, rs, cs, ld = _case(torch, rng, m, k, n)
        got = torch.empty(m * n, dtype=dt, device="cuda")
        want = torch.empty(m * n, dtype=dt, device="cuda")
        got.view(torch.uint8).fill_(0x7F)
        rc = L.dc_bgemm_dev_noalloc(comp.h, _p(xq), ld, _p(wt), ld, _p(rs), _p(cs), m, k, n, 1, flags, _p(got))
        assert rc == 0, L.dc_last_error(comp.h)
        rc = L.dc_bgemm_dev(comp.h, _p(xq), ld, _p(wt), ld, _p(rs), _p(cs), m, k, n, 1, flags, _p(want))
        assert rc == 0, L.dc_last_error(comp.h)
        comp.sync()
        assert torch.equal(got.view(torch.uint8), want.view(torch.uint8)), (m, k, n)


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
