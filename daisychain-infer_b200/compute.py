"""The compute core: the object ``Compute.initCompute`` returns in the reference.

Mirrors public/webgpu.js: ``init_compute`` (initCompute :284-648),
``load_luts`` (loadLUTs :247-257), ``kernel_probe`` (:1047-1060) and the
compute object's ``bgemm`` (gpuBgemmDP4 / gpuBgemmLUT :819-857), so that the
reference's vgemmBlock contract (public/verified_core.js:425-449) is met:

    out = compute.bgemm(Xq, Wq, rs, cs, dict(m=.., k=.., n=.., batch=1, relu=False, acc=False))

with host int8/f32 arrays in the reference's layouts; ``out`` is a fresh
int32 array (acc) or f32 array owned by the caller.  Errors carry the
reference's names: ``AccumulatorBoundError`` before any launch for
k > 131071, ``NonFiniteError`` for a non-finite quantiser input.

Device-resident entry points take torch CUDA tensors (torch is used only as
the device-memory allocator and for its current stream).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import DC_ACC, DC_RELU, DC_REQUANT, AccumulatorBoundError, NonFiniteError, raise_for  # noqa: F401


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data_as(C.c_void_p)
    return C.c_void_p(a.data_ptr())  # torch tensor


def flags_of(d: dict) -> int:
    f = 0
    if d.get("relu"):
        f |= DC_RELU
    if d.get("acc"):
        f |= DC_ACC
    if d.get("requant"):
        f |= DC_REQUANT
    return f


class Compute:
    """One B200 bound to one stream: ``backend``, ``label``, ``bgemm``."""

    backend = "cuda-sm100a"

    def __init__(self, device: int = 0, stream=None):
        self.L = _lib.load()
        self.device = device
        h = C.c_void_p()
        rc = self.L.dc_init(device, C.byref(h))
        if rc:
            raise_for(rc, "dc_init: " + (self.L.dc_init_error() or b"").decode())
        self.h = h
        if stream is not None:
            self.set_stream(stream)
        self.label = self.L.dc_backend_label(self.h).decode()

    # ---- plumbing -------------------------------------------------------------
    def _check(self, rc: int, where: str) -> None:
        if rc:
            raise_for(rc, f"{where}: " + (self.L.dc_last_error(self.h) or b"").decode())

    def set_stream(self, stream) -> None:
        """Launch on an existing stream (a torch.cuda.Stream or a raw handle)."""
        handle = getattr(stream, "cuda_stream", stream)
        # torch reports the legacy default stream as handle 0; CUDA names it cudaStreamLegacy (0x1)
        self._check(self.L.dc_set_stream(self.h, C.c_void_p(handle if handle else 1)), "dc_set_stream")

    def sync(self) -> None:
        self._check(self.L.dc_sync(self.h), "dc_sync")

    @property
    def tc_enabled(self) -> bool:
        return bool(self.L.dc_tc_enabled(self.h))

    def close(self) -> None:
        if getattr(self, "h", None):
            self.L.dc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- the LUT units ----------------------------------------------------------
    def luts(self) -> dict:
        """loadLUTs: {mul int16[65536], requant int8[65536], relu int8[256], shift 8},
        rebuilt by the library and checked against the reference's sha256 ids."""
        mul = np.empty(65536, np.int16)
        req = np.empty(65536, np.int8)
        relu = np.empty(256, np.int8)
        self._check(self.L.dc_luts(self.h, _ptr(mul), _ptr(req), _ptr(relu)), "dc_luts")
        return dict(mul=mul, requant=req, relu=relu, shift=8)

    # ---- compute.bgemm (host buffers) -------------------------------------------
    def bgemm(self, Xq, Wq, rs, cs, d: dict) -> np.ndarray:
        m, k, n = int(d["m"]), int(d["k"]), int(d["n"])
        batch = int(d.get("batch") or 1)
        flags = flags_of(d)
        if k > _lib.MAX_INT32_K:
            raise AccumulatorBoundError(f"bgemm: contraction length {k} exceeds the int32 accumulator headroom "
                                        f"{_lib.MAX_INT32_K} (the sum would wrap)")
        Xq = np.ascontiguousarray(Xq, np.int8).reshape(-1)
        Wq = np.ascontiguousarray(Wq, np.int8).reshape(-1)
        rs = np.ascontiguousarray(rs, np.float32).reshape(-1)
        cs = np.ascontiguousarray(cs, np.float32).reshape(-1)
        if Xq.size != batch * m * k or Wq.size != batch * k * n or rs.size != batch * m or cs.size != batch * n:
            raise ValueError("bgemm: buffer sizes do not match d")
        dt = np.int32 if flags & DC_ACC else (np.int8 if flags & DC_REQUANT else np.float32)
        out = np.empty(batch * m * n, dt)
        self._check(self.L.dc_bgemm(self.h, _ptr(Xq), _ptr(Wq), _ptr(rs), _ptr(cs), m, k, n, batch, flags,
                                    _ptr(out)), "bgemm")
        return out

    # ---- device-resident entry points (torch CUDA tensors) ---------------------
    def bgemm_dev(self, xq, ldx, wt, ldw, rs, cs, m, k, n, batch, flags, out, kind: int = 0) -> None:
        if kind:
            rc = self.L.dc_bgemm_dev_kind(self.h, _ptr(xq), ldx, _ptr(wt), ldw, _ptr(rs), _ptr(cs), m, k, n, batch,
                                          flags, _ptr(out), kind)
        else:
            rc = self.L.dc_bgemm_dev(self.h, _ptr(xq), ldx, _ptr(wt), ldw, _ptr(rs), _ptr(cs), m, k, n, batch, flags,
                                     _ptr(out))
        self._check(rc, "bgemm_dev")

    def bgemm_lut_dev(self, xq, wq, rs, cs, m, k, n, batch, flags, out) -> None:
        self._check(self.L.dc_bgemm_lut_dev(self.h, _ptr(xq), _ptr(wq), _ptr(rs), _ptr(cs), m, k, n, batch, flags,
                                            _ptr(out)), "bgemm_lut_dev")

    def quantize_rows_dev(self, X, rows, cols, q, ldq, s) -> None:
        self._check(self.L.dc_quantize_rows(self.h, _ptr(X), rows, cols, _ptr(q), ldq, _ptr(s)), "quantize_rows")

    def quantize_cols_t_dev(self, W, rows, cols, qt, ldq, s) -> None:
        self._check(self.L.dc_quantize_cols_t(self.h, _ptr(W), rows, cols, _ptr(qt), ldq, _ptr(s)),
                    "quantize_cols_t")

    def register_weight(self, W: np.ndarray, k: int, n: int) -> "Weight":
        return Weight(self, W, k, n)

    def vgemm_dev(self, X, m, w: "Weight", flags, out) -> None:
        self._check(self.L.dc_vgemm(self.h, _ptr(X), m, w.h, flags, _ptr(out)), "vgemm")

    def ordered_sum_dev(self, terms, rows, n, out) -> None:
        """out[r] = serial double sum of terms[r] in index order (infer.js:73-76, :100-104)."""
        self._check(self.L.dc_ordered_sum_dev(self.h, _ptr(terms), rows, n, _ptr(out)), "ordered_sum")

    def exp_dev(self, x, n, y, sel=False) -> None:
        """y = Math.exp(x) by the fdlibm method (sel True or 1: the branch-free form the kernels
        use; 2: the table-driven exp of the chunk softmax; 3: f32(Math.exp(x)) as that softmax
        settles it; 4, 5: the SwiGLU value of g = f32(x), u = f32(x/2 + 1/4), settled and exact)."""
        self._check(self.L.dc_exp_dev(self.h, _ptr(x), n, _ptr(y), int(sel)), "exp")

    def rmsnorm_dev(self, x, rows, cols, w, eps, y, exact_sum: bool = False) -> None:
        """infer.js rmsnorm (:70-80) of rows x cols f32 (exact_sum: always the serial-order sum)."""
        self._check(self.L.dc_rmsnorm_dev(self.h, _ptr(x), rows, cols, _ptr(w), float(eps), _ptr(y),
                                          1 if exact_sum else 0), "rmsnorm")

    def measure_capacity(self, spec=None, T: int = 16, seconds: float = 0.3) -> float:
        """The capacity the ring's planner apportions layers by, in the
        reference's unit: verified 32x64x64 GEMMs per second (app.js
        measureCapacity, :508-519).  Without ``spec`` it is that probe itself
        (vgemmBlock of the same X = sin(i)/2, W = cos(i)/2, each call waited
        for).  With a model ``spec`` it is measured at the real shapes: the
        four projection GEMMs of a T-row chunk (QKV, O, gate/up, down) on
        device-resident int8 weights, back to back, as MACs per second over the
        probe's 32*64*64 MACs -- the unit shard.estimate_lap_ms divides by."""
        import time

        import torch
        from .shard import UNIT_MACS
        dev = torch.device("cuda", self.device)
        if spec is None:
            m, k, n = 32, 64, 64
            X = torch.from_numpy((np.sin(np.arange(m * k)) * 0.5).astype(np.float32)).to(dev)
            w = self.register_weight((np.cos(np.arange(k * n)) * 0.5).astype(np.float32), k, n)
            out = torch.empty(m * n, dtype=torch.float32, device=dev)
            self.vgemm_dev(X, m, w, 0, out)
            self.sync()
            t0, it = time.perf_counter(), 0
            while time.perf_counter() - t0 < seconds:
                self.vgemm_dev(X, m, w, 0, out)
                self.sync()
                it += 1
            return it / (time.perf_counter() - t0)
        C_, hd = spec.hidden, spec.headDim or spec.hidden // spec.heads
        q, kv, I_ = spec.heads * hd, spec.kvHeads * hd, spec.inter
        g = torch.Generator(device=dev)
        g.manual_seed(0x5EED)
        ops = []
        for k, n in ((C_, q + 2 * kv), (q, C_), (C_, 2 * I_), (I_, C_)):
            ld = (k + 15) // 16 * 16
            wt = torch.randint(-127, 128, (n, ld), dtype=torch.int8, device=dev, generator=g)
            xq = torch.randint(-127, 128, (T, ld), dtype=torch.int8, device=dev, generator=g)
            cs = torch.rand(n, device=dev, generator=g) * 1e-3
            rs = torch.rand(T, device=dev, generator=g)
            out = torch.empty(T * n, dtype=torch.float32, device=dev)
            ops.append((xq, ld, wt, rs, cs, k, n, out))

        def one_pass():
            for xq, ld, wt, rs, cs, k, n, out in ops:
                self.bgemm_dev(xq, ld, wt, ld, rs, cs, T, k, n, 1, 0, out)

        one_pass()
        self.sync()
        t0, passes = time.perf_counter(), 0
        while True:
            for _ in range(8):
                one_pass()
            passes += 8
            self.sync()
            el = time.perf_counter() - t0
            if el >= seconds:
                break
        macs = T * sum(k * n for _, _, _, _, _, k, n, _ in ops)
        return macs * passes / UNIT_MACS / el

    def kernel_probe(self) -> int:
        """kernelProbe's int32 hash (webgpu.js:1047-1055, before the math fold)."""
        h = C.c_uint32()
        self._check(self.L.dc_kernel_probe(self.h, C.byref(h)), "kernel_probe")
        return h.value


class Weight:
    """A weight quantised once and resident in HBM (dc_weight_register)."""

    def __init__(self, comp: Compute, W: np.ndarray, k: int, n: int):
        self.comp = comp
        W = np.ascontiguousarray(W, np.float32).reshape(-1)
        if W.size != k * n:
            raise ValueError("weight: size does not match k x n")
        h = C.c_void_p()
        comp._check(comp.L.dc_weight_register(comp.h, _ptr(W), k, n, C.byref(h)), "weight_register")
        self.h = h
        self.k, self.n = k, n
        qt, ld, cs = C.c_void_p(), C.c_int(), C.c_void_p()
        comp.L.dc_weight_info(self.h, C.byref(qt), C.byref(ld), C.byref(cs), None, None)
        self.qt_ptr, self.ldw, self.cs_ptr = qt.value, ld.value, cs.value

    def __del__(self):
        try:
            if self.h:
                self.comp.L.dc_weight_free(self.h)
                self.h = None
        except Exception:
            pass


def init_compute(device: int = 0, stream=None) -> Compute:
    """initCompute (webgpu.js:284): a gated compute object, or an exception."""
    return Compute(device, stream)
