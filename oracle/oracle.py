"""CPU oracle for the verified INT8 W8A8 path (TEST INFRASTRUCTURE ONLY).

Python face of ``dc_oracle.c`` plus restatements of the reference's integer
host logic.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline legs may import this module; the product package never does, and
nothing here is a fallback for the CUDA path.

Restated reference behaviour (paths relative to the reference project):

* ``public/verified_core.js`` quantizeRows/quantizeCols/bgemmJS/epi/accBound
  (through the C library);
* ``public/infer.js`` layerForward, embedRows, logitsAt, pickToken (greedy),
  draftRows :371-380, generateLocal :448-460, generateLookahead :464-494,
  generateChunked :339-367;
* ``public/shard.js`` planStages :32-52, prefillChunks :345-361,
  promptLookupDraft :366-385, lookaheadFrame :391-398, acceptDraft :530-536,
  fnv1a/hashF32 :195-200;
* ``public/wire.js`` packAct/unpackAct :106-120, routeAfter/classifyAct :129-138;
* ``test_pipeline.js`` makeWeights :41-68 (mulberry32 weight fixtures).

Parity for values downstream of exp/pow/cos/sin is unpinned against V8 (see
the header of dc_oracle.c); everything else is pinned bit for bit.
"""
from __future__ import annotations

import ctypes as C
import math
import os
import struct
import subprocess
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

OK, E_ACCBOUND, E_NONFINITE, E_INVAL, E_NOMEM = 0, 1, 2, 3, 4
RELU, ACC, REQUANT = 1, 2, 4
MAX_INT32_K = 131071


class NonFiniteError(ValueError):
    """verified_core.js:21-24 ``NonFiniteError``."""


class AccumulatorBoundError(ValueError):
    """verified_core.js:44-47 ``AccumulatorBoundError``."""


def _check(rc: int, where: str) -> None:
    if rc == OK:
        return
    if rc == E_NONFINITE:
        raise NonFiniteError(f"non-finite input to {where}")
    if rc == E_ACCBOUND:
        raise AccumulatorBoundError(f"{where}: contraction length exceeds {MAX_INT32_K}")
    raise RuntimeError(f"{where}: oracle error {rc}")


def build() -> str:
    """Compile liboracle.so with the committed Makefile (gcc)."""
    so = os.path.join(_HERE, "liboracle.so")
    src = os.path.join(_HERE, "dc_oracle.c")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return so


def lib():
    global _LIB
    if _LIB is not None:
        return _LIB
    L = C.CDLL(build())
    p, i64, i32, u32, d, f = C.c_void_p, C.c_int64, C.c_int, C.c_uint32, C.c_double, C.c_float
    sig = {
        "orc_max_int32_k": (i32, []),
        "orc_acc_bound": (i32, [i64]),
        "orc_first_nonfinite": (i64, [p, i64]),
        "orc_js_round": (d, [d]),
        "orc_make_luts": (None, [p, p, p]),
        "orc_quantize_rows": (i32, [p, i64, i64, p, p]),
        "orc_quantize_cols": (i32, [p, i64, i64, p, p]),
        "orc_quantize_cols_t": (i32, [p, i64, i64, p, p]),
        "orc_bgemm_t": (i32, [p, p, p, p, i32, i32, i32, C.c_uint, p]),
        "orc_model_set_fast": (None, [p, i32]),
        "orc_model_synth": (i32, [p, C.c_uint64, d, i32, i32, i32, i32]),
        "orc_epi": (f, [i32, f, f]),
        "orc_bgemm": (i32, [p, p, p, p, i32, i32, i32, i32, C.c_uint, p, p, p, p]),
        "orc_exp": (d, [d]),
        "orc_fdl_sin": (d, [d]),
        "orc_fdl_cos": (d, [d]),
        "orc_fdl_pow": (d, [d, d]),
        "orc_rmsnorm": (None, [p, i32, i32, p, d, p]),
        "orc_rope_tables": (None, [i32, d, i32, p, p]),
        "orc_apply_rope": (None, [p, i32, i32, i32, p, p, i32]),
        "orc_softmax_causal": (None, [p, i32, i32, i32, d, p]),
        "orc_swiglu": (None, [p, p, i64, p]),
        "orc_vgemm": (i32, [p, p, i32, i32, i32, p]),
        "orc_model_new": (p, [i32, i32, i32, i32, i32, i32, i32, d, d]),
        "orc_model_free": (None, [p]),
        "orc_model_set_per_call_quant": (None, [p, i32]),
        "orc_model_set_head": (i32, [p, p, p, p]),
        "orc_model_set_layer": (i32, [p, i32, p, p, p, p, p, p, p, p, p]),
        "orc_kv_new": (p, [p, i32, i32, i32]),
        "orc_kv_free": (None, [p]),
        "orc_kv_len": (i32, [p, i32]),
        "orc_kv_read": (None, [p, i32, p, p]),
        "orc_run_layers": (i32, [p, i32, i32, p, i32, p, i32]),
        "orc_embed_rows": (None, [p, p, i32, p]),
        "orc_logits_rows": (i32, [p, p, i32, p, i32, p]),
        "orc_argmax": (i32, [p, i32]),
        "orc_fnv1a": (u32, [p, i64]),
        "orc_threads": (i32, []),
        "orc_probe_inputs": (None, [p, p]),
        "orc_mulberry_fill": (None, [u32, i64, d, p]),
        "orc_synth_fill": (None, [C.c_uint64, i64, i64, d, p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = L
    return L


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


# ---- units --------------------------------------------------------------------
def make_luts():
    mul = np.empty(65536, np.int16)
    req = np.empty(65536, np.int8)
    relu = np.empty(256, np.int8)
    lib().orc_make_luts(_p(mul), _p(req), _p(relu))
    return mul, req, relu


def js_round(v: float) -> float:
    return lib().orc_js_round(float(v))


def quantize_rows(X: np.ndarray, rows: int, cols: int):
    X = np.ascontiguousarray(X, np.float32).reshape(-1)
    q = np.empty(rows * cols, np.int8)
    s = np.empty(rows, np.float32)
    _check(lib().orc_quantize_rows(_p(X), rows, cols, _p(q), _p(s)), "quantizeRows")
    return q, s


def quantize_cols(W: np.ndarray, rows: int, cols: int):
    W = np.ascontiguousarray(W, np.float32).reshape(-1)
    q = np.empty(rows * cols, np.int8)
    s = np.empty(cols, np.float32)
    _check(lib().orc_quantize_cols(_p(W), rows, cols, _p(q), _p(s)), "quantizeCols")
    return q, s


def quantize_cols_t(W: np.ndarray, rows: int, cols: int):
    """quantizeCols with the values returned transposed (cols x rows)."""
    W = np.ascontiguousarray(W, np.float32).reshape(-1)
    qt = np.empty(rows * cols, np.int8)
    s = np.empty(cols, np.float32)
    _check(lib().orc_quantize_cols_t(_p(W), rows, cols, _p(qt), _p(s)), "quantizeCols")
    return qt, s


def bgemm_t(Xq, Wt, rs, cs, m, k, n, flags=0):
    """bgemmJS (batch 1) over a transposed weight (n x k) by exact products:
    the path the full-size golden fixtures use; equal to ``bgemm``."""
    Xq = np.ascontiguousarray(Xq, np.int8).reshape(-1)
    Wt = np.ascontiguousarray(Wt, np.int8).reshape(-1)
    rs = np.ascontiguousarray(rs, np.float32).reshape(-1)
    cs = np.ascontiguousarray(cs, np.float32).reshape(-1)
    dt = np.int32 if flags & ACC else (np.int8 if flags & REQUANT else np.float32)
    out = np.empty(m * n, dt)
    _check(lib().orc_bgemm_t(_p(Xq), _p(Wt), _p(rs), _p(cs), m, k, n, flags, _p(out)), "bgemmJS")
    return out


_LUTS = None


def bgemm(Xq, Wq, rs, cs, m, k, n, batch=1, flags=0):
    """bgemmJS (verified_core.js:241-266) with the declared requant rule."""
    global _LUTS
    if _LUTS is None:
        _LUTS = make_luts()
    mul, req, relu = _LUTS
    Xq = np.ascontiguousarray(Xq, np.int8).reshape(-1)
    Wq = np.ascontiguousarray(Wq, np.int8).reshape(-1)
    rs = np.ascontiguousarray(rs, np.float32).reshape(-1)
    cs = np.ascontiguousarray(cs, np.float32).reshape(-1)
    if flags & ACC:
        out = np.empty(batch * m * n, np.int32)
    elif flags & REQUANT:
        out = np.empty(batch * m * n, np.int8)
    else:
        out = np.empty(batch * m * n, np.float32)
    _check(lib().orc_bgemm(_p(Xq), _p(Wq), _p(rs), _p(cs), m, k, n, batch, flags, _p(mul), _p(req), _p(relu),
                           _p(out)), "bgemmJS")
    return out


def epi(s: int, a: float, b: float) -> float:
    return lib().orc_epi(int(s), float(a), float(b))


def exp(x: float) -> float:
    return lib().orc_exp(float(x))


def fdl_sin(x: float) -> float:
    """Math.sin by the fdlibm method (|x| <= 2^19 pi/2)."""
    return lib().orc_fdl_sin(float(x))


def fdl_cos(x: float) -> float:
    """Math.cos by the fdlibm method (|x| <= 2^19 pi/2)."""
    return lib().orc_fdl_cos(float(x))


def fdl_pow(x: float, y: float) -> float:
    """Math.pow by the fdlibm method (x > 0 finite, y finite)."""
    return lib().orc_fdl_pow(float(x), float(y))


def vgemm(X, W, m, k, n):
    """vgemmBlock with both operands quantised on this call."""
    X = np.ascontiguousarray(X, np.float32).reshape(-1)
    W = np.ascontiguousarray(W, np.float32).reshape(-1)
    out = np.empty(m * n, np.float32)
    _check(lib().orc_vgemm(_p(X), _p(W), m, k, n, _p(out)), "vgemmBlock")
    return out


def rmsnorm(x, rows, C_, w, eps):
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    w = np.ascontiguousarray(w, np.float32).reshape(-1)
    y = np.empty_like(x)
    lib().orc_rmsnorm(_p(x), rows, C_, _p(w), float(eps), _p(y))
    return y


def rope_tables(hd, theta, maxT):
    half = hd >> 1
    c = np.empty(maxT * half, np.float32)
    s = np.empty(maxT * half, np.float32)
    lib().orc_rope_tables(hd, float(theta), maxT, _p(c), _p(s))
    return c, s


def softmax_causal(scores, T, N, n0, scale):
    scores = np.ascontiguousarray(scores, np.float32).reshape(-1)
    a = np.empty(T * N, np.float32)
    lib().orc_softmax_causal(_p(scores), T, N, n0, float(scale), _p(a))
    return a


def swiglu(g, u):
    g = np.ascontiguousarray(g, np.float32).reshape(-1)
    u = np.ascontiguousarray(u, np.float32).reshape(-1)
    out = np.empty_like(g)
    lib().orc_swiglu(_p(g), _p(u), g.size, _p(out))
    return out


def threads() -> int:
    """Threads the C restatement's parallel loops use (OpenMP; 1 without it)."""
    return int(lib().orc_threads())


def fnv1a(b: bytes | np.ndarray) -> int:
    a = np.frombuffer(bytes(b), np.uint8) if not isinstance(b, np.ndarray) else np.ascontiguousarray(b).view(np.uint8)
    return int(lib().orc_fnv1a(_p(a), a.size))


def hash_f32(a: np.ndarray) -> int:
    """shard.js:200 hashF32: FNV-1a over the raw little-endian bytes."""
    return fnv1a(np.ascontiguousarray(a, np.float32))


def probe_inputs():
    """webgpu.js:998-1009."""
    Xq = np.empty(2 * 24 * 96, np.int8)
    Wq = np.empty(2 * 96 * 24, np.int8)
    lib().orc_probe_inputs(_p(Xq), _p(Wq))
    rs = np.ones(48, np.float32)
    cs = np.ones(48, np.float32)
    return Xq, Wq, rs, cs, dict(m=24, k=96, n=24, batch=2)


def probe_hash_int32() -> int:
    """FNV-1a of the probe's int32 accumulators (webgpu.js:1052-1055), before
    the transcendental fold, which needs V8's Math.* bits."""
    Xq, Wq, rs, cs, d = probe_inputs()
    acc = bgemm(Xq, Wq, rs, cs, d["m"], d["k"], d["n"], d["batch"], ACC)
    return fnv1a(acc)


def mulberry_fill(seed: int, n: int, scale: float) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_mulberry_fill(seed & 0xFFFFFFFF, n, float(scale), _p(out))
    return out


def synth_fill(seed: int, start: int, n: int, factor: float) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_synth_fill(seed & 0xFFFFFFFFFFFFFFFF, start, n, float(factor), _p(out))
    return out


# ---- model specs and fixtures ------------------------------------------------------
@dataclass
class Spec:
    """The normalised Llama-family spec fields of arch.js:50-71."""
    hidden: int
    layers: int
    heads: int
    kvHeads: int
    inter: int
    vocab: int
    headDim: int = 0
    normEps: float = 1e-5
    ropeTheta: float = 10000.0
    tie: bool = True
    maxPos: int = 2048

    def __post_init__(self):
        if not self.headDim:
            self.headDim = self.hidden // self.heads


LLAMA_TEST = Spec(hidden=64, layers=6, heads=4, kvHeads=2, inter=128, vocab=128, maxPos=64, tie=True)


def to_kn(w_out_in: np.ndarray, out_dim: int, in_dim: int) -> np.ndarray:
    """shard.js:70-76 toKN for torch's (out, in) layout."""
    return np.ascontiguousarray(w_out_in.reshape(out_dim, in_dim).T).reshape(-1)


def make_weights(spec: Spec) -> dict:
    """test_pipeline.js:41-68 for the Llama family: mulberry32 seeds from 7 in
    the reference's put() order; weights returned in k x n layout."""
    C_, q, kv, I_ = spec.hidden, spec.heads * spec.headDim, spec.kvHeads * spec.headDim, spec.inter
    seed = [7]

    def put(n, scale=0.08):
        a = mulberry_fill(seed[0], n, scale)
        seed[0] += 1
        return a

    w = {"emb": put(spec.vocab * C_, 0.05)}
    put(C_, 1)                                   # nrmF drawn, then overwritten with ones
    w["nrmF"] = np.ones(C_, np.float32)
    w["lm"] = None if spec.tie else to_kn(put(spec.vocab * C_, 0.05), spec.vocab, C_)
    w["layers"] = []
    for _ in range(spec.layers):
        ly = {"nrm1": np.ones(C_, np.float32), "nrm2": np.ones(C_, np.float32)}
        ly["Wq"] = to_kn(put(q * C_), q, C_)
        ly["Wk"] = to_kn(put(kv * C_), kv, C_)
        ly["Wv"] = to_kn(put(kv * C_), kv, C_)
        ly["Wo"] = to_kn(put(C_ * q), C_, q)
        ly["Wgate"] = to_kn(put(I_ * C_), I_, C_)
        ly["Wup"] = to_kn(put(I_ * C_), I_, C_)
        ly["Wdown"] = to_kn(put(C_ * I_), C_, I_)
        w["layers"].append(ly)
    return w


SYNTH_STD = 0.02
SYNTH_FACTOR = SYNTH_STD / (math.sqrt(4.0 / 12.0) * 4294967296.0)


def synth_tensor_seed(model_seed: int, layer: int, role: int) -> int:
    """Seed of one tensor of a synthetic benchmark model (shared formula with
    the CUDA model builder)."""
    return (model_seed * 1000003 + (layer + 1) * 64 + role) & 0xFFFFFFFFFFFFFFFF


SYNTH_ROLES = {"emb": 1, "lm": 2, "Wq": 3, "Wk": 4, "Wv": 5, "Wo": 6, "Wgate": 7, "Wup": 8, "Wdown": 9}


def synth_weight(model_seed: int, layer: int, role: str, k: int, n: int) -> np.ndarray:
    """One synthetic weight in k x n layout: element (row r of torch's (out, in)
    layout = column of k x n) ... generated directly in k x n order."""
    return synth_fill(synth_tensor_seed(model_seed, layer, SYNTH_ROLES[role]), 0, k * n, SYNTH_FACTOR)


# ---- the model --------------------------------------------------------------------
class Model:
    """A whole Llama-family model held by the C oracle (weights k x n f32)."""

    def __init__(self, spec: Spec, w: dict, per_call_quant: bool = False, fast: bool = False):
        self.spec = spec
        self._keep = []
        L = lib()
        self.h = L.orc_model_new(spec.hidden, spec.layers, spec.heads, spec.kvHeads, spec.headDim, spec.inter,
                                 spec.vocab, float(spec.normEps), float(spec.ropeTheta))
        if not self.h:
            raise ValueError("bad spec")
        L.orc_model_set_per_call_quant(self.h, 1 if per_call_quant else 0)
        L.orc_model_set_fast(self.h, 1 if fast else 0)
        if w is None:
            return

        def keep(a):
            if a is None:
                return None
            a = np.ascontiguousarray(a, np.float32)
            self._keep.append(a)
            return a

        _check(L.orc_model_set_head(self.h, _p(keep(w["emb"])), _p(keep(w["nrmF"])), _p(keep(w.get("lm")))),
               "set_head")
        for l, ly in enumerate(w["layers"]):
            _check(L.orc_model_set_layer(self.h, l, *[_p(keep(ly[k])) for k in
                                                      ("nrm1", "nrm2", "Wq", "Wk", "Wv", "Wo", "Wgate", "Wup",
                                                       "Wdown")]), "set_layer")

    def __del__(self):
        try:
            if self.h:
                lib().orc_model_free(self.h)
        except Exception:
            pass

    def embed_rows(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        x = np.empty(ids.size * self.spec.hidden, np.float32)
        lib().orc_embed_rows(self.h, _p(ids), ids.size, _p(x))
        return x

    def run_layers(self, x: np.ndarray, lo: int, hi: int, kv: "KV | None" = None, pos0: int = 0) -> np.ndarray:
        x = np.array(x, np.float32, copy=True).reshape(-1)
        T = x.size // self.spec.hidden
        _check(lib().orc_run_layers(self.h, lo, hi, _p(x), T, kv.h if kv else None, pos0), "runLayers")
        return x

    def logits_rows(self, x: np.ndarray, rows) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        T = x.size // self.spec.hidden
        rows = np.ascontiguousarray(rows, np.int32)
        out = np.empty(rows.size * self.spec.vocab, np.float32)
        _check(lib().orc_logits_rows(self.h, _p(x), T, _p(rows), rows.size, _p(out)), "logitsAt")
        return out.reshape(rows.size, self.spec.vocab)


class SynthModel(Model):
    """A synthetic benchmark model (the weights ``synth_weight`` gives) built
    inside the C oracle on the exact-product path: each weight is generated,
    quantised once and its f32 copy dropped, so full-size models fit in RAM."""

    def __init__(self, spec: Spec, model_seed: int, factor: float = None, lo: int = 0, hi: int | None = None,
                 head: bool = True):
        super().__init__(spec, None, fast=True)
        hi = spec.layers if hi is None else hi
        _check(lib().orc_model_synth(self.h, model_seed & 0xFFFFFFFFFFFFFFFF,
                                     float(SYNTH_FACTOR if factor is None else factor), 1 if spec.tie else 0, lo, hi,
                                     1 if head else 0), "synth model")


class KV:
    """Per-stage f32 K/V cache of the chunk path (infer.js:154-165)."""

    def __init__(self, model: Model, lo: int, hi: int, max_pos: int):
        self.model = model
        self.lo, self.hi = lo, hi
        self.h = lib().orc_kv_new(model.h, lo, hi, max_pos)

    def __del__(self):
        try:
            lib().orc_kv_free(self.h)
        except Exception:
            pass

    def read(self, layer: int):
        n = lib().orc_kv_len(self.h, layer)
        kvd = self.model.spec.kvHeads * self.model.spec.headDim
        k = np.empty(n * kvd, np.float32)
        v = np.empty(n * kvd, np.float32)
        lib().orc_kv_read(self.h, layer, _p(k), _p(v))
        return k, v


def argmax(logits: np.ndarray) -> int:
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_argmax(_p(logits), logits.size))


# ---- shard.js / infer.js host logic ------------------------------------------------------
def prefill_chunks(n_tokens: int, chunk_size: int, in_flight: int):
    """shard.js:345-361."""
    size = max(1, int(chunk_size))
    window = max(1, int(in_flight))
    n = max(1, math.ceil(max(n_tokens, 1) / size))
    base = n_tokens // n
    rem = n_tokens - base * n
    chunks, lo = [], 0
    for _ in range(n):
        ln = base + (1 if rem > 0 else 0)
        if rem > 0:
            rem -= 1
        if ln < 1:
            break
        chunks.append(dict(index=len(chunks), lo=lo, hi=lo + ln))
        lo += ln
    return dict(chunks=chunks, window=window, chunkSize=size)


def prompt_lookup_draft(ids, max_draft):
    """shard.js:366-385."""
    cap = max(0, int(max_draft))
    n = len(ids)
    if cap == 0 or n < 3:
        return []
    best, best_len = [], 0
    for ln in range(2, min(n - 1, 8) + 1):
        for i in range(0, n - ln):
            if any(ids[i + j] != ids[n - ln + j] for j in range(ln)):
                continue
            draft = []
            k = 0
            while k < cap and i + ln + k < n - ln:
                draft.append(ids[i + ln + k])
                k += 1
            if not draft:
                continue
            if ln > best_len:
                best, best_len = draft, ln
    return best


def lookahead_frame(ids, T, max_draft):
    """shard.js:391-398."""
    draft = prompt_lookup_draft(ids, max_draft)
    seq = list(ids) + list(draft)
    shown = seq[-T:] if T > 0 else []
    shown_draft = min(len(draft), max(0, len(shown) - 1))
    draft = draft[len(draft) - shown_draft:]
    return dict(draft=draft, shown=len(shown), win=list(shown))


def accept_draft(picked, draft):
    """shard.js:530-536."""
    out, i = [], 0
    while i < len(draft) and i < len(picked) and picked[i] == draft[i]:
        out.append(draft[i])
        i += 1
    if i < len(picked):
        out.append(picked[i])
    return out


def draft_rows(T, seq_len, draft_len):
    """infer.js:371-380."""
    rows = []
    first = seq_len - draft_len - 1
    for i in range(draft_len + 1):
        tok = first + i
        if tok < 0 or tok >= seq_len:
            break
        rows.append(T - seq_len + tok)
    return rows


def plan_stages(layers: int, caps):
    """shard.js:32-52: largest-remainder apportionment by measured capacity."""
    n = len(caps)
    if n < 1:
        raise ValueError("no devices to plan across")
    total = sum(max(1e-6, c["capacity"]) for c in caps)
    exact = [layers * max(1e-6, c["capacity"]) / total for c in caps]
    floor = [math.floor(e) for e in exact]
    left = layers - sum(floor)
    order = sorted(((e - floor[i], i) for i, e in enumerate(exact)), key=lambda t: (-t[0], t[1]))
    i = 0
    while i < len(order) and left > 0:
        floor[order[i][1]] += 1
        i += 1
        left -= 1
    stages, lo = [], 0
    for i in range(n):
        hi = lo + floor[i]
        stages.append(dict(id=caps[i]["id"], index=i, lo=lo, hi=hi, head=i == 0,
                           backend=caps[i].get("backend"), capacity=caps[i]["capacity"]))
        lo = hi
    kept = [s for s in stages if s["head"] or s["hi"] > s["lo"]]
    return [dict(s, index=i) for i, s in enumerate(kept)]


# ---- generation loops (infer.js), over stages given as (lo, hi) layer ranges ------
def _window(ids, T):
    win = np.zeros(T, np.int32)
    tail = ids[-T:]
    win[T - len(tail):] = tail
    return win


def generate_local(model: Model, stages, ids, n_tokens, T):
    """infer.js:448-460 (greedy)."""
    out = list(ids)
    for _ in range(n_tokens):
        x = model.embed_rows(_window(out, T))
        for lo, hi in stages:
            x = model.run_layers(x, lo, hi)
        out.append(argmax(model.logits_rows(x, [T - 1])[0]))
    return out


def generate_lookahead(model: Model, stages, ids0, n_new, T, max_draft=4, trace=None):
    """infer.js:464-494 (greedy).  ``trace`` (a dict), when given, receives the
    first lap's hidden state (``first_hidden``), scored rows (``first_rows``)
    and their logits (``first_logits``), the same of the last lap (``last_win``
    its window ids, ``last_hidden``, ``last_rows``, ``last_logits``), and the
    number of laps (``laps``)."""
    ids = list(ids0)
    produced = 0
    laps = 0
    while produced < n_new:
        frame = lookahead_frame(ids, T, max_draft)
        draft = frame["draft"]
        win = np.zeros(T, np.int32)
        win[T - len(frame["win"]):] = frame["win"]
        x = model.embed_rows(win)
        for lo, hi in stages:
            x = model.run_layers(x, lo, hi)
        rows = draft_rows(T, frame["shown"], len(draft))
        logits = model.logits_rows(x, rows)
        if trace is not None:
            if laps == 0:
                trace.update(first_hidden=x.copy(), first_rows=list(rows), first_logits=logits.copy())
            trace.update(last_win=[int(v) for v in win], last_hidden=x.copy(), last_rows=list(rows),
                         last_logits=logits.copy())
        laps += 1
        picked = [argmax(logits[i]) for i in range(len(rows))]
        got = accept_draft(picked, draft)
        if not got:
            break
        for t in got:
            ids.append(t)
            produced += 1
            if produced >= n_new:
                break
    if trace is not None:
        trace["laps"] = laps
    return ids


def generate_chunked(model: Model, stages, ids0, n_new, chunk_size, max_pos=None, trace=None):
    """infer.js:339-367 (greedy); per-stage KV caches.  ``trace`` (a dict), when
    given, receives the prefill's last hidden row (``prefill_last``), the
    logits row of the first pick (``first_logits``) and the stages' caches
    after the last lap (``caches``, one ``KV`` per stage)."""
    ids = list(ids0)
    max_pos = max_pos or (len(ids0) + n_new + 1)
    caches = [KV(model, lo, hi, max_pos) if hi > lo else None for lo, hi in stages]
    last = None
    for ch in prefill_chunks(len(ids), chunk_size, 1)["chunks"]:
        x = model.embed_rows(ids[ch["lo"]:ch["hi"]])
        for (lo, hi), kv in zip(stages, caches):
            if hi > lo:
                x = model.run_layers(x, lo, hi, kv, ch["lo"])
        last = x
    for n in range(n_new):
        rows = last.size // model.spec.hidden
        lg = model.logits_rows(last, [rows - 1])[0]
        if trace is not None and n == 0:
            trace.update(prefill_last=last[(rows - 1) * model.spec.hidden:].copy(), first_logits=lg.copy())
        t = argmax(lg)
        ids.append(t)
        pos = len(ids) - 1
        x = model.embed_rows([t])
        for (lo, hi), kv in zip(stages, caches):
            if hi > lo:
                x = model.run_layers(x, lo, hi, kv, pos)
        last = x
    if trace is not None:
        trace["caches"] = caches
    return ids


# ---- wire.js ------------------------------------------------------------------------
ACT, RETURN = -23, -1


def pack_act(seq, token_idx, next_index, hidden: np.ndarray, model_hash: int) -> bytes:
    """wire.js:106-112."""
    h = np.ascontiguousarray(hidden, np.float32)
    return struct.pack("<4i2I", ACT, seq, token_idx, next_index, hash_f32(h), model_hash & 0xFFFFFFFF) + h.tobytes()


def unpack_act(buf: bytes):
    """wire.js:113-120."""
    if len(buf) < 24:
        raise ValueError("act: truncated header")
    _, seq, tok, nxt, ah, mh = struct.unpack_from("<4i2I", buf, 0)
    hidden = np.frombuffer(buf[24:], np.float32).copy()
    if hash_f32(hidden) != ah:
        raise ValueError("act: payload failed its integrity hash")
    return dict(seq=seq, tokenIdx=tok, nextIndex=nxt, actHash=ah, modelHash=mh, hidden=hidden)
