"""safetensors model files for the stages (public/safetensors.js, arch.js, shard.js).

A file is ``[u64 header length][JSON header][tensor bytes]``; the header gives
every tensor's dtype, shape and byte range (safetensors.js:1-12).  A stage
reads only its own tensors -- the byte ranges of its layers (plus the head's
embedding, final norm and lm_head on stage 0), merged into a few contiguous
reads (``coalesce``) -- widens them exactly to f32 (BF16 and F16 widen without
rounding; F64 rounds to nearest) and arranges them as the forward pass wants
them: torch's (out, in) matrices become k x n (in x out), shard.js toKN
(:70-76).  ``Stage.load`` then quantises them on the GPU.

``save_weights`` writes a weight set (e.g. the test fixtures or a synthetic
model) under the Llama tensor names of arch.js (:86-119), F32 in (out, in)
order, so the reference's loader can read the same model.
"""
from __future__ import annotations

import json
import math
import struct

import numpy as np

BYTES = {"F64": 8, "F32": 4, "F16": 2, "BF16": 2, "I64": 8, "I32": 4, "I16": 2, "I8": 1, "U8": 1, "BOOL": 1}


# ---- dtype widening (safetensors.js:17-66) ---------------------------------------
def to_f32(dtype: str, raw) -> np.ndarray:
    """Raw little-endian tensor bytes -> f32.  BF16 is the top half of an f32
    (a shift), every F16 value is exactly representable in f32, F64 rounds to
    the nearest f32.  Other dtypes are refused, as the reference does."""
    b = bytes(raw)
    if dtype == "F32":
        return np.frombuffer(b, "<f4").astype(np.float32)
    if dtype == "BF16":
        return (np.frombuffer(b, "<u2").astype(np.uint32) << 16).view(np.float32)
    if dtype == "F16":
        return np.frombuffer(b, "<f2").astype(np.float32)
    if dtype == "F64":
        return np.frombuffer(b, "<f8").astype(np.float32)
    raise ValueError(f"tensor dtype {dtype} cannot be widened to f32 here (F32, F16, BF16 and F64 can)")


# ---- header (safetensors.js:68-103) ------------------------------------------------
def parse_header(head: bytes, file_size: int | None = None) -> dict:
    """Parse the header from the first bytes of a file (at least 8 + header
    length of them).  Tensor ``start``/``end`` are absolute file offsets.
    Raises ValueError for an implausible length, a truncated or non-JSON
    header, a malformed entry or a byte count that does not match its shape."""
    if len(head) < 8:
        raise ValueError("the file ends before its header does (truncated)")
    lo, hi = struct.unpack_from("<II", head, 0)
    if hi != 0:
        raise ValueError("the 64-bit header length is implausibly large (its upper word is set)")
    limit = (file_size if file_size is not None else len(head)) - 8
    if lo <= 0 or lo > limit or 8 + lo > len(head):
        raise ValueError("the file ends before its header does (truncated)")
    try:
        meta = json.loads(head[8:8 + lo].decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError):
        raise ValueError("the header bytes are not valid JSON text") from None
    if not isinstance(meta, dict):
        raise ValueError("the header is not valid JSON for this format (not an object of tensors)")
    data_start = 8 + lo
    tensors = {}
    for name, t in meta.items():
        if name == "__metadata__":
            continue
        if (not isinstance(t, dict) or not t.get("dtype") or not isinstance(t.get("shape"), list)
                or not isinstance(t.get("data_offsets"), list) or len(t["data_offsets"]) != 2):
            raise ValueError(f'header entry "{name}" is malformed: it needs a dtype, a shape and two data offsets')
        s, e = (int(v) for v in t["data_offsets"])
        elems = math.prod(int(d) for d in t["shape"])
        per = BYTES.get(t["dtype"], 0)
        if per and e - s != elems * per:
            raise ValueError(f'"{name}" spans {e - s} bytes, but a {"x".join(str(d) for d in t["shape"])} '
                             f'{t["dtype"]} tensor takes {elems * per} (expected {elems * per})')
        tensors[name] = dict(name=name, dtype=t["dtype"], shape=[int(d) for d in t["shape"]], elems=elems,
                             start=data_start + s, end=data_start + e, bytes=e - s)
    return dict(tensors=tensors, data_start=data_start, metadata=meta.get("__metadata__") or {})


def read_header(path: str) -> dict:
    """parse_header of a file, reading only its header bytes."""
    with open(path, "rb") as f:
        f.seek(0, 2)
        size = f.tell()
        f.seek(0)
        first = f.read(8)
        if len(first) < 8:
            raise ValueError("the file ends before its header does (truncated)")
        n = struct.unpack_from("<Q", first, 0)[0]
        if n > size:
            return parse_header(first, size)  # refused there: truncated or implausible
        return parse_header(first + f.read(n), size)


def f32_bytes(tensors) -> int:
    """Bytes the tensors take once widened to f32 (safetensors.js:105-111)."""
    return sum(t["elems"] * 4 for t in tensors)


def coalesce(tensors, slack: int | None = None) -> list:
    """Merge byte ranges whose gaps are at most ``slack`` (1 MiB) into runs
    (safetensors.js:113-126): one read per run."""
    gap = (1 << 20) if slack is None else slack
    runs = []
    for t in sorted(tensors, key=lambda t: t["start"]):
        if runs and t["start"] - runs[-1]["end"] <= gap:
            runs[-1]["end"] = max(runs[-1]["end"], t["end"])
            runs[-1]["tensors"].append(t)
        else:
            runs.append(dict(start=t["start"], end=t["end"], tensors=[t]))
    return runs


# ---- tensor names of the Llama family (arch.js:86-157) -----------------------------
def layer_tensors(i: int) -> dict:
    p = f"model.layers.{i}."
    return dict(nrm1=p + "input_layernorm.weight", nrm2=p + "post_attention_layernorm.weight",
                Wq=p + "self_attn.q_proj.weight", Wk=p + "self_attn.k_proj.weight",
                Wv=p + "self_attn.v_proj.weight", Wo=p + "self_attn.o_proj.weight",
                Wgate=p + "mlp.gate_proj.weight", Wup=p + "mlp.up_proj.weight", Wdown=p + "mlp.down_proj.weight")


def head_tensors(tie: bool) -> dict:
    return dict(emb="model.embed_tokens.weight", nrmF="model.norm.weight", lm=None if tie else "lm_head.weight")


def resolver(available):
    """Resolve a name against the tensors a file holds, trying the prefix
    variants exports differ by (arch.js:124-139)."""
    have = set(available)

    def resolve(name, optional=False):
        if name is None:
            return None
        if name in have:
            return name
        for alt in ("transformer." + name, name[len("model."):] if name.startswith("model.") else name,
                    "model." + name, name[len("transformer."):] if name.startswith("transformer.") else name):
            if alt in have:
                return alt
        if optional:
            return None
        raise ValueError(f'the weights do not contain "{name}" — this repo\'s layout is not one this build recognises')

    return resolve


def stage_tensors(header: dict, spec, lo: int, hi: int, head: bool) -> dict:
    """Role -> tensor entry for one stage (arch.js tensorsFor, :141-157)."""
    resolve = resolver(header["tensors"])

    def pick(name, optional=False):
        r = resolve(name, optional)
        return header["tensors"][r] if r else None

    out = {}
    if head:
        h = head_tensors(spec.tie)
        out["emb"] = pick(h["emb"])
        out["nrmF"] = pick(h["nrmF"], True)
        out["lm"] = pick(h["lm"], True) if h["lm"] else None
    for l in range(lo, hi):
        for role, name in layer_tensors(l).items():
            out[(l, role)] = pick(name)
    return out


def _to_kn(w: np.ndarray, out_dim: int, in_dim: int) -> np.ndarray:
    """shard.js toKN (:70-76): torch (out, in) -> k x n (in, out), flattened."""
    return np.ascontiguousarray(w.reshape(out_dim, in_dim).T).reshape(-1)


def read_stage_weights(path: str, spec, lo: int, hi: int, head: bool, slack: int | None = None) -> dict:
    """The weight dict ``infer.Stage.load`` takes, for layers [lo, hi) (and the
    head's tensors when ``head``), read from a safetensors file with one read
    per coalesced run (shard.js stageWeights :78-121)."""
    header = read_header(path)
    want = stage_tensors(header, spec, lo, hi, head)
    entries = [t for t in want.values() if t is not None]
    got = {}
    with open(path, "rb") as f:
        for run in coalesce(entries, slack):
            f.seek(run["start"])
            blob = f.read(run["end"] - run["start"])
            if len(blob) != run["end"] - run["start"]:
                raise ValueError("the file ends inside the byte range of a tensor its header lists (truncated)")
            for t in run["tensors"]:
                got[t["name"]] = to_f32(t["dtype"], blob[t["start"] - run["start"]:t["end"] - run["start"]])
    C_, q, kv, I_ = spec.hidden, spec.heads * spec.headDim, spec.kvHeads * spec.headDim, spec.inter
    dims = dict(Wq=(q, C_), Wk=(kv, C_), Wv=(kv, C_), Wo=(C_, q), Wgate=(I_, C_), Wup=(I_, C_), Wdown=(C_, I_))
    w = {"layers": [None] * spec.layers}
    for l in range(lo, hi):
        ly = {}
        for role in ("nrm1", "nrm2"):
            ly[role] = got[want[(l, role)]["name"]]
        for role, (o, i) in dims.items():
            t = want[(l, role)]
            if t["elems"] != o * i:
                raise ValueError(f'tensor "{t["name"]}" has {t["elems"]} elements, the spec wants {o}x{i}')
            ly[role] = _to_kn(got[t["name"]], o, i)
        w["layers"][l] = ly
    if head:
        w["emb"] = got[want["emb"]["name"]]
        w["nrmF"] = got[want["nrmF"]["name"]] if want["nrmF"] else np.ones(C_, np.float32)
        w["lm"] = _to_kn(got[want["lm"]["name"]], spec.vocab, C_) if want["lm"] is not None else None
    return w


def save_weights(path: str, w: dict, spec, metadata: dict | None = None) -> None:
    """Write a weight dict (k x n layout, as ``read_stage_weights`` returns and
    the oracle's fixtures hold) as a Llama-named F32 safetensors file, matrices
    in torch's (out, in) order, header padded to 8 bytes."""
    C_, q, kv, I_ = spec.hidden, spec.heads * spec.headDim, spec.kvHeads * spec.headDim, spec.inter
    dims = dict(Wq=(q, C_), Wk=(kv, C_), Wv=(kv, C_), Wo=(C_, q), Wgate=(I_, C_), Wup=(I_, C_), Wdown=(C_, I_))
    items = []  # (name, shape, f32 array in file order)
    h = head_tensors(spec.tie)
    items.append((h["emb"], [spec.vocab, C_], np.asarray(w["emb"], np.float32).reshape(-1)))
    items.append((h["nrmF"], [C_], np.asarray(w["nrmF"], np.float32)))
    if not spec.tie:
        lm = np.asarray(w["lm"], np.float32).reshape(C_, spec.vocab)  # k x n
        items.append((h["lm"], [spec.vocab, C_], np.ascontiguousarray(lm.T).reshape(-1)))
    for l, ly in enumerate(w["layers"]):
        names = layer_tensors(l)
        items.append((names["nrm1"], [C_], np.asarray(ly["nrm1"], np.float32)))
        items.append((names["nrm2"], [C_], np.asarray(ly["nrm2"], np.float32)))
        for role, (o, i) in dims.items():
            kn = np.asarray(ly[role], np.float32).reshape(i, o)
            items.append((names[role], [o, i], np.ascontiguousarray(kn.T).reshape(-1)))
    meta, off = {}, 0
    if metadata:
        meta["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    for name, shape, a in items:
        meta[name] = dict(dtype="F32", shape=shape, data_offsets=[off, off + a.nbytes])
        off += a.nbytes
    hdr = json.dumps(meta, separators=(",", ":")).encode("utf-8")
    hdr += b" " * (-len(hdr) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hdr)))
        f.write(hdr)
        for _, _, a in items:
            f.write(a.astype("<f4").tobytes())
