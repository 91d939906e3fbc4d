"""The forward pass split at layer boundaries: public/infer.js on the B200.

``Stage`` wraps a ``dc_stage`` (include/dcinfer.h): one contiguous layer range
of a Llama-family model resident in HBM with its KV cache.  The functions
mirror the reference's API and meaning:

    embed_rows (infer.js:298)   run_layers (:275)    run_layers_chunk (:288)
    logits_at (:324)            generate_local (:448)
    generate_lookahead (:464)   generate_chunked (:339)

Activations live on the device (torch tensors used as plain device buffers);
greedy picks come back to the host as token ids.  ``NonFiniteError`` is raised
for a non-finite activation, as runLayers does (:279-281).
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np

from . import shard
from ._lib import DcSpec, raise_for


# Synthetic benchmark weights: a sum of four uniform 32-bit draws (variance
# 4 * 2^64 / 12), centred, scaled once to standard deviation 0.02.
SYNTH_STD = 0.02
SYNTH_FACTOR = SYNTH_STD / (math.sqrt(4.0 / 12.0) * 4294967296.0)


@dataclass
class Spec:
    """The Llama-family fields of arch.js fromConfig (:50-71)."""
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
        if self.heads % self.kvHeads:
            raise ValueError(f"num_attention_heads ({self.heads}) is not a multiple of num_key_value_heads "
                             f"({self.kvHeads})")

    @classmethod
    def from_config(cls, cfg: dict) -> "Spec":
        """arch.js:30-81 for the Llama family; other families are refused by name."""
        t = str(cfg.get("model_type", "")).lower()
        if t not in {"llama", "mistral", "qwen2", "qwen3", "smollm", "tinyllama", "olmo", "phi3"}:
            raise ValueError(f'unsupported architecture "{cfg.get("model_type", "unknown")}"')
        need = ("hidden_size", "num_hidden_layers", "num_attention_heads", "vocab_size")
        if any(not cfg.get(k) for k in need):
            raise ValueError("config.json is missing hidden_size / num_hidden_layers / num_attention_heads / "
                             "vocab_size")
        if not cfg.get("intermediate_size"):
            raise ValueError("a gated MLP needs intermediate_size in config.json")
        h = cfg["hidden_size"]
        heads = cfg["num_attention_heads"]
        return cls(hidden=h, layers=cfg["num_hidden_layers"], heads=heads,
                   kvHeads=cfg.get("num_key_value_heads", heads), inter=cfg["intermediate_size"],
                   vocab=cfg["vocab_size"], headDim=cfg.get("head_dim", h // heads),
                   normEps=cfg.get("rms_norm_eps", 1e-5), ropeTheta=cfg.get("rope_theta", 10000.0),
                   tie=bool(cfg.get("tie_word_embeddings", False)), maxPos=cfg.get("max_position_embeddings", 2048))

    def c_spec(self) -> DcSpec:
        return DcSpec(self.hidden, self.layers, self.heads, self.kvHeads, self.headDim, self.inter, self.vocab,
                      float(self.normEps), float(self.ropeTheta), 1 if self.tie else 0)


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data_as(C.c_void_p)
    return C.c_void_p(a.data_ptr())


class Stage:
    """Layers [lo, hi) of one model on the compute core's device."""

    def __init__(self, comp, spec: Spec, lo: int, hi: int, head: bool, max_rows: int, max_pos: int):
        import torch
        self.torch = torch
        self.comp, self.spec, self.lo, self.hi, self.head = comp, spec, lo, hi, head
        self.max_rows, self.max_pos = max_rows, max_pos
        self.L = comp.L
        h = C.c_void_p()
        cs = spec.c_spec()
        self._check(self.L.dc_stage_create(comp.h, C.byref(cs), lo, hi, 1 if head else 0, max_rows, max_pos,
                                           C.byref(h)), "stage_create")
        self.h = h
        dev = torch.device("cuda", comp.device)
        self.dev = dev
        self._ids = torch.empty(max_rows, dtype=torch.int32, device=dev)
        self._picks = torch.empty(8, dtype=torch.int32, device=dev)
        self._logits = torch.empty(8 * spec.vocab, dtype=torch.float32, device=dev) if head else None

    def _check(self, rc, where):
        if rc:
            raise_for(rc, f"{where}: " + (self.L.dc_last_error(self.comp.h) or b"").decode())

    def close(self):
        if getattr(self, "h", None):
            self.L.dc_stage_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- weights ----------------------------------------------------------------
    def set_layer(self, layer: int, ly: dict) -> None:
        keys = ("nrm1", "nrm2", "Wq", "Wk", "Wv", "Wo", "Wgate", "Wup", "Wdown")
        arrs = [np.ascontiguousarray(ly[k], np.float32) for k in keys]
        self._check(self.L.dc_stage_set_layer(self.h, layer, *[_ptr(a) for a in arrs]), "stage_set_layer")

    def set_head(self, emb, nrmF, lm=None) -> None:
        e = np.ascontiguousarray(emb, np.float32)
        n = np.ascontiguousarray(nrmF, np.float32)
        m = None if lm is None else np.ascontiguousarray(lm, np.float32)
        self._check(self.L.dc_stage_set_head(self.h, _ptr(e), _ptr(n), _ptr(m)), "stage_set_head")

    def load(self, w: dict) -> None:
        """Weights as the oracle's fixtures hold them (k x n f32, reference layout)."""
        for l in range(self.lo, self.hi):
            self.set_layer(l, w["layers"][l])
        if self.head:
            self.set_head(w["emb"], w["nrmF"], w.get("lm"))

    def load_safetensors(self, path: str) -> None:
        """This stage's tensors of a safetensors model file: only their byte
        ranges are read (shard.js stageWeights :78-121), then quantised on the GPU."""
        from . import safetensors
        self.load(safetensors.read_stage_weights(path, self.spec, self.lo, self.hi, self.head))

    def synth(self, model_seed: int, factor: float | None = None) -> None:
        """Random-init weights of the synthetic benchmark models, generated on
        the GPU (``dc_stage_synth``); ``factor`` defaults to SYNTH_FACTOR."""
        if factor is None:
            factor = SYNTH_FACTOR
        self._check(self.L.dc_stage_synth(self.h, model_seed, float(factor)), "stage_synth")

    # ---- the pass -----------------------------------------------------------------
    def embed_rows(self, ids) -> "torch.Tensor":
        torch = self.torch
        ids = torch.as_tensor(np.asarray(ids, np.int32)).to(self.dev, non_blocking=False)
        T = ids.numel()
        x = torch.empty(T * self.spec.hidden, dtype=torch.float32, device=self.dev)
        self._check(self.L.dc_stage_embed(self.h, _ptr(ids), T, _ptr(x)), "stage_embed")
        return x

    def run_layers(self, x) -> "torch.Tensor":
        """Full-window pass of this stage's layers, in place on x (positions 0..T-1)."""
        T = x.numel() // self.spec.hidden
        self._check(self.L.dc_stage_forward(self.h, _ptr(x), T, 0, 0), "runLayers")
        return x

    def run_layers_chunk(self, x, pos0: int) -> "torch.Tensor":
        """One chunk at positions pos0.., appending to this stage's KV cache."""
        T = x.numel() // self.spec.hidden
        self._check(self.L.dc_stage_forward(self.h, _ptr(x), T, pos0, 1), "runLayersChunk")
        return x

    def run_layers_chunks(self, x, pos0: int, rows) -> "torch.Tensor":
        """Consecutive chunks (lengths ``rows``) at positions pos0.. in one pass
        over this stage's weights, appending to the KV cache; bit-identical to
        run_layers_chunk on each chunk in turn."""
        T = x.numel() // self.spec.hidden
        r = np.ascontiguousarray(rows, np.int32)
        if r.size == 1:
            return self.run_layers_chunk(x, pos0)
        self._check(self.L.dc_stage_forward_chunks(self.h, _ptr(x), T, pos0, _ptr(r), r.size), "runLayersChunk")
        return x

    def logits_at(self, x, rows):
        """Greedy picks (host list) and device logits of the given rows."""
        T = x.numel() // self.spec.hidden
        r = np.ascontiguousarray(rows, np.int32)
        self._check(self.L.dc_stage_logits(self.h, _ptr(x), T, _ptr(r), r.size, _ptr(self._logits),
                                           _ptr(self._picks)), "logitsAt")
        self.comp.sync()
        picks = self._picks[: r.size].cpu().tolist()
        return picks, self._logits[: r.size * self.spec.vocab].view(r.size, self.spec.vocab)

    # ---- device-resident token ids (no host round trip per decode lap) ------------
    def new_ids(self, n: int):
        return self.torch.zeros(max(n, 1), dtype=self.torch.int32, device=self.dev)

    def ids_buffer(self, n: int):
        return self.torch.zeros(n, dtype=self.torch.int32, device=self.dev)

    def pick_into(self, x, row: int, picks, n: int) -> None:
        """Greedy pick of one row of x written to picks[n] on the device."""
        T = x.numel() // self.spec.hidden
        r = np.array([row], np.int32)
        self._check(self.L.dc_stage_logits(self.h, _ptr(x), T, _ptr(r), 1, _ptr(self._logits),
                                           C.c_void_p(picks.data_ptr() + 4 * n)), "logitsAt")

    def embed_device(self, picks, n: int):
        """embedRows of the single id picks[n] (a device int32)."""
        x = self.torch.empty(self.spec.hidden, dtype=self.torch.float32, device=self.dev)
        self._check(self.L.dc_stage_embed(self.h, C.c_void_p(picks.data_ptr() + 4 * n), 1, _ptr(x)), "stage_embed")
        return x

    def decode_many(self, stages, last, n_new: int, use_graph: bool = True):
        """n_new chunked-decode laps over `stages` (this stage is the head, all on
        one device) from the last hidden row of `last`; returns the device ids."""
        picks = self.new_ids(n_new)
        row = last[last.numel() - self.spec.hidden:]
        arr = (C.c_void_p * len(stages))(*[s.h.value for s in stages])
        self._check(self.L.dc_decode_run(arr, len(stages), _ptr(row), n_new, _ptr(picks), 1 if use_graph else 0),
                    "decode_run")
        return picks

    def broadcast_ids(self, buf) -> None:
        import torch.distributed as dist
        dist.broadcast(buf, src=0)

    def kv_reset(self) -> None:
        self._check(self.L.dc_stage_kv_reset(self.h), "kv_reset")

    def set_row_graph(self, on: bool) -> None:
        """One-row cached forwards (decode steps) as a CUDA graph (default) or kernel by kernel."""
        self._check(self.L.dc_stage_set_row_graph(self.h, 1 if on else 0), "set_row_graph")

    def handoff(self, dst: "Stage", x, out) -> "torch.Tensor":
        """Hand this stage's output rows x to stage dst's buffer out (its device):
        the stage-to-stage hop, ordered after this stage's work and before dst's."""
        T = x.numel() // self.spec.hidden
        self._check(self.L.dc_stage_handoff(self.h, dst.h, _ptr(x), _ptr(out), T), "stage_handoff")
        return out

    def set_pass_attention(self, mode: int) -> None:
        """0: by size (default); 1: one CTA per (head, chunk) whenever it fits; 2: never."""
        self._check(self.L.dc_stage_set_pass_attention(self.h, int(mode)), "set_pass_attention")

    def set_row_fusion(self, on: bool) -> None:
        """Decode rows with the norm / SwiGLU / row quantisation fused into their
        GEMVs, or as separate kernels (default); the results are identical."""
        self._check(self.L.dc_stage_set_row_fusion(self.h, 1 if on else 0), "set_row_fusion")

    def set_timeline(self, buf=None, per_lap: int = 0, laps: int = 0) -> None:
        """Stamp %globaltimer after every launch of each decode lap this (head)
        stage runs through decode_many, into buf (device int64, laps x per_lap);
        set_timeline() turns it off.  A measurement aid: each stamp adds a
        one-thread launch to the lap."""
        self._check(self.L.dc_stage_set_timeline(self.h, _ptr(buf) if buf is not None else None,
                                                 per_lap if buf is not None else 0,
                                                 laps if buf is not None else 0), "stage_set_timeline")

    def timeline_info(self):
        """(kinds, bytes) of the stamps of one lap: for stamp i, the kind of the
        launch it closes (1 one-row GEMV, 3 tcgen05 GEMM, 0 other) and that
        GEMM's algorithmic bytes."""
        n = self.L.dc_stage_timeline_info(self.h, None, None, 0)
        kinds = (C.c_int * max(n, 1))()
        by = (C.c_double * max(n, 1))()
        self.L.dc_stage_timeline_info(self.h, kinds, by, n)
        return list(kinds)[:n], list(by)[:n]

    def kv_len(self) -> int:
        return self.L.dc_stage_kv_len(self.h)

    def kv_read(self, layer: int):
        n = self.kv_len()
        s = self.spec
        k8 = np.empty(s.kvHeads * n * s.headDim, np.int8)
        ks = np.empty(s.kvHeads * n, np.float32)
        v = np.empty(n * s.kvHeads * s.headDim, np.float32)
        self._check(self.L.dc_stage_kv_read(self.h, layer, _ptr(k8), _ptr(ks), _ptr(v)), "kv_read")
        return k8, ks, v


def _sync_check(stages):
    stages[0].comp.sync()


def run_ring(stages, x, chunk_pos=None, rows=None):
    """One lap through every stage in plan order (the hop is a device buffer);
    ``rows`` (chunk lengths) runs several chunks in one pass of each stage."""
    for S in stages:
        if S.hi > S.lo:
            if chunk_pos is None:
                x = S.run_layers(x)
            elif rows is not None and len(rows) > 1:
                x = S.run_layers_chunks(x, chunk_pos, rows)
            else:
                x = S.run_layers_chunk(x, chunk_pos)
    return x


def generate_local(stages, ids, n_tokens: int, T: int) -> list:
    """infer.js:448-460, greedy."""
    head = stages[0]
    out = list(ids)
    for _ in range(n_tokens):
        tail = out[-T:]
        win = [0] * (T - len(tail)) + tail
        x = run_ring(stages, head.embed_rows(win))
        picks, _ = head.logits_at(x, [T - 1])
        out.append(picks[0])
    return out


def generate_lookahead(stages, ids0, n_new: int, T: int, max_draft: int = 4) -> list:
    """infer.js:464-494, greedy: the prompt-lookup draft scored in the same lap."""
    head = stages[0]
    ids = list(ids0)
    produced = 0
    while produced < n_new:
        frame = shard.lookahead_frame(ids, T, max_draft)
        draft = frame["draft"]
        win = [0] * (T - len(frame["win"])) + frame["win"]
        x = run_ring(stages, head.embed_rows(win))
        rows = shard.draft_rows(T, frame["shown"], len(draft))
        picked, _ = head.logits_at(x, rows)
        got = shard.accept_draft(picked, draft)
        if not got:
            break
        for t in got:
            ids.append(t)
            produced += 1
            if produced >= n_new:
                break
    return ids


def generate_chunked(stages, ids0, n_new: int, chunk_size: int, use_device_loop: bool = True,
                     use_graph: bool = True, per_pass: int = 1) -> list:
    """infer.js:339-367, greedy: chunked prefill on per-stage KV, then one token per lap.
    The decode laps run on the device (dc_decode_run, optionally one CUDA graph
    replayed per lap); use_device_loop=False runs them from the host instead.
    per_pass > 1 runs that many consecutive chunks per pass over the weights
    (the same ids)."""
    head = stages[0]
    ids = list(ids0)
    for S in stages:
        S.kv_reset()
    last = None
    chunks = shard.prefill_chunks(len(ids), chunk_size, 1)["chunks"]
    for lo, hi, rows in shard.chunk_passes(chunks, per_pass):
        last = run_ring(stages, head.embed_rows(ids[lo:hi]), lo, rows)
    if use_device_loop:
        picks = head.decode_many(stages, last, n_new, use_graph)
        return ids + picks[:n_new].cpu().tolist()
    for _ in range(n_new):
        rows = last.numel() // head.spec.hidden
        picks, _ = head.logits_at(last, [rows - 1])
        ids.append(picks[0])
        pos = len(ids) - 1
        last = run_ring(stages, head.embed_rows([picks[0]]), pos)
    return ids
