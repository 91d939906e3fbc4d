"""The browser ring's activation frame (public/wire.js), for a B200 stage that
speaks it.

Between B200 ranks the hidden state moves as a bare f32 buffer over NCCL
(``pipeline.TorchP2P``).  A stage that exchanges activations with the
reference's peers instead frames every hop as wire.js does:

    [i32 ACT = -23, seq, tokenIdx, nextIndex][u32 actHash, modelHash][f32 hidden]

(wire.js:100-121), little-endian, 24 header bytes, actHash = FNV-1a of the
payload bytes (shard.js:195-200, computed natively by ``dc_fnv1a``), modelHash
= the model fingerprint of shard.js:206-213.  ``nextIndex`` is the receiving
stage's index, or RETURN (-1) on the leg back to the head (wire.js:129-138).
``WireTransport`` wraps a point-to-point transport so that ``pipeline.Ring``
sends and checks these frames; the layout, sentinels and hash are the
reference's, so the bytes are interchangeable with its codec.
"""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np

from . import _lib
from .pipeline import RETURN, classify_act, route_after

ACT = -23
_HDR = struct.Struct("<4i2I")
HEADER_BYTES = _HDR.size  # 24


def fnv1a(data) -> int:
    """FNV-1a (32-bit) of a bytes-like object or a contiguous numpy array."""
    a = np.ascontiguousarray(np.frombuffer(data, np.uint8) if isinstance(data, (bytes, bytearray, memoryview))
                             else data)
    return int(_lib.load().dc_fnv1a(a.ctypes.data_as(C.c_void_p), a.nbytes))


def hash_f32(hidden) -> int:
    """shard.js hashF32: FNV-1a over the bytes of an f32 array."""
    return fnv1a(np.ascontiguousarray(hidden, np.float32))


def pack_act(seq: int, token_idx: int, next_index: int, hidden, model_hash: int) -> bytes:
    """wire.js packAct (:106-112)."""
    h = np.ascontiguousarray(hidden, np.float32)
    return _HDR.pack(ACT, seq, token_idx, next_index, hash_f32(h), model_hash & 0xFFFFFFFF) + h.tobytes()


def unpack_act(buf) -> dict:
    """wire.js unpackAct (:113-120); the tag is checked too (wire.js tagOf
    dispatch).  Raises ValueError on a short, mistagged or corrupted frame."""
    b = bytes(buf)
    if len(b) < HEADER_BYTES:
        raise ValueError("act: truncated header")
    tag, seq, tok, nxt, ah, mh = _HDR.unpack_from(b, 0)
    if tag != ACT:
        raise ValueError(f"act: tag {tag} is not an activation frame")
    if (len(b) - HEADER_BYTES) % 4:
        raise ValueError("act: payload is not a whole number of floats")
    hidden = np.frombuffer(b, np.float32, offset=HEADER_BYTES).copy()
    if hash_f32(hidden) != ah:
        raise ValueError("act: payload failed its integrity hash")
    return dict(seq=seq, tokenIdx=tok, nextIndex=nxt, actHash=ah, modelHash=mh, hidden=hidden)


def model_fingerprint(repo: str, revision: str | None, tensors: dict) -> int:
    """shard.js modelFingerprint (:206-213): FNV-1a of "repo|revision|name:dtype:
    shape:start:end|..." over the tensor index in name order.  ``tensors`` maps
    names to dicts with dtype, shape, start, end (absolute byte offsets, as
    ``safetensors.parse_header`` returns them)."""
    parts = [repo, revision or "main"]
    for name in sorted(tensors):
        t = tensors[name]
        parts.append(f"{name}:{t['dtype']}:{'x'.join(str(d) for d in t['shape'])}:{t['start']}:{t['end']}")
    return fnv1a("|".join(parts).encode("utf-8"))


class _Done:
    def __init__(self, handle, keep, after=None):
        self.handle, self.keep, self.after = handle, keep, after

    def wait(self):
        if self.handle is not None:
            self.handle.wait()
            self.handle = None
        if self.after is not None:
            f, self.after = self.after, None
            f()
        return True


class WireTransport:
    """A point-to-point transport whose every hop is a wire.js activation frame.

    ``inner`` moves tensors (``pipeline.TorchP2P``: NCCL between GPUs, gloo on
    CPU).  ``plan`` is the ring's stage list (dicts with ``id`` and ``index``,
    as shard.plan_stages builds it) and ``my_index`` this rank's stage.  On
    send the frame carries the addressee from route_after (RETURN on the last
    stage's hop back to the head); on receipt the frame must pass its integrity
    hash, carry this ring's model hash, be addressed to this stage (``mine``,
    or ``return`` at the head: classify_act) and, when the caller names it,
    carry the expected token index.  A frame that fails raises ValueError from
    ``wait()``."""

    def __init__(self, inner, plan: list, my_index: int, model_hash: int, seq: int = 0):
        self.inner, self.plan, self.my_index = inner, plan, my_index
        self.model_hash, self.seq = model_hash & 0xFFFFFFFF, seq
        self.route = route_after(plan, my_index)

    def _frame_tensor(self, frame: bytes, like):
        import torch
        t = torch.frombuffer(bytearray(frame), dtype=torch.uint8)
        return t.to(like.device) if like.device.type != "cpu" else t

    def send(self, t, dst: int, token_idx: int = 0):
        hidden = t.detach().reshape(-1).to("cpu").numpy()
        frame = self._frame_tensor(pack_act(self.seq, token_idx, self.route["address"], hidden, self.model_hash), t)
        return _Done(self.inner.send(frame, dst), frame)

    def recv(self, t, src: int, token_idx: int | None = None):
        import torch
        frame = torch.empty(HEADER_BYTES + 4 * t.numel(), dtype=torch.uint8, device=t.device)
        handle = self.inner.recv(frame, src)

        def finish():
            a = unpack_act(frame.to("cpu").numpy().tobytes())
            if a["modelHash"] != self.model_hash:
                raise ValueError(f"act: model hash {a['modelHash']:#010x} is not this ring's {self.model_hash:#010x}")
            want = "return" if self.my_index == 0 else "mine"
            got = classify_act(a["nextIndex"], self.my_index)
            if got != want:
                raise ValueError(f"act: frame addressed to {a['nextIndex']} arrived at stage {self.my_index} ({got})")
            if token_idx is not None and a["tokenIdx"] != token_idx:
                raise ValueError(f"act: token index {a['tokenIdx']} where {token_idx} was due")
            if a["seq"] != self.seq:
                raise ValueError(f"act: sequence {a['seq']} is not the running {self.seq}")
            t.view(-1).copy_(torch.from_numpy(a["hidden"]).to(t.device))

        return _Done(handle, frame, finish)


__all__ = ["ACT", "RETURN", "HEADER_BYTES", "fnv1a", "hash_f32", "pack_act", "unpack_act", "model_fingerprint",
           "WireTransport"]
