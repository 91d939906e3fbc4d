"""Planner and scheduling helpers of public/shard.js and public/infer.js.

Pure host logic (integers and ids), the same functions the reference's
pipeline calls around its compute core:

* ``plan_stages`` (shard.js:32-52): largest-remainder apportionment of layers
  by measured capacity; stage 0 is the head; empty non-head stages dropped;
* ``prefill_chunks`` (shard.js:345-361): even prompt chunks, ``window`` in flight;
* ``prompt_lookup_draft`` (:366-385), ``lookahead_frame`` (:391-398),
  ``accept_draft`` (:530-536) and ``draft_rows`` (infer.js:371-380);
* ``ring_members`` (:215-222), ``estimate_lap_ms`` / ``estimate_plan_ms``
  (:224-256), ``head_can_hold`` / ``prefer_local`` (:258-272): who joins the
  ring, the lap-time budget check, and whether the head runs alone.
"""
from __future__ import annotations

import math


def plan_stages(layers: int, caps: list) -> list:
    n = len(caps)
    if n < 1:
        raise ValueError("no devices to plan across")
    total = sum(max(1e-6, c["capacity"]) for c in caps)
    exact = [layers * max(1e-6, c["capacity"]) / total for c in caps]
    floor = [math.floor(e) for e in exact]
    left = layers - sum(floor)
    order = sorted(((e - floor[i], i) for i, e in enumerate(exact)), key=lambda t: (-t[0], t[1]))
    for i in range(len(order)):
        if left <= 0:
            break
        floor[order[i][1]] += 1
        left -= 1
    stages, lo = [], 0
    for i, c in enumerate(caps):
        hi = lo + floor[i]
        stages.append(dict(id=c["id"], index=i, lo=lo, hi=hi, head=i == 0, backend=c.get("backend"),
                           capacity=c["capacity"]))
        lo = hi
    kept = [s for s in stages if s["head"] or s["hi"] > s["lo"]]
    return [dict(s, index=i) for i, s in enumerate(kept)]


def prefill_chunks(n_tokens: int, chunk_size: int, in_flight: int) -> dict:
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


def chunk_passes(chunks: list, per_pass: int) -> list:
    """Consecutive prefillChunks chunks, ``per_pass`` at a time, as the passes
    a stage runs them in (one pass over its weights each, the same ids as one
    chunk per pass): [(lo, hi, [chunk lengths])].  Every rank derives the same
    list from the same chunks."""
    n = max(1, int(per_pass))
    out = []
    for i in range(0, len(chunks), n):
        g = chunks[i:i + n]
        out.append((g[0]["lo"], g[-1]["hi"], [c["hi"] - c["lo"] for c in g]))
    return out


def prompt_lookup_draft(ids: list, max_draft: int) -> list:
    cap = max(0, int(max_draft))
    n = len(ids)
    if cap == 0 or n < 3:
        return []
    best, best_len = [], 0
    for ln in range(2, min(n - 1, 8) + 1):
        suffix = ids[n - ln:]
        for i in range(0, n - ln):
            if ids[i:i + ln] != suffix:
                continue
            draft = ids[i + ln:min(i + ln + cap, n - ln)]
            if draft and ln > best_len:
                best, best_len = list(draft), ln
    return best


def lookahead_frame(ids: list, T: int, max_draft: int) -> dict:
    draft = prompt_lookup_draft(ids, max_draft)
    shown = (list(ids) + draft)[-T:] if T > 0 else []
    shown_draft = min(len(draft), max(0, len(shown) - 1))
    draft = draft[len(draft) - shown_draft:]
    return dict(draft=draft, shown=len(shown), win=shown)


def accept_draft(picked: list, draft: list) -> list:
    out, i = [], 0
    while i < len(draft) and i < len(picked) and picked[i] == draft[i]:
        out.append(draft[i])
        i += 1
    if i < len(picked):
        out.append(picked[i])
    return out


def draft_rows(T: int, seq_len: int, draft_len: int) -> list:
    rows = []
    first = seq_len - draft_len - 1
    for i in range(draft_len + 1):
        tok = first + i
        if tok < 0 or tok >= seq_len:
            break
        rows.append(T - seq_len + tok)
    return rows


def ring_members(caps: list, probe_hash=None) -> list:
    """shard.js ringMembers: peers whose kernel probe disagrees with the head's
    are left out; the head (first) is always kept; a peer without a probe yet
    is not a disagreement."""
    if not caps:
        return []
    head, rest = caps[0], caps[1:]
    return [head] + [d for d in rest if not probe_hash or not d.get("probe") or d["probe"] == probe_hash]


UNIT_MACS = 32 * 64 * 64  # the capacity probe's verified GEMM (app.js:508-519)


def estimate_lap_ms(spec, T: int, gemm_per_sec: float) -> float:
    """shard.js estimateLapMs: the MACs of one T-row window through every
    layer, in capacity-probe units, at ``gemm_per_sec`` units per second."""
    C = spec.hidden
    inter = spec.inter or C * 4
    hd = spec.headDim or C // spec.heads
    q = spec.heads * hd
    kv = (spec.kvHeads or spec.heads) * hd
    mac_per_layer = (T * C * q + 2 * T * C * kv + T * q * C + 3 * T * C * inter
                     + spec.heads * (T * hd * T + T * T * hd))
    gemms = mac_per_layer * spec.layers / UNIT_MACS
    return gemms / max(gemm_per_sec, 1e-6) * 1000.0


def estimate_plan_ms(spec, T: int, stages: list) -> float:
    """shard.js estimatePlanMs: each stage pays for the layers it holds at its
    own capacity; a head without layers pays 5 % for embedding and readout."""
    layers = max(spec.layers, 1)
    ms = 0.0
    for s in stages:
        owned = max(0, int(s.get("hi", 0)) - int(s.get("lo", 0)))
        share = owned / layers if owned > 0 else (0.05 if s.get("head") else 0.0)
        ms += estimate_lap_ms(spec, T, s.get("capacity") or 0) * share
    return ms


def head_can_hold(tensors, device_gb: float) -> bool:
    """shard.js headCanHold: the whole model as f32 under a quarter of the
    device's memory; unknown memory says no (the ring is used)."""
    if not device_gb or device_gb <= 0:
        return False
    return sum(t["elems"] * 4 for t in tensors) < device_gb * 0.25 * 1073741824


def prefer_local(prompt_tokens: int, peer_count: int, fits: bool) -> bool:
    """shard.js preferLocal: run on the head alone when it can hold the model."""
    return bool(fits and peer_count > 0 and prompt_tokens > 0)
