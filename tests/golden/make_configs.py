#!/usr/bin/env python3
"""Golden fixtures of the four model configurations at full size, from the oracle.

    python tests/golden/make_configs.py [--only NAME[,NAME]] [--out DIR]

For each benchmark model (the synthetic random-init models of bench.py's
WORKLOADS, seeded weights, seeded prompt) this runs the CPU oracle's
restatement of the reference's generator, greedy, at the real shapes:

* smollm-135m-window: SmolLM-135M shape, full window T = 64, 24-token prompt,
  16 tokens through generateLookahead (maxDraft 4, what the app runs) and
  through generateLocal (maxDraft 0), public/infer.js:448-494;
* tinyllama-chunked: TinyLlama-1.1B shape, 512-token prompt prefilled in
  chunks of 16, 128 greedy decode tokens, public/infer.js:339-367;
* smollm-360m-lookahead: SmolLM-360M shape, T = 512, 256-token repeated
  8-gram prompt, 128 new tokens through generateLookahead;
* llama3-8b-chunked: Llama-3-8B shape, 2048-token prompt in chunks of 16,
  256 greedy decode tokens.

and writes tests/golden/configs/<name>.json: the model and schedule, the
prompt ids, the generated ids, and sha256 digests of bits along the way: the
first lap's hidden state and logits; for the chunked path the last layer's
cache after the last lap (f32 values, int8 keys and key scales over every
position, so the whole decode trajectory is pinned even when the greedy ids
repeat); for the lookahead path the last lap's window, hidden state and
logits.  The oracle runs on the exact-product path
(oracle/dc_oracle.c orc_bgemm_t, equal to the LUT path by test), so a
Llama-3-8B run takes minutes on a few cores and ~12 GB of RAM.  The GPU tests
(tests/test_configs_gpu.py) compare the B200 path with these files.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import numpy as np  # noqa: E402

import bench  # noqa: E402
import oracle as O  # noqa: E402

NAMES = ["smollm-135m-window", "tinyllama-chunked", "smollm-360m-lookahead", "llama3-8b-chunked"]
STAGES = {"smollm-135m-window": 3, "tinyllama-chunked": 2, "smollm-360m-lookahead": 4, "llama3-8b-chunked": 8}
MAX_DRAFT = 4


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def hexes(a: np.ndarray, n: int = 8):
    return [float(v).hex() for v in np.asarray(a, np.float32).reshape(-1)[:n]]


def fnv(ids) -> int:
    return bench.P_fnv(ids)


def kv_digests(kv: "O.KV", layer: int, spec: O.Spec) -> dict:
    """The cache of one layer in the device's read-out layout: f32 values
    [len][kvDim], int8 keys [kvHeads][len][headDim] and key scales
    [kvHeads][len] (quantizeCols of each head's kᵀ: one scale per key token)."""
    kf, vf = kv.read(layer)
    hd, nkv = spec.headDim, spec.kvHeads
    n = kf.size // (hd * nkv)
    kf = kf.reshape(n, nkv, hd)
    k8, ks = [], []
    for g in range(nkv):
        q, s = O.quantize_cols(kf[:, g, :].T.copy(), hd, n)
        k8.append(q.reshape(hd, n).T.copy())
        ks.append(s)
    return dict(len=n, v_sha256=sha(vf), k8_sha256=sha(np.stack(k8)), ks_sha256=sha(np.stack(ks)))


def spec_of(w: dict) -> O.Spec:
    s = w["spec"]
    return O.Spec(hidden=s["hidden"], layers=s["layers"], heads=s["heads"], kvHeads=s["kvHeads"], inter=s["inter"],
                  vocab=s["vocab"], ropeTheta=s["ropeTheta"], tie=s["tie"])


def make(name: str) -> dict:
    w = bench.WORKLOADS[name]
    spec = spec_of(w)
    prompt = bench.prompt_ids(w, spec.vocab)
    plan = O.plan_stages(spec.layers, [dict(id=f"gpu{i}", capacity=1.0) for i in range(STAGES[name])])
    t0 = time.time()
    model = O.SynthModel(spec, bench.MODEL_SEED)
    t_build = time.time() - t0
    out = dict(workload=name, spec=w["spec"], model_seed=bench.MODEL_SEED, synth_factor=O.SYNTH_FACTOR,
               mode=w["mode"], stages=[[s["lo"], s["hi"]] for s in plan], prompt=prompt)
    whole = [(0, spec.layers)]
    t0 = time.time()
    if w["mode"] == "chunked":
        tr = {}
        ids = O.generate_chunked(model, whole, prompt, w["new"], w["chunk"], trace=tr)
        gen = ids[len(prompt):]
        out.update(chunk=w["chunk"], new=w["new"], generated=gen, generated_fnv=fnv(gen),
                   prefill_last_row_sha256=sha(tr["prefill_last"]), first_logits_sha256=sha(tr["first_logits"]),
                   first_logits_head=hexes(tr["first_logits"]),
                   kv_last_layer=kv_digests(tr["caches"][0], spec.layers - 1, spec))
    else:
        T = w["T"]
        tr = {}
        ids = O.generate_lookahead(model, whole, prompt, w["new"], T, MAX_DRAFT, trace=tr)
        gen = ids[len(prompt):]
        out.update(T=T, new=w["new"], max_draft=MAX_DRAFT, generated=gen, generated_fnv=fnv(gen), laps=tr["laps"],
                   first_rows=tr["first_rows"], first_hidden_sha256=sha(tr["first_hidden"]),
                   first_logits_sha256=sha(tr["first_logits"]), first_logits_head=hexes(tr["first_logits"]),
                   last_win=tr["last_win"], last_rows=tr["last_rows"], last_hidden_sha256=sha(tr["last_hidden"]),
                   last_logits_sha256=sha(tr["last_logits"]))
        if name == "smollm-135m-window":
            loc = O.generate_local(model, whole, prompt, w["new"], T)
            out["generated_local"] = loc[len(prompt):]
    out["oracle_seconds"] = dict(build=round(t_build, 1), generate=round(time.time() - t0, 1),
                                 threads=O.threads())
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="")
    ap.add_argument("--out", default=os.path.join(HERE, "configs"))
    args = ap.parse_args()
    names = [n for n in args.only.split(",") if n] or NAMES
    os.makedirs(args.out, exist_ok=True)
    for name in names:
        t = time.time()
        d = make(name)
        path = os.path.join(args.out, name + ".json")
        with open(path, "w") as f:
            json.dump(d, f, indent=1)
            f.write("\n")
        print(f"{name}: {len(d['generated'])} ids, fnv {d['generated_fnv']}, {time.time() - t:.0f} s -> {path}",
              flush=True)


if __name__ == "__main__":
    main()
