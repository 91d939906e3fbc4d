"""Greedy generation of the benchmark models at full size, bit for bit against the oracle.

The golden files under tests/golden/configs/ come from the CPU oracle
(tests/golden/make_configs.py) on the synthetic random-init models of the
four model configurations, at their real shapes:

* SmolLM-135M shape, full window T = 64, 24-token prompt, 16 tokens
  (generateLookahead with maxDraft 4 and generateLocal), 3 stages;
* TinyLlama-1.1B shape, 512-token prompt in chunks of 16, 128 decode tokens,
  2 stages;
* SmolLM-360M shape, T = 512, 256-token 8-gram prompt, 128 new tokens through
  generateLookahead, 4 stages;
* Llama-3-8B shape, 2048-token prompt in chunks of 16, 256 decode tokens
  (the decode attention then spans nine 256-key blocks per head at head_dim
  128, on 4-CTA clusters), 8 stages.

Each runs on cuda:0 as one stage and as the configuration's stage split
(split invariance, test_pipeline.js:141-146, 264-280), and must give the
oracle's ids, and the sha256 of the bits of: the first lap's hidden state and
logits; for the chunked path the last layer's cache after the last lap (f32
values, int8 keys, key scales: the whole decode trajectory); for the lookahead
path the last lap's hidden state and logits.  Reference generators:
public/infer.js:339-367 (generateChunked), :448-494 (generateLocal,
generateLookahead).
"""
import glob
import hashlib
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "configs")
FILES = sorted(glob.glob(os.path.join(GOLDEN, "*.json")))


def sha(t) -> str:
    a = t.cpu().numpy() if hasattr(t, "cpu") else np.asarray(t)
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def first_diff(a, b):
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return min(len(a), len(b)) if len(a) != len(b) else None


def load(path):
    with open(path) as f:
        return json.load(f)


def build(P, comp, g, splits, per_pass=1):
    s = g["spec"]
    spec = P.infer.Spec(hidden=s["hidden"], layers=s["layers"], heads=s["heads"], kvHeads=s["kvHeads"],
                        inter=s["inter"], vocab=s["vocab"], ropeTheta=s["ropeTheta"], tie=s["tie"])
    if g["mode"] == "chunked":
        max_rows, max_pos = max(g["chunk"] * per_pass, 8), len(g["prompt"]) + g["new"] + 1
    else:
        max_rows, max_pos = g["T"], g["T"]
    stages = []
    for i, (lo, hi) in enumerate(splits):
        S = P.infer.Stage(comp, spec, lo, hi, head=(i == 0), max_rows=max_rows, max_pos=max_pos)
        S.synth(g["model_seed"], g["synth_factor"])
        stages.append(S)
    return spec, stages


def close(stages):
    for S in stages:
        S.close()


def check_chunked(P, comp, g, splits, per_pass=1):
    spec, stages = build(P, comp, g, splits, per_pass)
    try:
        prompt = g["prompt"]
        got = P.infer.generate_chunked(stages, prompt, g["new"], g["chunk"], per_pass=per_pass)[len(prompt):]
        assert got == g["generated"], f"ids differ from index {first_diff(got, g['generated'])}"
        kv = g["kv_last_layer"]
        k8, ks, v = stages[-1].kv_read(spec.layers - 1)
        assert stages[-1].kv_len() == kv["len"]
        assert sha(v) == kv["v_sha256"], "last layer's cached values differ"
        assert sha(k8) == kv["k8_sha256"], "last layer's int8 keys differ"
        assert sha(ks) == kv["ks_sha256"], "last layer's key scales differ"
        # the prefill alone: its last hidden row and the logits of the first pick
        for S in stages:
            S.kv_reset()
        last = None
        chunks = P.shard.prefill_chunks(len(prompt), g["chunk"], 1)["chunks"]
        for lo, hi, rows in P.shard.chunk_passes(chunks, per_pass):
            last = P.infer.run_ring(stages, stages[0].embed_rows(prompt[lo:hi]), lo, rows)
        rows = last.numel() // spec.hidden
        picks, logits = stages[0].logits_at(last, [rows - 1])
        assert sha(last[(rows - 1) * spec.hidden:]) == g["prefill_last_row_sha256"], "prefill hidden row differs"
        assert sha(logits) == g["first_logits_sha256"], "first logits differ"
        assert picks[0] == g["generated"][0]
    finally:
        close(stages)


def check_lookahead(P, comp, g, splits):
    spec, stages = build(P, comp, g, splits)
    try:
        prompt, T, md = g["prompt"], g["T"], g["max_draft"]
        got = P.infer.generate_lookahead(stages, prompt, g["new"], T, md)[len(prompt):]
        assert got == g["generated"], f"ids differ from index {first_diff(got, g['generated'])}"
        frame = P.shard.lookahead_frame(prompt, T, md)
        win = [0] * (T - len(frame["win"])) + frame["win"]
        x = P.infer.run_ring(stages, stages[0].embed_rows(win))
        _, logits = stages[0].logits_at(x, g["first_rows"])
        assert sha(x) == g["first_hidden_sha256"], "first lap's hidden state differs"
        assert sha(logits) == g["first_logits_sha256"], "first lap's logits differ"
        x = P.infer.run_ring(stages, stages[0].embed_rows(g["last_win"]))
        _, logits = stages[0].logits_at(x, g["last_rows"])
        assert sha(x) == g["last_hidden_sha256"], "last lap's hidden state differs"
        assert sha(logits) == g["last_logits_sha256"], "last lap's logits differ"
        if "generated_local" in g:
            loc = P.infer.generate_local(stages, prompt, g["new"], T)[len(prompt):]
            assert loc == g["generated_local"], f"generateLocal ids differ from {first_diff(loc, g['generated_local'])}"
    finally:
        close(stages)


def test_golden_files_present():
    names = {os.path.basename(p)[:-5] for p in FILES}
    assert names == {"smollm-135m-window", "tinyllama-chunked", "smollm-360m-lookahead", "llama3-8b-chunked"}


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(p)[:-5] for p in FILES])
@pytest.mark.parametrize("split", ["one-stage", "config-stages"])
def test_config_generation_matches_oracle(comp, P, path, split):
    g = load(path)
    splits = [(0, g["spec"]["layers"])] if split == "one-stage" else [tuple(s) for s in g["stages"]]
    if g["mode"] == "chunked":
        check_chunked(P, comp, g, splits)
    else:
        check_lookahead(P, comp, g, splits)


CHUNKED = [p for p in FILES if load(p)["mode"] == "chunked"]


@pytest.mark.parametrize("path", CHUNKED, ids=[os.path.basename(p)[:-5] for p in CHUNKED])
@pytest.mark.parametrize("per_pass,split", [(8, "one-stage"), (16, "config-stages")])
def test_chunk_passes_generation_matches_oracle(comp, P, path, per_pass, split):
    """The chunked configurations with several 16-token chunks per pass over
    the weights (dc_stage_forward_chunks) give the oracle's ids, prefill row,
    first logits and last-layer cache, which it computes one chunk at a time."""
    g = load(path)
    splits = [(0, g["spec"]["layers"])] if split == "one-stage" else [tuple(s) for s in g["stages"]]
    check_chunked(P, comp, g, splits, per_pass)


def test_bench_ring_matches_oracle(comp, P):
    """The benchmark's own call (pipeline.Ring, one GPU, two chunks in flight,
    decode laps as CUDA graphs) on the Llama-3-8B model gives the oracle's ids."""
    g = load(os.path.join(GOLDEN, "llama3-8b-chunked.json"))
    spec, stages = build(P, comp, g, [(0, g["spec"]["layers"])], per_pass=32)
    try:
        ring = P.pipeline.Ring(stages[0], 0, 1, spec.hidden)
        for per_pass in (1, 32, 32):  # the last run reuses the captured graphs
            picks = ring.generate_chunked(g["prompt"], g["new"], g["chunk"], 2, per_pass=per_pass)
            assert picks[:g["new"]].cpu().tolist() == g["generated"], per_pass
    finally:
        close(stages)
