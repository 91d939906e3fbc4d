"""The reference's pipeline-equivalence checks, on the oracle (CPU only).

Restates test_pipeline.js for the Llama family: bit-exact split invariance
(:130-146), the mutation checks that prove the comparison is not blind
(:150-160), chunked-prefill and lookahead split invariance (:264-280), the
planner (:182-202) and the scheduling helpers' known answers (:248-262).
"""
import numpy as np
import pytest

T, PROMPT = 16, [5, 11, 42, 7]


@pytest.fixture(scope="module")
def model(O):
    spec = O.LLAMA_TEST
    return O.Model(spec, O.make_weights(spec))


def splits_to_ranges(splits):
    out, lo = [], 0
    for n in splits:
        out.append((lo, lo + n))
        lo += n
    return out


def test_stage_boundary_changes_no_bit(O, model):
    win = np.zeros(T, np.int32)
    win[T - len(PROMPT):] = PROMPT
    a = model.run_layers(model.embed_rows(win), 0, 6)
    b = model.embed_rows(win)
    for lo, hi in splits_to_ranges([2, 2, 2]):
        b = model.run_layers(b, lo, hi)
    assert a.tobytes() == b.tobytes()


@pytest.mark.parametrize("splits", [[3, 3], [1, 2, 3], [0, 3, 3], [2, 1, 1, 1, 1], [1, 1, 1, 1, 1, 1]])
def test_generation_identical_across_splits(O, model, splits):
    ref = O.generate_local(model, [(0, 6)], PROMPT, 8, T)
    assert O.generate_local(model, splits_to_ranges(splits), PROMPT, 8, T) == ref


def test_mutations_are_caught(O, model):
    ref = O.generate_local(model, [(0, 6)], PROMPT, 8, T)
    dropped = [(0, 2), (2, 3), (4, 6)]  # the middle stage loses its second layer
    assert O.generate_local(model, dropped, PROMPT, 8, T) != ref
    reordered = [(0, 2), (4, 6), (2, 4)]
    assert O.generate_local(model, reordered, PROMPT, 8, T) != ref


def test_chunked_prefill_matches_across_split(O, model):
    prompt = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5, 8]
    whole = O.generate_chunked(model, [(0, 6)], prompt, 3, 4)
    split = O.generate_chunked(model, splits_to_ranges([2, 2, 2]), prompt, 3, 4)
    assert split == whole and len(whole) == len(prompt) + 3


def test_lookahead_split_invariant(O, model):
    prompt = [4, 4, 4, 7, 4, 4, 4]
    whole = O.generate_lookahead(model, [(0, 6)], prompt, 4, 16, 4)
    split = O.generate_lookahead(model, splits_to_ranges([1, 2, 3]), prompt, 4, 16, 4)
    assert split == whole and len(whole) == len(prompt) + 4


def test_lookahead_without_draft_is_local(O, model):
    # An empty draft is exactly one new token, the same window as generateLocal (infer.js:462-463).
    a = O.generate_lookahead(model, [(0, 6)], PROMPT, 5, T, 0)
    assert a == O.generate_local(model, [(0, 6)], PROMPT, 5, T)


def test_kv_cache_holds_rotated_keys(O, model):
    ids = [1, 2, 3, 4]
    kv = O.KV(model, 0, 6, 8)
    model.run_layers(model.embed_rows(ids), 0, 6, kv, 0)
    k, v = kv.read(0)
    assert k.size == 4 * 2 * 16 and v.size == k.size


def test_planning_is_deterministic_and_capacity_weighted(O):
    caps = [dict(id="p1", capacity=100), dict(id="p2", capacity=300), dict(id="p3", capacity=200)]
    a, b = O.plan_stages(6, caps), O.plan_stages(6, caps)
    assert a == b
    assert sum(s["hi"] - s["lo"] for s in a) == 6
    assert a[1]["hi"] - a[1]["lo"] > a[0]["hi"] - a[0]["lo"]
    assert a[0]["head"]
    # equal capacities over 30 layers and 8 devices: largest remainder
    eq = O.plan_stages(30, [dict(id=str(i), capacity=1.0) for i in range(8)])
    assert [s["hi"] - s["lo"] for s in eq] == [4, 4, 4, 4, 4, 4, 3, 3]


def test_empty_non_head_stage_is_dropped(O):
    plan = O.plan_stages(2, [dict(id="h", capacity=1), dict(id="a", capacity=1e-9), dict(id="b", capacity=1)])
    assert [s["id"] for s in plan] == ["h", "b"] and [s["index"] for s in plan] == [0, 1]


def test_prefill_chunks_drafts_and_accept(O):
    c = O.prefill_chunks(40, 16, 2)
    assert [x["hi"] - x["lo"] for x in c["chunks"]] == [14, 13, 13]
    assert c["chunks"][2]["hi"] == 40 and c["chunks"][0]["lo"] == 0 and c["window"] == 2
    assert [x["hi"] - x["lo"] for x in O.prefill_chunks(512, 16, 2)["chunks"]] == [16] * 32
    assert len(O.prefill_chunks(2048, 16, 2)["chunks"]) == 128
    frame = O.lookahead_frame([1, 2, 3, 9, 1, 2, 3], 16, 4)
    assert frame["draft"] == [9] and len(frame["win"]) == 8
    assert O.prompt_lookup_draft([1, 2, 3, 9, 1, 2, 3], 4) == [9]
    assert O.accept_draft([9, 4], [9]) == [9, 4]
    assert O.accept_draft([8, 4], [9]) == [8]
    assert O.draft_rows(16, 8, 1) == [14, 15]


def test_non_finite_activation_refused(O, model):
    bad = np.zeros(2 * 64, np.float32)
    bad[5] = np.nan
    with pytest.raises(O.NonFiniteError):
        model.run_layers(bad, 0, 0)
