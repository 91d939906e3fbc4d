"""Ring membership and the lap-time budget of public/shard.js (:215-272),
restated in shard.py: hand-computed values and the reference's rules."""
import pytest


@pytest.fixture(scope="module")
def S(P):
    return P.shard


@pytest.fixture(scope="module")
def spec(P):
    return P.infer.Spec(hidden=64, layers=6, heads=4, kvHeads=2, inter=128, vocab=128)


def test_probe_disagreement_leaves_a_peer_out(S):
    caps = [dict(id="head", probe=7), dict(id="a", probe=7), dict(id="b", probe=9), dict(id="c")]
    assert [c["id"] for c in S.ring_members(caps, 7)] == ["head", "a", "c"]  # no probe yet is kept
    assert [c["id"] for c in S.ring_members(caps, None)] == ["head", "a", "b", "c"]
    assert S.ring_members([dict(id="head", probe=1)], 7)[0]["id"] == "head"  # the head always stays
    assert S.ring_members([], 7) == []


def test_lap_estimate_counts_the_window_macs(S, spec):
    # per layer at T = 16: Q, K, V, O, gate/up/down and the two attention products
    C, q, kv, I, hd, T = 64, 64, 32, 128, 16, 16
    macs = T * C * q + 2 * T * C * kv + T * q * C + 3 * T * C * I + 4 * (T * hd * T + T * T * hd)
    assert macs == 622592
    assert S.estimate_lap_ms(spec, T, 1000.0) == pytest.approx(macs * 6 / (32 * 64 * 64))
    assert S.estimate_lap_ms(spec, T, 0) > 1e9  # no capacity: effectively never


def test_plan_estimate_charges_each_stage_at_its_rate(S, spec):
    full = S.estimate_lap_ms(spec, 16, 1000.0)
    two = [dict(lo=0, hi=2, head=True, capacity=1000.0), dict(lo=2, hi=6, capacity=500.0)]
    assert S.estimate_plan_ms(spec, 16, two) == pytest.approx(full * 2 / 6 + 2 * full * 4 / 6)
    bare_head = [dict(lo=0, hi=0, head=True, capacity=1000.0), dict(lo=0, hi=6, capacity=1000.0)]
    assert S.estimate_plan_ms(spec, 16, bare_head) == pytest.approx(full * 1.05)


def test_head_holds_the_model_under_a_quarter_of_its_memory(S):
    t = [dict(elems=1 << 28)]  # 1 GiB of f32
    assert S.head_can_hold(t, 4.0 + 1e-9) and not S.head_can_hold(t, 4.0)
    assert not S.head_can_hold(t, 0) and not S.head_can_hold(t, None)
    assert S.prefer_local(10, 2, True) and not S.prefer_local(10, 0, True) and not S.prefer_local(0, 2, True)
    assert not S.prefer_local(10, 2, False)


def test_plan_follows_measured_capacity(S):
    plan = S.plan_stages(32, [dict(id="b200", capacity=3.0e6), dict(id="laptop", capacity=1.0e6)])
    assert [(p["lo"], p["hi"]) for p in plan] == [(0, 24), (24, 32)]


def test_synthetic_weight_scale_matches_the_oracle(P, O):
    """The benchmark models' weight scale is the package's own constant; the
    oracle's restatement of the generator uses the same one."""
    assert P.infer.SYNTH_FACTOR == O.SYNTH_FACTOR and P.infer.SYNTH_STD == O.SYNTH_STD
