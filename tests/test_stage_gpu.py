"""The forward pass on the B200 against the CPU oracle, bit for bit.

The reference's pipeline checks (test_pipeline.js) run on the device: the
6-layer Llama fixture (hidden 64, 4/2 heads, inter 128, vocab 128, T = 16,
prompt [5, 11, 42, 7]) must give the oracle's hidden-state bits and token ids,
at every stage split, through the full-window, chunked-prefill and lookahead
paths; plus synthetic random-init models at head_dim 64 and 128.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

T, PROMPT = 16, [5, 11, 42, 7]


def ranges(splits):
    out, lo = [], 0
    for n in splits:
        out.append((lo, lo + n))
        lo += n
    return out


def make_stages(P, comp, spec, w, splits, max_rows=64, max_pos=64, synth=None):
    I = P.infer
    stages = []
    for i, (lo, hi) in enumerate(ranges(splits)):
        S = I.Stage(comp, spec, lo, hi, head=(i == 0), max_rows=max_rows, max_pos=max_pos)
        if synth is not None:
            S.synth(*synth)
        else:
            S.load(w)
        stages.append(S)
    return stages


@pytest.fixture(scope="module")
def fixture(O, P):
    ospec = O.LLAMA_TEST
    w = O.make_weights(ospec)
    spec = P.infer.Spec(hidden=ospec.hidden, layers=ospec.layers, heads=ospec.heads, kvHeads=ospec.kvHeads,
                        inter=ospec.inter, vocab=ospec.vocab, tie=True, maxPos=64)
    return ospec, spec, w, O.Model(ospec, w)


def win_of(ids, t=T):
    return [0] * (t - len(ids)) + list(ids)


def test_window_hidden_state_bits(comp, O, P, fixture):
    ospec, spec, w, om = fixture
    stages = make_stages(P, comp, spec, w, [6])
    x = stages[0].embed_rows(win_of(PROMPT))
    x = stages[0].run_layers(x)
    comp.sync()
    want = om.run_layers(om.embed_rows(np.array(win_of(PROMPT), np.int32)), 0, 6)
    assert x.cpu().numpy().tobytes() == want.tobytes()


def test_stage_boundary_changes_no_bit(comp, O, P, fixture):
    ospec, spec, w, om = fixture
    whole = make_stages(P, comp, spec, w, [6])
    split = make_stages(P, comp, spec, w, [2, 2, 2])
    a = P.infer.run_ring(whole, whole[0].embed_rows(win_of(PROMPT)))
    b = P.infer.run_ring(split, split[0].embed_rows(win_of(PROMPT)))
    comp.sync()
    assert a.cpu().numpy().tobytes() == b.cpu().numpy().tobytes()


def test_logits_bits_match_oracle(comp, O, P, fixture):
    ospec, spec, w, om = fixture
    stages = make_stages(P, comp, spec, w, [6])
    x = P.infer.run_ring(stages, stages[0].embed_rows(win_of(PROMPT)))
    picks, logits = stages[0].logits_at(x, [T - 1, 3, 0])
    xo = om.run_layers(om.embed_rows(np.array(win_of(PROMPT), np.int32)), 0, 6)
    want = om.logits_rows(xo, [T - 1, 3, 0])
    assert logits.cpu().numpy().tobytes() == want.tobytes()
    assert picks == [O.argmax(want[i]) for i in range(3)]


@pytest.mark.parametrize("splits", [[6], [3, 3], [1, 2, 3], [0, 3, 3], [2, 1, 1, 1, 1]])
def test_generation_matches_oracle_at_every_split(comp, O, P, fixture, splits):
    ospec, spec, w, om = fixture
    ref = O.generate_local(om, [(0, 6)], PROMPT, 8, T)
    got = P.infer.generate_local(make_stages(P, comp, spec, w, splits), PROMPT, 8, T)
    assert got == ref


def test_stages_load_their_slice_of_a_safetensors_file(comp, O, P, fixture, tmp_path):
    """The fixture model written as a safetensors file; every stage reads only
    its own tensors from it and the generation equals the oracle's."""
    ospec, spec, w, om = fixture
    path = str(tmp_path / "fixture.safetensors")
    P.safetensors.save_weights(path, w, spec)
    ref = O.generate_local(om, [(0, 6)], PROMPT, 8, T)
    for splits in ([6], [2, 4]):
        stages = []
        for i, (lo, hi) in enumerate(ranges(splits)):
            S = P.infer.Stage(comp, spec, lo, hi, head=(i == 0), max_rows=64, max_pos=64)
            S.load_safetensors(path)
            stages.append(S)
        assert P.infer.generate_local(stages, PROMPT, 8, T) == ref


def test_stage_handoff_carries_the_lap(comp, O, P, fixture):
    """dc_stage_handoff (the stage-to-stage hop) between two stages: layers
    0-2 on one stage, the hop into the next stage's buffer, layers 3-5 there;
    the hidden state equals the one-stage run and the oracle bit for bit."""
    import torch
    ospec, spec, w, om = fixture
    a, b = make_stages(P, comp, spec, w, [3, 3])
    x = a.run_layers(a.embed_rows(win_of(PROMPT)))
    y = torch.full_like(x, float("nan"))
    a.handoff(b, x, y)
    b.run_layers(y)
    comp.sync()
    want = om.run_layers(om.embed_rows(np.array(win_of(PROMPT), np.int32)), 0, 6)
    assert y.cpu().numpy().tobytes() == want.tobytes()


def test_mutations_are_caught_on_device(comp, O, P, fixture):
    ospec, spec, w, om = fixture
    ref = O.generate_local(om, [(0, 6)], PROMPT, 8, T)
    st = make_stages(P, comp, spec, w, [2, 2, 2])
    assert P.infer.generate_local([st[0], st[2], st[1]], PROMPT, 8, T) != ref
    dropped = make_stages(P, comp, spec, w, [2, 1])  # layers 3..5 never run
    assert P.infer.generate_local(dropped, PROMPT, 8, T) != ref


def test_chunked_prefill_matches_oracle(comp, O, P, fixture):
    ospec, spec, w, om = fixture
    prompt = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5, 8]
    ref = O.generate_chunked(om, [(0, 6)], prompt, 3, 4)
    for splits in ([6], [2, 2, 2]):
        got = P.infer.generate_chunked(make_stages(P, comp, spec, w, splits), prompt, 3, 4)
        assert got == ref


def test_decode_loop_modes_agree(comp, O, P, fixture):
    """The device decode loop, replayed as one CUDA graph per lap, equals the
    un-captured device loop and the host-driven loop (and the oracle)."""
    ospec, spec, w, om = fixture
    prompt = [9, 8, 7, 6, 5, 4, 3, 2, 1, 0, 11, 12, 13]
    ref = O.generate_chunked(om, [(0, 6)], prompt, 12, 5)
    for kw in (dict(use_device_loop=False), dict(use_graph=False), dict(use_graph=True)):
        for splits in ([6], [0, 3, 3]):
            got = P.infer.generate_chunked(make_stages(P, comp, spec, w, splits), prompt, 12, 5, **kw)
            assert got == ref, (kw, splits)
    # the host-driven loop with each stage's one-row forward kernel by kernel (no row graph)
    st = make_stages(P, comp, spec, w, [2, 4])
    for S in st:
        S.set_row_graph(False)
    assert P.infer.generate_chunked(st, prompt, 12, 5, use_device_loop=False) == ref


def test_decode_timeline_stamps_every_lap(comp, O, P, fixture):
    """dc_stage_set_timeline: the stamped decode (graph replays) still equals
    the oracle; every lap within the buffer has all its stamps, in time order;
    laps past the buffer write nothing; one stamp per lap closes each GEMV (six
    layers x four projections, and the lm_head), tagged with its bytes."""
    import torch
    ospec, spec, w, om = fixture
    prompt = [9, 8, 7, 6, 5, 4, 3, 2, 1, 0, 11, 12, 13]
    ref = O.generate_chunked(om, [(0, 6)], prompt, 12, 5)
    laps, per = 8, 256
    for splits in ([6], [0, 3, 3]):
        st = make_stages(P, comp, spec, w, splits)
        buf = torch.zeros(laps * per + 64, dtype=torch.int64, device="cuda")
        st[0].set_timeline(buf[:laps * per], per, laps)
        got = P.infer.generate_chunked(st, prompt, 12, 5)
        comp.sync()
        kinds, by = st[0].timeline_info()
        st[0].set_timeline()
        assert got == ref, splits
        n = len(kinds)
        assert 25 < n <= per
        assert kinds.count(1) == 6 * 4 + 1
        assert all(b > 0 for k, b in zip(kinds, by) if k == 1)
        t = buf.cpu().numpy()
        lapt = t[:laps * per].reshape(laps, per)
        assert (lapt[:, :n] > 0).all()
        assert (np.diff(lapt[:, :n].astype(np.int64), axis=1) >= 0).all()
        assert (lapt[:, n:] == 0).all() and (t[laps * per:] == 0).all()
        # and off again: the next generation runs (and replays) without stamps
        buf.zero_()
        assert P.infer.generate_chunked(st, prompt, 12, 5) == ref
        comp.sync()
        assert int(buf.abs().sum()) == 0


def test_kv_cache_contents_match_oracle(comp, O, P, fixture):
    ospec, spec, w, om = fixture
    ids = [1, 2, 3, 4, 5]
    st = make_stages(P, comp, spec, w, [6])
    x = st[0].run_layers_chunk(st[0].embed_rows(ids[:3]), 0)
    x = st[0].run_layers_chunk(st[0].embed_rows(ids[3:]), 3)
    comp.sync()
    kv = O.KV(om, 0, 6, 8)
    om.run_layers(om.embed_rows(ids[:3]), 0, 6, kv, 0)
    om.run_layers(om.embed_rows(ids[3:]), 0, 6, kv, 3)
    hd, nkv = ospec.headDim, ospec.kvHeads
    for layer in (0, 5):
        k8, ks, v = st[0].kv_read(layer)
        kf, vf = kv.read(layer)
        assert v.tobytes() == vf.tobytes()
        n = len(ids)
        kf = kf.reshape(n, nkv, hd)
        for g in range(nkv):
            q, s = O.quantize_cols(kf[:, g, :].T.copy(), hd, n)   # khᵀ: columns are key tokens
            assert ks.reshape(nkv, n)[g].tobytes() == s.tobytes()
            assert k8.reshape(nkv, n, hd)[g].tobytes() == q.reshape(hd, n).T.copy().tobytes()


def test_lookahead_matches_oracle(comp, O, P, fixture):
    ospec, spec, w, om = fixture
    prompt = [4, 4, 4, 7, 4, 4, 4]
    ref = O.generate_lookahead(om, [(0, 6)], prompt, 4, 16, 4)
    for splits in ([6], [1, 2, 3]):
        got = P.infer.generate_lookahead(make_stages(P, comp, spec, w, splits), prompt, 4, 16, 4)
        assert got == ref


def test_non_finite_activation_refused(comp, P, fixture):
    ospec, spec, w, om = fixture
    st = make_stages(P, comp, spec, w, [6])
    x = st[0].embed_rows(win_of(PROMPT))
    x[5] = float("nan")
    st[0].run_layers(x)
    with pytest.raises(P.NonFiniteError):
        comp.sync()


def synth_model(O, P, hidden, layers, heads, kv, inter, vocab, tie, theta=10000.0, seed=77):
    ospec = O.Spec(hidden=hidden, layers=layers, heads=heads, kvHeads=kv, inter=inter, vocab=vocab, tie=tie,
                   ropeTheta=theta)
    C_, q, kvd = hidden, heads * ospec.headDim, kv * ospec.headDim
    w = {"emb": O.synth_weight(seed, -1, "emb", vocab, C_), "nrmF": np.ones(C_, np.float32),
         "lm": None if tie else O.synth_weight(seed, -1, "lm", C_, vocab), "layers": []}
    for l in range(layers):
        w["layers"].append(dict(nrm1=np.ones(C_, np.float32), nrm2=np.ones(C_, np.float32),
                                Wq=O.synth_weight(seed, l, "Wq", C_, q), Wk=O.synth_weight(seed, l, "Wk", C_, kvd),
                                Wv=O.synth_weight(seed, l, "Wv", C_, kvd), Wo=O.synth_weight(seed, l, "Wo", q, C_),
                                Wgate=O.synth_weight(seed, l, "Wgate", C_, inter),
                                Wup=O.synth_weight(seed, l, "Wup", C_, inter),
                                Wdown=O.synth_weight(seed, l, "Wdown", inter, C_)))
    spec = P.infer.Spec(hidden=hidden, layers=layers, heads=heads, kvHeads=kv, inter=inter, vocab=vocab, tie=tie,
                        ropeTheta=theta)
    return ospec, spec, w


@pytest.mark.parametrize("cfg", [dict(hidden=256, layers=2, heads=4, kv=2, inter=512, vocab=1000, tie=True),
                                 dict(hidden=512, layers=2, heads=4, kv=1, inter=1024, vocab=777, tie=False,
                                      theta=500000.0),
                                 dict(hidden=4096, layers=1, heads=32, kv=8, inter=1024, vocab=512, tie=False,
                                      theta=500000.0)],
                         ids=["hd64-tied", "hd128-untied", "hidden4096"])
def test_synthetic_model_device_generator_matches_oracle(comp, O, P, cfg):
    ospec, spec, w = synth_model(O, P, **cfg)
    om = O.Model(ospec, w)
    seed = 77
    ids = list(np.random.default_rng(3).integers(0, cfg["vocab"], 40))
    for synth in (True, False):
        st = make_stages(P, comp, spec, w, [cfg["layers"]], max_rows=64, max_pos=96,
                         synth=(seed, O.SYNTH_FACTOR) if synth else None)
        x = P.infer.run_ring(st, st[0].embed_rows(ids))
        comp.sync()
        want = om.run_layers(om.embed_rows(np.array(ids, np.int32)), 0, cfg["layers"])
        assert x.cpu().numpy().tobytes() == want.tobytes(), f"synth={synth}"
        picks, logits = st[0].logits_at(x, [len(ids) - 1])
        assert logits.cpu().numpy().tobytes() == om.logits_rows(want, [len(ids) - 1]).tobytes()
    want = O.generate_chunked(om, [(0, cfg["layers"])], ids, 6, 16)
    for fused in (True, False):  # decode rows with the norm/SwiGLU/row quantisation fused into the GEMVs, or not
        for S in st:
            S.set_row_fusion(fused)
        got = P.infer.generate_chunked(st, ids, 6, 16)
        assert got == want, f"fused={fused}"
        got = P.infer.generate_chunked(st, ids, 6, 16, use_device_loop=False)  # one-row graphs per stage
        assert got == want, f"fused={fused}, host loop"


@pytest.mark.parametrize("cfg", [dict(hidden=256, layers=2, heads=4, kv=2, inter=512, vocab=1000, tie=True),
                                 dict(hidden=512, layers=2, heads=4, kv=1, inter=1024, vocab=777, tie=False,
                                      theta=500000.0)],
                         ids=["hd64", "hd128"])
def test_chunk_passes_match_oracle(comp, O, P, cfg):
    """dc_stage_forward_chunks: consecutive chunks in one pass over the weights
    give the oracle's rows (one chunk at a time, infer.js:339-367) bit for bit,
    each chunk's context under the value scales as of its own last row; the
    cache (f32 values, int8 keys and their scales) and the decode ids that
    follow agree too.  Ragged chunks (prefillChunks of 45 in 16s: 15, 15, 15;
    of 45 in 4s: twelve chunks of 3 and 4), passes of 2, 3, 5 and 16 chunks, a
    pass split over two stages, and chunks wider than 16 rows (one by one)."""
    ospec, spec, w = synth_model(O, P, **cfg)
    om = O.Model(ospec, w)
    L = cfg["layers"]
    ids = [int(v) for v in np.random.default_rng(11).integers(0, cfg["vocab"], 45)]
    for chunk, per_pass, splits in ((16, 3, [L]), (4, 5, [L]), (4, 16, [L]), (4, 2, [1, 1]), (23, 2, [L])):
        chunks = P.shard.prefill_chunks(len(ids), chunk, 1)["chunks"]
        kv = [O.KV(om, 0, L, 96)]
        want_rows = []
        for ch in chunks:
            x = om.run_layers(om.embed_rows(ids[ch["lo"]:ch["hi"]]), 0, L, kv[0], ch["lo"])
            want_rows.append(x)
        want = np.concatenate(want_rows)
        ref = O.generate_chunked(om, [(0, L)], ids, 6, chunk)
        for mode in (1, 2):  # the pass's attention by (head, chunk) CTAs, or by (head, row) CTAs
            st = make_stages(P, comp, spec, w, splits, max_rows=64, max_pos=96)
            for S in st:
                S.set_pass_attention(mode)
            got = []
            for lo, hi, rows in P.shard.chunk_passes(chunks, per_pass):
                got.append(P.infer.run_ring(st, st[0].embed_rows(ids[lo:hi]), lo, rows).cpu().numpy())
            comp.sync()
            case = (chunk, per_pass, splits, mode)
            assert np.concatenate(got).tobytes() == want.tobytes(), case
            k8, ks, v = st[-1].kv_read(L - 1)
            _, vf = kv[0].read(L - 1)
            assert v.tobytes() == vf.tobytes(), case
            assert st[-1].kv_len() == len(ids), case
            assert P.infer.generate_chunked(st, ids, 6, chunk, per_pass=per_pass) == ref, case


def test_chunk_pass_argument_checks(comp, P, fixture):
    ospec, spec, w, om = fixture
    st = make_stages(P, comp, spec, w, [6], max_rows=16)
    x = st[0].embed_rows(list(range(12)))
    with pytest.raises(P.DeviceError):
        st[0].run_layers_chunks(x, 0, [5, 5])      # rows do not sum to T
    with pytest.raises(P.DeviceError):
        st[0].run_layers_chunks(x, 3, [6, 6])      # not at the cached length
    with pytest.raises(P.DeviceError):
        st[0].run_layers_chunks(x, 0, [6, 0, 6])   # an empty chunk
    assert st[0].kv_len() == 0
    # head_dim 16 (the reference's fixture): the chunks run one by one, same rows
    st[0].run_layers_chunks(x, 0, [4, 4, 4])
    assert st[0].kv_len() == 12
