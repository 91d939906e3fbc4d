"""The oracle's exact-product path equals its LUT path, bit for bit.

The full-size golden fixtures (tests/golden/make_configs.py) run the oracle on
orc_bgemm_t: int8 dot products formed directly over a transposed weight,
instead of bgemmJS's mul-LUT triple loop (verified_core.js:241-266).  The mul
unit is the exact product (tests/test_oracle_units.py pins its sha256), and an
int32 sum of exact products within the k <= 131071 bound does not depend on
order, so the two must agree everywhere; these tests hold them to that on
ragged shapes, every output mode, and a whole synthetic model.
"""
import numpy as np
import pytest


@pytest.mark.parametrize("m,k,n", [(1, 576, 1536), (5, 100, 37), (16, 4096, 260), (17, 33, 9), (3, 0, 5),
                                   (4, 31, 4), (9, 1, 1), (2, 131071, 3)])
def test_fast_gemm_equals_lut_gemm(O, m, k, n):
    rng = np.random.default_rng(m * 7 + k)
    W = rng.standard_normal(k * n).astype(np.float32)
    X = rng.standard_normal(m * k).astype(np.float32)
    q, s = O.quantize_cols(W, k, n)
    qt, st = O.quantize_cols_t(W, k, n)
    assert s.tobytes() == st.tobytes()
    assert q.reshape(k, n).T.tobytes() == qt.tobytes()
    xq, xs = O.quantize_rows(X, m, k)
    for flags in (0, O.RELU, O.ACC, O.REQUANT, O.REQUANT | O.RELU):
        a = O.bgemm(xq, q, xs, s, m, k, n, 1, flags)
        b = O.bgemm_t(xq, qt, xs, s, m, k, n, flags)
        assert a.tobytes() == b.tobytes(), flags


def test_fast_gemm_extreme_values(O):
    """All -128 (the largest products) at the accumulator bound, and mixed signs."""
    k, n, m = 131071, 2, 1
    xq = np.full(k, -128, np.int8)
    q = np.full(k * n, -128, np.int8)
    q[1::2] = 127
    rs = np.ones(m, np.float32)
    cs = np.ones(n, np.float32)
    a = O.bgemm(xq, q, rs, cs, m, k, n, 1, O.ACC)
    b = O.bgemm_t(xq, q.reshape(k, n).T.copy(), rs, cs, m, k, n, O.ACC)
    assert a.tolist() == b.tolist() == [k * 16384, -k * 128 * 127]
    with pytest.raises(O.AccumulatorBoundError):
        O.bgemm_t(np.zeros(131072, np.int8), np.zeros(131072, np.int8), rs, cs, 1, 131072, 1, O.ACC)


def test_quantize_cols_t_refuses_non_finite(O):
    W = np.ones(12, np.float32)
    W[5] = np.inf
    with pytest.raises(O.NonFiniteError):
        O.quantize_cols_t(W, 3, 4)


@pytest.mark.parametrize("tie", [True, False])
def test_synth_model_equals_model_from_synth_weights(O, tie):
    """A model built inside the C oracle (exact-product path, f32 weights
    dropped) generates what the LUT-path model built from the same synthetic
    weights generates: hidden bits, logits bits, chunked and lookahead ids."""
    spec = O.Spec(hidden=128, layers=2, heads=4, kvHeads=2, inter=256, vocab=300, tie=tie, ropeTheta=500000.0)
    seed = 99
    C_, q, kvd, I_ = spec.hidden, spec.heads * spec.headDim, spec.kvHeads * spec.headDim, spec.inter
    w = {"emb": O.synth_weight(seed, -1, "emb", spec.vocab, C_), "nrmF": np.ones(C_, np.float32),
         "lm": None if tie else O.synth_weight(seed, -1, "lm", C_, spec.vocab), "layers": []}
    for l in range(spec.layers):
        w["layers"].append(dict(nrm1=np.ones(C_, np.float32), nrm2=np.ones(C_, np.float32),
                                Wq=O.synth_weight(seed, l, "Wq", C_, q), Wk=O.synth_weight(seed, l, "Wk", C_, kvd),
                                Wv=O.synth_weight(seed, l, "Wv", C_, kvd), Wo=O.synth_weight(seed, l, "Wo", q, C_),
                                Wgate=O.synth_weight(seed, l, "Wgate", C_, I_),
                                Wup=O.synth_weight(seed, l, "Wup", C_, I_),
                                Wdown=O.synth_weight(seed, l, "Wdown", I_, C_)))
    ref = O.Model(spec, w)
    fast = O.SynthModel(spec, seed)
    ids = list(np.random.default_rng(1).integers(0, spec.vocab, 37))
    xr = ref.run_layers(ref.embed_rows(ids), 0, spec.layers)
    xf = fast.run_layers(fast.embed_rows(ids), 0, spec.layers)
    assert xr.tobytes() == xf.tobytes()
    assert ref.logits_rows(xr, [36, 0]).tobytes() == fast.logits_rows(xf, [36, 0]).tobytes()
    assert (O.generate_chunked(ref, [(0, 2)], ids, 5, 16) == O.generate_chunked(fast, [(0, 1), (1, 2)], ids, 5, 16))
    assert O.generate_lookahead(ref, [(0, 2)], ids[:9], 6, 16) == O.generate_lookahead(fast, [(0, 2)], ids[:9], 6, 16)
