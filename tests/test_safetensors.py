"""safetensors model files for the stages (public/safetensors.js, arch.js
names, shard.js toKN), checked on CPU: a written model reads back bit for bit
at every stage split, only a stage's byte ranges are read, the widenings are
exact, malformed headers are refused, and the known answers of the
reference's own loader tests (test_loader.js:24-126) hold."""
import dataclasses
import json
import struct

import numpy as np
import pytest


@pytest.fixture(scope="module")
def ST(P):
    return P.safetensors


def spec_of(P, ospec, tie):
    return P.infer.Spec(hidden=ospec.hidden, layers=ospec.layers, heads=ospec.heads, kvHeads=ospec.kvHeads,
                        inter=ospec.inter, vocab=ospec.vocab, tie=tie, maxPos=64)


@pytest.mark.parametrize("tie", [True, False])
def test_model_round_trips_at_every_split(P, O, ST, tmp_path, tie):
    ospec = dataclasses.replace(O.LLAMA_TEST, tie=tie)
    w = O.make_weights(ospec)
    spec = spec_of(P, ospec, tie)
    path = str(tmp_path / "model.safetensors")
    ST.save_weights(path, w, spec, metadata={"format": "pt"})
    hdr = ST.read_header(path)
    assert hdr["metadata"] == {"format": "pt"}
    assert ("lm_head.weight" in hdr["tensors"]) == (not tie)
    for lo, hi in [(0, 6), (0, 2), (2, 6), (3, 4)]:
        got = ST.read_stage_weights(path, spec, lo, hi, head=lo == 0)
        for l in range(lo, hi):
            for k, v in w["layers"][l].items():
                assert got["layers"][l][k].tobytes() == np.asarray(v, np.float32).tobytes(), (l, k)
        if lo == 0:
            assert got["emb"].tobytes() == w["emb"].tobytes()
            assert got["nrmF"].tobytes() == w["nrmF"].tobytes()
            assert (got["lm"] is None) == tie
            if not tie:
                assert got["lm"].tobytes() == w["lm"].tobytes()
        else:
            assert "emb" not in got


def test_a_stage_reads_only_its_own_ranges(P, O, ST, tmp_path, monkeypatch):
    ospec = O.LLAMA_TEST
    spec = spec_of(P, ospec, True)
    path = str(tmp_path / "m.safetensors")
    ST.save_weights(path, O.make_weights(ospec), spec)
    hdr = ST.read_header(path)
    want = ST.stage_tensors(hdr, spec, 4, 6, head=False)
    runs = ST.coalesce([t for t in want.values() if t], 0)
    assert len(runs) == 1  # layers 4 and 5 are contiguous in the file
    lo = min(t["start"] for t in want.values())
    hi = max(t["end"] for t in want.values())
    assert (runs[0]["start"], runs[0]["end"]) == (lo, hi)
    assert hi - lo < 0.4 * (max(t["end"] for t in hdr["tensors"].values()) - hdr["data_start"])
    assert ST.f32_bytes(want.values()) == hi - lo  # F32 file: bytes read = bytes held


def test_coalesce_merges_small_gaps_only(ST):
    t = lambda n, s, e: dict(name=n, start=s, end=e)
    runs = ST.coalesce([t("c", 300, 400), t("a", 0, 100), t("b", 150, 200)], slack=50)
    assert [(r["start"], r["end"], [x["name"] for x in r["tensors"]]) for r in runs] == \
        [(0, 200, ["a", "b"]), (300, 400, ["c"])]
    assert len(ST.coalesce([t("a", 0, 100), t("b", 150, 200), t("c", 300, 400)])) == 1  # 1 MiB default


def test_widening_is_exact(ST):
    u16 = np.arange(65536, dtype=np.uint16)
    bf = ST.to_f32("BF16", u16.tobytes())
    assert (bf.view(np.uint32) == (u16.astype(np.uint32) << 16)).all()
    f16 = ST.to_f32("F16", u16.tobytes())
    ref = u16.view(np.float16).astype(np.float64)  # every f16 is an exact double
    fin = np.isfinite(ref)
    assert (f16[fin].astype(np.float64) == ref[fin]).all()
    assert np.isnan(f16[np.isnan(ref)]).all() and (f16[np.isinf(ref)] == ref[np.isinf(ref)]).all()
    # the reference's hand-written widening (safetensors.js:31-43), restated, on the finite values
    h = u16[fin].astype(np.int64)
    s, e, f = (h & 0x8000) >> 15, (h & 0x7C00) >> 10, h & 0x03FF
    v = np.where(e == 0, np.ldexp(f / 1024.0, -14), np.ldexp(1 + f / 1024.0, (e - 15).astype(np.int32)))
    assert (f16[fin] == np.where(s == 1, -v, v)).all()
    d = np.array([0.1, 1 / 3, 1e-40, 3.4e38, -2.5], np.float64)
    assert ST.to_f32("F64", d.tobytes()).tobytes() == d.astype(np.float32).tobytes()
    with pytest.raises(ValueError, match="cannot be widened"):
        ST.to_f32("I8", b"\x01")


def header_bytes(obj, pad=0):
    h = json.dumps(obj).encode() + b" " * pad
    return struct.pack("<Q", len(h)) + h


def test_malformed_headers_are_refused(ST):
    with pytest.raises(ValueError, match="implausibly large"):
        ST.parse_header(struct.pack("<II", 16, 1) + b"{}" * 8)
    with pytest.raises(ValueError, match="truncated"):
        ST.parse_header(struct.pack("<Q", 100) + b"{}")
    with pytest.raises(ValueError, match="not valid JSON"):
        ST.parse_header(struct.pack("<Q", 4) + b"{no]")
    with pytest.raises(ValueError, match="malformed"):
        ST.parse_header(header_bytes({"x": {"dtype": "F32", "shape": [2]}}))
    with pytest.raises(ValueError, match="expected 8"):
        ST.parse_header(header_bytes({"x": {"dtype": "F32", "shape": [2], "data_offsets": [0, 12]}}))
    ok = ST.parse_header(header_bytes({"__metadata__": {"a": "b"},
                                       "x": {"dtype": "BF16", "shape": [2, 3], "data_offsets": [0, 12]}}, pad=3))
    t = ok["tensors"]["x"]
    assert (t["elems"], t["start"] - ok["data_start"], t["bytes"]) == (6, 0, 12) and ok["metadata"] == {"a": "b"}


def test_names_resolve_across_export_prefixes(ST):
    r = ST.resolver(["layers.0.mlp.up_proj.weight", "model.norm.weight"])
    assert r("model.layers.0.mlp.up_proj.weight") == "layers.0.mlp.up_proj.weight"
    assert r("model.norm.weight") == "model.norm.weight"
    assert r("lm_head.weight", True) is None
    with pytest.raises(ValueError, match="do not contain"):
        r("model.layers.1.mlp.up_proj.weight")


def test_fingerprint_of_a_file(P, O, ST, tmp_path):
    spec = spec_of(P, O.LLAMA_TEST, True)
    path = str(tmp_path / "m.safetensors")
    ST.save_weights(path, O.make_weights(O.LLAMA_TEST), spec)
    t = ST.read_header(path)["tensors"]
    a = P.wire.model_fingerprint("test/llama", "main", t)
    assert a == P.wire.model_fingerprint("test/llama", None, t)
    t2 = dict(t)
    t2.pop("model.norm.weight")
    assert P.wire.model_fingerprint("test/llama", "main", t2) != a


# ---- the reference's loader tests (test_loader.js:24-126), restated --------------------
def build_file(entries):
    """test_loader.js buildFile: [(name, dtype, shape, bytes)] -> a safetensors buffer."""
    header, chunks, off = {}, [], 0
    for name, dtype, shape, raw in entries:
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + len(raw)]}
        chunks.append(raw)
        off += len(raw)
    hj = json.dumps(header).encode()
    return struct.pack("<II", len(hj), 0) + hj + b"".join(chunks)


def test_loader_parses_and_locates_every_tensor(ST):
    buf = build_file([("w.a", "F32", [2, 2], np.array([1, 2, 3, 4], "<f4").tobytes()),
                      ("w.b", "F32", [2], np.array([5, 6], "<f4").tobytes())])
    t = ST.parse_header(buf)["tensors"]
    assert len(t) == 2 and t["w.a"]["shape"] == [2, 2] and t["w.a"]["elems"] == 4
    a, b = t["w.a"], t["w.b"]
    assert list(ST.to_f32("F32", buf[a["start"]:a["end"]])) == [1, 2, 3, 4]
    assert list(ST.to_f32("F32", buf[b["start"]:b["end"]])) == [5, 6]


def test_loader_refuses_contradictions_and_junk(ST):
    with pytest.raises(ValueError, match="expected"):
        ST.parse_header(build_file([("w", "F32", [9, 9], np.arange(4, dtype="<f4").tobytes())]))
    junk = bytearray(64)
    junk[0:4] = struct.pack("<I", 16)
    with pytest.raises(ValueError, match="not valid JSON|not a safetensors"):
        ST.parse_header(bytes(junk))
    big = bytearray(16)
    big[4:8] = struct.pack("<I", 7)
    with pytest.raises(ValueError, match="implausibly large"):
        ST.parse_header(bytes(big))


def test_loader_known_widenings(ST):
    vals = np.array([1, -1, 0.5, -0.5, 2, 100, -0.0078125, 0], np.float32)
    bf = (vals.view(np.uint32) >> 16).astype("<u2")
    assert ST.to_f32("BF16", bf.tobytes()).tobytes() == vals.tobytes()
    cases = [(0x3C00, 1.0), (0xBC00, -1.0), (0x3800, 0.5), (0x0000, 0.0), (0x8000, -0.0),
             (0x0001, 2.0 ** -24), (0x7BFF, 65504.0)]
    out = ST.to_f32("F16", np.array([c[0] for c in cases], "<u2").tobytes())
    for (bits, want), got in zip(cases, out):
        assert got == want and np.signbit(got) == np.signbit(want), hex(bits)


def test_loader_coalescing_keeps_offsets(ST):
    mk = lambda s, e: dict(start=s, end=e, bytes=e - s, elems=(e - s) // 4, dtype="F32", name=f"t{s}")
    runs = ST.coalesce([mk(0, 100), mk(100, 200), mk(10_000_000, 10_000_100)], 1024)
    assert len(runs) == 2 and (runs[0]["start"], runs[0]["end"]) == (0, 200) and len(runs[0]["tensors"]) == 2
    assert (runs[1]["start"], runs[1]["end"]) == (10_000_000, 10_000_100)
    assert runs[0]["tensors"][1]["start"] - runs[0]["start"] == 100


def test_stage_byte_cost_from_the_header_alone(P, ST):
    spec = P.infer.Spec(hidden=64, layers=4, heads=4, kvHeads=4, inter=128, vocab=100)
    tensors = {}

    def add(name, elems):
        tensors[name] = dict(name=name, elems=elems, bytes=elems * 2, dtype="BF16", shape=[elems], start=0, end=0)

    h = ST.head_tensors(True)
    add(h["emb"], 100 * 64)
    add(h["nrmF"], 64)
    for l in range(4):
        lt = ST.layer_tensors(l)
        add(lt["nrm1"], 64)
        add(lt["nrm2"], 64)
        for r in ("Wq", "Wk", "Wv", "Wo"):
            add(lt[r], 64 * 64)
        add(lt["Wgate"], 128 * 64)
        add(lt["Wup"], 128 * 64)
        add(lt["Wdown"], 64 * 128)
    header = {"tensors": tensors}
    mid = ST.f32_bytes(t for t in ST.stage_tensors(header, spec, 1, 2, False).values() if t)
    head = ST.f32_bytes(t for t in ST.stage_tensors(header, spec, 0, 1, True).values() if t)
    assert mid == (4 * 64 * 64 + 3 * 128 * 64 + 2 * 64) * 4
    assert head > mid
