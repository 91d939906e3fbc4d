"""The activation frame a B200 stage exchanges with the reference's peers
(public/wire.js:100-138, shard.js fnv1a :195-200 and modelFingerprint
:206-213), against the oracle's restatement of the same codec (test_wire.js)."""
import numpy as np
import pytest
import torch


@pytest.fixture(scope="module")
def W(P):
    return P.wire


def test_fnv1a_matches_the_oracle(W, O):
    assert W.fnv1a(b"") == 0x811C9DC5 and W.fnv1a(b"a") == 0xE40C292C
    rng = np.random.default_rng(3)
    for n in (1, 7, 4096, 65537):
        b = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert W.fnv1a(b) == O.fnv1a(b)


def test_frame_is_byte_identical_to_the_oracle(W, O):
    rng = np.random.default_rng(5)
    hidden = rng.standard_normal(16 * 64).astype(np.float32)
    for seq, tok, nxt, mh in ((0, 0, 1, 0), (7, 2032, -1, 0xDEADBEEF), (3, 5, 2, 0x5150)):
        assert W.pack_act(seq, tok, nxt, hidden, mh) == O.pack_act(seq, tok, nxt, hidden, mh)
    a = W.unpack_act(O.pack_act(7, 3, 2, hidden, 0x5150))
    assert (a["seq"], a["tokenIdx"], a["nextIndex"], a["modelHash"]) == (7, 3, 2, 0x5150)
    assert a["hidden"].tobytes() == hidden.tobytes()


def test_corrupted_short_and_mistagged_frames_are_refused(W):
    buf = bytearray(W.pack_act(1, 0, 1, np.full(64, 1.5, np.float32), 9))
    v = np.frombuffer(bytes(buf[24 + 40:24 + 44]), np.float32)[0]
    buf[24 + 40:24 + 44] = np.float32(np.nextafter(v, np.float32(2))).tobytes()  # one ulp
    with pytest.raises(ValueError, match="integrity hash"):
        W.unpack_act(bytes(buf))
    with pytest.raises(ValueError, match="truncated"):
        W.unpack_act(bytes(23))
    good = bytearray(W.pack_act(1, 0, 1, np.zeros(4, np.float32), 9))
    good[0:4] = np.int32(-24).tobytes()  # a TOKEN message
    with pytest.raises(ValueError, match="not an activation"):
        W.unpack_act(bytes(good))


def test_negative_zero_is_distinguished(W):
    hidden = np.zeros(8, np.float32)
    hidden[3] = -0.0
    buf = bytearray(W.pack_act(1, 0, 1, hidden, 9))
    assert np.signbit(W.unpack_act(bytes(buf))["hidden"][3])
    buf[24 + 12:24 + 16] = np.float32(0.0).tobytes()
    with pytest.raises(ValueError, match="integrity hash"):
        W.unpack_act(bytes(buf))


def test_model_fingerprint_restates_shard_js(W, O):
    tensors = {"model.norm.weight": dict(dtype="F32", shape=[64], start=208, end=464),
               "model.embed_tokens.weight": dict(dtype="BF16", shape=[128, 64], start=464, end=16848)}
    want = O.fnv1a(("org/model|main|model.embed_tokens.weight:BF16:128x64:464:16848|"
                    "model.norm.weight:F32:64:208:464").encode())
    assert W.model_fingerprint("org/model", None, tensors) == want
    assert W.model_fingerprint("org/model", "v2", tensors) != want


class Loopback:
    """An in-process transport: frames queue up in order, optionally tampered."""

    def __init__(self, tamper=None):
        self.q, self.tamper = [], tamper

    class _H:
        def __init__(self, f):
            self.f = f

        def wait(self):
            if self.f:
                self.f()
                self.f = None

    def send(self, t, dst, token_idx=0):
        c = t.clone()
        if self.tamper:
            self.tamper(c)
        self.q.append(c)
        return self._H(None)

    def recv(self, t, src, token_idx=None):
        return self._H(lambda: t.copy_(self.q.pop(0)))


PLAN = [dict(id="head", index=0), dict(id="mid", index=1), dict(id="tail", index=2)]


def hop(W, sender, receiver, x, tok=16, tok_due=16, tamper=None, mh=(1, 1)):
    link = Loopback(tamper)
    tx = W.WireTransport(link, PLAN, sender, model_hash=mh[0], seq=4)
    rx = W.WireTransport(link, PLAN, receiver, model_hash=mh[1], seq=4)
    tx.send(x, receiver, token_idx=tok).wait()
    out = torch.empty_like(x)
    rx.recv(out, sender, token_idx=tok_due).wait()
    return out


def test_transport_delivers_the_hidden_bits(W):
    x = torch.from_numpy(np.random.default_rng(1).standard_normal(3 * 64).astype(np.float32))
    assert torch.equal(hop(W, 0, 1, x), x)      # head -> stage 1, addressed "mine"
    assert torch.equal(hop(W, 2, 0, x), x)      # last stage -> head, addressed RETURN


def test_transport_refuses_bad_frames(W):
    x = torch.ones(64)
    with pytest.raises(ValueError, match="integrity hash"):
        hop(W, 0, 1, x, tamper=lambda f: f.__setitem__(30, f[30] ^ 1))
    with pytest.raises(ValueError, match="model hash"):
        hop(W, 0, 1, x, mh=(1, 2))
    with pytest.raises(ValueError, match="addressed"):
        hop(W, 0, 2, x)                         # a frame for stage 1 arriving at stage 2
    with pytest.raises(ValueError, match="token index"):
        hop(W, 0, 1, x, tok=16, tok_due=32)


def test_sentinels_and_the_solo_ring(W, P):
    """test_wire.js:192-205: the activation tag is negative and outside the
    -2..-8 range of DaisyChain-Web; RETURN is not a stage index; a one-stage
    ring returns to itself at once."""
    assert W.ACT == -23 and W.ACT <= -20 and W.RETURN == -1
    hop = P.pipeline.route_after([dict(id="p0", index=0)], 0)
    assert hop["isReturn"] and hop["to"] == "p0" and hop["address"] == W.RETURN
