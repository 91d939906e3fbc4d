"""The activation codec and routing of public/wire.js, restated (test_wire.js)."""
import numpy as np
import pytest


def test_activation_round_trips_with_both_hashes(O):
    hidden = (np.cos(np.arange(16 * 32)) * 0.5).astype(np.float32)
    a = O.unpack_act(O.pack_act(7, 3, 2, hidden, 0x5150))
    assert (a["seq"], a["tokenIdx"], a["nextIndex"], a["modelHash"]) == (7, 3, 2, 0x5150)
    assert a["hidden"].tobytes() == hidden.tobytes()


def test_one_ulp_flip_is_caught(O):
    buf = bytearray(O.pack_act(1, 0, 1, np.full(64, 1.5, np.float32), 9))
    v = np.frombuffer(bytes(buf[24 + 40:24 + 44]), np.float32)[0]
    buf[24 + 40:24 + 44] = np.float32(np.nextafter(v, np.float32(2))).tobytes()
    with pytest.raises(ValueError, match="integrity hash"):
        O.unpack_act(bytes(buf))


def test_negative_zero_survives_and_is_distinguished(O):
    hidden = np.zeros(8, np.float32)
    hidden[3] = -0.0
    buf = bytearray(O.pack_act(1, 0, 1, hidden, 9))
    a = O.unpack_act(bytes(buf))
    assert np.signbit(a["hidden"][3])
    buf[24 + 12:24 + 16] = np.float32(0.0).tobytes()
    with pytest.raises(ValueError, match="integrity hash"):
        O.unpack_act(bytes(buf))


def test_fnv1a_known_values(O):
    assert O.fnv1a(b"") == 0x811C9DC5
    assert O.fnv1a(b"a") == 0xE40C292C
