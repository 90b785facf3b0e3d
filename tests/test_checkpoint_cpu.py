"""Checkpoint file format (host side): round trip, atomic replace and every
corruption the reader must refuse."""
import os

import numpy as np
import pytest

from forgellm import checkpoint as ck


def _sections(n=1000, seed=0):
    rng = np.random.default_rng(seed)
    return {"params": rng.standard_normal(n).astype(np.float32),
            "adam_m": rng.standard_normal(n).astype(np.float32),
            "adam_v": rng.random(n).astype(np.float32)}


def test_round_trip_bit_exact(tmp_path):
    path = str(tmp_path / "a.ck")
    sec = _sections()
    want = {k: v.copy() for k, v in sec.items()}
    ck.write_file(path, {"config": {"dim": 64}, "n_params": 1000, "adam": {"t": 7}}, sec)
    header, got = ck.read_file(path)
    assert header["config"] == {"dim": 64} and header["adam"]["t"] == 7
    assert list(got) == ["params", "adam_m", "adam_v"]
    for k in want:
        assert got[k].dtype == np.float32 and np.array_equal(got[k].view(np.uint32), want[k].view(np.uint32))
    assert [f for f in os.listdir(tmp_path) if ".tmp." in f] == []     # no temp file left behind


def test_overwrite_is_atomic_replace(tmp_path):
    path = str(tmp_path / "a.ck")
    ck.write_file(path, {"n": 1}, _sections(seed=1))
    ck.write_file(path, {"n": 2}, _sections(seed=2))
    header, got = ck.read_file(path)
    assert header["n"] == 2 and np.array_equal(got["params"], _sections(seed=2)["params"])


@pytest.mark.parametrize("damage", ["flip_data", "truncate", "magic", "header"])
def test_corruption_is_refused(tmp_path, damage):
    path = str(tmp_path / "a.ck")
    ck.write_file(path, {"n": 1}, _sections())
    blob = bytearray(open(path, "rb").read())
    if damage == "flip_data":
        blob[-5] ^= 0x01
    elif damage == "truncate":
        blob = blob[:-17]
    elif damage == "magic":
        blob[0] ^= 0xFF
    else:
        blob[14] = ord("#")
    open(path, "wb").write(bytes(blob))
    with pytest.raises(ValueError):
        ck.read_file(path)
