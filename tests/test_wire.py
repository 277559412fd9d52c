"""The packed download format (`src/model.rs:205-283`) on the host: the writer that makes a packed
model directory and the numpy `unpack_shard` agree byte for byte with the GPU-layout directory
written beside it."""
import json
import os

import numpy as np
import pytest

from strands_decider import model as M


@pytest.fixture(scope="module")
def packed_dirs(small_model, tmp_path_factory):
    root = tmp_path_factory.mktemp("wire")
    M.write_packed(small_model, str(root / "packed"), str(root / "unpacked"))
    return str(root / "packed"), str(root / "unpacked")


def test_unpack_shard_gives_the_converted_shard(packed_dirs):
    packed, unpacked = packed_dirs
    m = M.read_manifest(packed)
    shard = m["shards"][0]
    with open(os.path.join(packed, shard["path"]), "rb") as f:
        wire = f.read()
    assert len(wire) == shard["wire"]
    with open(os.path.join(unpacked, "weights.0.bin"), "rb") as f:
        want = f.read()
    assert M.unpack_shard(wire, shard, m["tensors"]) == want
    offs = [t["wire"] for t in m["tensors"].values() if "wire" in t]
    assert any(o % 4 for o in offs)  # unaligned wire offsets are exercised
    assert sum(bool(t.get("u8")) for t in m["tensors"].values()) >= 8
    assert not os.path.exists(os.path.join(packed, "weights.0.bin"))


def test_unpack_shard_out_of_range(packed_dirs):
    packed, _ = packed_dirs
    m = M.read_manifest(packed)
    shard = m["shards"][0]
    with open(os.path.join(packed, shard["path"]), "rb") as f:
        wire = f.read()
    with pytest.raises(ValueError, match="out of range"):
        M.unpack_shard(wire[: len(wire) // 2], shard, m["tensors"])


def test_decoded_scales_are_close(packed_dirs, small_model):
    """The 8-bit codes are a lossy format: decoded scales stay within one log step of the originals."""
    _, unpacked = packed_dirs
    m = M.read_manifest(small_model)
    t = m["tensors"]["layers.0.in_proj.s"]
    with open(os.path.join(small_model, "weights.0.bin"), "rb") as f:
        f.seek(t["offset"])
        a = np.frombuffer(f.read(t["bytes"]), np.float16).astype(np.float64)
    with open(os.path.join(unpacked, "weights.0.bin"), "rb") as f:
        f.seek(t["offset"])
        b = np.frombuffer(f.read(t["bytes"]), np.float16).astype(np.float64)
    assert np.all(np.sign(a) == np.sign(b))
    assert np.max(np.abs(np.log2(np.abs(b) / np.abs(a)))) < 0.05
    with open(os.path.join(unpacked, "manifest.json")) as f:
        assert json.load(f)["shards"][0]["path"] == "weights.0.bin"
