"""The wire format unpacked on the device (`src/model.rs:205-283`): `sd_decode_scales` against the
oracle's `decode_scales` bit for bit, an engine loaded from a packed shard against one loaded from the
converted shard, and the embedding's 8-bit scale codes decoded at load against an embedding stored
with the decoded fp16 scales (bit-identical hidden rows in both cases)."""
import json
import os

import numpy as np
import pytest

from oracle import oracle
from strands_decider import model as M

pytestmark = pytest.mark.gpu


def _codes(rng, n, g, jmax):
    m = rng.integers(0x0400, 0x7C00, n).astype(np.uint16)  # positive normal fp16
    m[::7] = rng.integers(1, 0x0400, len(m[::7]))          # and some subnormal ones
    j = rng.integers(1, jmax + 1, n).astype(np.uint16)
    j[0] = jmax
    hdr = np.stack([m, j], axis=1).astype("<u2").tobytes()
    codes = rng.integers(0, 256, (n, g)).astype(np.uint8)
    codes[0, :2] = [127, 255]
    return hdr + codes.tobytes()


@pytest.mark.parametrize("n,g,jmax", [(1, 64, 1), (3000, 64, 3000), (517, 40, 65535)])
def test_decode_scales_matches_oracle(n, g, jmax):
    import torch
    from strands_decider.engine import decode_scales
    src = _codes(np.random.default_rng(n), n, g, jmax)
    want = oracle.decode_scales(src, n, g).view(np.uint16)
    sd = torch.from_numpy(np.frombuffer(src, np.uint8).copy()).cuda()
    dd = torch.zeros((n, g), dtype=torch.int16, device="cuda")
    decode_scales(sd.data_ptr(), n, g, dd.data_ptr())
    torch.cuda.synchronize()
    got = dd.cpu().numpy().view(np.uint16)
    assert np.array_equal(got, want)


def _forward(path, ids, rows):
    from strands_decider.engine import Engine
    e = Engine.load(path)
    try:
        return e.forward(ids, rows).hidden
    finally:
        e.close()


def test_packed_shard_loads_as_converted(small_model, tmp_path):
    M.write_packed(small_model, str(tmp_path / "packed"), str(tmp_path / "unpacked"))
    rng = np.random.default_rng(3)
    ids = rng.integers(0, 8192, 333)
    rows = [0, 100, 332]
    a = _forward(str(tmp_path / "packed"), ids, rows)
    b = _forward(str(tmp_path / "unpacked"), ids, rows)
    assert np.isfinite(a).all()
    assert np.array_equal(a, b)


def test_packed_shard_errors(small_model, tmp_path):
    from strands_decider.engine import Engine, Error
    M.write_packed(small_model, str(tmp_path / "packed"), str(tmp_path / "unpacked"))
    p = tmp_path / "packed"
    m = json.loads((p / "manifest.json").read_text())
    # a tensor whose wire range runs past the packed file
    bad = json.loads(json.dumps(m))
    name = next(n for n, t in bad["tensors"].items() if t.get("u8"))
    bad["tensors"][name]["wire"] = bad["shards"][0]["wire"] - 10
    (p / "manifest.json").write_text(json.dumps(bad))
    with pytest.raises(Error, match="out of range"):
        Engine.load(str(p))
    # a compressed packed file
    gz = json.loads(json.dumps(m))
    gz["shards"][0]["path"] = "weights.0.wire.gz"
    os.symlink(p / "weights.0.wire", p / "weights.0.wire.gz")
    (p / "manifest.json").write_text(json.dumps(gz))
    with pytest.raises(Error, match="compressed"):
        Engine.load(str(p))


def test_embedding_u8_codes_decode_as_host(small_model_u8, tmp_path):
    """small_model_u8's embedding rows carry 8-bit scale codes; the same model with those codes
    decoded on the host (numpy `decode_scales`) into plain fp16 rows gives bit-identical hidden rows
    over ids spread across the vocabulary."""
    m = M.read_manifest(small_model_u8)
    e = m["embed"]
    qb, sb = e["parts"][0][1], e["parts"][1][1]
    rb = e["wire_row_bytes"]
    raw = np.fromfile(os.path.join(small_model_u8, e["rows"]), np.uint8).reshape(e["vocab"], rb)
    scales = np.stack([M.decode_scales_u8(raw[r, qb:].tobytes(), 1, sb // 2)[0] for r in range(e["vocab"])])
    rows = np.concatenate([raw[:, :qb], scales.view(np.uint8).reshape(e["vocab"], sb)], axis=1)
    for f in os.listdir(small_model_u8):
        if f not in ("manifest.json", e["rows"]):
            os.symlink(os.path.join(small_model_u8, f), tmp_path / f)
    rows.tofile(tmp_path / e["rows"])
    m2 = json.loads(json.dumps(m))
    m2["embed"]["u8"] = False
    m2["embed"].pop("wire_row_bytes")
    (tmp_path / "manifest.json").write_text(json.dumps(m2))
    ids = np.arange(5, e["vocab"], 7)[:1500]
    r = [0, 700, len(ids) - 1]
    a = _forward(small_model_u8, ids, r)
    b = _forward(str(tmp_path), ids, r)
    assert np.array_equal(a, b)
