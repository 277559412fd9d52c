"""Models whose layer matmuls use the reference's other weight formats (int3 and int2 codes, groups of
64 and 128 weights per scale, and asymmetric weights with a per-group f16 bias), which the reference
serves through its GEMV (`src/engine.rs:432-441`, `src/kernels.rs:545-635`): they load (each weight
repacked into the int4 tile layout with unchanged values) and their residual stream after every layer
matches the oracle, which takes the GEMV with f32 dequantization for these formats as the reference
does, within the 4-layer tests' 2e-2; the answer probabilities within 1e-3 with the same argmax."""
import os

import numpy as np
import pytest

from oracle import oracle
from strands_decider import model as M

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FORMATS = [(3, 32), (2, 64), (4, 128), (3, 64), (2, 32), (4, 32)]
# asymmetric (q * scale + bias) in most layer matmuls, one symmetric among them
FORMATS_ASYM = [(4, 32, True), (3, 64, True), (2, 32, True), (4, 128, True), (3, 32, False), (2, 64, True)]


def _model(name, seed, formats):
    path = os.path.join(ROOT, "_models", name)
    if not os.path.exists(os.path.join(path, "tokenizer.json")):
        M.write_synthetic(path, seed=seed, n_layers=4, vocab=4096, matmul_formats=formats)
        from strands_decider.tokenizer import write_synthetic_tokenizer
        write_synthetic_tokenizer(os.path.join(path, "tokenizer.json"), seed=0)
    return path


@pytest.fixture(scope="module")
def formats_model():
    return _model("formats_s7", 7, FORMATS)


@pytest.fixture(scope="module")
def asym_model():
    return _model("formats_asym_s8", 8, FORMATS_ASYM)


def test_the_model_uses_the_other_formats(formats_model, asym_model):
    m = M.read_manifest(formats_model)
    seen = {(t["bits"], t["group"]) for n, t in m["tensors"].items() if n.endswith(".q") and n != "embed.q"}
    assert {(3, 32), (2, 64), (4, 128)} <= seen
    m = M.read_manifest(asym_model)
    asym = [n for n, t in m["tensors"].items() if n.endswith(".q") and t.get("asym")]
    assert asym and all(n[:-2] + ".b" in m["tensors"] for n in asym)


@pytest.mark.parametrize("l", [11, 150])
@pytest.mark.parametrize("which", ["symmetric", "asymmetric"])
def test_other_formats_layers_match_oracle(formats_model, asym_model, which, l):
    from strands_decider.engine import Engine, Head
    path = formats_model if which == "symmetric" else asym_model
    gpu, cpu = Engine.load(path), oracle.Engine(path)
    rng = np.random.default_rng(l)
    ids = rng.integers(0, 4000, l)
    rows = sorted(set([0, l // 2, l - 1]))
    out = gpu.forward(ids, rows, trace=True)
    want, _, tr = cpu.forward(ids, rows, trace=True)
    per_layer = np.abs(out.trace - tr).max(axis=(1, 2))
    assert per_layer.max() < 2e-2, per_layer
    head = Head.load(os.path.join(path, "head.safetensors"))
    tensors = M.read_safetensors(os.path.join(path, "head.safetensors"))
    a = head.probs(out.hidden, 2048, 1.0)
    b = oracle.head_probs(want, tensors, 1.0)
    assert np.abs(a - b).max() < 1e-3 and np.argmax(a) == np.argmax(b)
    gpu.close()
