"""A model whose layer matmuls use the reference's other symmetric weight formats (int3 and int2 codes,
groups of 64 and 128 weights per scale), which the reference serves through its GEMV
(`src/engine.rs:432-441`, `src/kernels.rs:545-635`): it loads (each weight repacked into the int4 tile
layout with unchanged values) and its residual stream after every layer matches the oracle, which
takes the GEMV with f32 dequantization for these formats as the reference does, within the 4-layer
tests' 2e-2; the answer probabilities within 1e-3 with the same argmax."""
import os

import numpy as np
import pytest

from oracle import oracle
from strands_decider import model as M

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FORMATS = [(3, 32), (2, 64), (4, 128), (3, 64), (2, 32), (4, 32)]


@pytest.fixture(scope="module")
def formats_model():
    path = os.path.join(ROOT, "_models", "formats_s7")
    if not os.path.exists(os.path.join(path, "tokenizer.json")):
        M.write_synthetic(path, seed=7, n_layers=4, vocab=4096, matmul_formats=FORMATS)
        from strands_decider.tokenizer import write_synthetic_tokenizer
        write_synthetic_tokenizer(os.path.join(path, "tokenizer.json"), seed=0)
    return path


def test_the_model_uses_the_other_formats(formats_model):
    m = M.read_manifest(formats_model)
    seen = {(t["bits"], t["group"]) for n, t in m["tensors"].items() if n.endswith(".q") and n != "embed.q"}
    assert {(3, 32), (2, 64), (4, 128)} <= seen


@pytest.mark.parametrize("l", [11, 150])
def test_other_formats_layers_match_oracle(formats_model, l):
    from strands_decider.engine import Engine, Head
    gpu, cpu = Engine.load(formats_model), oracle.Engine(formats_model)
    rng = np.random.default_rng(l)
    ids = rng.integers(0, 4000, l)
    rows = sorted(set([0, l // 2, l - 1]))
    out = gpu.forward(ids, rows, trace=True)
    want, _, tr = cpu.forward(ids, rows, trace=True)
    per_layer = np.abs(out.trace - tr).max(axis=(1, 2))
    assert per_layer.max() < 2e-2, per_layer
    head = Head.load(os.path.join(formats_model, "head.safetensors"))
    tensors = M.read_safetensors(os.path.join(formats_model, "head.safetensors"))
    a = head.probs(out.hidden, 2048, 1.0)
    b = oracle.head_probs(want, tensors, 1.0)
    assert np.abs(a - b).max() < 1e-3 and np.argmax(a) == np.argmax(b)
    gpu.close()
