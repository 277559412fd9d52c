"""Other sizes of the model family. The reference reads every dim from the manifest's config
(`src/model.rs:31-47`) and sizes its dispatches from them (`src/engine.rs:463-522`); the kernels here fix
the head sizes (attention head dim 256, gated-delta heads of 128 x 128) and take any hidden size that is
a multiple of 64 up to 8192, any intermediate size that is a multiple of 128 and any head counts. Each
model loads, its residual stream after every layer matches the oracle within the 4-layer tests' 2e-2,
and its answer probabilities within 1e-3 with the same argmax; a snapshot continued matches the
full pass (prefix == full, `tests/engine_parity.rs:16-85` of the reference)."""
import os

import numpy as np
import pytest

from oracle import oracle
from strands_decider import model as M

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# hidden 1024 (one partial 2048-wide pass of the norms) with fewer heads; hidden 3072 (one full pass and
# a half one) with more; hidden 5120 (three passes, the last a half) with GQA 5:1.
DIMS = {
    "d1024": dict(hidden_size=1024, intermediate_size=3584, num_attention_heads=4, num_key_value_heads=1,
                  linear_num_key_heads=8),
    "d3072": dict(hidden_size=3072, intermediate_size=8192, num_attention_heads=16, num_key_value_heads=4,
                  linear_num_key_heads=24),
    "d5120": dict(hidden_size=5120, intermediate_size=1536, num_attention_heads=10, num_key_value_heads=2,
                  linear_num_key_heads=4),
}


def _model(name):
    path = os.path.join(ROOT, "_models", f"dims_{name}")
    if not os.path.exists(os.path.join(path, "tokenizer.json")):
        M.write_synthetic(path, seed=11, n_layers=4, vocab=4096, dims=DIMS[name])
        from strands_decider.tokenizer import write_synthetic_tokenizer
        write_synthetic_tokenizer(os.path.join(path, "tokenizer.json"), seed=0)
    return path


def test_writer_takes_other_dims():
    m = M.write_synthetic(os.path.join(ROOT, "_models", "dims_manifest_only"), seed=1, n_layers=4, vocab=256,
                          dims=DIMS["d1024"])
    c = m["config"]
    assert c["hidden_size"] == 1024 and c["linear_num_key_heads"] == 8
    t = m["tensors"]
    assert t["layers.0.in_proj.q"]["K"] == 1024 and t["layers.3.o_proj.q"]["K"] == 4 * 256
    assert t["layers.0.gate_up.q"]["N"] == 2 * 3584


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(DIMS))
def test_other_dims_layers_match_oracle(name):
    from strands_decider.engine import Engine, Head
    path = _model(name)
    gpu, cpu = Engine.load(path), oracle.Engine(path)
    d = DIMS[name]["hidden_size"]
    assert gpu.hidden_size() == d
    for l in (13, 150):
        rng = np.random.default_rng(l)
        ids = rng.integers(0, 4000, l)
        rows = sorted({0, l // 2, l - 1})
        out = gpu.forward(ids, rows, trace=True)
        want, _, tr = cpu.forward(ids, rows, trace=True)
        per_layer = np.abs(out.trace - tr).max(axis=(1, 2))
        assert per_layer.max() < 2e-2, (l, per_layer)
        head = Head.load(os.path.join(path, "head.safetensors"))
        tensors = M.read_safetensors(os.path.join(path, "head.safetensors"))
        a = head.probs(out.hidden, d, 1.0)
        b = oracle.head_probs(want, tensors, 1.0)
        assert np.abs(a - b).max() < 1e-3 and np.argmax(a) == np.argmax(b)
    gpu.close()


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["d1024", "d3072"])
def test_other_dims_prefix_equals_full(name):
    from strands_decider.engine import Engine
    gpu = Engine.load(_model(name))
    rng = np.random.default_rng(5)
    ids = rng.integers(0, 4000, 200)
    full = gpu.forward(ids, [199]).hidden
    first = gpu.forward(ids[:137], [], keep=True)
    cont = gpu.forward(ids[137:], [62], cache=first.snapshot).hidden
    assert np.abs(full - cont).max() < 2e-2
    gpu.close()
