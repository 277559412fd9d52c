"""Shared test set-up: import paths, the `gpu` marker and seeded synthetic model directories."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "strands-decider-rs_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

MODELS = os.path.join(ROOT, "_models")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path through the C ABI)")


@pytest.fixture(autouse=True)
def _kernel_status(request):
    """After every GPU test: no kernel of a standalone call gave up on a bounded wait (sd_op_status)."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch
    if not torch.cuda.is_available():
        return
    from strands_decider import engine
    engine.op_status()


@pytest.fixture(scope="session")
def small_model():
    """Production dims, 4 layers (3 gated-delta + 1 full attention), an 8192-row vocabulary."""
    from strands_decider import model
    return model.ensure_model(os.path.join(MODELS, "l4_v8192_s0"), seed=0, n_layers=4, vocab=8192)


@pytest.fixture(scope="session")
def full_model():
    """The benchmarked model: production dims, 24 layers ([3 gated-delta, 1 attention] x 6), the
    248320-row int3 embedding; seed 0, as bench.py generates it."""
    from strands_decider import model
    return model.ensure_model(os.path.join(MODELS, "full_s0"), seed=0)


@pytest.fixture(scope="session")
def small_model_u8():
    """As small_model, with the embedding's scales stored as 8-bit codes (`src/model.rs:219-236`)."""
    from strands_decider import model
    path = os.path.join(MODELS, "l4_v8192_s3_u8")
    if not os.path.exists(os.path.join(path, "tokenizer.json")):
        model.write_synthetic(path, seed=3, n_layers=4, vocab=8192, embed_u8=True)
        from strands_decider.tokenizer import write_synthetic_tokenizer
        write_synthetic_tokenizer(os.path.join(path, "tokenizer.json"), seed=0)
    return path


@pytest.fixture(scope="session")
def adapter_model():
    """Two layers: one gated-delta layer then one adapter layer (`src/engine.rs:466-472`)."""
    from strands_decider import model
    path = os.path.join(MODELS, "adapter_s5")
    if not os.path.exists(os.path.join(path, "tokenizer.json")):
        model.write_synthetic(path, seed=5, vocab=4096, layer_types=["linear_attention", "adapter", "full_attention"])
        from strands_decider.tokenizer import write_synthetic_tokenizer
        write_synthetic_tokenizer(os.path.join(path, "tokenizer.json"), seed=0)
    return path
