"""The C ABI library without a GPU: it loads, exports every entry point include/sd_b200.h declares,
reports the absence of a GPU as an error (no CPU fallback), and runs its host-only parts (the
pointer head) exactly as the oracle does."""
import ctypes
import os
import re

import numpy as np
import pytest

from strands_decider import engine as E

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sd_b200.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sd_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = E.lib()
    names = declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
        assert isinstance(getattr(lib, n), ctypes._CFuncPtr)


def test_engine_without_gpu_fails_loudly(small_model):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(E.Error) as ei:
        E.Engine.load(small_model)
    assert ei.value.code == -4 and "device" in str(ei.value).lower()


def test_head_matches_oracle(small_model):
    from oracle import oracle
    from strands_decider import model as M
    head = E.Head.load(os.path.join(small_model, "head.safetensors"))
    tensors = M.read_safetensors(os.path.join(small_model, "head.safetensors"))
    rng = np.random.default_rng(0)
    for n in (2, 3, 6):
        hidden = rng.standard_normal((n, 2048)).astype(np.float32) * 2
        for t in (1.0, 0.5):
            a = head.probs(hidden, 2048, t)
            b = oracle.head_probs(hidden, tensors, t)
            np.testing.assert_allclose(a, b, rtol=1e-10, atol=1e-13)


def test_head_load_errors(tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(b"\x05\x00\x00\x00\x00\x00\x00\x00{}")
    with pytest.raises(E.Error):
        E.Head.load(str(p))
    with pytest.raises(E.Error):
        E.Head.load(str(tmp_path / "missing.safetensors"))


def test_new_entry_points_reject_bad_arguments_without_touching_a_gpu():
    """The device-side head, the fork-with-head and the scale decoder validate their arguments on the
    host: a null engine, null buffers or impossible sizes come back as SD_ERR_INVALID with a message."""
    L = E.lib()
    L.sd_last_error.restype = ctypes.c_char_p
    buf = (ctypes.c_uint8 * 64)()
    # no engine
    assert L.sd_head_probs_dev(None, None, None, None, 1, None, None) == -1
    assert L.sd_forward_fork_multi_probs(None, None, None, None, 1, None, None, None, None, None) == -1
    # decode_scales: null buffers, negative rows, zero or huge group
    assert L.sd_decode_scales(None, 1, 64, buf, None) == -1
    assert L.sd_decode_scales(buf, -1, 64, buf, None) == -1
    assert L.sd_decode_scales(buf, 1, 0, buf, None) == -1
    assert L.sd_decode_scales(buf, 1, 1 << 21, buf, None) == -1
    assert b"sd_decode_scales" in L.sd_last_error()
    # no rows at all is a no-op, not an error
    assert L.sd_decode_scales(buf, 0, 64, buf, None) == 0
    # sd_matmul_ex: no weight, no output, an unknown algo
    assert L.sd_matmul_ex(None, buf, 4, buf, 64, 0, None, None, 0, 0, None) == -1
    assert L.sd_matmul_ex(None, buf, 4, None, 64, 0, None, None, 0, 3, None) == -1
    assert b"sd_matmul" in L.sd_last_error()
