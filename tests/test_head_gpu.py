"""The pointer head on the GPU (`sd_head_probs_dev`, `sd_forward_fork_multi_probs`) against the
oracle's `Head::probs` (`src/head.rs:55-77`, f64) and the host head, on the same hidden rows. The GPU
sums in tree order, so the bar is the one the host head meets against the oracle (f64 rounding): 1e-10
relative, 1e-13 absolute, on every probability."""
import json
import os

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-10, 1e-13


@pytest.fixture(scope="module")
def parts(small_model):
    from strands_decider import model as M
    from strands_decider.engine import Engine, Head
    return (Engine.load(small_model), Head.load(os.path.join(small_model, "head.safetensors")),
            M.read_safetensors(os.path.join(small_model, "head.safetensors")))


def test_head_dev_matches_oracle(parts):
    """Questions of 2 to 13 rows and one of 301 (more options than the block's threads), each with
    its own temperature, in one call; hidden rows of several scales, one row constant (zero variance)."""
    import torch
    eng, head, tensors = parts
    rng = np.random.default_rng(11)
    nrows = [2, 3, 5, 13, 4, 301, 2]
    temps = [1.0, 0.7, 2.5, 1e-9, 1.0, 0.3, 4.0]
    rows = [rng.standard_normal((n, 2048)).astype(np.float32) * rng.uniform(0.1, 30.0) for n in nrows]
    rows[2][1] = 0.5  # a constant row: LayerNorm of zero variance
    hidden = np.concatenate(rows)
    hd = torch.from_numpy(hidden).cuda()
    pd = torch.full((sum(nrows) - len(nrows),), float("nan"), dtype=torch.float64, device="cuda")
    torch.cuda.synchronize()
    eng.head_probs_dev(head, hd.data_ptr(), nrows, temps, pd.data_ptr())
    eng.synchronize()
    got = np.split(pd.cpu().numpy(), np.cumsum(np.array(nrows) - 1)[:-1])
    for r, t, g in zip(rows, temps, got):
        want = oracle.head_probs(r, tensors, t)
        np.testing.assert_allclose(g, want, rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(g, head.probs(r, 2048, t), rtol=RTOL, atol=ATOL)
        assert abs(g.sum() - 1.0) < 1e-12


def test_head_dev_many_questions(parts):
    """2000 questions of 2 to 12 rows in one call (grids of thousands of blocks), each against the
    host head."""
    import torch
    eng, head, _ = parts
    rng = np.random.default_rng(12)
    nrows = rng.integers(2, 13, 2000).tolist()
    temps = rng.uniform(0.5, 2.0, 2000).tolist()
    hidden = rng.standard_normal((sum(nrows), 2048)).astype(np.float32)
    hd = torch.from_numpy(hidden).cuda()
    pd = torch.full((sum(nrows) - len(nrows),), float("nan"), dtype=torch.float64, device="cuda")
    eng.head_probs_dev(head, hd.data_ptr(), nrows, temps, pd.data_ptr())
    eng.synchronize()
    got = np.split(pd.cpu().numpy(), np.cumsum(np.array(nrows) - 1)[:-1])
    row0 = np.concatenate([[0], np.cumsum(nrows)[:-1]])
    for i in range(0, 2000, 7):
        want = head.probs(hidden[row0[i]:row0[i] + nrows[i]], 2048, temps[i])
        np.testing.assert_allclose(got[i], want, rtol=RTOL, atol=ATOL)


def test_fork_probs_matches_fork_then_host_head(parts, small_model):
    """sd_forward_fork_multi_probs = sd_forward_fork_multi (the same pass, so the same hidden rows)
    followed by the host head, across two snapshots."""
    eng, head, _ = parts
    rng = np.random.default_rng(5)
    _, snaps = eng.forward_batch(None, [rng.integers(0, 8000, 300), rng.integers(0, 8000, 77)], [[], []], keep=True)
    lens = [40, 9, 130, 64, 17]
    ids = [rng.integers(0, 8000, n) for n in lens]
    rows = [sorted(set(rng.integers(0, n - 1, 1 + i % 4).tolist())) + [n - 1] for i, n in enumerate(lens)]
    caches = [snaps[i % 2] for i in range(len(lens))]
    temps = [1.0, 0.5, 1.0, 2.0, 1.0]
    got = eng.forward_fork_probs(caches, ids, rows, head, temps)
    hidden = eng.forward_fork(caches, ids, rows)
    for g, h, t in zip(got, hidden, temps):
        np.testing.assert_allclose(g, head.probs(h, 2048, t), rtol=RTOL, atol=ATOL)
    for s in snaps:
        s.close()


def test_fork_probs_rotated_torso(parts, small_model, tmp_path):
    """A rotated torso (`unrotate` in the manifest, src/engine.rs:652-660): the device maps the rows
    back (Walsh-Hadamard in f32 with the host's butterfly order, then the f64 factors) before the
    head, as the host does for sd_forward_fork's rows."""
    from strands_decider.engine import Engine
    _, head, _ = parts
    for name in os.listdir(small_model):
        if name != "manifest.json":
            os.symlink(os.path.join(small_model, name), tmp_path / name)
    with open(os.path.join(small_model, "manifest.json")) as f:
        m = json.load(f)
    rng = np.random.default_rng(2)
    m["config"]["unrotate"] = (rng.uniform(0.5, 1.5, 2048) / np.sqrt(2048)).tolist()
    with open(tmp_path / "manifest.json", "w") as f:
        json.dump(m, f)
    eng = Engine.load(str(tmp_path))
    _, snaps = eng.forward_batch(None, [rng.integers(0, 8000, 100)], [[]], keep=True)
    ids = [rng.integers(0, 8000, n) for n in (20, 33)]
    rows = [[3, 7, 19], [0, 32]]
    got = eng.forward_fork_probs([snaps[0]] * 2, ids, rows, head, [1.0, 0.8])
    hidden = eng.forward_fork([snaps[0]] * 2, ids, rows)
    for g, h, t in zip(got, hidden, [1.0, 0.8]):
        np.testing.assert_allclose(g, head.probs(h, 2048, t), rtol=RTOL, atol=ATOL)
    snaps[0].close()
    eng.close()


def test_head_dev_errors(parts):
    """Questions need two rows (options and the answer); the head's width must be the torso's."""
    import torch
    from strands_decider.engine import Error
    eng, head, _ = parts
    hd = torch.zeros((8, 2048), dtype=torch.float32, device="cuda")
    pd = torch.zeros(8, dtype=torch.float64, device="cuda")
    with pytest.raises(Error, match="2 or more"):
        eng.head_probs_dev(head, hd.data_ptr(), [3, 1], 1.0, pd.data_ptr())
    _, snaps = eng.forward_batch(None, [np.arange(10)], [[]], keep=True)
    with pytest.raises(Error, match="2 or more"):
        eng.forward_fork_probs([snaps[0]], [np.arange(5)], [[4]], head, 1.0)
    snaps[0].close()
    # the engine is still usable after the refusals
    eng.head_probs_dev(head, hd.data_ptr(), [4, 4], 1.0, pd.data_ptr())
    eng.synchronize()
