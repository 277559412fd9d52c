"""`sd_forward_batch`: many `Engine::forward` calls (src/engine.rs:529-662) in one packed pass: fresh
sequences and continuations of snapshots side by side, each with its own new snapshot. Checked
against separate sd_forward calls and against the CPU oracle; tolerance as the per-layer parity
target (2e-2 max-abs on the hidden rows). Lengths straddle the 64-token chunk (the single-pass scan
for sequences of at most two chunks, the two-phase scan beyond) and the attention blocks."""
import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engines(small_model):
    from strands_decider.engine import Engine
    return Engine.load(small_model), oracle.Engine(small_model)


def _rows(n):
    return sorted(set([0, n // 2, n - 1]))


def _close(a, b, tol=2e-2):
    assert a.shape == b.shape
    assert np.abs(a - b).max() < tol


def test_batch_of_fresh_sequences_matches_serial(engines):
    gpu, _ = engines
    rng = np.random.default_rng(40)
    lens = [1, 63, 64, 65, 200, 1000, 2100, 130]
    ids = [rng.integers(0, 8000, n) for n in lens]
    rows = [_rows(n) for n in lens]
    outs, snaps = gpu.forward_batch(None, ids, rows, keep=True)
    q = rng.integers(0, 8000, 37)
    for x, r, o, s in zip(ids, rows, outs, snaps):
        ref = gpu.forward(x, r, keep=True)
        _close(o, ref.hidden)
        assert s.len == len(x)
        # the batch's snapshot continues like the serial one
        _close(gpu.forward(q, [0, 36], cache=s).hidden, gpu.forward(q, [0, 36], cache=ref.snapshot).hidden)
        ref.snapshot.close()
        s.close()


def test_batch_of_continuations_matches_serial(engines):
    """Continuations of snapshots (long ones: the two-phase scan from each sequence's own state) and
    fresh sequences in one pass, every one kept."""
    gpu, _ = engines
    rng = np.random.default_rng(41)
    bases = [gpu.forward(rng.integers(0, 8000, n), [], keep=True).snapshot for n in (5, 300, 900)]
    caches = [bases[2], None, bases[0], bases[1], bases[2], None]
    lens = [400, 70, 129, 64, 3, 250]
    ids = [rng.integers(0, 8000, n) for n in lens]
    rows = [_rows(n) for n in lens]
    outs, snaps = gpu.forward_batch(caches, ids, rows, keep=True)
    q = rng.integers(0, 8000, 20)
    for c, x, r, o, s in zip(caches, ids, rows, outs, snaps):
        ref = gpu.forward(x, r, cache=c, keep=True)
        _close(o, ref.hidden)
        assert s.len == (c.len if c is not None else 0) + len(x)
        _close(gpu.forward(q, [19], cache=s).hidden, gpu.forward(q, [19], cache=ref.snapshot).hidden)
        ref.snapshot.close()
        s.close()
    for b in bases:
        b.close()


def test_batch_of_short_sequences_keeps_snapshots(engines):
    """At most two chunks per sequence (the single-pass scan, final states stored per sequence)."""
    gpu, _ = engines
    rng = np.random.default_rng(42)
    base = gpu.forward(rng.integers(0, 8000, 77), [], keep=True).snapshot
    lens = [10, 128, 2, 64, 100]
    caches = [None, base, base, None, base]
    ids = [rng.integers(0, 8000, n) for n in lens]
    rows = [[n - 1] for n in lens]
    outs, snaps = gpu.forward_batch(caches, ids, rows, keep=True)
    q = rng.integers(0, 8000, 9)
    for c, x, r, o, s in zip(caches, ids, rows, outs, snaps):
        ref = gpu.forward(x, r, cache=c, keep=True)
        _close(o, ref.hidden)
        _close(gpu.forward(q, [8], cache=s).hidden, gpu.forward(q, [8], cache=ref.snapshot).hidden)
        ref.snapshot.close()
        s.close()
    base.close()


def test_batch_matches_oracle(engines):
    gpu, cpu = engines
    rng = np.random.default_rng(43)
    state = rng.integers(0, 8000, 60)
    base = gpu.forward(state, [], keep=True).snapshot
    ids = [rng.integers(0, 8000, 150), rng.integers(0, 8000, 90)]
    rows = [[0, 75, 149], [89]]
    outs, _ = gpu.forward_batch([None, base], ids, rows)
    _close(outs[0], cpu.forward(ids[0], rows[0])[0])
    _close(outs[1], cpu.forward(np.concatenate([state, ids[1]]), [60 + 89])[0])
    base.close()


def test_batch_dev_matches_host(engines):
    import torch
    gpu, _ = engines
    rng = np.random.default_rng(44)
    lens = [300, 40, 700]
    ids = [rng.integers(0, 8000, n) for n in lens]
    rows = [_rows(n) for n in lens]
    want, snaps_h = gpu.forward_batch(None, ids, rows, keep=True)
    ids_d = torch.from_numpy(np.concatenate(ids).astype(np.int32)).cuda()
    hid = torch.empty((sum(len(r) for r in rows), gpu.hidden_size()), dtype=torch.float32, device="cuda")
    snaps_d = gpu.forward_batch_dev(None, ids_d.data_ptr(), lens, rows, hid.data_ptr(), keep=True)
    gpu.synchronize()
    assert np.array_equal(hid.cpu().numpy(), np.concatenate(want))
    q = rng.integers(0, 8000, 12)
    for a, b in zip(snaps_h, snaps_d):
        assert np.array_equal(gpu.forward(q, [11], cache=a).hidden, gpu.forward(q, [11], cache=b).hidden)
        a.close()
        b.close()


def test_batch_errors(engines, small_model):
    from strands_decider.engine import Engine, Error
    gpu, _ = engines
    rng = np.random.default_rng(45)
    x = rng.integers(0, 8000, 10)
    with pytest.raises(Error):
        gpu.forward_batch(None, [x, x[:0]], [[9], []])  # an empty sequence
    with pytest.raises(Error):
        gpu.forward_batch(None, [x], [[10]])  # row past the sequence
    with pytest.raises(Error):
        gpu.forward_batch(None, [x, rng.integers(0, 8000, 5000)], [[9], [0]])  # past the context
    other = Engine.load(small_model)
    c = other.forward(x, [], keep=True).snapshot
    with pytest.raises(Error):
        gpu.forward_batch([None, c], [x, x], [[9], [9]])  # another engine's snapshot
    outs, snaps = gpu.forward_batch([None], [x], [[9]], keep=True)
    assert outs[0].shape == (1, gpu.hidden_size()) and snaps[0].len == 10
    snaps[0].close()
    c.close()
