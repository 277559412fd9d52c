"""The batched fork (`sd_forward_fork`) against the serial loop it replaces (`Decider::ask_all`,
`src/lib.rs:192-198`: one `Engine::forward(ids, rows, Some(&snapshot), ..)` per question) and against
the CPU oracle. Questions of lengths around the 64-token chunk and attention-block boundaries are
packed together; tolerance as the per-layer parity target (2e-2 max-abs on the hidden rows)."""
import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engines(small_model):
    from strands_decider.engine import Engine
    return Engine.load(small_model), oracle.Engine(small_model)


def _questions(rng, lens):
    qs = [rng.integers(0, 8000, n) for n in lens]
    rows = [sorted(set([0, n // 2, n - 1])) for n in lens]
    return qs, rows


def test_fork_matches_serial_continuations(engines):
    gpu, _ = engines
    rng = np.random.default_rng(21)
    snap = gpu.forward(rng.integers(0, 8000, 300), [], keep=True).snapshot
    qs, rows = _questions(rng, [1, 5, 30, 63, 64, 65, 100, 130])
    got = gpu.forward_fork(snap, qs, rows)
    for q, r, g in zip(qs, rows, got):
        want = gpu.forward(q, r, cache=snap).hidden
        assert g.shape == want.shape
        assert np.abs(g - want).max() < 2e-2
    snap.close()


def test_fork_up_to_the_context_limit(engines):
    """Questions after a 4000-token snapshot, the longest ending exactly at the 4096-token context:
    the batched fork equals the serial continuations and, for the longest, the full forward."""
    gpu, _ = engines
    rng = np.random.default_rng(23)
    state = rng.integers(0, 8000, 4000)
    snap = gpu.forward(state, [], keep=True).snapshot
    qs, rows = _questions(rng, [96, 50, 130 - 34, 1])
    got = gpu.forward_fork(snap, qs, rows)
    for q, r, g in zip(qs, rows, got):
        assert np.abs(g - gpu.forward(q, r, cache=snap).hidden).max() < 2e-2
    full = gpu.forward(np.concatenate([state, qs[0]]), [4000 + i for i in rows[0]]).hidden
    assert np.abs(got[0] - full).max() < 2e-2
    snap.close()


def test_fork_matches_oracle(engines):
    gpu, cpu = engines
    rng = np.random.default_rng(22)
    state = rng.integers(0, 8000, 90)
    snap = gpu.forward(state, [], keep=True).snapshot
    qs, rows = _questions(rng, [17, 70])
    got = gpu.forward_fork(snap, qs, rows)
    for q, r, g in zip(qs, rows, got):
        want = cpu.forward(np.concatenate([state, q]), [len(state) + i for i in r])[0]
        assert np.abs(g - want).max() < 2e-2
    snap.close()


def test_fork_leaves_the_snapshot_unchanged(engines):
    gpu, _ = engines
    rng = np.random.default_rng(23)
    snap = gpu.forward(rng.integers(0, 8000, 120), [], keep=True).snapshot
    q = rng.integers(0, 8000, 40)
    before = gpu.forward(q, [39], cache=snap).hidden
    qs, rows = _questions(rng, [33, 80, 12])
    gpu.forward_fork(snap, qs, rows)
    after = gpu.forward(q, [39], cache=snap).hidden
    assert np.array_equal(before, after)
    snap.close()


def test_fork_config4_shapes(engines):
    """Config 4: a 512-token state, 64 questions of 24-48 tokens from one snapshot."""
    gpu, _ = engines
    rng = np.random.default_rng(24)
    snap = gpu.forward(rng.integers(0, 8000, 512), [], keep=True).snapshot
    lens = rng.integers(24, 49, 64)
    qs = [rng.integers(0, 8000, n) for n in lens]
    rows = [[n - 1] for n in lens]
    got = gpu.forward_fork(snap, qs, rows)
    assert len(got) == 64
    for i in rng.choice(64, 8, replace=False):
        want = gpu.forward(qs[i], rows[i], cache=snap).hidden
        assert np.abs(got[i] - want).max() < 2e-2
    snap.close()


def test_fork_dev_matches_host(engines):
    """sd_forward_fork_dev (ids on the GPU, rows to device memory, asynchronous) back to back."""
    import torch
    gpu, _ = engines
    rng = np.random.default_rng(26)
    snap = gpu.forward(rng.integers(0, 8000, 200), [], keep=True).snapshot
    outs = []
    for lens in ([12, 70, 3], [64, 65], [40] * 9):
        qs, rows = _questions(rng, lens)
        want = np.concatenate(gpu.forward_fork(snap, qs, rows))
        ids_d = torch.from_numpy(np.concatenate(qs).astype(np.int32)).cuda()
        hid = torch.empty((len(want), gpu.hidden_size()), dtype=torch.float32, device="cuda")
        outs.append((want, ids_d, hid))
        gpu.forward_fork_dev(snap, ids_d.data_ptr(), lens, rows, hid.data_ptr())
    gpu.synchronize()
    for want, _, hid in outs:
        assert np.array_equal(hid.cpu().numpy(), want)
    snap.close()


def test_fork_errors(engines, small_model):
    from strands_decider.engine import Engine, Error, Snapshot
    gpu, _ = engines
    rng = np.random.default_rng(25)
    snap = gpu.forward(rng.integers(0, 8000, 50), [], keep=True).snapshot
    q = rng.integers(0, 8000, 10)
    with pytest.raises(Error):
        gpu.forward_fork(snap, [q], [[10]])  # row past the question
    with pytest.raises(Error):
        gpu.forward_fork(snap, [q, q[:0]], [[9], []])  # an empty question
    with pytest.raises(Error):
        gpu.forward_fork(Snapshot(None), [q], [[9]])  # no snapshot
    with pytest.raises(Error):
        gpu.forward_fork(snap, [q, rng.integers(0, 8000, 4096)], [[9], [0]])  # past the context
    other = Engine.load(small_model)
    with pytest.raises(Error):
        other.forward_fork(snap, [q], [[9]])  # another engine's snapshot
    # the engine still works after the rejected calls
    assert gpu.forward_fork(snap, [q], [[9]])[0].shape == (1, gpu.hidden_size())
    snap.close()


def test_fork_across_snapshots_matches_serial(engines):
    """sd_forward_fork_multi: questions of several requests (snapshots of 3 to 1100 tokens, the
    longest with its keys split across CTAs) in one pass, interleaved, each equal to its own serial
    continuation."""
    gpu, _ = engines
    rng = np.random.default_rng(27)
    snaps = [gpu.forward(rng.integers(0, 8000, n), [], keep=True).snapshot for n in (3, 64, 300, 1100)]
    order = [2, 0, 3, 1, 2, 3, 0, 1, 3]
    qs, rows = _questions(rng, [5, 63, 64, 65, 1, 130, 30, 12, 77])
    got = gpu.forward_fork([snaps[i] for i in order], qs, rows)
    for i, q, r, g in zip(order, qs, rows, got):
        want = gpu.forward(q, r, cache=snaps[i]).hidden
        assert g.shape == want.shape
        assert np.abs(g - want).max() < 2e-2
    # the same questions through one call per snapshot agree (a batch of another size takes other
    # GEMM split-K and attention key-split plans, so f32 summation orders differ: parity tolerance)
    for s in range(4):
        idx = [j for j, i in enumerate(order) if i == s]
        one = gpu.forward_fork(snaps[s], [qs[j] for j in idx], [rows[j] for j in idx])
        for j, g in zip(idx, one):
            assert np.abs(g - got[j]).max() < 2e-2
    for s in snaps:
        s.close()


def test_fork_across_snapshots_matches_oracle(engines):
    gpu, cpu = engines
    rng = np.random.default_rng(28)
    states = [rng.integers(0, 8000, n) for n in (40, 150)]
    snaps = [gpu.forward(s, [], keep=True).snapshot for s in states]
    qs, rows = _questions(rng, [20, 66, 9])
    order = [1, 0, 1]
    got = gpu.forward_fork([snaps[i] for i in order], qs, rows)
    for i, q, r, g in zip(order, qs, rows, got):
        want = cpu.forward(np.concatenate([states[i], q]), [len(states[i]) + k for k in r])[0]
        assert np.abs(g - want).max() < 2e-2
    for s in snaps:
        s.close()


def test_fork_across_snapshots_dev_matches_host(engines):
    import torch
    gpu, _ = engines
    rng = np.random.default_rng(29)
    snaps = [gpu.forward(rng.integers(0, 8000, n), [], keep=True).snapshot for n in (100, 700)]
    qs, rows = _questions(rng, [50, 3, 90, 64])
    caches = [snaps[0], snaps[1], snaps[1], snaps[0]]
    want = np.concatenate(gpu.forward_fork(caches, qs, rows))
    ids_d = torch.from_numpy(np.concatenate(qs).astype(np.int32)).cuda()
    hid = torch.empty((len(want), gpu.hidden_size()), dtype=torch.float32, device="cuda")
    gpu.forward_fork_dev(caches, ids_d.data_ptr(), [len(q) for q in qs], rows, hid.data_ptr())
    gpu.synchronize()
    assert np.array_equal(hid.cpu().numpy(), want)
    for s in snaps:
        s.close()


def test_fork_across_snapshots_errors(engines, small_model):
    from strands_decider.engine import Engine, Error, Snapshot
    gpu, _ = engines
    rng = np.random.default_rng(30)
    a = gpu.forward(rng.integers(0, 8000, 50), [], keep=True).snapshot
    b = gpu.forward(rng.integers(0, 8000, 4000), [], keep=True).snapshot
    q = rng.integers(0, 8000, 10)
    with pytest.raises(Error):
        gpu.forward_fork([a, Snapshot(None)], [q, q], [[9], [9]])  # one question without a snapshot
    with pytest.raises(Error):
        gpu.forward_fork([a, b], [q, rng.integers(0, 8000, 200)], [[9], [0]])  # past the context of b
    other = Engine.load(small_model)
    c = other.forward(q, [], keep=True).snapshot
    with pytest.raises(Error):
        gpu.forward_fork([a, c], [q, q], [[9], [9]])  # another engine's snapshot
    assert len(gpu.forward_fork([a, b], [q, q[:5]], [[9], [4]])) == 2
    for s in (a, b, c):
        s.close()
