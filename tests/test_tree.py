"""The tree pass (`sd_forward_tree`, `sd_forward_tree_probs`): a request's state and its questions in one
packed pass, each question continuing its state within the same launch sequence, against the two
passes it replaces (`Engine::forward` of the state kept as a snapshot, then each question continued
from it: the question loop of `Decider::ask_all`, `src/lib.rs:192-198`) and against the CPU oracle.
Tolerances as the per-layer parity target: 2e-2 max-abs on the hidden rows, 1e-3 on probabilities
with the same argmax."""
import os

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engines(small_model):
    from strands_decider.engine import Engine
    return Engine.load(small_model), oracle.Engine(small_model)


def _rows(n):
    return sorted({0, n // 2, n - 1})


def test_tree_matches_state_then_fork(engines):
    """Three requests in one call: fresh states of 40, 300 and 1000 tokens (the longest several
    64-token chunks and 128-query blocks), each with questions of lengths around the chunk and block
    boundaries; one request has no questions. Every row equals the state's kept snapshot continued by
    the question on its own, and the states' own rows equal their plain forwards."""
    gpu, _ = engines
    rng = np.random.default_rng(31)
    states = [rng.integers(0, 8000, n) for n in (40, 300, 1000)]
    qlens = {0: [5, 64], 1: [1, 65, 30], 2: []}
    seqs, parents, rows = [], [], []
    for s in states:
        seqs.append(s), parents.append(-1), rows.append(_rows(len(s)))
    for r, ls in qlens.items():
        for n in ls:
            seqs.append(rng.integers(0, 8000, n)), parents.append(r), rows.append(_rows(n))
    got = gpu.forward_tree(None, parents, seqs, rows)
    for b in range(3):
        want = gpu.forward(seqs[b], rows[b]).hidden
        assert np.abs(got[b] - want).max() < 2e-2
    snaps = [gpu.forward(s, [], keep=True).snapshot for s in states]
    for b in range(3, len(seqs)):
        want = gpu.forward(seqs[b], rows[b], cache=snaps[parents[b]]).hidden
        assert got[b].shape == want.shape
        assert np.abs(got[b] - want).max() < 2e-2
    for s in snaps:
        s.close()


def test_tree_from_snapshots_matches_oracle(engines):
    """Roots that continue snapshots themselves (a second turn of a conversation), their questions
    after them, against the oracle's full forward of snapshot + root + question."""
    gpu, cpu = engines
    rng = np.random.default_rng(32)
    prefixes = [rng.integers(0, 8000, n) for n in (70, 150)]
    snaps = [gpu.forward(p, [], keep=True).snapshot for p in prefixes]
    roots = [rng.integers(0, 8000, n) for n in (20, 90)]
    qs = [rng.integers(0, 8000, n) for n in (17, 40, 70)]
    par = [-1, -1, 0, 1, 1]
    seqs = roots + qs
    rows = [[], [89]] + [_rows(len(q)) for q in qs]
    got = gpu.forward_tree(snaps + [None] * 3, par, seqs, rows)
    assert got[0].shape == (0, gpu.hidden_size())
    full1 = np.concatenate([prefixes[1], roots[1]])
    assert np.abs(got[1] - cpu.forward(full1, [len(full1) - 1])[0]).max() < 2e-2
    for b in range(2, 5):
        r = par[b]
        full = np.concatenate([prefixes[r], roots[r], seqs[b]])
        want = cpu.forward(full, [len(full) - len(seqs[b]) + i for i in rows[b]])[0]
        assert np.abs(got[b] - want).max() < 2e-2
    for s in snaps:
        s.close()


def test_tree_probs_match_fork_probs(engines, small_model):
    """sd_forward_tree_probs (one pass and the pointer head on the GPU) against the state pass plus
    sd_forward_fork_multi_probs, the path it replaces: 1e-3, same argmax; the snapshots given to the
    roots are left unchanged."""
    from strands_decider.engine import Head
    gpu, _ = engines
    head = Head.load(os.path.join(small_model, "head.safetensors"))
    rng = np.random.default_rng(33)
    states = [rng.integers(0, 8000, n) for n in (130, 257)]
    qs, par, qrows, temps = [], [], [], []
    for r, ls in enumerate([[30, 45, 24], [33, 48]]):
        for n in ls:
            qs.append(rng.integers(0, 8000, n)), par.append(r)
            qrows.append([n // 3, 2 * n // 3, n - 1]), temps.append(1.0 + 0.25 * len(qs))
    got = gpu.forward_tree_probs(None, [-1, -1] + par, states + qs, [[], []] + qrows, head, [1.0, 1.0] + temps)
    snaps = [gpu.forward(s, [], keep=True).snapshot for s in states]
    want = gpu.forward_fork_probs([snaps[r] for r in par], qs, qrows, head, temps)
    assert len(got) == len(want) == len(qs)
    for a, b in zip(got, want):
        assert np.abs(a - b).max() < 1e-3 and np.argmax(a) == np.argmax(b)
    for s in snaps:
        s.close()


def test_tree_errors(engines):
    from strands_decider.engine import Error
    gpu, _ = engines
    rng = np.random.default_rng(34)
    a, b, c = (rng.integers(0, 8000, n) for n in (20, 10, 5))
    snap = gpu.forward(a, [], keep=True).snapshot
    with pytest.raises(Error):
        gpu.forward_tree(None, [1, -1], [a, b], [[0], [0]])  # a parent after its child
    with pytest.raises(Error):
        gpu.forward_tree(None, [-1, 0, 1], [a, b, c], [[0], [0], [0]])  # a child of a child
    with pytest.raises(Error):
        gpu.forward_tree([None, snap], [-1, 0], [a, b], [[0], [0]])  # a child with a snapshot too
    with pytest.raises(Error):
        gpu.forward_tree(None, [-1, 0], [a, rng.integers(0, 8000, 4080)], [[0], [0]])  # past the context
    # the engine still works after the rejected calls
    got = gpu.forward_tree(None, [-1, 0], [a, b], [[19], [9]])
    assert np.abs(got[1] - gpu.forward(b, [9], cache=snap).hidden).max() < 2e-2
    snap.close()
