"""GPU parity on exactly what the bench measures: the 24-layer model, the benchmark configurations'
shapes, and a long state. The reference's own invariants (`tests/engine_parity.rs:16-85`: the same
top answer, |dp| < 0.01, prefix forward == full forward) and this build's targets: answer
probabilities within 2e-3 with the same argmax, kernels as in tests/test_gpu_parity.py (attention
outputs within 4e-3; the chunked gated-delta scan within 5e-3 relative), and the residual stream after
every layer within 2e-2 max-abs of the oracle, or within DRIFT_FACTOR (3) times the oracle's own
drift where that is larger (and the probabilities of the 24-layer model likewise within 2e-3, or 3
times the oracle's drift of them).

The drift: this random-init 24-layer model carries any f16-level perturbation forward and grows it
layer by layer. The oracle with nothing changed but the order of its f32 matmul sums
(`oracle.set_sum_reversed`) moves 2.3e-2 max-abs away from itself by layer 24, so past the first
dozen layers 2e-2 is below what any implementation that is not bit-identical to the reference's
summation order can reach. Each 24-layer test measures that drift on its own inputs and bounds layer
i by max(2e-2, 3 x drift_i).

Each test prints the worst error it saw (pytest -rP shows it)."""
import os

import numpy as np
import pytest

from oracle import oracle
from strands_decider import model as M

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
LAYER_TOL = 2e-2
# The reference's own parity test of probabilities between two implementations allows 0.01
# (tests/engine_parity.rs:55); the probabilities here must agree within 2e-3, or DRIFT_FACTOR times
# the oracle's own drift where that is larger. One question's probabilities move by up to ~1.5e-3
# between GPU builds that differ only in f16 rounding points (each within the per-layer bounds), while
# the oracle's single reordering moved them by 4e-4 to 1.7e-3: one perturbation's size is a noisy
# estimate of the spread.
PROB_TOL = 2e-3
# How many times the oracle's own sum-order drift a comparison may reach: the GPU path differs from
# the oracle in several independent f16-level ways (every GEMM's summation order, attention's f16
# probabilities, the chunked scan's operands), each of about the size of one such reordering, and
# independent perturbations of one size add up to about the square root of their count times it.
DRIFT_FACTOR = 3.0


@pytest.fixture(scope="module")
def torch():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def layer_bound(drift):
    """Per-layer bound on |GPU - oracle|: 2e-2, or DRIFT_FACTOR times the oracle's own sum-order drift."""
    return np.maximum(LAYER_TOL, DRIFT_FACTOR * np.asarray(drift))


@pytest.fixture(scope="module")
def full(full_model):
    oracle.set_threads(os.cpu_count() or 1)
    return full_model, oracle.Engine(full_model)


WORDS = ("payout", "failing", "account", "billing", "urgent", "refund", "customer", "support", "invoice", "delay",
         "error", "card", "bank", "transfer", "status", "pending", "help", "days", "please", "order", "ticket",
         "escalate", "charge", "merchant", "dashboard", "settings", "email", "phone", "reply", "waiting")


def _state_text(tokenizer, n_tokens, seed):
    """A state of random words whose rendering is n_tokens tokens or just over."""
    from strands_decider import prompt
    rng = np.random.default_rng(seed)
    words = []
    while len(tokenizer.encode(prompt.render_state(" ".join(words))).ids) < n_tokens:
        words.append(WORDS[int(rng.integers(len(WORDS)))])
    return " ".join(words)


def test_config1_ask_all_on_the_24_layer_model(full):
    """Config 1: `Decider::ask_all` (`src/lib.rs:141-198`) on a 128-token state with three questions
    (noul; choice over 3; score over 3) through the GPU engine, against the same pipeline through the
    oracle: every layer's residual stream of the state and of each question continued from the
    state's snapshot, then the answers."""
    from strands_decider import Decider, Question
    from strands_decider import prompt
    path, cpu = full
    dec = Decider.load(path)
    state = _state_text(dec.tokenizer, 128, seed=1)
    qs = [Question.noul("Does this convey urgency?"),
          Question.choice("Which team should handle this?", ["billing", "technical", "sales"]),
          Question.score("How frustrated is the writer?", ["calm", "frustrated", "very angry"])]
    answers = dec.ask_all(state, qs)
    rendered, sids, qencs, options = dec.encode(state, [(str(i), q) for i, q in enumerate(qs)])
    assert 128 <= len(sids) <= 132
    gpu = dec.engine
    tensors = M.read_safetensors(os.path.join(path, "head.safetensors"))

    out = gpu.forward(sids, [len(sids) - 1], keep=True, trace=True)
    _, snap, tr = cpu.forward(sids, [len(sids) - 1], keep=True, trace=True)
    oracle.set_sum_reversed(True)
    try:
        _, snap_r, tr_r = cpu.forward(sids, [len(sids) - 1], keep=True, trace=True)
        drift, drift_p = [np.abs(tr_r - tr).max(axis=(1, 2))], []
        for i, q in enumerate(qencs):
            rows = list(options[i]) + [len(q.ids) - 1]
            h_r, _, t_r = cpu.forward(q.ids, rows, cache=snap_r, trace=True)
            oracle.set_sum_reversed(False)
            h_f, _, t_f = cpu.forward(q.ids, rows, cache=snap, trace=True)
            oracle.set_sum_reversed(True)
            drift.append(np.abs(t_r - t_f).max(axis=(1, 2)))
            temp = dec._temperature(rendered[i])
            drift_p.append(float(np.abs(oracle.head_probs(h_r, tensors, temp) - oracle.head_probs(h_f, tensors, temp)).max()))
    finally:
        oracle.set_sum_reversed(False)
    worst_layer = np.abs(out.trace - tr).max(axis=(1, 2))
    assert (worst_layer < layer_bound(drift[0])).all(), (worst_layer, drift[0])
    worst_p = 0.0
    for i, (q, a) in enumerate(zip(qencs, answers)):
        rows = list(options[i]) + [len(q.ids) - 1]
        got = gpu.forward(q.ids, rows, cache=out.snapshot, trace=True)
        want_h, _, want_tr = cpu.forward(q.ids, rows, cache=snap, trace=True)
        per_layer = np.abs(got.trace - want_tr).max(axis=(1, 2))
        worst_layer = np.maximum(worst_layer, per_layer)
        assert (per_layer < layer_bound(drift[i + 1])).all(), (i, per_layer, drift[i + 1])
        want_p = oracle.head_probs(want_h, tensors, dec._temperature(rendered[i]))
        got_p = dec.head.probs(got.hidden, 2048, dec._temperature(rendered[i]))
        p_tol = max(PROB_TOL, DRIFT_FACTOR * drift_p[i])
        worst_p = max(worst_p, float(np.abs(got_p - want_p).max()))
        assert np.abs(got_p - want_p).max() < p_tol, (i, got_p, want_p, drift_p[i])
        assert np.argmax(got_p) == np.argmax(want_p)
        want = prompt.to_answer(rendered[i], want_p, dec.cfg["ordinal_smoothing"])
        gp = dict(a.probabilities) if a.probabilities else {"true": a.noul}
        wp = dict(want.probabilities) if want.probabilities else {"true": want.noul}
        for kk in wp:
            assert abs(gp[kk] - wp[kk]) <= p_tol + 1e-4, (kk, gp, wp, drift_p[i])  # answers carry 4 decimals
        if a.kind == "choice":
            assert a.choice == want.choice
    out.snapshot.close()
    d = np.maximum.reduce(drift)
    print(f"config 1 (24 layers, {len(sids)}-token state, 3 questions): worst per-layer max-abs "
          f"{worst_layer.max():.2e} (layer {int(worst_layer.argmax())}; the oracle's sum-order drift there "
          f"{d[int(worst_layer.argmax())]:.2e}, at layer 12 {worst_layer[11]:.2e} vs {d[11]:.2e}), worst |dp| {worst_p:.2e} "
          f"(the oracle's sum-order drift of the probabilities: {max(drift_p):.2e})")


def test_config2_attention_exact_shape(torch):
    """Config 2: B=4, S=2048, 8 query / 2 KV heads x 256, causal and gated, one sd_attention_batch
    launch, against the oracle's attention per sequence (`src/kernels.rs:453-541`)."""
    from strands_decider.engine import attention_batch
    B, S, hq, hk, hd = 4, 2048, 8, 2, 256
    rng = np.random.default_rng(2)
    q = rng.standard_normal((B, hq, S, hd)).astype(np.float16)
    k = rng.standard_normal((B, hk, S, hd)).astype(np.float16)
    v = rng.standard_normal((B, hk, S, hd)).astype(np.float16)
    gw = hq * 2 * hd
    gate = rng.standard_normal((B, S, gw)).astype(np.float16)
    qd, kd, vd, gd = (dev(torch, x.view(np.uint16)) for x in (q, k, v, gate))
    out = torch.zeros((B, S, hq * hd), dtype=torch.float16, device="cuda")
    attention_batch(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), gd.data_ptr(), gw, hd, 2 * hd, out.data_ptr(), B, S, 0, S,
                    hq, hk, hd)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float32)
    worst = 0.0
    for b in range(B):
        want = oracle.attn(q[b], k[b], v[b], gate[b], gw, hd, 2 * hd).astype(np.float32)
        err = float(np.abs(got[b] - want).max())
        worst = max(worst, err)
        assert np.isfinite(got[b]).all() and err < 4e-3, (b, err)
    print(f"config 2 (B=4, S=2048): worst |out - oracle| {worst:.2e}")


def _config3_inputs():
    B, L, H = 16, 1024, 16
    rng = np.random.default_rng(3)
    q = rng.standard_normal((B, L, H, 128)).astype(np.float32)
    k = rng.standard_normal((B, L, H, 128)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, L, H, 128)).astype(np.float32)
    q, k, v = (x.astype(np.float16) for x in (q, k, v))
    beta = (1 / (1 + np.exp(-rng.standard_normal((B, L, H))))).astype(np.float32)
    g = (-np.log1p(np.exp(rng.standard_normal((B, L, H))))).astype(np.float32)
    return q, k, v, beta, g


def test_config3_gdn_exact_shape(torch):
    """Config 3: B=16, L=1024, 16 heads of 128 x 128, f16 q/k/v (q, k L2-normalised N(0,1), v N(0,1)),
    beta = sigmoid(N(0,1)), g = -softplus(N(0,1)), the final state written, through sd_gdn, against
    the oracle's token-serial recurrence (`src/kernels.rs:257-302`) per sequence."""
    from strands_decider.engine import gdn
    q, k, v, beta, g = _config3_inputs()
    B, L, H = beta.shape
    qd, kd, vd, bd, gd = (dev(torch, x) for x in (q, k, v, beta, g))
    st = torch.zeros((B, H, 128, 128), dtype=torch.float32, device="cuda")
    od = torch.zeros((B, L, H * 128), dtype=torch.float32, device="cuda")
    gdn(qd.data_ptr(), kd.data_ptr(), H * 128, vd.data_ptr(), H * 128, bd.data_ptr(), gd.data_ptr(), st.data_ptr(), False,
        od.data_ptr(), L, H, batch=B, seq_qk=L * H * 128, seq_v=L * H * 128, in_f16=True)
    torch.cuda.synchronize()
    got_o, got_s = od.cpu().numpy(), st.cpu().numpy()
    worst = 0.0
    for b in range(B):
        o_want, s_want = oracle.gdn(q[b].astype(np.float32), k[b].astype(np.float32), v[b].astype(np.float32), beta[b],
                                    np.exp(g[b]), None)
        eo = np.linalg.norm(got_o[b] - o_want) / np.linalg.norm(o_want)
        es = np.linalg.norm(got_s[b] - s_want) / np.linalg.norm(s_want)
        worst = max(worst, eo, es)
        assert eo < 5e-3 and es < 5e-3, (b, eo, es)
    print(f"config 3 (B=16, L=1024): worst relative error of outputs and final states {worst:.2e}")


@pytest.fixture(scope="module")
def long_state(full_model):
    import sys
    sys.path.insert(0, os.path.join(HERE, "golden"))
    from make_long_state import fingerprint
    fx = dict(np.load(os.path.join(HERE, "golden", "long_state_s0.npz")))
    assert str(fx["fingerprint"]) == fingerprint(full_model), "the model files differ from the fixture's"
    return fx


def test_long_state_and_continuation_match_fixture(full_model, long_state):
    """A 3000-token state and a 48-token question continued from its snapshot on the 24-layer model,
    against the oracle's outputs committed in tests/golden/long_state_s0.npz (make_long_state.py):
    the state's residual stream after every layer at two rows (sd_forward), the same state through
    sd_forward_batch (packed, kept as a snapshot) and the question through sd_forward_fork_multi, and
    the pointer head's probabilities on the GPU."""
    from strands_decider.engine import Engine, Head
    fx = long_state
    gpu = Engine.load(full_model)
    state, question = fx["state"], fx["question"]
    srows, qrows = fx["state_rows"].tolist(), fx["q_rows"].tolist()
    out = gpu.forward(state, srows, trace=True)
    per_layer = np.abs(out.trace[:, srows, :] - fx["trace_state"]).max(axis=(1, 2))
    bound_s, bound_q = layer_bound(fx["drift_state"]), layer_bound(fx["drift_q"])
    assert (per_layer < bound_s).all(), (per_layer, fx["drift_state"])
    assert np.abs(out.hidden - fx["hidden_state"]).max() < bound_s[-1]
    del out
    hid, snaps = gpu.forward_batch(None, [state], [srows], keep=True)
    assert np.abs(hid[0] - fx["hidden_state"]).max() < bound_s[-1]
    got_q = gpu.forward_fork([snaps[0]], [question], [qrows])[0]
    err_q = float(np.abs(got_q - fx["hidden_q"]).max())
    assert err_q < bound_q[-1]
    qt = gpu.forward(question, qrows, cache=snaps[0], trace=True)
    per_layer_q = np.abs(qt.trace[:, [qrows[-1]], :] - fx["trace_q"]).max(axis=(1, 2))
    assert (per_layer_q < bound_q).all(), (per_layer_q, fx["drift_q"])
    head = Head.load(os.path.join(full_model, "head.safetensors"))
    probs = gpu.forward_fork_probs([snaps[0]], [question], [qrows], head, 1.0)[0]
    dp = float(np.abs(probs - fx["probs"]).max())
    p_tol = max(PROB_TOL, DRIFT_FACTOR * float(fx["drift_p"]))
    assert dp < p_tol and np.argmax(probs) == np.argmax(fx["probs"]), (dp, float(fx["drift_p"]))
    snaps[0].close()
    gpu.close()
    print(f"3000-token state (24 layers): worst per-layer max-abs {per_layer.max():.2e} (state rows; the oracle's "
          f"sum-order drift {fx['drift_state'].max():.2e}), {per_layer_q.max():.2e} (question; drift "
          f"{fx['drift_q'].max():.2e}); fork hidden {err_q:.2e}; |dp| {dp:.2e} (drift {float(fx['drift_p']):.2e})")
