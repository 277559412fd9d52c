"""Makes tests/golden/long_state_s0.npz: the oracle's answers for a 3000-token state and a question
continued from it on the full 24-layer synthetic model (seed 0), for the GPU parity test of long
states (tests/test_parity_configs.py). The oracle takes minutes on this length, longer than a GPU
test should, so its outputs are computed once here and committed.

    python tests/golden/make_long_state.py

The model directory is regenerated from its seed wherever the tests run; the fixture carries a
fingerprint of the model files so a test can tell that it checks against the same weights.
"""
import hashlib
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (ROOT, os.path.join(ROOT, "strands-decider-rs_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

STATE_LEN = 3000
STATE_ROWS = (1499, 2999)  # rows whose residual stream is kept after every layer
Q_LEN = 48
Q_ROWS = (20, 31, 40, 47)  # option rows and the answer row of the question
VOCAB_IDS = 240000  # ids drawn from [6003, VOCAB_IDS): above the synthetic tokenizer's added tokens
SEED = 3000


def fingerprint(path: str) -> str:
    """sha256 over the manifest, and the first and last MiB of the weight shard and the embedding."""
    h = hashlib.sha256()
    with open(os.path.join(path, "manifest.json"), "rb") as f:
        h.update(f.read())
    for name in ("weights.0.bin", "embed.bin"):
        with open(os.path.join(path, name), "rb") as f:
            h.update(f.read(1 << 20))
            f.seek(-(1 << 20), os.SEEK_END)
            h.update(f.read(1 << 20))
    return h.hexdigest()


def inputs():
    rng = np.random.default_rng(SEED)
    state = rng.integers(6003, VOCAB_IDS, STATE_LEN).astype(np.uint32)
    question = rng.integers(6003, VOCAB_IDS, Q_LEN).astype(np.uint32)
    return state, question


def main():
    from oracle import oracle
    from strands_decider import model
    path = model.ensure_model(os.path.join(ROOT, "_models", "full_s0"), seed=0)
    oracle.set_threads(os.cpu_count() or 1)
    eng = oracle.Engine(path)
    state, question = inputs()
    t0 = time.time()
    hidden_s, snap, tr = eng.forward(state, list(STATE_ROWS), keep=True, trace=True)
    trace_rows = np.ascontiguousarray(tr[:, list(STATE_ROWS), :])
    del tr
    t1 = time.time()
    hidden_q, _, trq = eng.forward(question, list(Q_ROWS), cache=snap, trace=True)
    trace_q = np.ascontiguousarray(trq[:, [Q_ROWS[-1]], :])
    tensors = model.read_safetensors(os.path.join(path, "head.safetensors"))
    probs = oracle.head_probs(hidden_q, tensors, 1.0)
    # the oracle's own drift under a change of its f32 summation order (the floor of any comparison)
    oracle.set_sum_reversed(True)
    _, snap_r, tr_r = eng.forward(state, list(STATE_ROWS), keep=True, trace=True)
    drift_state = np.abs(tr_r[:, list(STATE_ROWS), :] - trace_rows).max(axis=(1, 2))
    del tr_r
    hidden_q_r, _, trq_r = eng.forward(question, list(Q_ROWS), cache=snap_r, trace=True)
    drift_q = np.abs(trq_r[:, [Q_ROWS[-1]], :] - trace_q).max(axis=(1, 2))
    drift_p = float(np.abs(oracle.head_probs(hidden_q_r, tensors, 1.0) - probs).max())
    oracle.set_sum_reversed(False)
    t2 = time.time()
    out = os.path.join(HERE, "long_state_s0.npz")
    np.savez_compressed(out, fingerprint=np.array(fingerprint(path)), state=state, question=question,
                        state_rows=np.array(STATE_ROWS, np.int32), q_rows=np.array(Q_ROWS, np.int32),
                        hidden_state=hidden_s, trace_state=trace_rows, hidden_q=hidden_q, trace_q=trace_q, probs=probs,
                        drift_state=drift_state.astype(np.float32), drift_q=drift_q.astype(np.float32),
                        drift_p=np.float32(drift_p))
    print(f"state forward {t1 - t0:.0f} s, question and drift {t2 - t1:.0f} s -> {out} ({os.path.getsize(out) / 1e3:.0f} KB); "
          f"sum-order drift at the last layer {drift_state[-1]:.2e} (state), {drift_q[-1]:.2e} (question); "
          f"of the probabilities {drift_p:.2e}")


if __name__ == "__main__":
    main()
