"""sd_decider_ask_all (the C++ Decider in the library) against the Python Decider on the same model:
the same System One requests give the same response bodies (both drive the same engine and head)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_native_decider_matches_python(small_model):
    from strands_decider import Decider, NativeDecider, Request
    py = Decider.load(small_model)
    nat = NativeDecider.load(small_model)
    requests = [
        {"state": "Help! My payouts have been failing for 3 days!",
         "questions": {"urgent": {"type": "noul", "instructions": "Does this convey urgency?"}}},
        {"state": {"ticket": 4812, "text": "Refund please — charged twice", "amount": 12.5, "tags": ["billing", None]},
         "questions": {"team": {"type": "choice", "instructions": "Which team should handle this?",
                                "criteria": {"billing": "money", "technical": "", "sales": None}},
                       "mood": {"type": "score", "instructions": "How upset is the customer?",
                                "criteria": ["calm", "annoyed", "furious"]},
                       "urgent": {"instructions": "Is it urgent?"}}},
    ]
    for req in requests:
        want = py.evaluate(Request.from_json(req)).to_json()
        got = nat.ask_all(req)
        assert got == want
    with pytest.raises(Exception, match="questions must be a non-empty object"):
        nat.ask_all({"state": "x", "questions": {}})
    nat.close()


def _close_answers(a, b, tol=3e-3):
    """Two response bodies from different batchings: same keys, labels and choices, numbers within tol.
    A request alone and the same request in a packed batch can take different gated-delta kernels (the
    fused scan or the two-phase one, chosen per layer by the batch's shape), whose f16 rounding points
    differ; each is checked against the oracle on its own."""
    assert a.keys() == b.keys()
    assert a["model"] == b["model"] and a["usage"] == b["usage"]
    for name in a["answers"]:
        x, y = a["answers"][name], b["answers"][name]
        assert x.keys() == y.keys() and x["type"] == y["type"]
        for k in x:
            if isinstance(x[k], float):
                assert abs(x[k] - y[k]) <= tol, (name, k)
            elif k == "probabilities":
                assert x[k].keys() == y[k].keys()
                assert max(abs(x[k][o] - y[k][o]) for o in x[k]) <= tol
            elif k != "choice":
                assert x[k] == y[k], (name, k)


def test_native_decider_batch_matches_one_by_one(small_model):
    """sd_decider_ask_batch: many requests (one question, several, invalid ones) in packed passes give
    each request's own ask_all answers; the failures come back in place as {"error": ...}."""
    from strands_decider import NativeDecider
    nat = NativeDecider.load(small_model)
    rng = np.random.default_rng(7)
    words = ["payout", "refund", "charged", "twice", "help", "urgent", "billing", "login", "error", "slow", "café", "日本"]
    qs = {"urgent": {"type": "noul", "instructions": "Does this convey urgency?"},
          "team": {"type": "choice", "instructions": "Which team?", "criteria": {"billing": "money", "tech": "", "sales": None}},
          "mood": {"type": "score", "instructions": "How upset?", "criteria": ["calm", "annoyed", "furious"]}}
    requests = []
    for i in range(10):
        state = " ".join(rng.choice(words, int(rng.integers(3, 400))))
        names = list(qs)[: 1 + i % 3]
        requests.append({"state": state, "questions": {n: qs[n] for n in names}})
    requests.insert(3, {"state": "x", "questions": {}})
    requests.insert(7, {"state": 5, "questions": qs})
    requests.append({"state": "word " * 5000, "questions": qs})  # past the context window
    got = nat.ask_batch(requests)
    assert len(got) == len(requests)
    for req, g in zip(requests, got):
        try:
            want = nat.ask_all(req)
        except Exception as e:
            assert g == {"error": str(e)}
            continue
        _close_answers(g, want)
    assert nat.ask_batch([]) == []
    with pytest.raises(Exception, match="JSON array"):
        nat.ask_batch({"state": "x"})
    nat.close()


def test_native_decider_batch_spans_several_passes(small_model):
    """Twenty requests of ~3500-token states (over 65536 tokens in all, so the states run in more
    than one packed pass) and one to three questions each, prepared on host threads: every
    request's answers match its own ask_all."""
    from strands_decider import NativeDecider
    nat = NativeDecider.load(small_model)
    rng = np.random.default_rng(11)
    words = ["payout", "refund", "charged", "twice", "help", "urgent", "billing", "login", "error", "slow"]
    qs = {"urgent": {"type": "noul", "instructions": "Does this convey urgency?"},
          "team": {"type": "choice", "instructions": "Which team?", "criteria": {"billing": "money", "tech": "", "sales": None}},
          "mood": {"type": "score", "instructions": "How upset?", "criteria": ["calm", "annoyed", "furious"]}}
    requests = []
    for i in range(20):
        state = " ".join(rng.choice(words, 1300))
        names = list(qs)[: 1 + i % 3]
        requests.append({"state": state, "questions": {n: qs[n] for n in names}})
    got = nat.ask_batch(requests)
    assert sum(g["usage"]["input_tokens"] for g in got) > 65536
    for req, g in zip(requests, got):
        _close_answers(g, nat.ask_all(req))
    nat.close()
