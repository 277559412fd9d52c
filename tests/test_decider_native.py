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
