"""Prompt rendering and answer formulas against the reference's fixtures and unit tests.

Golden data: tests/golden/prompt_cases.json, extracted by tests/golden/make_golden.py from the
reference's tests/fixtures/expected.json (renderings by the official package); the vectors in
test_python_formatting and test_renders_like_python are the reference's own unit-test vectors
(`src/prompt.rs:378-398`).
"""
import json
import os
import unicodedata

import pytest

from strands_decider import prompt
from strands_decider.prompt import Question

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "prompt_cases.json")


def cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["name"])
def test_renders_questions_like_the_official_package(case):
    """`tests/parity.rs:28-38`: ours is NFC up front, the official text is normalized the same way."""
    qs = [Question.from_json(q) for q in case["request"]["questions"].values()]
    assert len(qs) == len(case["question_text"])
    for q, want in zip(qs, case["question_text"]):
        r = prompt.render_question(q)
        assert r.text == unicodedata.normalize("NFC", want)
        # spans are byte ranges of whole option lines
        b = r.text.encode()
        for i, (lo, hi) in enumerate(r.spans):
            assert b[lo:hi].decode().startswith(f"{i + 1}. ")
            assert b[hi:hi + 1] == b"\n"


def test_python_formatting():
    """The reference's `python_formatting` vectors (`src/prompt.rs:379-388`)."""
    for x, s in [(0.1, "0.1"), (1.0, "1.0"), (0.0001, "0.0001"), (1e-5, "1e-05"), (1.2345678901234568e17, "1.2345678901234568e+17"),
                 (1e15, "1000000000000000.0"), (-2.5e-7, "-2.5e-07"), (0.8442, "0.8442")]:
        assert prompt.py_float(x) == s
        assert prompt.py_float(x) == repr(x)
    v = json.loads('{"a": [1, 2.5, {"b": null}], "c": "é\\n\\u0001\\"", "d": {}, "e": [], "g": 1e-5, "i": 100.0, "a": 7}')
    assert prompt.py_dumps(v) == '{\n  "a": 7,\n  "c": "é\\n\\u0001\\"",\n  "d": {},\n  "e": [],\n  "g": 1e-05,\n  "i": 100.0\n}'


def test_py_float_matches_repr_widely():
    import random
    r = random.Random(0)
    for _ in range(3000):
        x = r.choice([r.uniform(-1, 1), r.uniform(-1e20, 1e20), 10 ** r.uniform(-30, 30), r.random() * 1e-5, float(r.randint(0, 10**17))])
        assert prompt.py_float(x) == repr(x)


def test_renders_like_python():
    """The reference's `renders_like_python` (`src/prompt.rs:390-398`)."""
    q = Question.from_json({"type": "choice", "instructions": "  Route it. ", "criteria": {"billing": "money\n matters", "sales": None}})
    r = prompt.render_question(q)
    assert r.text == "<question type=\"choice\">\nSelect exactly one option.\nRoute it.\n<options>\n1. billing — money matters\n2. sales\n</options>\n</question>\n<answer>"
    assert r.text.encode()[r.spans[1][0]:r.spans[1][1]].decode() == "2. sales"
    assert prompt.choice_confidence([0.5, 0.5]) == 0.0
    assert abs(prompt.score_confidence([0.0, 1.0, 0.0], 0.1) - 1.0) < 1e-12


def test_question_validation_errors():
    bad = [
        ({"type": "choice", "instructions": "x", "criteria": {"a": ""}}, "between 2 and 255"),
        ({"type": "score", "instructions": "x", "criteria": ["a"]}, "between 2 and 10"),
        ({"type": "score", "instructions": "x", "criteria": {"a": "b"}}, "list of level"),
        ({"type": "noul", "instructions": "x", "criteria": {"maybe": "b"}}, "subset"),
        ({"type": "other", "instructions": "x"}, "noul, choice or score"),
        ({"type": "noul", "instructions": 3}, "instructions must be"),
        ({"type": "choice", "instructions": "x", "criteria": {"a": 1, "b": ""}}, "descriptions must be"),
        ("nope", "must be an object"),
    ]
    for q, msg in bad:
        with pytest.raises(prompt.PromptError, match=msg):
            Question.from_json(q)
    # kind inference without "type" (`src/prompt.rs:111-116`)
    assert Question.from_json({"instructions": "x"}).kind == "noul"
    assert Question.from_json({"instructions": "x", "criteria": ["a", "b"]}).kind == "score"
    assert Question.from_json({"instructions": "x", "criteria": {"true": "y"}}).kind == "noul"
    assert Question.from_json({"instructions": "x", "criteria": {"a": "", "b": ""}}).kind == "choice"


def test_answers():
    rq = prompt.render_question(Question.noul("x"))
    a = prompt.to_answer(rq, [0.25, 0.75], 0.0)
    assert a.to_json() == {"type": "noul", "noul": 0.75} and str(a) == "P(true) = 0.750"
    rq = prompt.render_question(Question.choice("x", ["a", "b", "c"]))
    a = prompt.to_answer(rq, [0.2, 0.5, 0.3], 0.0)
    assert a.choice == "b" and a.confidence == 0.25
    rq = prompt.render_question(Question.score("x", ["lo", "mid", "hi"]))
    a = prompt.to_answer(rq, [0.0, 0.5, 0.5], 0.0)
    assert a.score == 1.5 and a.legend == [("0", "lo"), ("1", "mid"), ("2", "hi")]
    j = a.to_json()
    assert list(j) == ["type", "score", "legend", "probabilities", "confidence"]
