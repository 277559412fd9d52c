"""Prompt rendering and answer reading: a question becomes numbered option lines, and the head's
distribution over those options is read back as a noul probability, a choice or a score.

Mirrors the reference's `src/prompt.rs` (itself a port of the official package's ``prompting.py``
and ``schema.py``): ``Question`` (`:28-140`), ``render_content``/``render_state``/
``render_question`` (`:159-200`), ``option_token_index`` (`:203-213`), ``Answer`` and ``to_answer``
(`:215-296`), and Python's JSON/float formatting (`:309-372`). JSON objects keep insertion order, as
the reference's ``serde_json`` ``preserve_order`` feature does (`Cargo.toml:27`).
"""
from __future__ import annotations

import decimal
import json
import math
import unicodedata
from dataclasses import dataclass, field
from typing import Any


class PromptError(ValueError):
    pass


NOUL, CHOICE, SCORE = "noul", "choice", "score"

NOUL_DEFAULT = [("false", "the statement does not hold for this state"), ("true", "the statement holds for this state")]


def _is_content(v: Any) -> bool:
    return isinstance(v, (str, dict, list))


@dataclass
class Question:
    """A question about a state: its instructions and its options as (label, description) pairs
    (`src/prompt.rs:28-33`)."""
    kind: str
    instructions: Any
    options: list = field(default_factory=list)

    @staticmethod
    def noul(instructions) -> "Question":
        """Yes or no: is the statement true of the state? Answers P(true) (`src/prompt.rs:66-70`)."""
        return Question(NOUL, instructions, [(l, d) for l, d in NOUL_DEFAULT])

    @staticmethod
    def choice(instructions, options) -> "Question":
        """One of 2 to 255 options, each a label or a (label, description) pair (`:72-75`)."""
        opts = []
        for o in options:
            opts.append((o, None) if isinstance(o, str) else (str(o[0]), o[1]))
        return Question(CHOICE, instructions, opts)

    @staticmethod
    def score(instructions, levels) -> "Question":
        """A level on an ordered scale of 2 to 10 descriptions, lowest first (`:77-81`)."""
        return Question(SCORE, instructions, [(str(i), str(d)) for i, d in enumerate(levels)])

    def validate(self) -> None:
        """Checks the question as the official schema does (`src/prompt.rs:83-100`)."""
        if not _is_content(self.instructions):
            raise PromptError("question instructions must be a string, object or array")
        if any(d is not None and not _is_content(d) for _, d in self.options):
            raise PromptError("option descriptions must be strings, objects, arrays or null")
        n = len(self.options)
        if self.kind == NOUL and [l for l, _ in self.options] != ["false", "true"]:
            raise PromptError("noul options must be false, true")
        if self.kind == CHOICE and not 2 <= n <= 255:
            raise PromptError("choice requires between 2 and 255 options")
        if self.kind == CHOICE and len({l for l, _ in self.options}) != n:
            raise PromptError("choice options must be unique")
        if self.kind == SCORE and not 2 <= n <= 10:
            raise PromptError("score requires between 2 and 10 levels")
        if self.kind == SCORE and any(not isinstance(d, str) for _, d in self.options):
            raise PromptError("score levels must be strings")

    @staticmethod
    def from_json(v) -> "Question":
        """A question as the System One API takes it (``{"type", "instructions", "criteria"}``),
        validated as the official schema does (`src/prompt.rs:104-139`)."""
        if not isinstance(v, dict):
            raise PromptError("a question must be an object")
        criteria = v.get("criteria")
        t = v.get("type", Ellipsis)
        if t is Ellipsis:
            if criteria is None:
                kind = NOUL
            elif isinstance(criteria, list):
                kind = SCORE
            elif isinstance(criteria, dict) and all(k in ("true", "false") for k in criteria):
                kind = NOUL
            else:
                kind = CHOICE
        elif t in (NOUL, CHOICE, SCORE):
            kind = t
        else:
            raise PromptError("question type must be noul, choice or score")
        instructions = v.get("instructions")
        if kind == NOUL:
            if criteria is None:
                q = Question.noul(instructions)
            elif isinstance(criteria, dict) and all(k in ("true", "false") for k in criteria):
                q = Question.noul(instructions)
                q.options = [(l, criteria[l] if l in criteria else d) for l, d in q.options]
            else:
                raise PromptError("noul criteria keys must be a subset of {'true', 'false'}")
        elif kind == CHOICE:
            if not isinstance(criteria, dict):
                raise PromptError("choice criteria must map option names to descriptions")
            q = Question(CHOICE, instructions, list(criteria.items()))
        else:
            if not (isinstance(criteria, list) and all(isinstance(c, str) for c in criteria)):
                raise PromptError("score criteria must be a list of level descriptions")
            q = Question.score(instructions, criteria)
        q.validate()
        return q


@dataclass
class Rendered:
    """A question as prompt text, with what is needed to read the answer back (`:142-151`).
    ``spans`` are UTF-8 byte ranges of each option's line in ``text``."""
    text: str
    kind: str
    labels: list
    descriptions: list
    spans: list


def py_float(x: float) -> str:
    """Python's ``repr(float)`` (`src/prompt.rs:348-372`): shortest round-trip digits, exponent form
    below 1e-4 and from 1e16."""
    if not math.isfinite(x):
        return "NaN" if math.isnan(x) else ("Infinity" if x > 0 else "-Infinity")
    sign = "-" if math.copysign(1.0, x) < 0 else ""
    if x == 0.0:
        return sign + "0.0"
    # shortest round-trip decimal digits and the position of the decimal point
    t = decimal.Decimal(repr(abs(x))).normalize().as_tuple()
    digits = "".join(map(str, t.digits))
    n = len(digits)
    point = n + t.exponent
    if point <= -4 or point > 16:
        frac = "." + digits[1:] if n > 1 else ""
        body = f"{digits[0]}{frac}e{'+' if point > 0 else '-'}{abs(point - 1):02d}"
    elif point <= 0:
        body = "0." + "0" * (-point) + digits
    elif point >= n:
        body = digits + "0" * (point - n) + ".0"
    else:
        body = digits[:point] + "." + digits[point:]
    return sign + body


def py_dumps(v) -> str:
    """Python's ``json.dumps(v, indent=2, ensure_ascii=False)`` (`src/prompt.rs:309-346`)."""
    def dump(v, level, out):
        pad = "  "
        if isinstance(v, bool) or v is None:
            out.append(json.dumps(v))
        elif isinstance(v, float):
            out.append(py_float(v))
        elif isinstance(v, int):
            out.append(str(v))
        elif isinstance(v, str):
            out.append(json.dumps(v, ensure_ascii=False))
        elif isinstance(v, list) and v:
            out.append("[")
            for i, x in enumerate(v):
                out.append("\n" if i == 0 else ",\n")
                out.append(pad * (level + 1))
                dump(x, level + 1, out)
            out.append("\n" + pad * level + "]")
        elif isinstance(v, dict) and v:
            out.append("{")
            for i, (k, x) in enumerate(v.items()):
                out.append("\n" if i == 0 else ",\n")
                out.append(pad * (level + 1) + json.dumps(k, ensure_ascii=False) + ": ")
                dump(x, level + 1, out)
            out.append("\n" + pad * level + "}")
        else:
            out.append("[]" if isinstance(v, list) else "{}")
    out: list[str] = []
    dump(v, 0, out)
    return "".join(out)


def render_content(v) -> str:
    """Strings stripped, structured content as Python's indented JSON (`src/prompt.rs:159-165`)."""
    if v is None:
        return ""
    if isinstance(v, str):
        return v.strip()
    return py_dumps(v)


def render_state(state) -> str:
    """`render_state` (`src/prompt.rs:167-169`)."""
    return f"<state>\n{render_content(state)}\n</state>\n"


_HEADERS = {
    NOUL: "Decide whether the statement is true of the state.",
    CHOICE: "Select exactly one option.",
    SCORE: "Rate the state against the ordered levels below (lowest first).",
}


def render_question(q: Question) -> Rendered:
    """`render_question` (`src/prompt.rs:171-200`): pieces are NFC-normalized first, so byte offsets
    of the tokenized text are offsets into ``text``."""
    def nfc(s):
        return unicodedata.normalize("NFC", s)
    text = f'<question type="{q.kind}">\n{_HEADERS[q.kind]}\n{nfc(render_content(q.instructions))}\n<options>\n'
    nbytes = len(text.encode())
    spans = []
    for i, (name, desc) in enumerate(q.options):
        d = " ".join(render_content(desc).split())
        line = f"{i + 1}. {nfc(name)}"
        if d:
            line += f" — {nfc(d)}"
        lb = len(line.encode())
        spans.append((nbytes, nbytes + lb))
        text += line + "\n"
        nbytes += lb + 1
    text += "</options>\n</question>\n<answer>"
    return Rendered(text, q.kind, [n for n, _ in q.options], [render_content(d) for _, d in q.options], spans)


def option_token_index(offsets, spans) -> list[int]:
    """The last token that lies inside each option's line (`src/prompt.rs:203-213`)."""
    out = []
    for a, b in spans:
        idx = None
        for i in range(len(offsets) - 1, -1, -1):
            lo, hi = offsets[i]
            if hi > lo and lo >= a and hi <= b:
                idx = i
                break
        if idx is None:
            raise PromptError(f"option span ({a},{b}) has no tokens left; the prompt was truncated through its option list")
        out.append(idx)
    return out


def round4(x: float) -> float:
    """Python's ``round(x, 4)`` as the reference computes it (`src/prompt.rs:222-225`)."""
    return float(f"{x:.4f}")


def choice_confidence(p) -> float:
    """`derive_confidence` (`src/prompt.rs:227-235`)."""
    n = len(p)
    if n <= 1:
        return 1.0
    return min(max((n * max(p) - 1.0) / (n - 1.0), 0.0), 1.0)


def score_confidence(p, ordinal_smoothing: float) -> float:
    """`derive_score_confidence` (`src/prompt.rs:237-256`)."""
    n = len(p)
    if n <= 1:
        return 1.0
    total = sum(p)
    if total <= 0.0:
        return 0.0
    p = [x / total for x in p]
    mean = sum(i * pi for i, pi in enumerate(p))
    sigma = math.sqrt(sum(pi * (i - mean) ** 2 for i, pi in enumerate(p)))
    mx = (n - 1) / 2.0
    floor = math.sqrt(ordinal_smoothing) if ordinal_smoothing > 0.0 else 0.0
    if mx <= floor:
        return 1.0 if sigma <= floor else 0.0
    return min(max((mx - sigma) / (mx - floor), 0.0), 1.0)


@dataclass
class Answer:
    """`Answer` (`src/prompt.rs:215-220`): kind noul (``noul``), choice (``choice``,
    ``probabilities``, ``confidence``) or score (``score``, ``legend``, ``probabilities``,
    ``confidence``)."""
    kind: str
    noul: float | None = None
    choice: str | None = None
    score: float | None = None
    legend: list | None = None
    probabilities: list | None = None
    confidence: float | None = None

    def to_json(self) -> dict:
        """`Answer::to_json` (`src/prompt.rs:279-296`)."""
        if self.kind == NOUL:
            return {"type": "noul", "noul": self.noul}
        probs = {k: v for k, v in self.probabilities}
        if self.kind == CHOICE:
            return {"type": "choice", "choice": self.choice, "probabilities": probs, "confidence": self.confidence}
        return {"type": "score", "score": self.score, "legend": {k: v for k, v in self.legend},
                "probabilities": probs, "confidence": self.confidence}

    def __str__(self) -> str:
        """One line, as the reference's ``Display`` (`src/prompt.rs:298-307`)."""
        if self.kind == NOUL:
            return f"P(true) = {self.noul:.3f}"
        if self.kind == CHOICE:
            return f"{self.choice} (confidence {self.confidence:.3f})"
        return f"{self.score:.2f} (confidence {self.confidence:.3f})"


def to_answer(rq: Rendered, probs, ordinal_smoothing: float) -> Answer:
    """`to_answer` (`src/prompt.rs:258-277`)."""
    if rq.kind == NOUL:
        return Answer(NOUL, noul=round4(probs[rq.labels.index("true")]))
    if rq.kind == CHOICE:
        best = 0
        for i in range(len(probs)):
            if probs[i] > probs[best]:
                best = i
        return Answer(CHOICE, choice=rq.labels[best], probabilities=[(l, round4(p)) for l, p in zip(rq.labels, probs)],
                      confidence=round4(choice_confidence(probs)))
    return Answer(SCORE, score=round4(sum(i * p for i, p in enumerate(probs))),
                  legend=list(zip(rq.labels, rq.descriptions)),
                  probabilities=[(l, round4(p)) for l, p in zip(rq.labels, probs)],
                  confidence=round4(score_confidence(probs, ordinal_smoothing)))
