"""strands-decider on B200: the reference's public surface (`src/lib.rs`) over the C-ABI engine.

`Decider.load/ask/ask_all/evaluate`, `Question`, `Answer`, `Request`, `Response` and `Timings` keep
the reference's names, arguments, error behaviour and answer formulas. The torso runs through
libsdb200.so (include/sd_b200.h); tokenizer, prompt and head are host code as in the reference.
"""
from __future__ import annotations

import json
import os
import time
from dataclasses import dataclass, field

from . import prompt
from .engine import CONTEXT, Engine, Error, Head, NativeDecider, Snapshot
from .prompt import Answer, Question
from .tokenizer import Tokenizer

__all__ = ["Decider", "NativeDecider", "Question", "Answer", "Request", "Response", "Timings", "Engine", "Snapshot", "Error",
           "CONTEXT"]

MAX_BATCH = 32  # questions per batched fork; the reference's constant, which there only sets the token count (`src/lib.rs:107-108`)


@dataclass
class Request:
    """A System One request: a state and named questions about it, in order (`src/lib.rs:46-63`)."""
    state: object
    questions: list

    @staticmethod
    def from_json(v: dict) -> "Request":
        state = v.get("state") if isinstance(v, dict) else None
        if not isinstance(state, (str, dict, list)):
            raise Error("state must be a string, object or array")
        if isinstance(v.get("images"), list) and v["images"]:
            raise Error("this engine has no vision tower; images are not supported")
        qs = v.get("questions")
        if not isinstance(qs, dict) or not qs:
            raise Error("questions must be a non-empty object")
        out = []
        for name, q in qs.items():
            try:
                out.append((name, Question.from_json(q)))
            except prompt.PromptError as e:
                raise Error(f"question {name}: {e}") from None
        return Request(state, out)


@dataclass
class Timings:
    tokenize_ms: float = 0.0
    forward_ms: float = 0.0
    total_ms: float = 0.0


@dataclass
class Response:
    answers: list
    input_tokens: int
    timings: Timings = field(default_factory=Timings)

    def to_json(self) -> dict:
        """The System One response body (`src/lib.rs:78-87`)."""
        return {"model": "strands-decider-rs-0.1.0",  # the reference's crate name and version (`Cargo.toml:2-3`)
                "answers": {k: a.to_json() for k, a in self.answers},
                "usage": {"input_tokens": self.input_tokens, "output_tokens": len(self.answers)}}


class Decider:
    """`Decider` (`src/lib.rs:100-209`)."""

    def __init__(self, engine: Engine, tokenizer: Tokenizer, head: Head, cfg: dict):
        self.engine = engine
        self.tokenizer = tokenizer
        self.head = head
        self.cfg = cfg

    @classmethod
    def load(cls, model_dir: str, device: int = 0) -> "Decider":
        """`Decider::load` (`src/lib.rs:120-134`)."""
        def read(name):
            try:
                with open(os.path.join(model_dir, name), "rb") as f:
                    return f.read()
            except OSError as e:
                raise Error(f"{os.path.join(model_dir, name)}: {e}") from None
        tok = Tokenizer.from_json(read("tokenizer.json").decode("utf-8", errors="replace"))
        engine = Engine.load(model_dir, device)
        head = Head.load(os.path.join(model_dir, "head.safetensors"))
        try:
            cfg = json.loads(read("hobson_config.json"))
            cfg = {"max_length": int(cfg["max_length"]), "temperature": float(cfg["temperature"]),
                   "temperature_by_kind": dict(cfg.get("temperature_by_kind", {})),
                   "ordinal_smoothing": float(cfg.get("ordinal_smoothing", 0.0))}
        except (ValueError, KeyError, TypeError) as e:
            raise Error(f"hobson_config.json: {e}") from None
        return cls(engine, tok, head, cfg)

    def ask(self, state, question: Question) -> Answer:
        """Answers a question about `state` (`src/lib.rs:136-139`)."""
        return self.ask_all(state, [question])[0]

    def ask_all(self, state, questions) -> list:
        """Answers several questions about one state, in order; the state is encoded once
        (`src/lib.rs:141-145`)."""
        named = [(str(i), q) for i, q in enumerate(questions)]
        return [a for _, a in self._run(state, named).answers]

    def evaluate(self, req: Request) -> Response:
        """Answers a System One request (`src/lib.rs:147-150`)."""
        return self._run(req.state, req.questions)

    def _temperature(self, rq) -> float:
        return float(self.cfg["temperature_by_kind"].get(rq.kind, self.cfg["temperature"]))

    def encode(self, state, named):
        """Rendering, tokenization, context check and option rows (`src/lib.rs:158-181`)."""
        if not isinstance(state, (str, dict, list)):
            raise Error("state must be a string, object or array")
        if not named:
            raise Error("ask at least one question")
        for _, q in named:
            try:
                q.validate()
            except prompt.PromptError as e:
                raise Error(str(e)) from None
        rendered = [prompt.render_question(q) for _, q in named]
        sids = self.tokenizer.encode(prompt.render_state(state)).ids
        qencs = [self.tokenizer.encode(r.text) for r in rendered]
        longest = max(len(q.ids) for q in qencs)
        if len(sids) + longest > self.cfg["max_length"]:
            raise Error(f"prompt of {len(sids) + longest} tokens ({len(sids)} state + {longest} question) exceeds the "
                        f"context window of {self.cfg['max_length']} tokens")
        try:
            options = [prompt.option_token_index(q.offsets, r.spans) for q, r in zip(qencs, rendered)]
        except prompt.PromptError as e:
            raise Error(str(e)) from None
        return rendered, sids, qencs, options

    def _run(self, state, named) -> Response:
        """`Decider::run` (`src/lib.rs:156-208`): one forward for a single question; otherwise the
        state and every question in one tree pass, each question continuing the state
        (`sd_forward_tree`; the reference runs the state with a snapshot, then the questions one after
        another), or, past one pass's limits, the state once with a snapshot, then the questions
        continued from it, MAX_BATCH at a time in one batched fork each (`sd_forward_fork`)."""
        t0 = time.perf_counter()
        rendered, sids, qencs, options = self.encode(state, named)
        t1 = time.perf_counter()
        d = self.engine.hidden_size()
        answers = []
        smooth = self.cfg["ordinal_smoothing"]
        if len(qencs) == 1:
            ids = list(sids) + list(qencs[0].ids)
            rows = [len(sids) + i for i in options[0]] + [len(ids) - 1]
            out = self.engine.forward(ids, rows)
            probs = self.head.probs(out.hidden, d, self._temperature(rendered[0]))
            answers.append((named[0][0], prompt.to_answer(rendered[0], probs, smooth)))
        elif len(sids) + sum(len(q.ids) for q in qencs) <= 65536 and len(qencs) < 4096:
            rows = [[]] + [list(options[i]) + [len(qencs[i].ids) - 1] for i in range(len(qencs))]
            hidden = self.engine.forward_tree(None, [-1] + [0] * len(qencs), [sids] + [q.ids for q in qencs], rows)
            for i in range(len(qencs)):
                probs = self.head.probs(hidden[i + 1], d, self._temperature(rendered[i]))
                answers.append((named[i][0], prompt.to_answer(rendered[i], probs, smooth)))
        else:
            prefix = self.engine.forward(sids, [], keep=True).snapshot
            try:
                for c in range(0, len(qencs), MAX_BATCH):
                    idx = range(c, min(len(qencs), c + MAX_BATCH))
                    hidden = self.engine.forward_fork(prefix, [qencs[i].ids for i in idx],
                                                      [list(options[i]) + [len(qencs[i].ids) - 1] for i in idx])
                    for i, h in zip(idx, hidden):
                        probs = self.head.probs(h, d, self._temperature(rendered[i]))
                        answers.append((named[i][0], prompt.to_answer(rendered[i], probs, smooth)))
            finally:
                prefix.close()
        input_tokens = 0
        for c in range(0, len(qencs), MAX_BATCH):
            chunk = qencs[c:c + MAX_BATCH]
            input_tokens += len(sids) + sum(len(q.ids) for q in chunk) if len(chunk) > 1 else len(sids) + len(chunk[0].ids)
        t2 = time.perf_counter()
        ms = lambda a, b: (b - a) * 1e3  # noqa: E731
        return Response(answers, input_tokens, Timings(ms(t0, t1), ms(t1, t2), ms(t0, t2)))
