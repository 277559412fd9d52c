"""The tokenizer mirror (`src/tokenizer.rs`) against Hugging Face `tokenizers` 0.22.2 on the synthetic
byte-level BPE vocabulary, in the style of the reference's `tests/parity.rs:57-70`: ids must be
identical; offsets must be identical where NFC leaves the text unchanged (the mirror's offsets are
into the NFC text). Inputs: the reference's 21 raw edge-case strings (tests/golden/prompt_cases.json)
and every rendered fixture prompt.
"""
import json
import os
import unicodedata

import pytest

from strands_decider import prompt
from strands_decider.tokenizer import Tokenizer, TokenizerError, write_synthetic_tokenizer

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "prompt_cases.json")


@pytest.fixture(scope="module")
def toks(tmp_path_factory):
    from tokenizers import Tokenizer as HF
    p = tmp_path_factory.mktemp("tok") / "tokenizer.json"
    write_synthetic_tokenizer(str(p), seed=0)
    text = p.read_text()
    return Tokenizer.from_json(text), HF.from_str(text), text


def texts():
    with open(GOLDEN) as f:
        g = json.load(f)
    out = list(g["raw_texts"])
    for c in g["cases"]:
        out.append(prompt.render_state(c["request"]["state"]))
        for q in c["request"]["questions"].values():
            out.append(prompt.render_question(prompt.Question.from_json(q)).text)
    out += ["<|im_start|>user<|im_end|><|endoftext|>", "<|im_start|<|im_end|>>", "é́x", "ﬁ ＡＢＣ ⅻ"]
    return out


def test_ids_and_offsets_match_hugging_face(toks):
    mine, hf, _ = toks
    n_off = 0
    for s in texts():
        e = mine.encode(s)
        h = hf.encode(s, add_special_tokens=False)
        assert e.ids == h.ids, repr(s)
        if unicodedata.normalize("NFC", s) == s:
            b = [len(s[:i].encode()) for i in range(len(s) + 1)]
            assert e.offsets == [(b[lo], b[hi]) for lo, hi in h.offsets], repr(s)
            n_off += 1
    assert n_off > 50


def test_option_token_index_on_rendered_questions(toks):
    """Every option line of every fixture question keeps at least one token (`src/prompt.rs:203-213`)."""
    mine, _, _ = toks
    with open(GOLDEN) as f:
        g = json.load(f)
    for c in g["cases"]:
        for q in c["request"]["questions"].values():
            r = prompt.render_question(prompt.Question.from_json(q))
            e = mine.encode(r.text)
            idx = prompt.option_token_index(e.offsets, r.spans)
            assert len(idx) == len(r.spans) and idx == sorted(idx) and idx[-1] < len(e.ids) - 1


def test_rejects_unsupported_files(toks):
    _, _, text = toks
    base = json.loads(text)
    for path, val, what in [(("normalizer",), {"type": "NFKC"}, "normalizer"), (("model", "type"), "WordPiece", "model"),
                            (("pre_tokenizer", "type"), "ByteLevel", "pre_tokenizer")]:
        d = json.loads(text)
        cur = d
        for k in path[:-1]:
            cur = cur[k]
        cur[path[-1]] = val
        with pytest.raises(TokenizerError, match=what):
            Tokenizer.from_json(json.dumps(d))
    d = json.loads(text)
    d["added_tokens"][0]["lstrip"] = True
    with pytest.raises(TokenizerError, match="added token options"):
        Tokenizer.from_json(json.dumps(d))
    assert base["model"]["type"] == "BPE"
