"""The C++ host layer of the library (tokenizer, Unicode/NFC, JSON formatting, prompt rendering: the
part of the reference's `Decider` above the engine) against the Python mirror and the golden
fixtures, without a GPU. The Python mirror is itself pinned against Hugging Face `tokenizers` (the
tokenizer) and the reference's fixtures and unit vectors (the prompt)."""
import ctypes as C
import json
import os
import random
import unicodedata

import pytest

from strands_decider import engine as E
from strands_decider import prompt
from strands_decider.prompt import Question
from strands_decider.tokenizer import Tokenizer

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "prompt_cases.json")


def lib():
    L = E.lib()
    L.sd_tokenizer_load.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
    L.sd_tokenizer_free.argtypes = [C.c_void_p]
    L.sd_tokenizer_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_int64,
                                      C.POINTER(C.c_int64)]
    L.sd_tokenizer_encode_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_void_p,
                                            C.c_void_p, C.c_int64, C.c_void_p]
    L.sd_prompt_render.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
    L.sd_string_free.argtypes = [C.c_void_p]
    L.sd_host_last_error.restype = C.c_char_p
    return L


class CppTokenizer:
    def __init__(self, path):
        self.L = lib()
        self.h = C.c_void_p()
        rc = self.L.sd_tokenizer_load(path.encode(), C.byref(self.h))
        if rc != 0:
            raise ValueError(self.L.sd_host_last_error().decode())

    def encode(self, text: str):
        b = text.encode()
        n = C.c_int64()
        cap = 4 * len(b) + 8
        ids = (C.c_uint32 * cap)()
        offs = (C.c_uint32 * (2 * cap))()
        rc = self.L.sd_tokenizer_encode(self.h, b, len(b), ids, offs, cap, C.byref(n))
        if rc != 0:
            raise ValueError(self.L.sd_host_last_error().decode())
        return list(ids[:n.value]), [(offs[2 * i], offs[2 * i + 1]) for i in range(n.value)]

    def encode_batch(self, texts, threads=0, cap=None):
        bs = [t if isinstance(t, bytes) else t.encode() for t in texts]
        n = len(bs)
        ptrs = (C.c_char_p * n)(*bs)
        lens = (C.c_size_t * n)(*[len(b) for b in bs])
        cap = sum(4 * len(b) + 8 for b in bs) if cap is None else cap
        ids = (C.c_uint32 * max(cap, 1))()
        offs = (C.c_uint32 * max(2 * cap, 1))()
        counts = (C.c_int64 * max(n, 1))()
        rc = self.L.sd_tokenizer_encode_batch(self.h, ptrs, lens, n, threads, ids, offs, cap, counts)
        if rc != 0:
            raise ValueError(self.L.sd_host_last_error().decode())
        out, at = [], 0
        for i in range(n):
            c = counts[i]
            out.append((list(ids[at:min(at + c, cap)]), [(offs[2 * k], offs[2 * k + 1]) for k in range(at, min(at + c, cap))], c))
            at += c
        return out

    def close(self):
        self.L.sd_tokenizer_free(self.h)


def render_cpp(request) -> dict:
    L = lib()
    out = C.c_void_p()
    rc = L.sd_prompt_render(json.dumps(request).encode(), C.byref(out))
    if rc != 0:
        raise ValueError(L.sd_host_last_error().decode())
    s = C.string_at(out.value).decode()
    L.sd_string_free(out)
    return json.loads(s)


@pytest.fixture(scope="module")
def tokenizers(small_model):
    path = os.path.join(small_model, "tokenizer.json")
    with open(path) as f:
        py = Tokenizer.from_json(f.read())
    cpp = CppTokenizer(path)
    yield py, cpp
    cpp.close()


def _texts(seed: int, n: int):
    r = random.Random(seed)
    pieces = ["Help! My payouts have been failing for 3 days!", "billing", " the ", "payout", "12345", "3.14", "x=1;",
              "\n", "\r\n", "\t", "  ", " ", "　", " ", "\x1c", "\x85", "​",
              "é", "é", "Å", "Å", "ẛ̣", "q̣̇", "각",
              "각", "日本語", "支付", "über", "ñu", "çа", "😀", "👍🏽", "<|im_start|>", "<|im_end|>", "<|endoftext|>",
              "<question type=\"noul\">", "—", "'s", "'LL", "don't", "ſ", "K", "١٢٣", "Ⅻ", "½", "…", "«»", "{}", "[]"]
    for _ in range(n):
        yield "".join(r.choice(pieces) for _ in range(r.randint(1, 12)))


def test_tokenizer_matches_the_mirror(tokenizers):
    py, cpp = tokenizers
    for t in _texts(1, 600):
        e = py.encode(t)
        ids, offs = cpp.encode(t)
        assert ids == e.ids, t
        assert offs == [tuple(o) for o in e.offsets], t


@pytest.mark.parametrize("threads", [1, 4, 0])
def test_tokenizer_batch_matches_one_by_one(tokenizers, threads):
    """sd_tokenizer_encode_batch on host threads = sd_tokenizer_encode text by text (ids, offsets,
    counts), including empty texts; a cap cuts the written tokens, not the counts."""
    _, cpp = tokenizers
    texts = list(_texts(3, 300)) + ["", "".join(_texts(4, 200))]
    got = cpp.encode_batch(texts, threads)
    for t, (ids, offs, c) in zip(texts, got):
        want_ids, want_offs = cpp.encode(t)
        assert (ids, offs, c) == (want_ids, want_offs, len(want_ids)), t
    short = cpp.encode_batch(texts[:5], threads, cap=7)
    assert [c for _, _, c in short] == [len(cpp.encode(t)[0]) for t in texts[:5]]
    assert sum(len(i) for i, _, _ in short) == min(7, sum(c for _, _, c in short))
    with pytest.raises(ValueError, match="text 1: text is not UTF-8"):
        cpp.encode_batch(["ok", b"bad \xff\xfe", b"\xff"], threads)


def test_tokenizer_on_long_text(tokenizers):
    py, cpp = tokenizers
    t = "".join(_texts(2, 400)) + " " * 5000 + "\n" * 300 + "end"
    e = py.encode(t)
    ids, offs = cpp.encode(t)
    assert ids == e.ids and offs == [tuple(o) for o in e.offsets]


def test_nfc_through_the_tokenizer(tokenizers):
    """Offsets are into the NFC text: a decomposed input has the byte length of its NFC form."""
    py, cpp = tokenizers
    r = random.Random(3)
    marks = [0x0300, 0x0301, 0x0308, 0x0323, 0x0327, 0x031B, 0x0345, 0x05B7, 0x093C, 0x3099]
    for _ in range(300):
        s = "".join(chr(r.choice([0x41, 0x61, 0x4F, 0x55, 0x3B1, 0x3C9, 0x415, 0x5D0, 0x915, 0x304B, 0x1100, 0x1161, 0x11A8]))
                    + "".join(chr(r.choice(marks)) for _ in range(r.randint(0, 3))) for _ in range(r.randint(1, 8)))
        ids, offs = cpp.encode(s)
        assert offs[-1][1] == len(unicodedata.normalize("NFC", s).encode())
        assert ids == py.encode(s).ids


def test_tokenizer_rejects_bad_files(tmp_path):
    bad = tmp_path / "t.json"
    bad.write_text(json.dumps({"model": {"type": "Unigram"}}))
    with pytest.raises(ValueError):
        CppTokenizer(str(bad))
    bad.write_text("{not json")
    with pytest.raises(ValueError):
        CppTokenizer(str(bad))


def cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["name"])
def test_cpp_renders_like_the_official_package(case):
    got = render_cpp({"state": case["request"]["state"], "questions": list(case["request"]["questions"].values())})
    assert len(got["questions"]) == len(case["question_text"])
    for g, want in zip(got["questions"], case["question_text"]):
        assert g["text"] == unicodedata.normalize("NFC", want)
    for g, q in zip(got["questions"], case["request"]["questions"].values()):
        assert [list(s) for s in prompt.render_question(Question.from_json(q)).spans] == g["spans"]
    assert got["state"] == prompt.render_state(case["request"]["state"])


def test_cpp_state_rendering_matches_python():
    """JSON content as Python's json.dumps(indent=2, ensure_ascii=False) with repr floats."""
    r = random.Random(4)
    leaves = [0.1, 1.0, 1e-5, 1e16, 1.2345678901234568e17, -0.0, -2.5e-7, 123, -7, 0, True, False, None, "é\n\u0001\"\\",
              "  padded  ", "\t", "日本", "😀", 3.0e-310, 1.7976931348623157e308]
    def tree(d):
        if d == 0 or r.random() < 0.3:
            return r.choice(leaves)
        if r.random() < 0.5:
            return [tree(d - 1) for _ in range(r.randint(0, 3))]
        return {r.choice(["a", "b", "c", "é", "k" + str(r.randint(0, 9))]): tree(d - 1) for _ in range(r.randint(0, 3))}
    for _ in range(200):
        state = tree(4)
        if not isinstance(state, (dict, list, str)):
            state = [state]
        got = render_cpp({"state": state, "questions": []})
        assert got["state"] == prompt.render_state(state), state
    for s in ["  Help me  ", " x　", "", "a b"]:
        assert render_cpp({"state": s, "questions": []})["state"] == prompt.render_state(s)


def test_cpp_question_errors():
    for q, msg in [({"type": "choice", "instructions": "x", "criteria": {"a": ""}}, "between 2 and 255"),
                   ({"type": "score", "instructions": "x", "criteria": ["a", 1]}, "list of level descriptions"),
                   ({"type": "noul", "instructions": "x", "criteria": {"yes": "a"}}, "subset of"),
                   ({"type": "quiz", "instructions": "x"}, "noul, choice or score"),
                   ({"instructions": 5}, "instructions must be a string"),
                   ([1], "must be an object")]:
        with pytest.raises(ValueError, match=msg):
            render_cpp({"state": "s", "questions": [q]})
