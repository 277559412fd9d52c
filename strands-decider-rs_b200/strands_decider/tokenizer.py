"""Byte-level BPE from a ``tokenizer.json``: added tokens, NFC, the Split pre-tokenizer regex, then
byte-level BPE, encode direction only, with byte offsets into the normalized text.

Mirrors the reference's `src/tokenizer.rs:14-246` (`Tokenizer::from_json`, `encode`, `bpe`): the
same accepted file shape (`:84-131`), added tokens matched leftmost-longest before anything else
(`:157-165`), NFC per segment between added tokens (`:135-155`), regex gaps encoded as their own
pieces (`:167-181`), lowest-rank merge first with leftmost tie-break (`:185-232`), and offsets that
widen a partial character to the whole character (`:233-244`).

The reference's own vocabulary is not available here (there is no network), so
:func:`write_synthetic_tokenizer` trains a byte-level BPE of the accepted shape on seeded synthetic
text with Hugging Face ``tokenizers``; ids and offsets of this mirror are tested against that library.
"""
from __future__ import annotations

import heapq
import json
import unicodedata

import regex

# Printable stand-ins for the 256 byte values, as byte-level BPE vocabularies are written
# (`src/tokenizer.rs:67-81`).
def _byte_chars() -> list[str]:
    out = []
    n = 0
    for b in range(256):
        printable = 0x21 <= b <= 0x7E or 0xA1 <= b <= 0xAC or 0xAE <= b <= 0xFF
        if printable:
            out.append(chr(b))
        else:
            n += 1
            out.append(chr(255 + n))
    return out


class TokenizerError(ValueError):
    pass


class Encoding:
    __slots__ = ("ids", "offsets")

    def __init__(self):
        self.ids: list[int] = []
        self.offsets: list[tuple[int, int]] = []


class Tokenizer:
    """`Tokenizer` (`src/tokenizer.rs:14-21`)."""

    def __init__(self, byte_id, merges, added, split):
        self.byte_id = byte_id
        self.merges = merges
        self.added = added
        self.split = split

    @classmethod
    def from_json(cls, text: str) -> "Tokenizer":
        """`Tokenizer::from_json` (`src/tokenizer.rs:84-131`), with its checks on the file shape."""
        try:
            f = json.loads(text)
        except json.JSONDecodeError as e:
            raise TokenizerError(f"tokenizer.json: {e}") from None

        def unsupported(what):
            return TokenizerError(f"tokenizer.json: unsupported {what}")

        norm = f.get("normalizer")
        if norm is not None and norm != {"type": "NFC"}:
            raise unsupported("normalizer")
        p = f.get("pre_tokenizer") or {}
        pts = p.get("pretokenizers")
        ok = p.get("type") == "Sequence" and isinstance(pts, list) and len(pts) == 2
        split = pts[0] if ok else {}
        bl = pts[1] if ok else {}
        pattern = (split.get("pattern") or {}).get("Regex") if ok else None
        if not (ok and split.get("type") == "Split" and split.get("behavior") == "Isolated"
                and split.get("invert") is False and isinstance(pattern, str)
                and bl.get("type") == "ByteLevel" and bl.get("add_prefix_space") is False
                and bl.get("use_regex") is False):
            raise unsupported("pre_tokenizer")
        m = f["model"]
        if m.get("type") != "BPE" or m.get("byte_fallback", False) or m.get("ignore_merges", False):
            raise unsupported("model")
        added_tokens = f.get("added_tokens", [])
        if any(t.get("single_word") or t.get("lstrip") or t.get("rstrip") or t.get("normalized") for t in added_tokens):
            raise unsupported("added token options")
        vocab = m["vocab"]
        chars = _byte_chars()
        byte_id = []
        for c in chars:
            if c not in vocab:
                raise unsupported("vocabulary (missing a byte)")
            byte_id.append(vocab[c])
        merges = {}
        for rank, mg in enumerate(m["merges"]):
            if isinstance(mg, list):
                a, b = mg
            else:
                if " " not in mg:
                    raise unsupported("merge")
                a, b = mg.split(" ", 1)
            try:
                merges[(vocab[a], vocab[b])] = (rank, vocab[a + b])
            except KeyError:
                raise unsupported("merge (token not in vocabulary)") from None
        added = sorted(((t["content"], t["id"]) for t in added_tokens), key=lambda x: -len(x[0].encode()))
        try:
            rx = regex.compile(pattern)
        except regex.error as e:
            raise TokenizerError(f"tokenizer.json: pre-tokenizer regex: {e}") from None
        return cls(byte_id, merges, added, rx)

    def encode(self, text: str) -> Encoding:
        """`Tokenizer::encode` (`src/tokenizer.rs:135-155`): ids and byte offsets into the NFC text."""
        enc = Encoding()
        base = 0
        rest = text
        while rest:
            gap, special = self._next_added(rest)
            segment = unicodedata.normalize("NFC", rest[:gap])
            self._encode_segment(segment, base, enc)
            base += len(segment.encode())
            if special is None:
                break
            content, tid = special
            n = len(content.encode())
            enc.ids.append(tid)
            enc.offsets.append((base, base + n))
            base += n
            rest = rest[gap + len(content):]
        return enc

    def _next_added(self, s: str):
        """Leftmost added token (the longest one there), `src/tokenizer.rs:157-165`."""
        if not self.added:
            return len(s), None
        for i in range(len(s)):
            for t, tid in self.added:
                if s.startswith(t, i):
                    return i, (t, tid)
        return len(s), None

    def _encode_segment(self, s: str, base: int, enc: Encoding):
        """Regex pieces and the gaps between them, `src/tokenizer.rs:167-181`."""
        b = s.encode()
        # character index -> byte index
        cb = [0]
        for ch in s:
            cb.append(cb[-1] + len(ch.encode()))
        last = 0
        for m in self.split.finditer(s):
            st, en = cb[m.start()], cb[m.end()]
            if st > last:
                self._bpe(b, last, st, base, enc)
            if en > st:
                self._bpe(b, st, en, base, enc)
            last = en
        if last < len(b):
            self._bpe(b, last, len(b), base, enc)

    def _bpe(self, b: bytes, frm: int, to: int, base: int, enc: Encoding):
        """Byte-level BPE of one piece, lowest rank first, leftmost on ties (`src/tokenizer.rs:185-232`)."""
        n = to - frm
        ids = [self.byte_id[x] for x in b[frm:to]]
        start = list(range(n))
        ln = [1] * n
        prev = [i - 1 for i in range(n)]
        nxt = [i + 1 if i + 1 < n else -1 for i in range(n)]
        q = []
        merges = self.merges
        for i in range(n - 1):
            m = merges.get((ids[i], ids[i + 1]))
            if m is not None:
                q.append((m[0], i, m[1]))
        heapq.heapify(q)
        while q:
            _, pos, new_id = heapq.heappop(q)
            nx = nxt[pos]
            if ln[pos] == 0 or nx == -1:
                continue
            m = merges.get((ids[pos], ids[nx]))
            if m is None or m[1] != new_id:
                continue
            ids[pos] = new_id
            ln[pos] += ln[nx]
            nxt[pos] = nxt[nx]
            ln[nx] = 0
            after = nxt[pos]
            if after != -1:
                prev[after] = pos
            pv = prev[pos]
            if pv != -1:
                m2 = merges.get((ids[pv], new_id))
                if m2 is not None:
                    heapq.heappush(q, (m2[0], pv, m2[1]))
            if after != -1:
                m2 = merges.get((new_id, ids[after]))
                if m2 is not None:
                    heapq.heappush(q, (m2[0], pos, m2[1]))
        for i in range(n):
            if ln[i] == 0:
                continue
            lo, hi = frm + start[i], frm + start[i] + ln[i]
            # a token holding part of a UTF-8 character spans the whole character
            while lo > 0 and (b[lo] & 0xC0) == 0x80:
                lo -= 1
            while hi < len(b) and (b[hi] & 0xC0) == 0x80:
                hi += 1
            enc.ids.append(ids[i])
            enc.offsets.append((base + lo, base + hi))


# ---------------------------------------------------------------------------------------------
# Synthetic vocabulary
# ---------------------------------------------------------------------------------------------

# The pre-tokenizer split pattern of the synthetic vocabulary (written for this build): letter runs
# with one optional leading non-letter, single digits, punctuation runs with trailing newlines,
# newline runs, and whitespace that leaves one space for the next piece.
SPLIT_PATTERN = r"[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+"
SPECIAL_TOKENS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]

_SYLLABLES = ["ba", "be", "bi", "bo", "ka", "ke", "ki", "ko", "la", "le", "li", "lo", "ma", "me", "mi",
              "mo", "na", "ne", "ni", "no", "ra", "re", "ri", "ro", "sa", "se", "si", "so", "ta", "te",
              "ti", "to", "va", "ve", "vi", "str", "th", "an", "en", "in", "on", "ion", "ing", "er", "ly",
              "pay", "out", "fail", "day", "team", "bill", "sale", "help", "urg", "ent", "ca", "fé",
              "über", "ñu", "çа", "日", "本", "語", "支", "付"]
_TEMPLATE_WORDS = ["<state>", "</state>", "<question", "type=", "\"noul\"", "\"choice\"", "\"score\"", ">",
                   "</question>", "<options>", "</options>", "<answer>", "Decide whether the statement is true of the state.",
                   "Select exactly one option.", "Rate the state against the ordered levels below (lowest first).",
                   "the statement does not hold for this state", "the statement holds for this state",
                   "false", "true", "—", "1.", "2.", "3.", "4.", "5."]


def synthetic_corpus(seed: int = 0, n_words: int = 120_000) -> list[str]:
    import random
    r = random.Random(seed)
    lines = []
    words = []
    for _ in range(n_words):
        x = r.random()
        if x < 0.06:
            w = str(r.randint(0, 99999))
        elif x < 0.10:
            w = r.choice([".", ",", "!", "?", ":", ";", "(", ")", "\"", "'s", "-", "{", "}", "[", "]"])
        elif x < 0.14:
            w = r.choice(_TEMPLATE_WORDS)
        else:
            w = "".join(r.choice(_SYLLABLES) for _ in range(r.choice([1, 1, 2, 2, 2, 3, 3, 4])))
            if r.random() < 0.1:
                w = w.capitalize()
        words.append(w)
        if r.random() < 0.05:
            lines.append(" ".join(words))
            words = []
    lines.append(" ".join(words))
    return lines


def write_synthetic_tokenizer(path: str, seed: int = 0, vocab_size: int = 6000) -> None:
    """Trains a byte-level BPE of the shape `Tokenizer::from_json` accepts on :func:`synthetic_corpus`
    and writes it to ``path``."""
    from tokenizers import Regex, Tokenizer as HFTokenizer, models, normalizers, pre_tokenizers, trainers, decoders

    tok = HFTokenizer(models.BPE())
    tok.normalizer = normalizers.NFC()
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(SPLIT_PATTERN), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False),
    ])
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=vocab_size, min_frequency=2, show_progress=False,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), special_tokens=[])
    tok.train_from_iterator(synthetic_corpus(seed), trainer=trainer)
    tok.add_special_tokens(SPECIAL_TOKENS)
    data = json.loads(tok.to_str())
    for t in data["added_tokens"]:
        t["normalized"] = False
    with open(path, "w") as f:
        json.dump(data, f, ensure_ascii=False)
