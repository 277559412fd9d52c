"""Extracts the reference's prompt and tokenizer fixtures into tests/golden/prompt_cases.json.

Run in a container where the reference checkout is mounted (its path is the first argument); the
output is committed, because the reference is not available where the GPU tests run.

    python tests/golden/make_golden.py <reference checkout>

From tests/fixtures/expected.json (made by the reference's tests/fixtures/make.py from the official
package) it keeps, per case: the request, the official rendering of each question, the state and
question token counts (the real vocabulary's, kept only as length distributions) and the option
token indices; and the 21 raw tokenizer edge-case strings (their ids are for the real vocabulary,
which is not available here, so only the texts are kept).
"""
import json
import os
import sys

ref = sys.argv[1]
with open(os.path.join(ref, "tests/fixtures/expected.json")) as f:
    d = json.load(f)
cases = [{
    "name": c["name"],
    "request": c["request"],
    "question_text": c["question_text"],
    "state_len": len(c["state_ids"]),
    "question_lens": [len(q) for q in c["question_ids"]],
    "option_idx": c["option_idx"],
} for c in d["cases"]]
raw = [r["text"] for r in d["raw"]]
out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "prompt_cases.json")
with open(out, "w") as f:
    json.dump({"source": "reference tests/fixtures/expected.json", "cases": cases, "raw_texts": raw}, f,
              ensure_ascii=False, indent=0)
print(len(cases), "cases,", len(raw), "raw strings ->", out)
