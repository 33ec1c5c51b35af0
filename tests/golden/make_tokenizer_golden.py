"""Writes tests/golden/tokenizer_vectors.json from the reference crate's own tokenizer test data:
the 12 records of tests/data/reference_test_vectors.json (raw text, query or document, ids), the
7 long texts of tests/data/long_texts.txt with the ids of tests/data/long_reference_vectors.json,
and the vocabulary entries (model/vocab.txt) those ids use. Greedy longest-match WordPiece picks
the same pieces from this subset as from the full vocabulary for these texts, because every
piece it picked from the full vocabulary is in the subset.

    python tests/golden/make_tokenizer_golden.py <reference crate directory>
"""
import json
import os
import sys

ref = sys.argv[1]
short = json.load(open(os.path.join(ref, "tests/data/reference_test_vectors.json")))
long_ids = json.load(open(os.path.join(ref, "tests/data/long_reference_vectors.json")))
long_texts = open(os.path.join(ref, "tests/data/long_texts.txt"), encoding="utf-8").read().splitlines()
vocab = open(os.path.join(ref, "model/vocab.txt"), encoding="utf-8").read().split("\n")
if vocab and vocab[-1] == "":
    vocab.pop()
records = [{"kind": r["kind"], "text": r["raw_text"], "ids": r["ids"]} for r in short]
records += [{"kind": "document", "text": t, "ids": r["ids"], "name": r["name"]} for r, t in zip(long_ids, long_texts)]
used = {0, 100, 101, 102, 103}
for r in records:
    used.update(r["ids"])
out = {"source": "reference crate tests/data + model/vocab.txt", "vocab_size": len(vocab),
       "vocab_subset": {str(i): vocab[i] for i in sorted(used)}, "records": records}
path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tokenizer_vectors.json")
with open(path, "w", encoding="utf-8") as f:
    json.dump(out, f, ensure_ascii=False, indent=0)
print(path, len(records), "records,", len(used), "vocabulary entries")
