"""Writes tests/golden/tokenizer_vocab.json: a small HF-style BPE vocabulary
(the layout of the reference's lib/symbio_vocab.json: model.vocab,
model.merges as [a, b] pairs, the eight special tokens at ids 0-7, U+2581
word prefix) learnt by plain BPE merges on a seeded synthetic corpus.  Test
fixture only; run once: python tests/golden/make_tokenizer_vocab.py"""
import collections
import json
import os

import numpy as np

META = "▁"
SPECIALS = ["<unk>", "<pad>", "<s>", "</s>", "\n", "[USER]", "[SYMBIO]", "[SYSTEM]"]


def main(n_merges=600, seed=11):
    rng = np.random.default_rng(seed)
    letters = list("abcdefghijklmnopqrstuvwxyzäöüß") + list("ABCDEFGHIJKLMNOPQRSTUVWXYZ") + list("0123456789.,:;!?()'\"-_=+*/")
    probs = np.array([8 if c in "aeinrst" else 3 if c.islower() else 1 for c in letters], dtype=np.float64)
    probs /= probs.sum()
    words = collections.Counter()
    for _ in range(6000):
        w = "".join(rng.choice(letters, size=int(rng.integers(1, 9)), p=probs))
        words[META + w] += int(rng.integers(1, 20))
    vocab = {s: i for i, s in enumerate(SPECIALS)}
    for ch in [META] + letters:
        vocab.setdefault(ch, len(vocab))
    seqs = {w: list(w) for w in words}
    merges = []
    for _ in range(n_merges):
        pairs = collections.Counter()
        for w, f in words.items():
            s = seqs[w]
            for a, b in zip(s, s[1:]):
                pairs[(a, b)] += f
        if not pairs:
            break
        (a, b), _ = max(pairs.items(), key=lambda kv: (kv[1], kv[0]))
        merges.append([a, b])
        vocab.setdefault(a + b, len(vocab))
        for w in seqs:
            s, out, i = seqs[w], [], 0
            while i < len(s):
                if i + 1 < len(s) and s[i] == a and s[i + 1] == b:
                    out.append(a + b)
                    i += 2
                else:
                    out.append(s[i])
                    i += 1
            seqs[w] = out
    doc = {"version": "1.0", "truncation": None, "padding": None,
           "added_tokens": [{"id": i, "content": s, "special": True} for i, s in enumerate(SPECIALS)],
           "model": {"type": "BPE", "unk_token": "<unk>", "vocab": vocab, "merges": merges}}
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tokenizer_vocab.json")
    with open(path, "w", encoding="utf-8") as f:
        json.dump(doc, f, ensure_ascii=False, indent=1)
    print(path, len(vocab), "tokens", len(merges), "merges")


if __name__ == "__main__":
    main()
