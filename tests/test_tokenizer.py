"""The C++ BPE tokenizer of libcortex (cortex_tokenizer_*) against the
oracle's restatement of src/snai_tokenizer.php (oracle/tokenizer.py):
hand-derived known answers on a tiny vocabulary, random texts on a seeded
BPE vocabulary (tests/golden/tokenizer_vocab.json), and the reference's own
round-trip check (src/snai_tokenizer.php:202-227) when its vocabulary file
is at hand.  Host code only: runs without a GPU."""
import ctypes
import json
import os

import numpy as np
import pytest

from conftest import ROOT
from oracle.tokenizer import Tokenizer

FIXTURE = os.path.join(ROOT, "tests", "golden", "tokenizer_vocab.json")
REF_VOCAB = "/root/reference/lib/symbio_vocab.json"  # used only when present
META = "▁"


class CTok:
    def __init__(self, path):
        from snai_b200 import load
        self.lib = load()
        self.h = self.lib.cortex_tokenizer_load(str(path).encode())
        assert self.h, self.lib.cortex_last_error()

    def encode(self, text):
        raw = text.encode("utf-8") if isinstance(text, str) else text
        n = self.lib.cortex_tokenizer_encode(self.h, raw, len(raw), None, 0)
        ids = np.zeros(max(n, 1), dtype=np.int32)
        assert self.lib.cortex_tokenizer_encode(self.h, raw, len(raw), ids.ctypes.data_as(ctypes.c_void_p), n) == n
        return ids[:n].tolist()

    def decode(self, ids, trim=False):
        a = np.ascontiguousarray(ids, dtype=np.int32)
        n = self.lib.cortex_tokenizer_decode(self.h, a.ctypes.data_as(ctypes.c_void_p), len(a), int(trim), None, 0)
        buf = ctypes.create_string_buffer(n + 1)
        assert self.lib.cortex_tokenizer_decode(self.h, a.ctypes.data_as(ctypes.c_void_p), len(a), int(trim), buf,
                                                n + 1) == n
        return buf.raw[:n].decode("utf-8")

    def close(self):
        self.lib.cortex_tokenizer_free(self.h)


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    vocab = {s: i for i, s in enumerate(["<unk>", "<pad>", "<s>", "</s>", "\n", "[USER]", "[SYMBIO]", "[SYSTEM]"])}
    for t in [META, "a", "b", "c", META + "a", "ab", META + "ab", "?", "ä", META + "ä"]:
        vocab[t] = len(vocab)
    merges = [[META, "a"], ["a", "b"], [META + "a", "b"], [META, "ä"]]
    p = tmp_path_factory.mktemp("tok") / "tiny.json"
    p.write_text(json.dumps({"model": {"vocab": vocab, "merges": merges}}, ensure_ascii=False), encoding="utf-8")
    return str(p), vocab


def test_known_answers(tiny, built):
    path, v = tiny
    c = CTok(path)
    assert c.lib.cortex_tokenizer_vocab_size(c.h) == len(v)
    # "ab" -> " ab" -> "▁ab": (▁,a) rank 0 -> [▁a, b], then (▁a,b) rank 2 -> [▁ab]
    assert c.encode("ab") == [v[META + "ab"]]
    # "abab": " abab" -> [▁a, b, a, b] -> ▁a b merged first (rank 2 < ... no: (a,b) rank 1 < (▁a,b) 2)
    assert c.encode("abab") == Tokenizer(path).encode("abab")
    # a special token and a part with no leading space: the part is dropped (preg_match_all)
    assert c.encode("[USER]ab") == [v["[USER]"]]
    assert c.encode("[USER] ab\n[SYMBIO] c") == [v["[USER]"], v[META + "ab"], v["\n"], v["[SYMBIO]"], v[META],
                                                 v["c"]]
    # unknown pieces -> <unk>; invalid UTF-8 -> '?'
    assert c.encode("zz") == [v[META], v["<unk>"], v["<unk>"]]
    assert c.encode(b"\xff") == [v[META], v["?"]]
    assert c.encode(" ä") == [v[META + "ä"]]
    assert c.encode("") == []
    # decode: U+2581 -> ' ', unknown ids skipped, trim
    assert c.decode([v[META + "ab"], 999, v["\n"]]) == " ab\n"
    assert c.decode([v[META + "ab"], v["\n"]], trim=True) == "ab"
    c.close()


def test_random_texts_match_oracle(built):
    c, o = CTok(FIXTURE), Tokenizer(FIXTURE)
    rng = np.random.default_rng(0)
    alphabet = list("abcdeinrstäöüß ABC0123.,!?'\n") + ["[USER]", "[SYMBIO]", "</s>", "<s>", "  ", "\t", "€", "漢",
                                                            META, META + "a", "<", "[", "<s", "[US", "</"]
    for i in range(300):
        text = "".join(rng.choice(alphabet, size=int(rng.integers(0, 60))))
        if i % 7 == 0:
            raw = text.encode("utf-8") + bytes(rng.integers(0, 256, 3).tolist())  # invalid bytes
            assert c.encode(raw) == o.encode(raw), raw
        else:
            ids = c.encode(text)
            assert ids == o.encode(text), text
            assert c.decode(ids) == o.decode(ids)
            assert c.decode(ids, trim=True) == o.decode(ids, trim=True)
    c.close()


def test_long_text_matches_oracle(built):
    """One long text of many distinct words (the per-chunk memo grows and
    rehashes several times), encoded twice (the second time from the memo)."""
    c, o = CTok(FIXTURE), Tokenizer(FIXTURE)
    rng = np.random.default_rng(2)
    letters = list("abcdeinrstäöüßABC")
    words = ["".join(rng.choice(letters, size=int(rng.integers(1, 9)))) for _ in range(6000)]
    text = " ".join(words[int(i)] + ("\n" if k % 13 == 12 else "") for k, i in enumerate(rng.integers(0, 6000, 20000)))
    want = o.encode(text)
    assert c.encode(text) == want
    assert c.encode(text) == want
    c.close()


@pytest.mark.skipif(not os.path.exists(REF_VOCAB), reason="the reference's vocabulary file is not here")
def test_reference_vocabulary_round_trip(built):
    """src/snai_tokenizer.php:202-227: its test string survives encode ->
    decode exactly; the ids equal the oracle's."""
    c, o = CTok(REF_VOCAB), Tokenizer(REF_VOCAB)
    s = "[USER] Definiere eine Python Funktion:\n[SYMBIO] def hallo():\n    print('Test')</s>"
    ids = c.encode(s)
    assert c.lib.cortex_tokenizer_vocab_size(c.h) == 16384
    assert ids == o.encode(s)
    assert c.decode(ids) == s
    rng = np.random.default_rng(1)
    words = ["der", "die", "und", "Symbio", "Python", "def", "print", "(", ")", ":", "\n", " ", "[USER]", "ß", "ü"]
    for _ in range(50):
        t = " ".join(rng.choice(words, size=20))
        assert c.encode(t) == o.encode(t)
    c.close()
