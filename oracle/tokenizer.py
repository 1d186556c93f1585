"""TEST INFRASTRUCTURE ONLY: a Python restatement of the reference's BPE
tokenizer (src/snai_tokenizer.php), the checker of the library's C++
tokenizer (cortex_tokenizer_*).  Imported by tests/ only.

Restates, step for step:
  __construct :23-38   vocab = model.vocab, bpe_ranks["a b"] = index of the
                       merge (a later duplicate overwrites), inverse = flip
  bpe         :56-116  split into code points, repeatedly merge the
                       lowest-ranked adjacent pair (every occurrence, left to
                       right), memoised
  encode      :118-185 invalid UTF-8 -> '?', a leading ' ' unless the text
                       starts with ' ', '[' or '<', split on the special
                       tokens present in the vocab (first alternative of the
                       list order that matches at the leftmost position), ' '
                       -> U+2581, chunks (U+2581|\\n)[^U+2581\\n]* (text before
                       a part's first U+2581 is dropped, as preg_match_all
                       does), each chunk's BPE pieces looked up (<unk>, else 0)
  decode      :187-199 concatenate, U+2581 -> ' ', optional trim
NFKC (:128-130) is applied by the PHP code only when the intl extension is
loaded; neither version applies it.  Parity unpinned: PHP is not available
to run the reference itself.
"""
import json
import re

META = "▁"
SPECIALS = ["<unk>", "<pad>", "<s>", "</s>", "\n", "[USER]", "[SYMBIO]", "[SYSTEM]"]


def sanitize_utf8(raw):
    """mb_convert_encoding(text, 'UTF-8', 'UTF-8'): every invalid byte
    sequence (maximal subpart) becomes '?'."""
    if isinstance(raw, str):
        return raw
    out, i, n = [], 0, len(raw)
    while i < n:
        b = raw[i]
        if b < 0x80:
            out.append(chr(b))
            i += 1
            continue
        if 0xC2 <= b <= 0xDF:
            need, lo, hi = 1, 0x80, 0xBF
        elif b == 0xE0:
            need, lo, hi = 2, 0xA0, 0xBF
        elif 0xE1 <= b <= 0xEC or b in (0xEE, 0xEF):
            need, lo, hi = 2, 0x80, 0xBF
        elif b == 0xED:
            need, lo, hi = 2, 0x80, 0x9F
        elif b == 0xF0:
            need, lo, hi = 3, 0x90, 0xBF
        elif 0xF1 <= b <= 0xF3:
            need, lo, hi = 3, 0x80, 0xBF
        elif b == 0xF4:
            need, lo, hi = 3, 0x80, 0x8F
        else:
            out.append("?")
            i += 1
            continue
        j = i + 1
        ok = True
        for k in range(need):
            if j >= n:
                ok = False
                break
            c = raw[j]
            l, h = (lo, hi) if k == 0 else (0x80, 0xBF)
            if not l <= c <= h:
                ok = False
                break
            j += 1
        if ok:
            out.append(raw[i:j].decode("utf-8"))
            i = j
        else:
            out.append("?")
            i = j if j > i + 1 else i + 1
    return "".join(out)


class Tokenizer:
    def __init__(self, path):
        data = json.load(open(path, encoding="utf-8"))
        self.vocab = dict(data["model"]["vocab"])
        self.inverse = {}
        for k, v in data["model"]["vocab"].items():
            self.inverse[v] = k
        self.ranks = {}
        for i, m in enumerate(data["model"].get("merges", [])):
            self.ranks[" ".join(m) if isinstance(m, list) else str(m)] = i
        self.cache = {}

    def vocab_size(self):
        return len(self.vocab)

    def bpe(self, token):
        if token in self.cache:
            return self.cache[token]
        word = list(token)
        if len(word) < 2:
            return token
        while True:
            best, best_rank = None, None
            for a, b in zip(word, word[1:]):
                r = self.ranks.get(a + " " + b)
                if r is not None and (best_rank is None or r < best_rank):
                    best, best_rank = (a, b), r
            if best is None:
                break
            first, second = best
            new, i = [], 0
            while i < len(word):
                try:
                    j = word.index(first, i)
                except ValueError:
                    new.extend(word[i:])
                    break
                new.extend(word[i:j])
                i = j
                if i < len(word) - 1 and word[i] == first and word[i + 1] == second:
                    new.append(first + second)
                    i += 2
                else:
                    new.append(word[i])
                    i += 1
            word = new
            if len(word) == 1:
                break
        out = " ".join(word)
        self.cache[token] = out
        return out

    def encode(self, text):
        text = sanitize_utf8(text)
        if text and text[0] not in (" ", "[", "<"):
            text = " " + text
        specials = [s for s in SPECIALS if s in self.vocab]
        if specials:
            parts = [p for p in re.split("(" + "|".join(re.escape(s) for s in specials) + ")", text) if p != ""]
        else:
            parts = [text]
        unk = self.vocab.get("<unk>", 0)
        ids = []
        for part in parts:
            if part in specials:
                ids.append(self.vocab[part])
                continue
            work = part.replace(" ", META)
            for chunk in re.findall("(?:" + META + "|\n)[^" + META + "\n]*", work):
                for piece in self.bpe(chunk).split(" "):
                    ids.append(self.vocab.get(piece, unk))
        return ids

    def decode(self, ids, trim=False):
        text = "".join(self.inverse[i] for i in ids if i in self.inverse).replace(META, " ")
        return text.strip(" \t\n\r\0\x0b") if trim else text
