"""Host-side tokenizer of the nomic-bert embedder (internal/embed/tokenizer.go).

The reference keeps tokenisation on the host and hands token ids to the
forward pass; this module is that host step for the Python host.  It follows
tokenizer.go exactly:

* Encode (tokenizer.go:47-80): lowercase (Go's per-rune simple case mapping),
  split into words on whitespace and punctuation (punctuation characters are
  words of their own), encode each word, frame with [CLS]=101 / [SEP]=102,
  and when longer than maxLen keep the first maxLen ids with [SEP] last.
* encodeWord (tokenizer.go:84-142): the whole word with the SentencePiece
  prefix U+2581 if it is in the vocabulary, else greedy longest match over
  the word's UTF-8 *bytes* (pieces at most the longest vocabulary entry; the
  first piece carries the prefix), falling back to single bytes (prefixed,
  then bare) and [UNK]=100 per byte.
* preTokenize / isBertPunct (tokenizer.go:150-191): Go's unicode.IsSpace;
  ASCII punctuation, Unicode category P and the CJK ideograph blocks count as
  punctuation.
* LoadTokenizer (tokenizer.go:24-44, 194-330): the vocabulary is the GGUF
  string array "tokenizer.ggml.tokens"; token -> id with later duplicates
  winning, as a Go map assignment does.
"""
from __future__ import annotations

import struct
import unicodedata

PREFIX = "\u2581".encode()
CLS, SEP, UNK = 101, 102, 100

# unicode.IsSpace: the Latin-1 spaces and the White_Space property above it.
_GO_SPACE = frozenset("\t\n\v\f\r \x85\xa0\u1680\u2000\u2001\u2002\u2003\u2004\u2005\u2006\u2007\u2008"
                      "\u2009\u200a\u2028\u2029\u202f\u205f\u3000")


def _go_lower(text: str) -> str:
    """strings.ToLower: unicode.ToLower per rune (the simple mapping; unlike
    str.lower() no multi-character results and no final-sigma context)."""
    out = []
    for ch in text:
        if ch < "\x80":
            out.append(ch.lower())
            continue
        if ch == "\u0130":  # LATIN CAPITAL LETTER I WITH DOT ABOVE -> 'i'
            out.append("i")
            continue
        lo = ch.lower()
        out.append(lo if len(lo) == 1 else ch)
    return "".join(out)


def _is_bert_punct(ch: str) -> bool:
    o = ord(ch)
    if 0x21 <= o <= 0x2F or 0x3A <= o <= 0x40 or 0x5B <= o <= 0x60 or 0x7B <= o <= 0x7E:
        return True
    if unicodedata.category(ch).startswith("P"):
        return True
    return 0x4E00 <= o <= 0x9FFF or 0x3400 <= o <= 0x4DBF or 0x20000 <= o <= 0x2A6DF


def pre_tokenize(text: str) -> list[str]:
    """preTokenize (tokenizer.go:150-174)."""
    text = _go_lower(text)
    words, cur = [], []
    for ch in text:
        if ch in _GO_SPACE:
            if cur:
                words.append("".join(cur))
                cur = []
        elif _is_bert_punct(ch):
            if cur:
                words.append("".join(cur))
                cur = []
            words.append(ch)
        else:
            cur.append(ch)
    if cur:
        words.append("".join(cur))
    return words


def read_gguf_string_array(path: str, key: str) -> list[bytes]:
    """readGGUFStringArray (tokenizer.go:194-250): scan the KV section for an
    array of strings named `key`; values returned as raw bytes."""
    with open(path, "rb") as f:
        buf = f.read()
    pos = 24
    if buf[:4] != b"GGUF":
        raise ValueError("gguf: invalid magic")
    n_kv = struct.unpack_from("<Q", buf, 16)[0]
    sizes = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}

    def string():
        nonlocal pos
        n = struct.unpack_from("<Q", buf, pos)[0]
        s = buf[pos + 8:pos + 8 + n]
        pos += 8 + n
        return s

    def skip(vt):
        nonlocal pos
        if vt in sizes:
            pos += sizes[vt]
        elif vt == 8:
            string()
        elif vt == 9:
            et, n = struct.unpack_from("<IQ", buf, pos)
            pos += 12
            for _ in range(n):
                skip(et)
        else:
            raise ValueError(f"gguf: unknown value type {vt}")

    for _ in range(n_kv):
        k = string()
        vt = struct.unpack_from("<I", buf, pos)[0]
        pos += 4
        if k == key.encode() and vt == 9:
            et, n = struct.unpack_from("<IQ", buf, pos)
            pos += 12
            if et != 8:
                raise ValueError(f"expected string array, got element type {et}")
            return [string() for _ in range(n)]
        skip(vt)
    raise KeyError(f"key {key!r} not found in GGUF metadata")


class WordPieceTokenizer:
    """WordPieceTokenizer (tokenizer.go:13-19)."""

    def __init__(self, tokens: list[bytes]):
        self.vocab = {}
        for i, t in enumerate(tokens):
            self.vocab[t] = i
        self.id_to_tok = tokens
        self.max_token = max((len(t) for t in tokens), default=0)

    @classmethod
    def Load(cls, path: str) -> "WordPieceTokenizer":
        return cls(read_gguf_string_array(path, "tokenizer.ggml.tokens"))

    def VocabSize(self) -> int:
        return len(self.id_to_tok)

    def encode_word(self, word: str) -> list[int]:
        """encodeWord (tokenizer.go:84-142), over the word's UTF-8 bytes."""
        w = word.encode()
        tid = self.vocab.get(PREFIX + w)
        if tid is not None:
            return [tid]
        ids = []
        start, n = 0, len(w)
        while start < n:
            end = min(n, start + self.max_token)
            found = False
            while end > start:
                cand = (PREFIX + w[start:end]) if start == 0 else w[start:end]
                tid = self.vocab.get(cand)
                if tid is not None:
                    ids.append(tid)
                    start = end
                    found = True
                    break
                end -= 1
            if not found:
                if start == 0:
                    tid = self.vocab.get(PREFIX + w[0:1])
                    if tid is not None:
                        ids.append(tid)
                        start += 1
                        continue
                tid = self.vocab.get(w[start:start + 1])
                ids.append(UNK if tid is None else tid)
                start += 1
        return ids

    def Encode(self, text: str, max_len: int) -> tuple[list[int], list[int]]:
        """Encode (tokenizer.go:47-80): token ids and the all-ones mask."""
        ids = [CLS]
        for word in pre_tokenize(text):
            ids.extend(self.encode_word(word))
        ids.append(SEP)
        if len(ids) > max_len:
            ids = ids[:max_len]
            ids[max_len - 1] = SEP
        return ids, [1] * len(ids)
