"""Host tokenizer (internal/embed/tokenizer.go) on the synthetic vocabulary.

Expected token strings are worked out by hand from tokenizer.go's rules
(greedy longest match over UTF-8 bytes, U+2581 on the first piece, byte-wise
[UNK] fallback, Go's IsSpace and BERT punctuation, truncation keeping [SEP]);
the reference's own TestTokenizer (embedder_test.go:147-176) pins only the
[CLS]/[SEP] framing, the all-ones mask and the vocabulary size, checked too.
"""
import pytest

from llm_embed_b200 import synth
from llm_embed_b200.tokenizer import WordPieceTokenizer, _go_lower, pre_tokenize

P = "▁"


@pytest.fixture(scope="module")
def tok():
    path = synth.cached_model(synth.ModelSpec(layers=1, vocab=30522, seed=5))
    return WordPieceTokenizer.Load(path)


def strings(tok, ids):
    return [tok.id_to_tok[i].decode("utf-8", "replace") for i in ids]


def test_reference_tokenizer_contract(tok):
    """embedder_test.go:147-176."""
    assert tok.VocabSize() == 30522
    ids, mask = tok.Encode("hello world", 512)
    assert len(ids) >= 3 and ids[0] == 101 and ids[-1] == 102
    assert mask == [1] * len(ids)


@pytest.mark.parametrize("text,expected", [
    ("Hello, World!", [P + "hello", P + ",", P + "world", P + "!"]),
    ("search_query: what is machine learning",
     [P + "search", P + "_", P + "query", P + ":", P + "what", P + "is", P + "machine", P + "learning"]),
    ("tokenization", [P + "token", "ization"]),
    ("tokenizer", [P + "token", "izer"]),
    ("unable", [P + "un", "able"]),
    ("café", [P + "caf", "[UNK]", "[UNK]"]),
    ("Über", [P + "über"]),
    ("中文", [P + "中", P + "文"]),
    ("xyz", [P + "x", "y", "z"]),
    ("hello world", [P + "hello", P + "world"]),
    ("hello\x1cworld", [P + "hello", "[UNK]", "wor", "ld"]),
    ("  \t\n", []),
    ("", []),
])
def test_encode_known_answers(tok, text, expected):
    ids, _ = tok.Encode(text, 512)
    assert ids[0] == 101 and ids[-1] == 102
    assert strings(tok, ids[1:-1]) == expected


def test_truncation_keeps_sep(tok):
    ids, mask = tok.Encode("hello world", 3)
    assert strings(tok, ids) == ["[CLS]", P + "hello", "[SEP]"]
    assert len(mask) == 3
    ids, _ = tok.Encode("hello world", 4)
    assert strings(tok, ids) == ["[CLS]", P + "hello", P + "world", "[SEP]"]


def test_go_lowercase_and_split():
    assert _go_lower("HeLLo") == "hello"
    assert _go_lower("İ") == "i"            # unicode.ToLower(U+0130) = 'i'
    assert _go_lower("ΟΔΟΣ") == "οδοσ"  # no final-sigma rule
    assert pre_tokenize("a.b  c") == ["a", ".", "b", "c"]
    assert pre_tokenize("x　y z") == ["x", "y", "z"]   # White_Space above Latin-1
    assert pre_tokenize("¿qué?") == ["¿", "qué", "?"]  # category P


# ------------------------------------------------ the C++ host tokenizer --

def _random_texts(n, seed):
    """Texts mixing vocabulary words, unknown words, mixed case, Unicode
    letters with and without simple lowercase mappings, punctuation of every
    kind, CJK and unusual whitespace."""
    import numpy as np
    rng = np.random.default_rng(seed)
    pieces = ["hello", "World", "MACHINE", "learning", "tokenization", "unable", "café", "Über", "straße",
              "İstanbul", "ΟΔΟΣ", "Σίσυφος", "中文", "日本語", "x", "qzx", "caf́e", "a.b", "(x)", "¿qué?",
              "—", "…", "«quote»", "!!", "$5", "e=mc²", " ", "　", "\t", " ", "\u0085", "ǅ",
              "ǈ", "ﬁ", "K", "Å", "\U0001F600", "\U00020000", "naïve", "ß"]
    out = []
    for _ in range(n):
        k = int(rng.integers(0, 12))
        seps = [" ", "", "  ", "\n", "　"]
        out.append("".join(pieces[int(rng.integers(len(pieces)))] + seps[int(rng.integers(len(seps)))]
                           for _ in range(k)))
    return out


@pytest.fixture(scope="module")
def native(tok):
    from llm_embed_b200.embed import Tokenizer
    path = synth.cached_model(synth.ModelSpec(layers=1, vocab=30522, seed=5))
    t = Tokenizer.Load(path)
    yield t
    t.close()


def test_native_matches_restatement(tok, native):
    """le_tokenize gives the Python restatement's ids on the known-answer
    texts and on 2,000 random texts, one at a time and as one threaded batch,
    at several truncation lengths."""
    texts = ["Hello, World!", "search_query: what is machine learning", "tokenization", "café", "Über", "中文",
             "xyz", "hello\x1cworld", "  \t\n", ""] + _random_texts(2000, 7)
    assert native.VocabSize() == tok.VocabSize()
    for max_len in (512, 9, 2):
        ids, offs = native.encode_batch(texts, max_len, prefix="search_query: ", nthreads=8)
        for i, t in enumerate(texts):
            want = tok.Encode("search_query: " + t, max_len)[0]
            assert ids[offs[i]:offs[i + 1]].tolist() == want, (max_len, t)
    for t in texts[:50]:
        assert native.Encode(t, 512)[0] == tok.Encode(t, 512)[0]


def test_native_invalid_utf8_reads_as_replacement_char(native):
    """Go's range loop reads each byte of an invalid UTF-8 sequence as U+FFFD
    (strings.ToLower writes it as EF BF BD); U+FFFD is not in the vocabulary,
    so each becomes three byte pieces, here [UNK] each."""
    ids, offs = native.encode_batch([b"ab\xffcd", b"\xe2\x82"], 512)
    a = ids[offs[0]:offs[1]].tolist()
    b = ids[offs[1]:offs[2]].tolist()
    assert a[0] == 101 and a[-1] == 102 and b == [101, 100, 100, 100, 100, 100, 100, 102]
    ref, _ = native.encode_batch(["ab�cd"], 512)
    assert a == ref.tolist()


def test_native_duplicates_later_wins_and_capacity():
    """A later duplicate token takes the id (a Go map assignment); too small
    an ids buffer is reported with the needed size in the offsets."""
    import ctypes as C

    import numpy as np

    from llm_embed_b200.embed import LlmEmbedError, Tokenizer, lib
    vocab = ["[PAD]"] * 100 + ["[UNK]", "[CLS]", "[SEP]", "▁ab", "▁ab", "c"]
    t = Tokenizer.from_tokens(vocab)
    try:
        assert t.Encode("ab abc", 16)[0] == [101, 104, 104, 105, 102]
        toffs = np.array([0, 6], np.int64)
        offs = np.zeros(2, np.int32)
        ids = np.zeros(2, np.int32)
        rc = lib().le_tokenize(t._h, b"ab abc", toffs.ctypes.data_as(C.POINTER(C.c_int64)), 1, None, 16,
                               ids.ctypes.data_as(C.POINTER(C.c_int32)), 2, offs.ctypes.data_as(C.POINTER(C.c_int32)),
                               1)
        assert rc == -1 and offs[-1] == 5
    finally:
        t.close()
    with pytest.raises(LlmEmbedError):
        Tokenizer.Load("/nonexistent.gguf")
