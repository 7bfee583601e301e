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
