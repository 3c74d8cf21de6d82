"""Text I/O (aion_tokenizer_*, aion_encode, aion_decode) against its CPU
restatement (oracle/tokenizer_ref.py) on a synthetic llama2.c-format
vocabulary: byte-fallback pieces, single characters, multi-byte UTF-8
characters and scored merges.  Encodings must be identical, and decoding
an encoding must give the text back."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import tokenizer_ref as T


def vocab():
    pieces = [b"<unk>", b"\n<s>\n", b"\n</s>\n"] + [b"<0x%02X>" % b for b in range(256)]
    singles = [bytes([c]) for c in range(32, 127)] + ["é".encode(), "中".encode(), "ß".encode(), b"\n"]
    merges = [b" t", b"th", b" th", b"he", b"the", b" the", b"in", b"ing", b" a", b"an", b"and", b" and",
              b"er", b" w", b"wor", b"ld", b" world", b"es", b"est", b"  ", b"    ", "é t".encode(), b"ab", b"abc"]
    pieces += singles + merges
    rng = np.random.default_rng(3)
    scores = np.concatenate([np.zeros(259), -np.arange(len(singles), dtype=np.float32),
                             rng.uniform(1, 10, len(merges)).astype(np.float32)]).astype(np.float32)
    return pieces, scores


TEXTS = ["", "the world", "Hello, the world and the rest!", "  indented    text\nnext line",
         "café été", "中文 and ß", "emoji \U0001F600 and \U0001F680", "tab\there", "abcabc ab a",
         "é té test", "x" * 50]


@pytest.fixture(scope="module")
def tok(built, tmp_path_factory):
    import aion_b200 as A
    pieces, scores = vocab()
    p = tmp_path_factory.mktemp("tok") / "tokenizer.bin"
    T.write_tokenizer(p, pieces, scores)
    t = A.Tokenizer(p, len(pieces))
    yield t, pieces, scores
    t.close()


@pytest.mark.parametrize("text", TEXTS)
@pytest.mark.parametrize("bos,eos", [(True, False), (False, False), (True, True)])
def test_encode_matches_restatement(tok, text, bos, eos):
    t, pieces, scores = tok
    assert t.encode(text, bos, eos) == T.encode(pieces, scores, text, bos, eos)


@pytest.mark.parametrize("text", TEXTS)
def test_decode_round_trip(tok, text):
    t, pieces, _ = tok
    ids = t.encode(text, True, True)
    assert t.decode(ids) == text
    assert T.decode(pieces, ids) == text.encode("utf-8")


def test_byte_fallback_and_bounds(tok):
    t, _, _ = tok
    ids = t.encode("\U0001F600", False, False)         # 4 bytes, not in the vocabulary
    assert len(ids) == 5 and ids[1:] == [b + 3 for b in "\U0001F600".encode()]
    assert t.decode_bytes(-1, 3 + 0x41) == b"A"
    with pytest.raises(ValueError):
        t.decode_bytes(-1, 10 ** 6)


def test_truncated_file_is_rejected(built, tmp_path):
    import aion_b200 as A
    pieces, scores = vocab()
    p = tmp_path / "tok.bin"
    T.write_tokenizer(p, pieces, scores)
    p.write_bytes(p.read_bytes()[:-5])
    with pytest.raises(A.AionError):
        A.Tokenizer(p, len(pieces))
