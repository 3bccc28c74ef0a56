"""The tokenizer restatement (jieyu_b200/tokenizer.py) against the
reference's own json_libs::Tokenizer (libs/tokenizer_libs/include/
tokenizer.h, compiled from its sources into oracle/_ref): for the same
vocab.json / merges.txt files, the same ids for every text (ASCII, CJK,
full-width punctuation, 4-byte characters, invalid and truncated UTF-8,
special tokens inside the text, added special tokens, random bytes), the same
bytes back from decode, and the same special-token ids and vocabulary size.
The vocabularies are trained here by a small byte-level BPE (any valid files
serve: the test pins the reading and the encoding, not the training), written
with JSON \\u escapes, with and without the "</w>" word-end token.
"""
import collections
import ctypes as C
import json
import os

import numpy as np
import pytest

from jieyu_b200 import tokenizer as T
from oracle.bind import REF_SO

CORPUS = [
    "The quick brown fox jumps over the lazy dog. The dog sleeps; the fox runs!",
    "Hello, world -- hello again?  Two  spaces,\tand a tab.\nNew line (parens) [brackets] {braces}.",
    "我们今天学习分词器。你好，世界！这是一个测试：中文、标点和数字 123。",
    "naïve café résumé — “quotes” … ellipsis ¿qué? ¡sí! 😀 🚀 emoji",
    "def f(x): return x * 2 + 1  # code-like text with == and != and ->",
    "ＦｕｌｌＷｉｄｔｈ　ｓｐａｃｅ　ａｎｄ　ｐｕｎｃｔ！？",
]

TEXTS = CORPUS + [
    "", " ", "  ", " leading space", "trailing space ", "a . b , c", " .", "x　y", "tab\t\tend",
    "The fox. 我们的狐狸！", "<unk> inside <unk>", "no specials here",
    T.BOS_TOKEN.decode() + "hello" + T.EOS_TOKEN.decode(), "mixed " + T.EOS_TOKEN.decode() + " tail",
    b"\xff\xfe invalid bytes \xc3", b"truncated \xe4\xb8", b"\xf0\x9f\x98", b"\x00\x01\x7f ctrl",
]


def _train(corpus, merges_n, word_end):
    """Byte-level BPE: words by the reference's split, symbols = byte-level
    characters (+ "</w>"), greedy most-frequent pair merges."""
    words = collections.Counter()
    for text in corpus:
        data = text.encode()
        for a, b in T.split_word_ranges(data):
            sym = tuple(T._TO_CHAR[c] for c in data[a:b]) + ((T.WORD_END_TOKEN,) if word_end else ())
            words[sym] += 1
    vocab = {p: i for i, p in enumerate(T._TO_CHAR)}
    if word_end:
        vocab[T.WORD_END_TOKEN] = len(vocab)
    merges = []
    for _ in range(merges_n):
        pairs = collections.Counter()
        for w, c in words.items():
            for x, y in zip(w, w[1:]):
                pairs[(x, y)] += c
        if not pairs:
            break
        (x, y), _c = max(pairs.items(), key=lambda kv: (kv[1], kv[0]))
        merges.append((x, y))
        vocab.setdefault(x + y, len(vocab))
        new = collections.Counter()
        for w, c in words.items():
            out, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and w[i] == x and w[i + 1] == y:
                    out.append(x + y)
                    i += 2
                else:
                    out.append(w[i])
                    i += 1
            new[tuple(out)] += c
        words = new
    return vocab, merges


def _write(d, vocab, merges, extra=()):
    os.makedirs(d, exist_ok=True)
    v = {p.decode("utf-8", "surrogatepass"): i for p, i in vocab.items()}
    for p in extra:
        v.setdefault(p, len(v))
    with open(os.path.join(d, "vocab.json"), "w", encoding="ascii") as f:
        json.dump(v, f, ensure_ascii=True)  # \\u escapes for every non-ASCII piece
    with open(os.path.join(d, "merges.txt"), "wb") as f:
        f.write(b"#version: test\n")
        for x, y in merges:
            f.write(x + b" " + y + b"\n")
    return os.path.join(d, "vocab.json"), os.path.join(d, "merges.txt")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_SO):
        pytest.skip("reference harness not built (reference tree absent)")
    lib = C.CDLL(REF_SO)
    P = C.c_void_p
    lib.jyref_tok_load.restype = P
    lib.jyref_tok_load.argtypes = [C.c_char_p, C.c_char_p]
    lib.jyref_tok_free.argtypes = [P]
    lib.jyref_tok_encode.restype = C.c_int
    lib.jyref_tok_encode.argtypes = [P, C.c_char_p, C.c_int, P, C.c_int]
    lib.jyref_tok_decode.restype = C.c_int
    lib.jyref_tok_decode.argtypes = [P, P, C.c_int, P, C.c_int]
    lib.jyref_tok_info.argtypes = [P, P]
    lib.jyref_tok_add_special.restype = C.c_int
    lib.jyref_tok_add_special.argtypes = [P, C.c_char_p]
    return lib


def _ref_encode(lib, h, data: bytes):
    out = np.zeros(4 * len(data) + 16, np.int32)
    n = lib.jyref_tok_encode(h, data, len(data), out.ctypes.data, len(out))
    return [int(x) for x in out[:n]]


def _ref_decode(lib, h, ids):
    a = np.asarray(ids, np.int32)
    buf = C.create_string_buffer(64 * len(ids) + 16)
    n = lib.jyref_tok_decode(h, a.ctypes.data, len(a), buf, len(buf))
    return buf.raw[:n]


@pytest.mark.parametrize("word_end", [True, False])
def test_tokenizer_matches_reference(ref, tmp_path, word_end):
    vocab, merges = _train(CORPUS, 400, word_end)
    vp, mp = _write(str(tmp_path), vocab, merges, extra=["<|im_end|>"])
    h = ref.jyref_tok_load(vp.encode(), mp.encode())
    assert h
    try:
        tok = T.Tokenizer()
        assert tok.load(vp, mp)
        info = np.zeros(5, np.int32)
        ref.jyref_tok_info(h, info.ctypes.data)
        assert [tok.bos_id, tok.eos_id, tok.unk_id, tok.word_end_id, tok.vocab_size] == [int(x) for x in info]
        assert (tok.word_end_id >= 0) == word_end
        rng = np.random.default_rng(7)
        pool = [t if isinstance(t, bytes) else t.encode() for t in TEXTS]
        fuzz = [bytes(rng.integers(0, 256, size=int(rng.integers(1, 40)), dtype=np.uint8)) for _ in range(150)]
        mixed = [b"".join(pool[int(i)][: int(rng.integers(0, 20))] for i in rng.integers(0, len(pool), 4))
                 for _ in range(100)]
        # long words (no spaces): many merges interact within one word
        joined = "".join(CORPUS).replace(" ", "").replace("\n", "")
        letters = sorted(set(joined))
        long_words = [("".join(rng.choice(letters, size=n))).encode() for n in (64, 257, 1000)]
        long_words += [b"abab" * 300, joined[:1500].encode()]
        for data in pool + fuzz + mixed + long_words:
            want = _ref_encode(ref, h, data)
            got = tok.encode(data)
            assert got == want, data
            assert tok.decode(got) == _ref_decode(ref, h, want), data
        # an added special token is matched before the words
        assert tok.add_special_token(b"<|im_end|>") == ref.jyref_tok_add_special(h, b"<|im_end|>") >= 0
        for data in [b"chat<|im_end|>next", b"<|im_end|><|im_end|>", b"a <|im_end|> b"]:
            assert tok.encode(data) == _ref_encode(ref, h, data)
    finally:
        ref.jyref_tok_free(h)


def test_tokenizer_round_trips_text(tmp_path):
    vocab, merges = _train(CORPUS, 300, True)
    vp, mp = _write(str(tmp_path), vocab, merges)
    tok = T.Tokenizer()
    assert tok.load(vp, mp)
    for text in CORPUS:
        ids = tok.encode(text)
        assert len(ids) < len(text.encode())  # the merges compress
        assert tok.decode(ids) == text.encode()
    assert not T.Tokenizer().load(str(tmp_path / "missing.json"), mp)
