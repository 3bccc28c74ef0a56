"""Text layer pieces on the CPU (jieyu_b200.text): the byte-level vocabulary
writer gives the same files as the reference's write_byte_level_vocab
(libs/tokenizer_libs/include/byte_vocab.h, compiled into oracle/_ref); over
them the tokenizer meets the reference's check_pipeline cases 2-5
(libs/text/text.h:963-990: 259 tokens, decode(encode(text)) == text for
English and Chinese, encode("abc") == {97, 98, 99}); the stop-marker scan
follows pipeline.h:201-217."""
import ctypes as C
import os

import pytest

from jieyu_b200 import text as X
from jieyu_b200.tokenizer import Tokenizer
from oracle.bind import REF_SO


def test_byte_vocab_matches_reference_writer(tmp_path):
    if not os.path.exists(REF_SO):
        pytest.skip("reference harness not built (reference tree absent)")
    lib = C.CDLL(REF_SO)
    lib.jyref_write_byte_vocab.argtypes = [C.c_char_p, C.c_char_p]
    lib.jyref_write_byte_vocab.restype = C.c_int
    X.write_byte_level_vocab(str(tmp_path / "v.json"), str(tmp_path / "m.txt"))
    assert lib.jyref_write_byte_vocab(str(tmp_path / "rv.json").encode(), str(tmp_path / "rm.txt").encode()) == 0
    for a, b in (("v.json", "rv.json"), ("m.txt", "rm.txt")):
        assert (tmp_path / a).read_bytes() == (tmp_path / b).read_bytes()


def test_check_pipeline_tokenizer_cases(tmp_path):
    X.write_byte_level_vocab(str(tmp_path / "vocab.json"), str(tmp_path / "merges.txt"))
    tok = Tokenizer()
    assert tok.load(str(tmp_path / "vocab.json"), str(tmp_path / "merges.txt"))
    assert tok.vocab_size == 259
    for s in ("Hello, JieYu AI!", "你好，世界！昆仑分词器。"):
        assert tok.decode(tok.encode(s)) == s.encode()
    assert tok.encode("abc") == [97, 98, 99]


@pytest.mark.parametrize("s,stops,want", [
    (b"hello world", [], -1),
    (b"answer<|im_end|>", [], 6),
    (b"a<|", [], -1),                       # no marker character after "<|"
    (b"a<|x", [], 1),
    (b"text END more", [b"END"], 5),
    (b"x<|y END", [b"END"], 1),              # the earlier of the two
    (b"<| <|ok", [], 3),
])
def test_marker_at(s, stops, want):
    assert X.marker_at(s, stops) == want


class _Script:
    """A generator with generate()'s contract that emits a fixed id list
    (stopping early on EOS or when the callback asks)."""

    def __init__(self, new_ids):
        self.new_ids = list(new_ids)
        self.calls = []

    def __call__(self, ids, max_new, eos=None, temperature=0.0, repetition_penalty=1.0, cb=None):
        self.calls.append((list(ids), max_new, list(eos or []), temperature, repetition_penalty))
        seq = list(ids)
        for t in self.new_ids[:max_new]:
            seq.append(t)
            if (eos and t in eos) or (cb and cb(t)):
                break
        return seq


@pytest.fixture
def bytetok(tmp_path):
    X.write_byte_level_vocab(str(tmp_path / "vocab.json"), str(tmp_path / "merges.txt"))
    tok = Tokenizer()
    assert tok.load(str(tmp_path / "vocab.json"), str(tmp_path / "merges.txt"))
    return tok


def test_generate_text_rules(bytetok):
    tok = bytetok
    V = 259
    plain = X.ChatStrings()
    # BOS first, EOS list = {eos, 0 (text_end absent, as register_special gives 0)}
    g = _Script([ord(c) for c in "hi there"])
    assert X.generate_text(tok, "ab", V, 64, True, plain, g, 8, 0.0, 1.0) == (8, b"hi there")
    ids, max_new, eos, _, _ = g.calls[0]
    assert ids == [tok.bos_id, 97, 98] and max_new == 8 and eos == [tok.eos_id, 0]
    # max_new clamped by max_seq; a prompt longer than max_seq is cut
    g = _Script([ord("z")] * 50)
    assert X.generate_text(tok, "abcdef", V, 10, False, plain, g, 20, 0.0, 1.0)[0] == 4
    assert X.generate_text(tok, "x" * 30, V, 10, False, plain, g, 5, 0.0, 1.0) == (0, b"")
    # a chat string in the output ends it (cut before the string) and stops the loop
    chat = X.ChatStrings(s_end=b"END")
    g = _Script([ord(c) for c in "okENDmore"])
    n, out = X.generate_text(tok, "q", V, 64, False, chat, g, 20, 0.0, 1.0)
    assert out == b"ok" and n == 5
    # a "<|name" marker too
    g = _Script([ord(c) for c in "fine<|im_end|>tail"])
    n, out = X.generate_text(tok, "q", V, 64, False, plain, g, 30, 0.0, 1.0)
    assert out == b"fine" and n == len("fine<|i")
    # a registered stop token ends the text without being added
    chat = X.ChatStrings(id_end=258)
    g = _Script([ord("a"), 258, ord("b")])
    assert X.generate_text(tok, "q", V, 64, False, chat, g, 10, 0.0, 1.0) == (2, b"a")
    # ids outside the model's vocabulary: -1
    assert X.generate_text(tok, "q", 100, 64, False, plain, _Script([]), 4, 0.0, 1.0) == (-1, b"")
    assert X.generate_text(tok, "", V, 64, False, plain, _Script([]), 4, 0.0, 1.0) == (0, b"")
