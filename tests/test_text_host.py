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
