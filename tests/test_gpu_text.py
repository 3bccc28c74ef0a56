"""Text in, text out on the device (jieyu_b200.text.TextModel over a model
directory): the reference's check_pipeline cases 6 and 7
(libs/text/text.h:993-1013) on its shift-by-one demo model (converter.h:
422-503, identity byte embedding, lm_head[v][v-1] = 1) with its byte-level
vocabulary: "abcdefgh" -> "ijklmnopqrstuvwx" (16 tokens) and, with
max_new = 5, "abc" -> "defgh"."""
import json

import pytest

from jieyu_b200 import bfile
from jieyu_b200.model import HostWeights
from jieyu_b200.text import TextModel, write_byte_level_vocab

pytestmark = pytest.mark.gpu


def test_check_pipeline_text_cases(cuda, tmp_path):
    d = str(tmp_path)
    bfile.save_model_dir(HostWeights.shift_demo_kat(), d)
    write_byte_level_vocab(str(tmp_path / "vocab.json"), str(tmp_path / "merges.txt"))
    with open(tmp_path / "model_info.json") as f:
        info = json.load(f)
    info["max_position_embeddings"] = "1024"
    with open(tmp_path / "model_info.json", "w") as f:
        json.dump(info, f)
    m = TextModel(d)
    try:
        assert m.hw.cfg.max_seq == 1024
        assert m.generate("abcdefgh", max_new=16, temperature=0.0, repetition_penalty=1.0) == (16, b"ijklmnopqrstuvwx")
        assert m.generate("abc", max_new=5, temperature=0.0, repetition_penalty=1.0) == (5, b"defgh")
    finally:
        m.close()


def _shift_dir(tmp_path):
    d = str(tmp_path)
    bfile.save_model_dir(HostWeights.shift_demo_kat(), d)
    write_byte_level_vocab(str(tmp_path / "vocab.json"), str(tmp_path / "merges.txt"))
    return d


def test_text_c_abi_check_pipeline(cuda, tmp_path):
    """The same cases through the reference's text C ABI (jieyu_load /
    jieyu_generate, main.hpp:85-177), with its buffer rules: out = NULL
    copies nothing, a short buffer gets cap-1 bytes plus NUL, the return
    is the new-token count."""
    import ctypes as C

    from jieyu_b200 import _capi

    lib = _capi.load()
    d = _shift_dir(tmp_path)
    h = lib.jieyu_load(d.encode(), 0)
    assert h, lib.jieyu_last_error(None)
    try:
        assert lib.jieyu_context_length(h) == 1024  # the directory's max_position_embeddings
        assert lib.jieyu_model_dir(h) == d.encode()
        buf = C.create_string_buffer(64)
        assert lib.jieyu_generate(h, b"abcdefgh", buf, 64, 16, 0.0, 1.0) == 16
        assert buf.value == b"ijklmnopqrstuvwx"
        assert lib.jieyu_generate(h, b"abc", buf, 64, 5, 0.0, 1.0) == 5 and buf.value == b"defgh"
        assert lib.jieyu_generate(h, b"abc", None, 0, 5, 0.0, 1.0) == 5
        small = C.create_string_buffer(4)
        assert lib.jieyu_generate(h, b"abc", small, 4, 5, 0.0, 1.0) == 5 and small.value == b"def"
        # a second handle on the same directory shares the model
        h2 = lib.jieyu_load(d.encode(), 0)
        assert h2
        lib.jieyu_free(h2)
        assert lib.jieyu_generate(h, b"xyz", buf, 64, 3, 0.0, 1.0) == 3 and buf.value == b"{|}"
        # JSONL chat prompt: the feed is "u\nabc\n" (no chat strings in this
        # directory), so the shift model continues from "\n" (byte 10)
        jl = tmp_path / "chat.jsonl"
        jl.write_text('{"name": "u", "message": "abc"}\n\nnot json\n')
        assert lib.jieyu_generate_jsonl(h, str(jl).encode(), b"", b"", buf, 64, 3, 0.0, 1.0) == 3
        assert buf.value == b"\x0b\x0c\x0d"
        empty = tmp_path / "empty.jsonl"
        empty.write_text("\n{}\n")
        assert lib.jieyu_generate_jsonl(h, str(empty).encode(), b"", b"", buf, 64, 3, 0.0, 1.0) == -1
        assert b"jsonl_no_srch" in lib.jieyu_last_error(h)
    finally:
        lib.jieyu_free(h)


def test_python_wrapper(cuda, tmp_path):
    from jieyu_b200.text import Jieyu

    d = _shift_dir(tmp_path)
    with Jieyu(d) as j:
        assert j.context_length() == 1024 and j.dir() == d
        assert j.generate("abcdefgh", max_new=16, temperature=0.0, repetition_penalty=1.0) == b"ijklmnopqrstuvwx"
        assert j.last_error() == ""
    assert not j.is_open()
