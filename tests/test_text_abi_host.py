"""CPU: the text C ABI's host side (include/jieyu.h, jieyu_b200/csrc/text.cpp).
Its tokenizer gives the same ids and bytes as the restatement that is pinned
to the reference's own tokenizer (tokenizer_host tests), and as the reference
itself when oracle/_ref is built; model-directory problems are rejected
before any device work with the reference's error behaviour (NULL handle,
the reason in jieyu_last_error(NULL)); NULL handles and paths give -1."""
import ctypes as C
import os

import numpy as np
import pytest

from jieyu_b200 import _capi, bfile
from jieyu_b200 import tokenizer as T
from jieyu_b200.model import HostWeights
from jieyu_b200.text import write_byte_level_vocab
from oracle.bind import REF_SO
from test_tokenizer_host import CORPUS, TEXTS, _train, _write


def _enc(lib, h, data: bytes):
    n = lib.jyt_tok_encode(h, data, len(data), None, 0)
    out = np.zeros(max(n, 1), np.int32)
    assert lib.jyt_tok_encode(h, data, len(data), out.ctypes.data, n) == n
    return [int(x) for x in out[:n]]


def _dec(lib, h, ids):
    a = np.asarray(ids, np.int32)
    n = lib.jyt_tok_decode(h, a.ctypes.data, len(a), None, 0)
    buf = C.create_string_buffer(max(n, 1))
    assert lib.jyt_tok_decode(h, a.ctypes.data, len(a), buf, n) == n
    return buf.raw[:n]


@pytest.mark.parametrize("word_end", [True, False])
def test_native_tokenizer_matches_restatement(tmp_path, word_end):
    lib = _capi.load()
    vocab, merges = _train(CORPUS, 400, word_end)
    vp, mp = _write(str(tmp_path), vocab, merges, extra=["<|im_end|>"])
    h = lib.jyt_tok_load(vp.encode(), mp.encode())
    assert h
    try:
        tok = T.Tokenizer()
        assert tok.load(vp, mp)
        info = np.zeros(6, np.int32)
        assert lib.jyt_tok_info(h, info.ctypes.data) == 0
        assert [int(x) for x in info] == [tok.vocab_size, tok.bos_id, tok.eos_id, tok.unk_id, tok.word_end_id,
                                          len(tok.merge_result)]
        rng = np.random.default_rng(11)
        pool = [t if isinstance(t, bytes) else t.encode() for t in TEXTS]
        fuzz = [bytes(rng.integers(0, 256, size=int(rng.integers(1, 40)), dtype=np.uint8)) for _ in range(150)]
        mixed = [b"".join(pool[int(i)][: int(rng.integers(0, 20))] for i in rng.integers(0, len(pool), 4))
                 for _ in range(100)]
        for data in pool + fuzz + mixed:
            ids = _enc(lib, h, data)
            assert ids == tok.encode(data), data
            assert _dec(lib, h, ids) == tok.decode(ids), data
        assert lib.jyt_tok_add_special(h, b"<|im_end|>", 10) == tok.add_special_token(b"<|im_end|>") >= 0
        assert lib.jyt_tok_add_special(h, b"<|absent|>", 10) == -1
        for data in [b"chat<|im_end|>next", b"<|im_end|><|im_end|>", b"a <|im_end|> b"]:
            assert _enc(lib, h, data) == tok.encode(data)
        # ids outside the vocabulary decode to nothing
        assert _dec(lib, h, [-5, 10 ** 8]) == b""
    finally:
        lib.jyt_tok_free(h)
    assert not lib.jyt_tok_load(str(tmp_path / "missing.json").encode(), mp.encode())


def test_native_tokenizer_matches_reference(tmp_path):
    if not os.path.exists(REF_SO):
        pytest.skip("reference harness not built (reference tree absent)")
    ref = C.CDLL(REF_SO)
    P = C.c_void_p
    ref.jyref_tok_load.restype = P
    ref.jyref_tok_load.argtypes = [C.c_char_p, C.c_char_p]
    ref.jyref_tok_free.argtypes = [P]
    ref.jyref_tok_encode.restype = C.c_int
    ref.jyref_tok_encode.argtypes = [P, C.c_char_p, C.c_int, P, C.c_int]
    lib = _capi.load()
    vocab, merges = _train(CORPUS, 300, True)
    vp, mp = _write(str(tmp_path), vocab, merges)
    hr = ref.jyref_tok_load(vp.encode(), mp.encode())
    h = lib.jyt_tok_load(vp.encode(), mp.encode())
    # long words (no spaces) over the corpus' letters: many merges interact
    # within one word, ties of equal rank included
    rng = np.random.default_rng(5)
    joined = "".join(CORPUS).replace(" ", "").replace("\n", "")
    letters = sorted(set(joined))
    long_words = ["".join(rng.choice(letters, size=int(n))) for n in (64, 257, 1000)]
    long_words += ["abab" * 300, joined[:1500]]
    try:
        for text in list(TEXTS) + long_words:
            data = text if isinstance(text, bytes) else text.encode()
            out = np.zeros(4 * len(data) + 16, np.int32)
            n = ref.jyref_tok_encode(hr, data, len(data), out.ctypes.data, len(out))
            assert _enc(lib, h, data) == [int(x) for x in out[:n]], data
    finally:
        ref.jyref_tok_free(hr)
        lib.jyt_tok_free(h)


def test_byte_level_vocabulary_ids(tmp_path):
    lib = _capi.load()
    write_byte_level_vocab(str(tmp_path / "v.json"), str(tmp_path / "m.txt"))
    h = lib.jyt_tok_load(str(tmp_path / "v.json").encode(), str(tmp_path / "m.txt").encode())
    try:
        data = bytes(range(256))
        tok = T.Tokenizer()
        assert tok.load(str(tmp_path / "v.json"), str(tmp_path / "m.txt"))
        assert _enc(lib, h, data) == tok.encode(data)
        assert _dec(lib, h, list(range(256))) == data
    finally:
        lib.jyt_tok_free(h)


def _model_dir(tmp_path, drop=None, reshape=None):
    hw = HostWeights.shift_demo_kat()
    d = str(tmp_path)
    bfile.save_model_dir(hw, d)
    header, ts = bfile.model_dir_tensors(hw)
    if drop or reshape:
        out = []
        for name, dt, shape, data in ts:
            if name == drop:
                continue
            if name == reshape:
                shape = tuple(reversed(shape))
            out.append((name, dt, shape, data))
        bfile.write_bfile(os.path.join(d, "model.bf"), header, out)
    write_byte_level_vocab(os.path.join(d, "vocab.json"), os.path.join(d, "merges.txt"))
    return d


@pytest.mark.parametrize("case", ["no_dir", "missing", "shape", "no_vocab"])
def test_load_rejects_bad_directories(tmp_path, case):
    """Each case fails before the device upload, with the same rejection the
    restatement (bfile.load_model_dir / load_tokenizer) gives."""
    lib = _capi.load()
    if case == "no_dir":
        d, want = str(tmp_path / "absent"), b"model.bf"
    elif case == "missing":
        d, want = _model_dir(tmp_path, drop="model.layers.1.mlp.up_proj.weight"), b"missing tensor"
    elif case == "shape":
        d, want = _model_dir(tmp_path, reshape="model.layers.0.self_attn.k_proj.weight"), b"shape"
    else:
        d = _model_dir(tmp_path)
        os.remove(os.path.join(d, "vocab.json"))
        want = None  # the device upload comes first; on a CPU host it is what fails
    if case != "no_vocab":
        with pytest.raises((bfile.BFileError, OSError, ValueError)):
            bfile.load_model_dir(d)
    h = lib.jieyu_load(d.encode(), 0)
    assert not h
    err = lib.jieyu_last_error(None)
    assert err
    if want is not None:
        assert want in err, err


def test_null_arguments_and_version():
    lib = _capi.load()
    assert lib.jieyu_version() == b"1.0.0"
    assert lib.jieyu_context_length(None) == 0
    assert lib.jieyu_model_dir(None) == b""
    assert not lib.jieyu_load(None, 0)
    assert lib.jieyu_last_error(None) == b"dir is NULL"
    assert lib.jieyu_generate(None, b"x", None, 0, 4, 0.0, 1.0) == -1
    assert lib.jieyu_last_error(None) == b"handle is NULL"
    assert lib.jieyu_generate_jsonl(None, b"x.jsonl", b"", b"", None, 0, 4, 0.0, 1.0) == -1
    lib.jieyu_free(None)
    assert lib.jyt_tok_encode(None, b"x", 1, None, 0) == -1


def test_header_builds_as_c_and_cpp(tmp_path):
    """include/jieyu.h compiles as C and as C++ (with the RAII wrapper), and a
    program links against the library: a failed load throws jieyu::error
    carrying the load error."""
    import shutil
    import subprocess

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if not shutil.which("gcc") or not shutil.which("g++"):
        pytest.skip("no host compiler")
    inc, libdir = os.path.join(root, "include"), os.path.join(root, "jieyu_b200")
    c_src = tmp_path / "t.c"
    c_src.write_text('#include "jieyu.h"\n#include <stdio.h>\nint main(void){jieyu_model h=jieyu_load("/nonexistent",0);'
                     'printf("%d %s %s\\n",h==0,jieyu_last_error(0),jieyu_version());return 0;}\n')
    cpp_src = tmp_path / "t.cpp"
    cpp_src.write_text('#include "jieyu.h"\n#include <cstdio>\nint main(){try{jieyu m("/nonexistent");return 1;}'
                       'catch(const jieyu::error& e){std::printf("%s\\n",e.what());}'
                       'jieyu none; try{none.generate("x");}catch(const jieyu::error&){std::printf("closed\\n");}'
                       'return jieyu::version()=="1.0.0"?0:2;}\n')
    outs = []
    for cc, src, std in (("gcc", c_src, "-std=c99"), ("g++", cpp_src, "-std=c++17")):
        exe = str(tmp_path / (src.name + ".out"))
        subprocess.run([cc, std, "-I", inc, str(src), "-o", exe, "-L", libdir, "-ljieyu_b200",
                        f"-Wl,-rpath,{libdir}"], check=True, capture_output=True)
        r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
        assert r.returncode == 0, r.stderr
        outs.append(r.stdout)
    assert outs[0].startswith("1 /nonexistent/model.bf: cannot open 1.0.0")
    assert "load failed: /nonexistent/model.bf: cannot open" in outs[1] and "closed" in outs[1]


def test_python_wrapper_errors(tmp_path):
    from jieyu_b200.text import Jieyu, JieyuError

    assert Jieyu.version() == "1.0.0"
    j = Jieyu()
    assert not j.is_open() and j.context_length() == 0 and j.dir() == ""
    with pytest.raises(JieyuError, match="no model loaded"):
        j.generate("x")
    with pytest.raises(JieyuError, match="cannot open"):
        j.open(str(tmp_path / "absent"))
    assert not j.is_open()


def _probe(lib, d, max_seq=0):
    out = np.zeros(13, np.int32)
    err = C.create_string_buffer(256)
    r = lib.jyt_model_dir_probe(d.encode(), max_seq, out.ctypes.data, err, 256)
    return r, [int(x) for x in out], err.value.decode()


def _bfile_models():
    from test_bfile_host import _models
    return _models()


@pytest.mark.parametrize("model", ["bind_kat", "q8_tied_bias", "q8_separate", "f32_rect", "kquant_mixed"])
def test_native_binding_matches_restatement(tmp_path, model):
    """jieyu_load's binding (without the device upload) reads every model
    directory the restatement reads, with the same hyper-parameters, bias,
    tied head, weight formats and RoPE base."""
    lib = _capi.load()
    hw = _bfile_models()[model]
    d = str(tmp_path)
    bfile.save_model_dir(hw, d)
    got = bfile.load_model_dir(d)
    c = got.cfg
    r, v, err = _probe(lib, d)
    assert r == 0, err
    kinds = {bfile.Q8_0} if c.wtype == "q8" else None
    assert v[:8] == [c.layers, c.hidden, c.heads, c.kv_heads, c.head_dim, c.inter, c.vocab, c.max_seq]
    assert v[8] == int(c.qkv_bias) and v[9] == int(c.embed == "tied") and v[11] == int(c.theta)
    if kinds:
        assert v[10] == 1 << bfile.Q8_0
    elif c.wtype == "f32":
        assert v[10] == 1 << bfile.F32
    else:
        assert v[10] & ~((1 << bfile.F32) | (1 << bfile.Q4K) | (1 << bfile.Q5K) | (1 << bfile.Q6K)) == 0
    assert (v[12] & 1) == int(got.t["head"].dtype == np.uint8)
    r2, v2, _ = _probe(lib, d, 77)
    assert r2 == 0 and v2[7] == 77


def test_native_binding_rejects_what_the_restatement_rejects(tmp_path):
    from test_bfile_host import CORRUPT, _save

    lib = _capi.load()
    hw = _bfile_models()["q8_tied_bias"]
    for how, corrupt in CORRUPT.items():
        d = tmp_path / how
        d.mkdir()
        path = _save(hw, d)
        corrupt(path, os.path.getsize(path))
        with pytest.raises(bfile.BFileError):
            bfile.load_model_dir(str(d))
        r, _, err = _probe(lib, str(d))
        assert r == -1 and err, how


@pytest.mark.parametrize("info,want", [({"max_position_embeddings": "100000"}, 4096),
                                       ({"max_position_embeddings": 10}, 64),
                                       ({"max_position_embeddings": "2048"}, 2048), ({}, 1024),
                                       ({"max_position_embeddings": 3900.5}, 3900),
                                       ({"max_position_embeddings": "4e3"}, 64),
                                       ({"max_position_embeddings": " 300x"}, 300),
                                       ({"max_position_embeddings": True}, 1024)])
def test_max_seq_rule_native_and_restatement(tmp_path, info, want):
    import json

    lib = _capi.load()
    hw = _bfile_models()["f32_rect"]
    bfile.save_model_dir(hw, str(tmp_path))
    with open(tmp_path / "model_info.json", "w") as f:
        json.dump(info, f)
    assert bfile.load_model_dir(str(tmp_path)).cfg.max_seq == want
    r, v, err = _probe(lib, str(tmp_path))
    assert r == 0 and v[7] == want, err
