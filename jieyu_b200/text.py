"""Text in, text out on the device path: the reference's `jieyu_load` /
`jieyu_generate` flow (main.hpp:85-227 over pipeline.h:280-436
`load_model_dir` + `generate_text`) with the token loop on the GPU.

A model directory is bound as the reference binds it: weights from
`model.bf` (jieyu_b200.bfile.load_model_dir), the tokenizer from vocab.json /
merges.txt (jieyu_b200.tokenizer), and from model_info.json the BOS rule
(add_bos_token, default 1) and the chat strings (message_start,
message_end, text_end, user_start, assistant_start, bos_text, turn_end), each
registered as a special token when the vocabulary holds it.

`TextModel.generate` follows generate_text: encode the prompt, prepend BOS,
reject ids outside the model's vocabulary (-1), keep at most max_seq prompt
tokens and at most max_seq - prompt tokens of output, stop on the tokenizer's
EOS and the registered text_end / message_end ids, and build the output text
token by token: a registered message_start / message_end / text_end token
ends the text without being added; otherwise the token's bytes are added and
the text is cut (and generation stops) at the first chat string or "<|name"
marker it now holds.
"""
from __future__ import annotations

import os
from typing import Optional

from .bfile import _info_int, _info_text, _read_info, load_model_dir
from .model import DeviceModel
from .tokenizer import _TO_CHAR, Tokenizer, load_tokenizer


def write_byte_level_vocab(vocab_path: str, merges_path: str) -> None:
    """The reference's byte-level vocabulary (tokenizer_libs/include/
    byte_vocab.h): byte b's symbol has id b; no merges."""
    parts = []
    for b, piece in enumerate(_TO_CHAR):
        esc = piece.replace(b"\\", b"\\\\").replace(b'"', b'\\"')
        parts.append(b'"' + esc + b'":' + str(b).encode())
    with open(vocab_path, "wb") as f:
        f.write(b"{" + b",".join(parts) + b"}")
    with open(merges_path, "wb") as f:
        f.write(b"#version: 0.2\n")


def _is_marker_char(c: int) -> bool:
    return 0x61 <= c <= 0x7A or 0x41 <= c <= 0x5A or 0x30 <= c <= 0x39 or c in (0x5F, 0x2D)


def marker_at(s: bytes, stops: list) -> int:
    """First position of a chat string or of "<|" + 1..24 marker characters
    (pipeline.h:201-217); -1 when there is none."""
    best = -1
    for st in stops:
        if st:
            at = s.find(st)
            if at >= 0 and (best < 0 or at < best):
                best = at
    lt = s.find(b"<|")
    while lt >= 0:
        n = 0
        while lt + 2 + n < len(s) and n < 24 and _is_marker_char(s[lt + 2 + n]):
            n += 1
        if n >= 1 and (best < 0 or lt < best):
            best = lt
        lt = s.find(b"<|", lt + 1)
    return best


class TextModel:
    """A reference model directory bound for text generation on the device."""

    def __init__(self, path: str, max_seq: int = 0, tokenizer: Optional[Tokenizer] = None):
        self.hw = load_model_dir(path, max_seq=max_seq)
        self.tok = tokenizer or load_tokenizer(path)
        info = _read_info(os.path.join(path, "model_info.json"))

        def text(key: str) -> bytes:  # read_info_str (pipeline.h:155-160)
            return _info_text(info, key).encode("utf-8", "surrogatepass")

        self.add_bos = _info_int(info, "add_bos_token", 1) != 0
        self.s_start, self.s_end, self.s_text = text("message_start"), text("message_end"), text("text_end")
        self.s_user, self.s_asst, self.s_turn = text("user_start"), text("assistant_start"), text("turn_end")
        s_bos = text("bos_text")

        def register(piece: bytes) -> int:  # register_special: 0 when absent
            i = self.tok.add_special_token(piece) if piece else -1
            return i if i >= 0 else 0

        self.id_start = register(self.s_start)
        self.id_end = register(self.s_end)
        self.id_text = register(self.s_text)
        for piece in (self.s_user, self.s_asst, s_bos, self.s_turn):
            register(piece)
        self.model = DeviceModel(self.hw)

    def close(self) -> None:
        self.model.close()

    def generate(self, prompt, max_new: int = 256, temperature: float = 0.7,
                 repetition_penalty: float = 1.1) -> tuple[int, bytes]:
        """(new tokens, generated text bytes); (0, b"") when nothing can be
        produced, (-1, b"") when the prompt's ids do not fit the model."""
        chat = ChatStrings(self.s_start, self.s_end, self.s_text, self.s_user, self.s_asst, self.s_turn,
                           self.id_start, self.id_end, self.id_text)
        return generate_text(self.tok, prompt, self.hw.cfg.vocab, self.hw.cfg.max_seq, self.add_bos, chat,
                             self.model.generate, max_new, temperature, repetition_penalty)


class ChatStrings:
    """model_info.json's chat strings and the ids of the three registered as
    stop tokens (0 when the vocabulary lacks them, as register_special)."""

    def __init__(self, s_start=b"", s_end=b"", s_text=b"", s_user=b"", s_asst=b"", s_turn=b"",
                 id_start=0, id_end=0, id_text=0):
        self.stops = [x for x in (s_start, s_end, s_text, s_user, s_asst, s_turn) if x]
        self.id_start, self.id_end, self.id_text = id_start, id_end, id_text


def generate_text(tok: Tokenizer, prompt, vocab: int, max_seq: int, add_bos: bool, chat: ChatStrings, gen,
                  max_new: int = 256, temperature: float = 0.7, repetition_penalty: float = 1.1) -> tuple[int, bytes]:
    """The reference's generate_text (pipeline.h:280-374) over a token
    generator `gen(ids, max_new, eos=, temperature=, repetition_penalty=, cb=)`
    with generate()'s contract (returns prompt + new ids; cb(id) -> True
    stops after that token)."""
    ids = tok.encode(prompt)
    if add_bos and 0 <= tok.bos_id < vocab:
        ids.insert(0, tok.bos_id)
    if not ids:
        return 0, b""
    if max_new <= 0:
        max_new = max_seq
    if any(i < 0 or i >= vocab for i in ids):
        return -1, b""
    ids = ids[:max_seq]
    if len(ids) + max_new > max_seq:
        max_new = max_seq - len(ids)
    if max_new <= 0:
        return 0, b""
    eos: list = []
    for e in (tok.eos_id, chat.id_text, chat.id_end):  # want_eos: in range, distinct, at most 3
        if 0 <= e < vocab and e not in eos and len(eos) < 3:
            eos.append(e)
    specials = [i for i in (chat.id_start, chat.id_end, chat.id_text) if i != 0]
    out = bytearray()

    def on_token(i: int) -> bool:  # echo_token (pipeline.h:230-260): True stops the loop
        if i in specials:
            return True
        out.extend(tok.decode([i]))
        at = marker_at(bytes(out), chat.stops)
        if at >= 0:
            del out[at:]
            return True
        return False

    seq = gen(ids, max_new, eos=eos or None, temperature=temperature, repetition_penalty=repetition_penalty,
              cb=on_token)
    return len(seq) - len(ids), bytes(out)


class JieyuError(RuntimeError):
    """jieyu::error (JieyuAI_api.h:76-79)."""


class Jieyu:
    """The reference's `class jieyu` (JieyuAI_api.h:74-142) over the text C
    ABI of libjieyu_b200.so (include/jieyu.h): one model per process shared
    by every open handle, text handling in C++, token steps on the GPU."""

    def __init__(self, path: Optional[str] = None, max_seq: int = 0):
        from . import _capi

        self._lib = _capi.load()
        self._h = None
        if path is not None:
            self.open(path, max_seq)

    def open(self, path: str, max_seq: int = 0) -> None:
        self.close()
        h = self._lib.jieyu_load(os.fsencode(path), max_seq)
        if not h:
            raise JieyuError("load failed: " + self._lib.jieyu_last_error(None).decode("utf-8", "replace"))
        self._h = h

    def close(self) -> None:
        if self._h:
            self._lib.jieyu_free(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def is_open(self) -> bool:
        return bool(self._h)

    def context_length(self) -> int:
        return self._lib.jieyu_context_length(self._h) if self._h else 0

    def dir(self) -> str:
        return self._lib.jieyu_model_dir(self._h).decode("utf-8", "replace") if self._h else ""

    def last_error(self) -> str:
        return self._lib.jieyu_last_error(self._h).decode("utf-8", "replace")

    @staticmethod
    def version() -> str:
        from . import _capi

        return _capi.load().jieyu_version().decode()

    def _buffer(self, max_new: int):
        import ctypes

        return ctypes.create_string_buffer((max_new if max_new > 0 else 4096) * 16 + 256)

    def generate(self, prompt, max_new: int = 256, temperature: float = 0.7,
                 repetition_penalty: float = 1.1) -> bytes:
        """The generated text (bytes: the model's output need not be valid
        UTF-8); raises JieyuError when jieyu_generate returns -1."""
        if not self._h:
            raise JieyuError("no model loaded (call open first)")
        p = prompt.encode("utf-8") if isinstance(prompt, str) else bytes(prompt)
        buf = self._buffer(max_new)
        if self._lib.jieyu_generate(self._h, p, buf, len(buf), max_new, temperature, repetition_penalty) < 0:
            raise JieyuError(self.last_error())
        return buf.value

    def generate_jsonl(self, jsonl: str, qb: str = "", qe: str = "", max_new: int = 256,
                       temperature: float = 0.7, repetition_penalty: float = 1.1) -> bytes:
        if not self._h:
            raise JieyuError("no model loaded (call open first)")
        buf = self._buffer(max_new)
        if self._lib.jieyu_generate_jsonl(self._h, os.fsencode(jsonl), qb.encode(), qe.encode(), buf, len(buf),
                                          max_new, temperature, repetition_penalty) < 0:
            raise JieyuError(self.last_error())
        return buf.value
