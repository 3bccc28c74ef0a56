"""Byte-level BPE tokenizer of the reference (libs/tokenizer_libs/include/
tokenizer.h), restated for the host side of the device path: the same
vocab.json / merges.txt files give the same ids, so a prompt string reaches
the GPU token loop exactly as the reference's `generate_text`
(libs/model_libs/pipeline.h:280-374) would feed it.

Everything works on bytes, as the reference works on std::string:
  * bytes map to byte-level symbols (tokenizer.h:69-125: printable bytes are
    their own code point, the others 256, 257, ... in order);
  * text splits into words (tokenizer.h:152-222): runs of white space
    (a single ' ' joins the following word, or the following punctuation
    character), single punctuation characters, and runs of other characters;
  * each word is its bytes' symbols plus "</w>" when the vocabulary has it,
    merged by merges.txt rank with the lowest (rank, position) first
    (tokenizer.h:483-600);
  * the special pieces (BOS, EOS, UNK and any added) are matched in the text
    first, the earliest and then the longest (tokenizer.h:457-481).
UTF-8 is decoded with the reference's rules (json_libs/file_util.h:36-73):
an invalid or truncated sequence yields its lead byte as one code point.
"""
from __future__ import annotations

import heapq
import json
import os

BOS_TOKEN = b"<\xef\xbd\x9cbegin\xe2\x96\x81of\xe2\x96\x81sentence\xef\xbd\x9c>"
EOS_TOKEN = b"<\xef\xbd\x9cend\xe2\x96\x81of\xe2\x96\x81sentence\xef\xbd\x9c>"
UNK_TOKEN = b"<unk>"
WORD_END_TOKEN = b"</w>"


def utf8_encode(cp: int) -> bytes:
    if cp <= 0x7F:
        return bytes([cp])
    if cp <= 0x7FF:
        return bytes([0xC0 | (cp >> 6), 0x80 | (cp & 0x3F)])
    if cp <= 0xFFFF:
        return bytes([0xE0 | (cp >> 12), 0x80 | ((cp >> 6) & 0x3F), 0x80 | (cp & 0x3F)])
    return bytes([0xF0 | (cp >> 18), 0x80 | ((cp >> 12) & 0x3F), 0x80 | ((cp >> 6) & 0x3F), 0x80 | (cp & 0x3F)])


def utf8_decode(data: bytes, i: int) -> tuple[int, int]:
    """(code point, length) at data[i] with the reference's lenient rules."""
    b0 = data[i]
    n = len(data) - i
    if b0 < 0x80:
        return b0, 1
    if (b0 & 0xE0) == 0xC0:
        if n >= 2 and (data[i + 1] & 0xC0) == 0x80:
            return ((b0 & 0x1F) << 6) | (data[i + 1] & 0x3F), 2
        return b0, 1
    if (b0 & 0xF0) == 0xE0:
        if n >= 3 and (data[i + 1] & 0xC0) == 0x80 and (data[i + 2] & 0xC0) == 0x80:
            return ((b0 & 0x0F) << 12) | ((data[i + 1] & 0x3F) << 6) | (data[i + 2] & 0x3F), 3
        return b0, 1
    if (b0 & 0xF8) == 0xF0:
        if n >= 4 and all((data[i + j] & 0xC0) == 0x80 for j in (1, 2, 3)):
            return (((b0 & 0x07) << 18) | ((data[i + 1] & 0x3F) << 12) | ((data[i + 2] & 0x3F) << 6)
                    | (data[i + 3] & 0x3F)), 4
        return b0, 1
    return b0, 1


def _printable(b: int) -> bool:
    return 33 <= b <= 126 or 161 <= b <= 172 or 174 <= b <= 255


_TO_CHAR: list[bytes] = []
_TO_BYTE: list[int] = []  # code point 256 + slot -> byte
for _b in range(256):
    if _printable(_b):
        _TO_CHAR.append(utf8_encode(_b))
    else:
        _TO_CHAR.append(utf8_encode(256 + len(_TO_BYTE)))
        _TO_BYTE.append(_b)


def byte_level_decode(cp: int) -> int:
    if cp < 256:
        return cp if _printable(cp) else -1
    slot = cp - 256
    return _TO_BYTE[slot] if slot < len(_TO_BYTE) else -1


def _is_space(cp: int) -> bool:
    return cp in (0x20, 0x09, 0x0A, 0x0B, 0x0C, 0x0D, 0x3000)


def _is_punct(cp: int) -> bool:
    return (0x21 <= cp <= 0x2F or 0x3A <= cp <= 0x40 or 0x5B <= cp <= 0x60 or 0x7B <= cp <= 0x7E
            or 0x2010 <= cp <= 0x2027 or 0x2030 <= cp <= 0x205E or 0x3001 <= cp <= 0x303F
            or 0xFF01 <= cp <= 0xFF0F or 0xFF1A <= cp <= 0xFF20 or 0xFF3B <= cp <= 0xFF40
            or 0xFF5B <= cp <= 0xFF65)


def split_word_ranges(text: bytes) -> list[tuple[int, int]]:
    """Word boundaries of tokenizer.h:152-222 (byte offsets)."""
    ranges = []
    size = len(text)
    i = 0
    while i < size:
        cp, ln = utf8_decode(text, i)
        if _is_space(cp):
            nxt = i
            while nxt < size:
                c2, l2 = utf8_decode(text, nxt)
                if not _is_space(c2):
                    break
                nxt += l2
            if nxt - i == 1 and text[i] == 0x20 and nxt < size:
                stop = nxt
                after, al = utf8_decode(text, stop)
                if _is_punct(after):
                    stop += al
                else:
                    while stop < size:
                        c2, l2 = utf8_decode(text, stop)
                        if _is_space(c2) or _is_punct(c2):
                            break
                        stop += l2
                ranges.append((i, stop))
                i = stop
            else:
                ranges.append((i, nxt))
                i = nxt
            continue
        if _is_punct(cp):
            ranges.append((i, i + ln))
            i += ln
            continue
        stop = i
        while stop < size:
            c2, l2 = utf8_decode(text, stop)
            if _is_space(c2) or _is_punct(c2):
                break
            stop += l2
        ranges.append((i, stop))
        i = stop
    return ranges


def _strtol(text: str) -> int | None:
    """The integer prefix strtol(value, &end, 10) accepts (None when it accepts none)."""
    s = text.lstrip(" \t\n\r\f\v")
    j = 0
    if j < len(s) and s[j] in "+-":
        j += 1
    k = j
    while k < len(s) and s[k].isdigit() and s[k] in "0123456789":
        k += 1
    if k == j:
        return None
    return int(s[:k])


def _json_value_text(v) -> str:
    """json_file's value_to_string for the values a vocabulary holds."""
    if isinstance(v, str):
        return v
    if isinstance(v, bool):
        return "true" if v else "false"
    if v is None:
        return "null"
    return str(v)


class Tokenizer:
    """The reference's Tokenizer: load(vocab, merges), encode, decode."""

    def __init__(self):
        self.piece_to_id: dict[bytes, int] = {}
        self.id_to_piece: list[bytes] = []
        self.merge_rank: dict[tuple[int, int], int] = {}
        self.merge_result: list[int] = []
        self.byte_id = [-1] * 256
        self.word_end_id = self.bos_id = self.eos_id = self.unk_id = -1
        self.special_pieces: list[bytes] = []
        self.special_ids: list[int] = []

    # -- loading (tokenizer.h:340-455) --------------------------------------
    def _ensure(self, piece: bytes) -> int:
        i = self.piece_to_id.get(piece)
        if i is not None:
            return i
        i = len(self.id_to_piece)
        self.id_to_piece.append(piece)
        self.piece_to_id[piece] = i
        return i

    def load(self, vocab_path: str, merges_path: str) -> bool:
        self.__init__()
        try:
            with open(merges_path, "rb") as f:
                merges = f.read()
            with open(vocab_path, "rb") as f:
                pairs = json.loads(f.read().decode("utf-8", "surrogatepass"), object_pairs_hook=lambda p: p)
        except (OSError, ValueError):
            return False
        if not isinstance(pairs, list):
            return False
        count = 0
        for key, value in pairs:
            i = _strtol(_json_value_text(value))
            if i is None or i < 0:
                continue
            piece = key.encode("utf-8", "surrogatepass")
            if i >= len(self.id_to_piece):
                self.id_to_piece.extend([b""] * (i + 1 - len(self.id_to_piece)))
            self.id_to_piece[i] = piece
            self.piece_to_id.setdefault(piece, i)
            count += 1
        if count == 0:
            return False
        self.bos_id = self._ensure(BOS_TOKEN)
        self.eos_id = self._ensure(EOS_TOKEN)
        self.unk_id = self._ensure(UNK_TOKEN)
        self.word_end_id = self.piece_to_id.get(WORD_END_TOKEN, -1)
        for b in range(256):
            self.byte_id[b] = self.piece_to_id.get(_TO_CHAR[b], self.unk_id)
        lines = merges.split(b"\n") if merges else []
        if merges.endswith(b"\n"):
            lines = lines[:-1]
        for raw in lines:
            line = raw[:-1] if raw.endswith(b"\r") else raw
            if not line or line[:1] == b"#":
                continue
            sp = line.find(b" ")
            if sp < 0:
                continue
            left, right = line[:sp], line[sp + 1:]
            if not right:
                continue
            key = (self._ensure(left), self._ensure(right))
            if key in self.merge_rank:
                continue
            merged = self._ensure(left + right)
            self.merge_rank[key] = len(self.merge_result)
            self.merge_result.append(merged)
        self.special_pieces = sorted([BOS_TOKEN, EOS_TOKEN, UNK_TOKEN], key=lambda p: (-len(p), p))
        self.special_ids = [self._ensure(p) for p in self.special_pieces]
        return True

    def add_special_token(self, piece: bytes) -> int:
        if not piece:
            return -1
        i = self.piece_to_id.get(piece, -1)
        if i < 0:
            return -1
        if piece not in self.special_pieces:
            self.special_pieces.append(piece)
            self.special_ids.append(i)
        return i

    @property
    def vocab_size(self) -> int:
        return len(self.piece_to_id)

    def token_to_piece(self, i: int) -> bytes:
        return self.id_to_piece[i] if 0 <= i < len(self.id_to_piece) else b""

    # -- encoding ----------------------------------------------------------
    def _find_special(self, text: bytes, start: int):
        found, best_at, best_len = -1, -1, 0
        for i, p in enumerate(self.special_pieces):
            at = text.find(p, start)
            if at < 0:
                continue
            if found < 0 or at < best_at or (at == best_at and len(p) > best_len):
                found, best_at, best_len = i, at, len(p)
        return found, best_at, best_len

    def _merge_word(self, symbols: list[int]) -> list[int]:
        """Byte-pair merging of one word by the rule of tokenizer.h:483-600:
        while two adjacent symbols form a known merge, apply the one of lowest
        rank, the leftmost of equal ranks; a merge whose result is not in the
        vocabulary never applies. Candidates sit in a heap keyed (rank, left
        position); cur[p] is the rank of the pair now starting at p (-1: none),
        so an entry is acted on only while it still describes the word. A
        merge keeps its left position, so position 0 always heads the word."""
        n = len(symbols)
        if n < 2 or not self.merge_rank:
            return list(symbols)
        sym = list(symbols)
        left = list(range(-1, n - 1))
        right = list(range(1, n)) + [-1]
        cur = [-1] * n
        heap: list[tuple[int, int]] = []

        def refresh(p: int) -> None:
            if p < 0:
                return
            q, r = right[p], -1
            if q >= 0:
                got = self.merge_rank.get((sym[p], sym[q]))
                if got is not None and self.merge_result[got] >= 0:
                    r = got
            cur[p] = r
            if r >= 0:
                heapq.heappush(heap, (r, p))

        for i in range(n - 1):
            refresh(i)
        while heap:
            r, p = heapq.heappop(heap)
            if cur[p] != r:
                continue
            q = right[p]
            sym[p] = self.merge_result[r]
            cur[q] = -1
            right[p] = right[q]
            if right[q] >= 0:
                left[right[q]] = p
            refresh(p)
            refresh(left[p])
        out = []
        i = 0
        while i >= 0:
            out.append(sym[i])
            i = right[i]
        return out

    def encode(self, text) -> list[int]:
        data = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        ids: list[int] = []
        cur = 0
        while cur < len(data):
            si, at, ln = self._find_special(data, cur)
            end = at if si >= 0 else len(data)
            if end > cur:
                seg = data[cur:end]
                for a, b in split_word_ranges(seg):
                    if b <= a:
                        continue
                    symbols = [self.byte_id[c] for c in seg[a:b]]
                    if self.word_end_id >= 0:
                        symbols.append(self.word_end_id)
                    ids.extend(self._merge_word(symbols))
            if si < 0:
                break
            ids.append(self.special_ids[si])
            cur = at + ln
        return ids

    def decode(self, ids) -> bytes:
        out = bytearray()
        for i in ids:
            i = int(i)
            if i < 0 or i >= len(self.id_to_piece):
                continue
            if i in (self.bos_id, self.eos_id, self.unk_id):
                out += self.id_to_piece[i]
                continue
            body = self.id_to_piece[i]
            if len(body) >= 4 and body.endswith(WORD_END_TOKEN):
                body = body[:-4]
            j = 0
            while j < len(body):
                cp, ln = utf8_decode(body, j)
                b = byte_level_decode(cp)
                if b >= 0:
                    out.append(b)
                j += ln
        return bytes(out)


def load_tokenizer(model_dir: str) -> Tokenizer:
    """vocab.json + merges.txt of a reference model directory."""
    tok = Tokenizer()
    if not tok.load(os.path.join(model_dir, "vocab.json"), os.path.join(model_dir, "merges.txt")):
        raise ValueError(f"{model_dir}: tokenizer files missing or unreadable")
    return tok
