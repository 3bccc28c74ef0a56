// Text C ABI: the reference's jieyu_load / jieyu_generate flow
// (main.hpp:85-227 over model_libs/pipeline.h:280-436) on the device path.
// Host work only: JSON reading, the byte-level BPE tokenizer, the model.bf
// directory binding and the output rules of generate_text; the token loop
// is jyc_generate (the device model, model.cu).
#include "jieyu.h"
#include "jieyu_b200.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <climits>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>
#include <set>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// JSON: values keep their source text (the reference's parser does,
// json_libs/json_parser.h:99), objects keep members in order.
struct JVal {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    std::string text;  // a string's decoded bytes; for the rest, the source text
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;

    const JVal* find(const std::string& k) const {  // first match, as json_file::find
        if (kind != OBJ) return nullptr;
        for (const auto& m : obj)
            if (m.first == k) return &m.second;
        return nullptr;
    }
};

void put_utf8(std::string& s, uint32_t cp) {
    if (cp <= 0x7F) {
        s += (char)cp;
    } else if (cp <= 0x7FF) {
        s += (char)(0xC0 | (cp >> 6));
        s += (char)(0x80 | (cp & 0x3F));
    } else if (cp <= 0xFFFF) {
        s += (char)(0xE0 | (cp >> 12));
        s += (char)(0x80 | ((cp >> 6) & 0x3F));
        s += (char)(0x80 | (cp & 0x3F));
    } else {
        s += (char)(0xF0 | (cp >> 18));
        s += (char)(0x80 | ((cp >> 12) & 0x3F));
        s += (char)(0x80 | ((cp >> 6) & 0x3F));
        s += (char)(0x80 | (cp & 0x3F));
    }
}

class JParser {
public:
    JParser(const char* p, size_t n) : b_(p), p_(p), e_(p + n) {}
    bool parse(JVal& v) {
        ws();
        if (!value(v, 0)) return false;
        ws();
        return p_ == e_;
    }

private:
    const char *b_, *p_, *e_;
    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* w) {
        size_t n = strlen(w);
        if ((size_t)(e_ - p_) < n || memcmp(p_, w, n) != 0) return false;
        p_ += n;
        return true;
    }
    bool hex4(uint32_t& cp) {
        if (e_ - p_ < 4) return false;
        cp = 0;
        for (int i = 0; i < 4; ++i) {
            char c = p_[i];
            int h = (c >= '0' && c <= '9') ? c - '0' : (c >= 'a' && c <= 'f') ? c - 'a' + 10
                  : (c >= 'A' && c <= 'F') ? c - 'A' + 10 : -1;
            if (h < 0) return false;
            cp = cp * 16 + (uint32_t)h;
        }
        p_ += 4;
        return true;
    }
    bool str(std::string& s) {
        ++p_;
        while (p_ < e_) {
            unsigned char c = (unsigned char)*p_++;
            if (c == '"') return true;
            if (c != '\\') {
                if (c < 0x20) return false;
                s += (char)c;
                continue;
            }
            if (p_ >= e_) return false;
            char x = *p_++;
            switch (x) {
                case '"': s += '"'; break;
                case '\\': s += '\\'; break;
                case '/': s += '/'; break;
                case 'b': s += '\b'; break;
                case 'f': s += '\f'; break;
                case 'n': s += '\n'; break;
                case 'r': s += '\r'; break;
                case 't': s += '\t'; break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00 && e_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                        const char* save = p_;
                        p_ += 2;
                        uint32_t lo;
                        if (hex4(lo) && lo >= 0xDC00 && lo < 0xE000)
                            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                        else
                            p_ = save;
                    }
                    put_utf8(s, cp);  // a lone surrogate becomes its 3-byte form
                    break;
                }
                default: return false;
            }
        }
        return false;
    }
    bool number() {
        const char* s = p_;
        if (p_ < e_ && *p_ == '-') ++p_;
        if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
        if (*p_ == '0') ++p_;
        else while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
        if (p_ < e_ && *p_ == '.') {
            ++p_;
            if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
            while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ < e_ && (*p_ == 'e' || *p_ == 'E')) {
            ++p_;
            if (p_ < e_ && (*p_ == '+' || *p_ == '-')) ++p_;
            if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
            while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        return p_ > s;
    }
    bool value(JVal& v, int depth) {
        if (depth > 256 || p_ >= e_) return false;
        const char* start = p_;
        char c = *p_;
        if (c == '{') {
            v.kind = JVal::OBJ;
            ++p_;
            ws();
            if (p_ < e_ && *p_ == '}') { ++p_; v.text.assign(start, p_); return true; }
            for (;;) {
                ws();
                if (p_ >= e_ || *p_ != '"') return false;
                std::string key;
                if (!str(key)) return false;
                ws();
                if (p_ >= e_ || *p_ != ':') return false;
                ++p_;
                ws();
                v.obj.emplace_back(std::move(key), JVal());
                if (!value(v.obj.back().second, depth + 1)) return false;
                ws();
                if (p_ < e_ && *p_ == ',') { ++p_; continue; }
                if (p_ < e_ && *p_ == '}') { ++p_; break; }
                return false;
            }
            v.text.assign(start, p_);
            return true;
        }
        if (c == '[') {
            v.kind = JVal::ARR;
            ++p_;
            ws();
            if (p_ < e_ && *p_ == ']') { ++p_; v.text.assign(start, p_); return true; }
            for (;;) {
                ws();
                v.arr.emplace_back();
                if (!value(v.arr.back(), depth + 1)) return false;
                ws();
                if (p_ < e_ && *p_ == ',') { ++p_; continue; }
                if (p_ < e_ && *p_ == ']') { ++p_; break; }
                return false;
            }
            v.text.assign(start, p_);
            return true;
        }
        if (c == '"') { v.kind = JVal::STR; return str(v.text); }
        if (lit("true") || lit("false")) { v.kind = JVal::BOOL; v.text.assign(start, p_); return true; }
        if (lit("null")) { v.kind = JVal::NUL; v.text = "null"; return true; }
        if (!number()) return false;
        v.kind = JVal::NUM;
        v.text.assign(start, p_);
        return true;
    }
};

bool read_file(const std::string& path, std::string& out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::ostringstream ss;
    ss << f.rdbuf();
    out = ss.str();
    return true;
}

bool read_json(const std::string& path, JVal& v) {
    std::string s;
    if (!read_file(path, s)) return false;
    return JParser(s.data(), s.size()).parse(v);
}

// json_file::GetJsonData (json.h:57-63): a string's text, else the source text.
std::string info_text(const JVal& info, const char* key) {
    const JVal* v = info.find(key);
    return v ? v->text : std::string();
}

// std::stoi of GetJsonInt (json.h:73-83): the fallback when the text is
// empty, has no leading digits or leaves the int range.
int stoi_or(const std::string& s, int fallback) {
    if (s.empty()) return fallback;
    errno = 0;
    char* end = nullptr;
    long v = strtol(s.c_str(), &end, 10);
    if (end == s.c_str() || errno == ERANGE || v < INT_MIN || v > INT_MAX) return fallback;
    return (int)v;
}

// ---------------------------------------------------------------------------
// Byte-level BPE (tokenizer_libs/include/tokenizer.h).
const char kBos[] = "<\xef\xbd\x9c" "begin\xe2\x96\x81of\xe2\x96\x81sentence\xef\xbd\x9c>";
const char kEos[] = "<\xef\xbd\x9c" "end\xe2\x96\x81of\xe2\x96\x81sentence\xef\xbd\x9c>";
const char kUnk[] = "<unk>";
const char kWordEnd[] = "</w>";

// Lenient UTF-8 (json_libs/file_util.h:36-73): an invalid or truncated
// sequence yields its lead byte as one code point.
uint32_t utf8_at(const unsigned char* d, size_t n, size_t i, size_t* len) {
    unsigned b0 = d[i];
    size_t left = n - i;
    auto cont = [&](size_t j) { return (d[i + j] & 0xC0) == 0x80; };
    if (b0 < 0x80) { *len = 1; return b0; }
    if ((b0 & 0xE0) == 0xC0 && left >= 2 && cont(1)) {
        *len = 2;
        return ((b0 & 0x1F) << 6) | (d[i + 1] & 0x3F);
    }
    if ((b0 & 0xF0) == 0xE0 && left >= 3 && cont(1) && cont(2)) {
        *len = 3;
        return ((b0 & 0x0F) << 12) | ((d[i + 1] & 0x3F) << 6) | (d[i + 2] & 0x3F);
    }
    if ((b0 & 0xF8) == 0xF0 && left >= 4 && cont(1) && cont(2) && cont(3)) {
        *len = 4;
        return ((b0 & 0x07) << 18) | ((d[i + 1] & 0x3F) << 12) | ((d[i + 2] & 0x3F) << 6) | (d[i + 3] & 0x3F);
    }
    *len = 1;
    return b0;
}

bool printable_byte(int b) { return (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255); }

struct ByteMap {  // tokenizer.h:69-125: printable bytes are their own code point, the rest 256, 257, ...
    std::string sym[256];
    int back[256];  // code point 256 + slot -> byte
    int nback = 0;
    ByteMap() {
        for (int b = 0; b < 256; ++b) {
            if (printable_byte(b)) {
                put_utf8(sym[b], (uint32_t)b);
            } else {
                put_utf8(sym[b], (uint32_t)(256 + nback));
                back[nback++] = b;
            }
        }
    }
    int decode(uint32_t cp) const {
        if (cp < 256) return printable_byte((int)cp) ? (int)cp : -1;
        uint32_t slot = cp - 256;
        return slot < (uint32_t)nback ? back[slot] : -1;
    }
};
const ByteMap& byte_map() {
    static const ByteMap m;
    return m;
}

bool is_space(uint32_t cp) {
    return cp == 0x20 || cp == 0x09 || cp == 0x0A || cp == 0x0B || cp == 0x0C || cp == 0x0D || cp == 0x3000;
}
bool is_punct(uint32_t cp) {
    return (cp >= 0x21 && cp <= 0x2F) || (cp >= 0x3A && cp <= 0x40) || (cp >= 0x5B && cp <= 0x60) ||
           (cp >= 0x7B && cp <= 0x7E) || (cp >= 0x2010 && cp <= 0x2027) || (cp >= 0x2030 && cp <= 0x205E) ||
           (cp >= 0x3001 && cp <= 0x303F) || (cp >= 0xFF01 && cp <= 0xFF0F) || (cp >= 0xFF1A && cp <= 0xFF20) ||
           (cp >= 0xFF3B && cp <= 0xFF40) || (cp >= 0xFF5B && cp <= 0xFF65);
}

// Word boundaries of tokenizer.h:152-222: runs of white space (a single ' '
// joins the following word, or the following punctuation character), single
// punctuation characters, and runs of other characters.
void split_words(const unsigned char* t, size_t size, std::vector<std::pair<size_t, size_t>>& out) {
    size_t i = 0, ln;
    auto run_other = [&](size_t s) {
        while (s < size) {
            uint32_t c = utf8_at(t, size, s, &ln);
            if (is_space(c) || is_punct(c)) break;
            s += ln;
        }
        return s;
    };
    while (i < size) {
        uint32_t cp = utf8_at(t, size, i, &ln);
        if (is_space(cp)) {
            size_t nxt = i;
            while (nxt < size) {
                size_t l2;
                uint32_t c2 = utf8_at(t, size, nxt, &l2);
                if (!is_space(c2)) break;
                nxt += l2;
            }
            if (nxt - i == 1 && t[i] == 0x20 && nxt < size) {
                size_t al;
                uint32_t after = utf8_at(t, size, nxt, &al);
                size_t stop = is_punct(after) ? nxt + al : run_other(nxt);
                out.emplace_back(i, stop);
                i = stop;
            } else {
                out.emplace_back(i, nxt);
                i = nxt;
            }
            continue;
        }
        if (is_punct(cp)) {
            out.emplace_back(i, i + ln);
            i += ln;
            continue;
        }
        size_t stop = run_other(i);
        out.emplace_back(i, stop);
        i = stop;
    }
}

}  // namespace

struct jyt_tokenizer {
    std::unordered_map<std::string, int> piece_to_id;
    std::vector<std::string> id_to_piece;
    std::unordered_map<uint64_t, int> merge_rank;
    std::vector<int> merge_result;
    int byte_id[256];
    int word_end_id = -1, bos_id = -1, eos_id = -1, unk_id = -1;
    std::vector<std::string> special_pieces;
    std::vector<int> special_ids;

    static uint64_t pair_key(int a, int b) { return ((uint64_t)(uint32_t)a << 32) | (uint32_t)b; }

    int ensure(const std::string& p) {
        auto it = piece_to_id.find(p);
        if (it != piece_to_id.end()) return it->second;
        int i = (int)id_to_piece.size();
        id_to_piece.push_back(p);
        piece_to_id.emplace(p, i);
        return i;
    }
    int id_of(const std::string& p, int fallback) const {
        auto it = piece_to_id.find(p);
        return it == piece_to_id.end() ? fallback : it->second;
    }

    // tokenizer.h:340-455
    bool load(const std::string& vocab_path, const std::string& merges_path) {
        std::string merges;
        JVal vocab;
        if (!read_file(merges_path, merges) || !read_json(vocab_path, vocab) || vocab.kind != JVal::OBJ) return false;
        int count = 0;
        for (const auto& m : vocab.obj) {
            const std::string& v = m.second.text;  // value_to_string
            errno = 0;
            char* end = nullptr;
            long i = strtol(v.c_str(), &end, 10);
            if (end == v.c_str() || errno == ERANGE || i < 0 || i > (1L << 28)) continue;
            if ((size_t)i >= id_to_piece.size()) id_to_piece.resize((size_t)i + 1);
            id_to_piece[(size_t)i] = m.first;
            piece_to_id.emplace(m.first, (int)i);
            ++count;
        }
        if (count == 0) return false;
        bos_id = ensure(kBos);
        eos_id = ensure(kEos);
        unk_id = ensure(kUnk);
        word_end_id = id_of(kWordEnd, -1);
        for (int b = 0; b < 256; ++b) byte_id[b] = id_of(byte_map().sym[b], unk_id);
        size_t start = 0;
        while (start < merges.size()) {
            size_t nl = merges.find('\n', start);
            size_t stop = nl == std::string::npos ? merges.size() : nl;
            std::string line = merges.substr(start, stop - start);
            start = nl == std::string::npos ? merges.size() : nl + 1;
            if (!line.empty() && line.back() == '\r') line.pop_back();
            if (line.empty() || line[0] == '#') continue;
            size_t sp = line.find(' ');
            if (sp == std::string::npos) continue;
            std::string left = line.substr(0, sp), right = line.substr(sp + 1);
            if (right.empty()) continue;
            uint64_t key = pair_key(ensure(left), ensure(right));
            if (merge_rank.count(key)) continue;
            int merged = ensure(left + right);
            merge_rank.emplace(key, (int)merge_result.size());
            merge_result.push_back(merged);
        }
        special_pieces = {kBos, kEos, kUnk};
        std::sort(special_pieces.begin(), special_pieces.end(), [](const std::string& a, const std::string& b) {
            return a.size() != b.size() ? a.size() > b.size() : a < b;
        });
        for (const auto& p : special_pieces) special_ids.push_back(ensure(p));
        return true;
    }

    int add_special(const std::string& piece) {
        if (piece.empty()) return -1;
        int i = id_of(piece, -1);
        if (i < 0) return -1;
        if (std::find(special_pieces.begin(), special_pieces.end(), piece) == special_pieces.end()) {
            special_pieces.push_back(piece);
            special_ids.push_back(i);
        }
        return i;
    }

    // The earliest special piece from `start`, the longest at equal position.
    int find_special(const std::string& text, size_t start, size_t* at, size_t* len) const {
        int found = -1;
        for (size_t i = 0; i < special_pieces.size(); ++i) {
            size_t a = text.find(special_pieces[i], start);
            if (a == std::string::npos) continue;
            if (found < 0 || a < *at || (a == *at && special_pieces[i].size() > *len)) {
                found = (int)i;
                *at = a;
                *len = special_pieces[i].size();
            }
        }
        return found;
    }

    // Byte-pair merging of one word by the rule of tokenizer.h:483-600: while
    // two adjacent symbols form a known merge, apply the one of lowest rank,
    // the leftmost of equal ranks; a merge whose result is not in the
    // vocabulary never applies. The candidate pairs live in an ordered set
    // keyed (rank, left position), updated as each merge joins two symbols;
    // a merge keeps the left position, so position 0 always heads the word.
    void merge_word(std::vector<int>& sym, std::vector<int>& out) const {
        const int n = (int)sym.size();
        if (n < 2 || merge_rank.empty()) {
            out.insert(out.end(), sym.begin(), sym.end());
            return;
        }
        std::vector<int> left(n), right(n);  // neighbours in the live sequence (-1: none)
        for (int i = 0; i < n; ++i) {
            left[i] = i - 1;
            right[i] = i + 1 < n ? i + 1 : -1;
        }
        std::vector<int> in_set(n, -1);  // rank under which the pair starting at i is in `cand`
        std::set<std::pair<int, int>> cand;
        auto pair_rank = [&](int p) {
            const int q = right[p];
            if (q < 0) return -1;
            auto it = merge_rank.find(pair_key(sym[p], sym[q]));
            if (it == merge_rank.end() || merge_result[(size_t)it->second] < 0) return -1;
            return it->second;
        };
        auto add = [&](int p) {
            if (p < 0) return;
            in_set[p] = pair_rank(p);
            if (in_set[p] >= 0) cand.emplace(in_set[p], p);
        };
        auto drop = [&](int p) {
            if (p < 0 || in_set[p] < 0) return;
            cand.erase({in_set[p], p});
            in_set[p] = -1;
        };
        for (int i = 0; i + 1 < n; ++i) add(i);
        while (!cand.empty()) {
            const int r = cand.begin()->first, p = cand.begin()->second, q = right[p];
            drop(left[p]);
            drop(p);
            drop(q);
            sym[p] = merge_result[(size_t)r];
            right[p] = right[q];
            if (right[q] >= 0) left[right[q]] = p;
            add(left[p]);
            add(p);
        }
        for (int i = 0; i >= 0; i = right[i]) out.push_back(sym[i]);
    }

    std::vector<int> encode(const std::string& data) const {
        std::vector<int> ids, symbols;
        std::vector<std::pair<size_t, size_t>> words;
        size_t cur = 0;
        while (cur < data.size()) {
            size_t at = 0, len = 0;
            int si = find_special(data, cur, &at, &len);
            size_t end = si >= 0 ? at : data.size();
            if (end > cur) {
                const unsigned char* seg = reinterpret_cast<const unsigned char*>(data.data()) + cur;
                words.clear();
                split_words(seg, end - cur, words);
                for (const auto& w : words) {
                    if (w.second <= w.first) continue;
                    symbols.clear();
                    for (size_t k = w.first; k < w.second; ++k) symbols.push_back(byte_id[seg[k]]);
                    if (word_end_id >= 0) symbols.push_back(word_end_id);
                    merge_word(symbols, ids);
                }
            }
            if (si < 0) break;
            ids.push_back(special_ids[(size_t)si]);
            cur = at + len;
        }
        return ids;
    }

    void decode_one(int i, std::string& out) const {
        if (i < 0 || (size_t)i >= id_to_piece.size()) return;
        const std::string& piece = id_to_piece[(size_t)i];
        if (i == bos_id || i == eos_id || i == unk_id) {
            out += piece;
            return;
        }
        size_t n = piece.size();
        if (n >= 4 && piece.compare(n - 4, 4, kWordEnd) == 0) n -= 4;
        const unsigned char* d = reinterpret_cast<const unsigned char*>(piece.data());
        for (size_t j = 0, ln; j < n; j += ln) {
            int b = byte_map().decode(utf8_at(d, n, j, &ln));
            if (b >= 0) out += (char)b;
        }
    }
};

namespace {

// ---------------------------------------------------------------------------
// model.bf (bfile.h:141-204 View::open) bound as load_model_dir binds it
// (load_weights.h:55-155, pipeline.h:63-153).
enum BDtype { BF32 = 0, BF16_ = 1, BBF16 = 2, BI8 = 3, BI32 = 4, BQ4K = 5, BQ5K = 6, BQ6K = 7, BQ8_0 = 8 };

struct BTensor {
    int dtype = 0;
    std::vector<uint64_t> shape;
    const uint8_t* data = nullptr;
};

bool block_dtype(int dt, uint64_t* elems, uint64_t* bytes) {
    switch (dt) {
        case BQ4K: *elems = 256; *bytes = 144; return true;
        case BQ5K: *elems = 256; *bytes = 176; return true;
        case BQ6K: *elems = 256; *bytes = 210; return true;
        case BQ8_0: *elems = 32; *bytes = 34; return true;
        default: return false;
    }
}

uint64_t tensor_bytes(int dt, uint64_t elems) {
    uint64_t be, bb;
    if (block_dtype(dt, &be, &bb)) return elems % be ? 0 : elems / be * bb;
    switch (dt) {
        case BF32: case BI32: return elems * 4;
        case BF16_: case BBF16: return elems * 2;
        case BI8: return elems;
        default: return 0;
    }
}

int kq_code(int dt) { return dt == BQ4K ? JYC_Q4K : dt == BQ5K ? JYC_Q5K : dt == BQ6K ? JYC_Q6K : -1; }

struct BFile {
    void* map = nullptr;
    size_t size = 0;
    uint64_t hidden = 0, layers = 0, vocab = 0;
    int heads = 0, kv_heads = 0, head_dim = 0;
    uint32_t inter = 0;
    std::unordered_map<std::string, BTensor> tensors;

    ~BFile() {
        if (map) munmap(map, size);
    }
    const BTensor* get(const std::string& n) const {
        auto it = tensors.find(n);
        return it == tensors.end() ? nullptr : &it->second;
    }
    void open(const std::string& path) {
        int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) throw std::runtime_error(path + ": cannot open");
        struct stat st;
        if (fstat(fd, &st) != 0) {
            ::close(fd);
            throw std::runtime_error(path + ": cannot stat");
        }
        size = (size_t)st.st_size;
        if (size < 64) {
            ::close(fd);
            throw std::runtime_error(path + ": shorter than the 64-byte header");
        }
        map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (map == MAP_FAILED) {
            map = nullptr;
            throw std::runtime_error(path + ": mmap failed");
        }
        const uint8_t* h = static_cast<const uint8_t*>(map);
        auto u32 = [&](size_t o) { uint32_t v; memcpy(&v, h + o, 4); return v; };
        auto u64 = [&](size_t o) { uint64_t v; memcpy(&v, h + o, 8); return v; };
        if (memcmp(h, "JYAIBF", 6) != 0) throw std::runtime_error(path + ": not a JYAIBF file");
        hidden = u64(6);
        layers = u64(14);
        heads = h[23];
        kv_heads = h[24];
        head_dim = h[25];
        inter = u32(26);
        vocab = u64(30);
        uint32_t version = u32(38), count = u32(42), data_off = u32(46), esize = u32(50);
        if (version < 2) throw std::runtime_error(path + ": version " + std::to_string(version) + " has no tensor directory");
        if (esize != 104) throw std::runtime_error(path + ": directory entries of " + std::to_string(esize) + " bytes");
        if (data_off < 64 || data_off > size) throw std::runtime_error(path + ": data offset outside the file");
        if (64 + (uint64_t)count * 104 > data_off) throw std::runtime_error(path + ": directory does not fit");
        for (uint32_t e = 0; e < count; ++e) {
            const uint8_t* ent = h + 64 + (size_t)e * 104;
            std::string name(reinterpret_cast<const char*>(ent), strnlen(reinterpret_cast<const char*>(ent), 64));
            int dt = ent[64], nd = ent[65];
            if (nd > 4) throw std::runtime_error(path + ": " + name + ": more than 4 dimensions");
            uint64_t be, bb;
            if (tensor_bytes(dt, 1) == 0 && !block_dtype(dt, &be, &bb))
                throw std::runtime_error(path + ": " + name + ": unknown dtype " + std::to_string(dt));
            BTensor t;
            t.dtype = dt;
            uint64_t elems = 1;
            for (int d = 0; d < nd; ++d) {
                uint32_t s;
                memcpy(&s, ent + 68 + 4 * d, 4);
                t.shape.push_back(s);
                elems *= s;
            }
            uint64_t off, nb;
            memcpy(&off, ent + 88, 8);
            memcpy(&nb, ent + 96, 8);
            if (tensor_bytes(dt, elems) != nb) throw std::runtime_error(path + ": " + name + ": shape does not match its byte count");
            if (off % 64) throw std::runtime_error(path + ": " + name + ": data offset not a multiple of 64");
            if (data_off + off + nb > size) throw std::runtime_error(path + ": " + name + ": data runs past the end of the file");
            t.data = h + data_off + off;
            tensors.emplace(name, std::move(t));  // first match wins, as find()
        }
    }
};

std::string shape_str(const std::vector<uint64_t>& s) {
    std::string o = "[";
    for (size_t i = 0; i < s.size(); ++i) o += (i ? ", " : "") + std::to_string(s[i]);
    return o + "]";
}

// A model directory bound to a device-model descriptor whose pointers
// reach into the mapped file; throws with the reason on failure.
struct BoundDir {
    BFile bf;
    std::vector<jyc_layer_weights> lw;
    std::vector<float> cos_t, sin_t;
    jyc_model_desc d{};
    bool bias = false, tied = false;
    unsigned kinds = 0;  // bit per bfile dtype of the layer weights
    int theta = 0;
};

void bind_dir(const std::string& dir, int max_seq, BoundDir& b) {
    BFile& bf = b.bf;
    bf.open(dir + "/model.bf");
    const int L = (int)bf.layers, D = (int)bf.hidden, H = bf.heads, KV = bf.kv_heads, hd = bf.head_dim;
    const int F = (int)bf.inter, V = (int)bf.vocab;
    if (L <= 0 || D <= 0 || hd <= 0 || H <= 0) throw std::runtime_error(dir + ": header hyper-parameters are not valid");
    const int qd = H * hd, kvd = KV * hd;
    auto need = [&](const std::string& k) -> const BTensor& {
        const BTensor* t = bf.get(k);
        if (!t) throw std::runtime_error(dir + ": missing tensor " + k);
        return *t;
    };
    auto expect = [&](const std::string& k, const BTensor& t, std::vector<uint64_t> s) {
        if (t.shape != s) throw std::runtime_error(dir + ": " + k + " has shape " + shape_str(t.shape) + ", expected " + shape_str(s));
    };
    std::vector<int> kinds;
    auto linear = [&](const std::string& k, int inn, int out) {
        const BTensor& t = need(k);
        jyc_wmat w{};
        uint64_t be, bb;
        if (block_dtype(t.dtype, &be, &bb)) {
            expect(k, t, {(uint64_t)out, (uint64_t)inn});
            w.q = t.data;
            w.qt = (uint8_t)(t.dtype == BQ8_0 ? JYC_Q8_0 : kq_code(t.dtype));
        } else if (t.dtype == BF32) {
            expect(k, t, {(uint64_t)inn, (uint64_t)out});
            w.f = reinterpret_cast<const float*>(t.data);
        } else {
            throw std::runtime_error(dir + ": " + k + ": this device path runs Q8_0, Q4_K, Q5_K, Q6_K and f32 weights");
        }
        if (std::find(kinds.begin(), kinds.end(), t.dtype) == kinds.end()) kinds.push_back(t.dtype);
        return w;
    };
    auto f32 = [&](const std::string& k, int n) {
        const BTensor& t = need(k);
        if (t.dtype != BF32) throw std::runtime_error(dir + ": " + k + " must be f32");
        expect(k, t, {(uint64_t)n});
        return reinterpret_cast<const float*>(t.data);
    };
    auto lname = [](int l, const char* s) { return "model.layers." + std::to_string(l) + "." + s; };
    std::vector<jyc_layer_weights>& lw = b.lw;
    lw.resize((size_t)L);
    const bool bias = b.bias = bf.get(lname(0, "self_attn.q_proj.bias")) != nullptr;  // bind_biases: layer 0 decides
    for (int l = 0; l < L; ++l) {
        jyc_layer_weights& w = lw[(size_t)l];
        w.rms1_weight = f32(lname(l, "input_layernorm.weight"), D);
        w.rms2_weight = f32(lname(l, "post_attention_layernorm.weight"), D);
        w.Wq = linear(lname(l, "self_attn.q_proj.weight"), D, qd);
        w.Wk = linear(lname(l, "self_attn.k_proj.weight"), D, kvd);
        w.Wv = linear(lname(l, "self_attn.v_proj.weight"), D, kvd);
        w.Wo = linear(lname(l, "self_attn.o_proj.weight"), qd, D);
        w.W1 = linear(lname(l, "mlp.gate_proj.weight"), D, F);
        w.W2 = linear(lname(l, "mlp.down_proj.weight"), F, D);
        w.W3 = linear(lname(l, "mlp.up_proj.weight"), D, F);
        if (bias) {
            w.bq = f32(lname(l, "self_attn.q_proj.bias"), qd);
            w.bk = f32(lname(l, "self_attn.k_proj.bias"), kvd);
            w.bv = f32(lname(l, "self_attn.v_proj.bias"), kvd);
        }
    }
    if (std::find(kinds.begin(), kinds.end(), (int)BQ8_0) != kinds.end() && kinds.size() > 1)
        throw std::runtime_error(dir + ": Q8_0 linear weights mixed with other types; the device path runs Q8_0 models alone");
    const BTensor& emb = need("model.embed_tokens.weight");
    expect("model.embed_tokens.weight", emb, {(uint64_t)V, (uint64_t)D});
    auto as_wmat = [&](const char* k, const BTensor& t) {
        jyc_wmat w{};
        uint64_t be, bb;
        if (t.dtype == BF32) {
            w.f = reinterpret_cast<const float*>(t.data);
        } else if (block_dtype(t.dtype, &be, &bb)) {
            w.q = t.data;
            w.qt = (uint8_t)(t.dtype == BQ8_0 ? JYC_Q8_0 : kq_code(t.dtype));
        } else {
            throw std::runtime_error(dir + ": " + k + ": the device path reads f32, Q8_0 or K-quant here");
        }
        return w;
    };
    jyc_wmat embed = as_wmat("model.embed_tokens.weight", emb);
    const BTensor* head = bf.get("lm_head.weight");
    const char* head_name = "lm_head.weight";
    if (!head) {  // bind_lm_head's fallback (load_weights.h:142-144)
        b.tied = true;
        head = &emb;
        head_name = "model.embed_tokens.weight";
    }
    uint64_t be, bb;
    if (block_dtype(head->dtype, &be, &bb)) {
        expect(head_name, *head, {(uint64_t)V, (uint64_t)D});
    } else if (head->dtype == BF32) {
        expect(head_name, *head, {(uint64_t)D, (uint64_t)V});
    } else {
        throw std::runtime_error(dir + ": " + head_name + ": the device path runs block-quantised and f32 heads");
    }
    jyc_wmat lm_head = as_wmat(head_name, *head);
    const float* final_norm = f32("model.norm.weight", D);

    JVal info;
    if (!read_json(dir + "/model_info.json", info)) throw std::runtime_error(dir + "/model_info.json: missing or not JSON");
    if (max_seq <= 0)
        max_seq = std::max(64, std::min(stoi_or(info_text(info, "max_position_embeddings"), 1024), 4096));
    b.theta = stoi_or(info_text(info, "rope_theta"), 10000);
    const float theta = (float)b.theta;
    std::vector<float>& cos_t = b.cos_t;
    std::vector<float>& sin_t = b.sin_t;
    cos_t.assign((size_t)max_seq * (hd / 2), 0.f);
    sin_t.assign(cos_t.size(), 0.f);
    if (jyc_rope_table(max_seq, hd, theta, cos_t.data(), sin_t.data()) != JYC_OK)
        throw std::runtime_error(std::string("RoPE table: ") + jyc_last_error());

    for (int k : kinds) b.kinds |= 1u << k;
    jyc_model_desc& d = b.d;
    d.layers = lw.data();
    d.num_layers = L;
    d.embed = embed;
    d.lm_head = lm_head;
    d.final_rms_weight = final_norm;
    d.cos_table = cos_t.data();
    d.sin_table = sin_t.data();
    d.max_seq = max_seq;
    d.vocab_size = V;
    d.hidden = D;
    d.num_heads = H;
    d.num_kv_heads = KV;
    d.head_dim = hd;
    d.intermediate = F;
}

// The device model of a model directory (every weight uploaded; the file
// mapping is released on return).
jyc_model* bind_model_dir(const std::string& dir, int max_seq, int* vocab_out) {
    BoundDir b;
    bind_dir(dir, max_seq, b);
    jyc_model* m = jyc_model_create(&b.d);
    if (!m) throw std::runtime_error(std::string("device upload failed: ") + jyc_last_error());
    *vocab_out = b.d.vocab_size;
    return m;
}

// ---------------------------------------------------------------------------
// The loaded model (main.hpp:15-28): one per process, shared by the handles.
struct Loaded {
    std::string dir;
    jyc_model* model = nullptr;
    jyt_tokenizer tok;
    int vocab = 0, max_seq = 0;
    bool add_bos = true;
    std::string s_start, s_end, s_text, s_user, s_asst, s_turn;
    int id_start = 0, id_end = 0, id_text = 0;

    void release() {
        if (model) jyc_model_free(model);
        model = nullptr;
        tok = jyt_tokenizer();
        dir.clear();
    }
};

Loaded& loaded() {
    static Loaded l;
    return l;
}
int& handle_count() {
    static int n = 0;
    return n;
}
bool& model_ready() {
    static bool r = false;
    return r;
}

void set_text(char* dst, size_t cap, const char* src) {  // main.hpp:37-43
    if (!dst || cap == 0) return;
    size_t n = src ? strlen(src) : 0, k = n < cap - 1 ? n : cap - 1;
    if (k) memcpy(dst, src, k);
    dst[k] = '\0';
}
char* load_error() {
    static thread_local char text[JIEYU_ERR_MAX] = {0};
    return text;
}
void set_load_error(const std::string& m) { set_text(load_error(), JIEYU_ERR_MAX, m.c_str()); }
void set_error(jieyu_ctx* h, const char* m) {
    if (h) set_text(h->error, JIEYU_ERR_MAX, m);
}

int copy_out(const std::string& text, char* out, int cap) {  // main.hpp:76-83
    if (!out || cap <= 0) return (int)text.size();
    size_t room = (size_t)cap - 1, n = text.size() < room ? text.size() : room;
    memcpy(out, text.data(), n);
    out[n] = '\0';
    return (int)text.size();
}

bool marker_char(unsigned char c) {
    return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '_' || c == '-';
}

// First position of a chat string or of "<|" + 1..24 marker characters
// (pipeline.h:201-217); npos when there is none.
size_t marker_at(const std::string& s, const std::vector<const std::string*>& stops) {
    size_t best = std::string::npos;
    for (const std::string* st : stops) {
        if (st->empty()) continue;
        size_t at = s.find(*st);
        if (at < best) best = at;
    }
    for (size_t lt = s.find("<|"); lt != std::string::npos; lt = s.find("<|", lt + 1)) {
        size_t n = 0;
        while (lt + 2 + n < s.size() && n < 24 && marker_char((unsigned char)s[lt + 2 + n])) ++n;
        if (n >= 1 && lt < best) best = lt;
    }
    return best;
}

struct Echo {  // echo_token (pipeline.h:230-260)
    const Loaded* m;
    std::string* out;
    std::vector<int> specials;
    std::vector<const std::string*> stops;
};

int echo_token(int id, void* ud) {
    Echo* e = static_cast<Echo*>(ud);
    if (std::find(e->specials.begin(), e->specials.end(), id) != e->specials.end()) return 1;
    e->m->tok.decode_one(id, *e->out);
    size_t at = marker_at(*e->out, e->stops);
    if (at != std::string::npos) {
        e->out->resize(at);
        return 1;
    }
    return 0;
}

// generate_text (pipeline.h:280-374): new-token count, 0 when nothing can be
// produced, -1 for prompt ids outside the model's vocabulary, -2 when the
// device loop failed.
int generate_text(const Loaded& m, const std::string& prompt, int max_new, float temperature, float rep_pen,
                  std::string& out) {
    out.clear();
    std::vector<int> ids = m.tok.encode(prompt);
    if (m.add_bos && m.tok.bos_id >= 0 && m.tok.bos_id < m.vocab) ids.insert(ids.begin(), m.tok.bos_id);
    if (ids.empty()) return 0;
    if (max_new <= 0) max_new = m.max_seq;
    for (int i : ids)
        if (i < 0 || i >= m.vocab) return -1;
    if ((int)ids.size() > m.max_seq) ids.resize((size_t)m.max_seq);
    if ((int)ids.size() + max_new > m.max_seq) max_new = m.max_seq - (int)ids.size();
    if (max_new <= 0) return 0;
    std::vector<int> eos;
    for (int e : {m.tok.eos_id, m.id_text, m.id_end})  // in range, distinct, at most 3
        if (e >= 0 && e < m.vocab && std::find(eos.begin(), eos.end(), e) == eos.end() && eos.size() < 3)
            eos.push_back(e);
    Echo echo{&m, &out, {}, {&m.s_start, &m.s_end, &m.s_text, &m.s_user, &m.s_asst, &m.s_turn}};
    for (int i : {m.id_start, m.id_end, m.id_text})
        if (i != 0) echo.specials.push_back(i);
    std::vector<int> seq((size_t)m.max_seq + 1);
    int n = jyc_generate(m.model, ids.data(), (int)ids.size(), eos.data(), (int)eos.size(), max_new, temperature,
                         seq.data(), rep_pen, echo_token, &echo);
    if (n < 0) return -2;
    return n - (int)ids.size();
}

int finish_generate(jieyu_model h, int produced, const std::string& text, char* out, int cap) {
    if (produced == -2) {
        std::string e = std::string("generation failed on the device: ") + jyc_last_error();
        set_error(h, e.c_str());
        return -1;
    }
    if (produced < 0) {
        set_error(h, "generation failed (the prompt has tokens outside the vocabulary)");
        return -1;
    }
    if (produced == 0) set_error(h, "nothing produced (empty prompt or full context)");
    copy_out(text, out, cap);
    return produced;
}

}  // namespace

extern "C" {

JIEYU_API jieyu_model jieyu_load(const char* dir, int max_seq) {
    if (!dir) {
        set_load_error("dir is NULL");
        return nullptr;
    }
    const std::string d(dir);
    Loaded& m = loaded();
    if (model_ready() && m.dir != d) {  // another directory unbinds the loaded one (main.hpp:98-102)
        m.release();
        model_ready() = false;
    }
    jieyu_ctx* ctx = new (std::nothrow) jieyu_ctx();
    if (!ctx) {
        set_load_error("out of memory");
        return nullptr;
    }
    set_text(ctx->dir, JIEYU_PATH_MAX, d.c_str());
    if (max_seq > 0) {
        ctx->max_seq = max_seq;
    } else {  // jieyu_auto_max_seq (main.hpp:64-67)
        JVal info;
        int want = read_json(d + "/model_info.json", info) ? stoi_or(info_text(info, "max_position_embeddings"), 1024)
                                                            : 1024;
        ctx->max_seq = std::max(64, std::min(want, 4096));
    }
    if (!model_ready()) {
        try {
            m.release();
            m.dir = d;
            m.max_seq = ctx->max_seq;
            m.model = bind_model_dir(d, ctx->max_seq, &m.vocab);
            if (!m.tok.load(d + "/vocab.json", d + "/merges.txt"))
                throw std::runtime_error("tokenizer load failed: " + d + "/vocab.json / " + d + "/merges.txt");
            JVal info;
            read_json(d + "/model_info.json", info);
            m.add_bos = stoi_or(info_text(info, "add_bos_token"), 1) != 0;
            m.s_start = info_text(info, "message_start");
            m.s_end = info_text(info, "message_end");
            m.s_text = info_text(info, "text_end");
            m.s_user = info_text(info, "user_start");
            m.s_asst = info_text(info, "assistant_start");
            m.s_turn = info_text(info, "turn_end");
            auto reg = [&](const std::string& p) {  // register_special: 0 when absent
                int i = p.empty() ? -1 : m.tok.add_special(p);
                return i < 0 ? 0 : i;
            };
            m.id_start = reg(m.s_start);
            m.id_end = reg(m.s_end);
            m.id_text = reg(m.s_text);
            reg(m.s_user);
            reg(m.s_asst);
            reg(info_text(info, "bos_text"));
            reg(m.s_turn);
        } catch (const std::exception& e) {
            m.release();
            set_load_error(e.what());
            delete ctx;
            return nullptr;
        }
        model_ready() = true;
    }
    handle_count()++;
    set_load_error("");
    return ctx;
}

JIEYU_API void jieyu_free(jieyu_model h) {
    if (!h) return;
    if (handle_count() > 0 && --handle_count() <= 0) {
        loaded().release();
        model_ready() = false;
    }
    delete h;
}

JIEYU_API const char* jieyu_last_error(jieyu_model h) { return h ? h->error : load_error(); }

JIEYU_API const char* jieyu_version(void) { return "1.0.0"; }

JIEYU_API int jieyu_context_length(jieyu_model h) { return h ? h->max_seq : 0; }

JIEYU_API const char* jieyu_model_dir(jieyu_model h) { return h ? h->dir : ""; }

JIEYU_API int jieyu_generate(jieyu_model h, const char* prompt, char* out, int cap, int max_new, float temperature,
                             float repetition_penalty) {
    if (!h) {
        set_load_error("handle is NULL");
        return -1;
    }
    if (!prompt) {
        set_error(h, "prompt is NULL");
        return -1;
    }
    if (!model_ready()) {
        set_error(h, "no model loaded (call jieyu_load first)");
        return -1;
    }
    set_error(h, "");
    std::string text;
    int produced = generate_text(loaded(), prompt, max_new, temperature, repetition_penalty, text);
    return finish_generate(h, produced, text, out, cap);
}

JIEYU_API int jieyu_generate_jsonl(jieyu_model h, const char* jsonl, const char* qb, const char* qe, char* out,
                                   int cap, int max_new, float temperature, float repetition_penalty) {
    if (!h) {
        set_load_error("handle is NULL");
        return -1;
    }
    if (!jsonl) {
        set_error(h, "jsonl path is NULL");
        return -1;
    }
    if (!model_ready()) {
        set_error(h, "no model loaded (call jieyu_load first)");
        return -1;
    }
    set_error(h, "");
    const Loaded& m = loaded();
    // json_ochat_build (jsonl_ochat.h:7-27): one JSON object per line
    std::string content, feed;
    const std::string pre = (qb && *qb) ? qb : m.s_start, suf = (qe && *qe) ? qe : m.s_end;
    if (read_file(jsonl, content)) {
        size_t start = 0;
        while (start < content.size()) {
            size_t nl = content.find('\n', start), stop = nl == std::string::npos ? content.size() : nl;
            JVal v;
            if (JParser(content.data() + start, stop - start).parse(v)) {
                std::string name = info_text(v, "name"), msg = info_text(v, "message");
                if (!name.empty() || !msg.empty()) feed += pre + name + '\n' + msg + suf + '\n';
            }
            if (nl == std::string::npos) break;
            start = nl + 1;
        }
    }
    if (feed.empty()) {
        set_error(h, "jsonl_no_srch (the file has no usable name/message)");
        return -1;
    }
    if (!m.s_asst.empty()) feed += m.s_asst;
    else if (m.s_start == "<|im_start|>") feed += m.s_start + "assistant\n";
    std::string text;
    int produced = generate_text(m, feed, max_new, temperature, repetition_penalty, text);
    return finish_generate(h, produced, text, out, cap);
}

JIEYU_API jyt_tokenizer* jyt_tok_load(const char* vocab_path, const char* merges_path) {
    if (!vocab_path || !merges_path) return nullptr;
    jyt_tokenizer* t = new (std::nothrow) jyt_tokenizer();
    if (t && !t->load(vocab_path, merges_path)) {
        delete t;
        t = nullptr;
    }
    return t;
}

JIEYU_API void jyt_tok_free(jyt_tokenizer* t) { delete t; }

JIEYU_API int jyt_tok_encode(const jyt_tokenizer* t, const char* text, int len, int* ids, int cap) {
    if (!t || (!text && len > 0) || len < 0) return -1;
    std::vector<int> v = t->encode(std::string(text ? text : "", (size_t)len));
    if (ids)
        for (int i = 0; i < cap && i < (int)v.size(); ++i) ids[i] = v[(size_t)i];
    return (int)v.size();
}

JIEYU_API int jyt_tok_decode(const jyt_tokenizer* t, const int* ids, int n, char* out, int cap) {
    if (!t || (!ids && n > 0) || n < 0) return -1;
    std::string s;
    for (int i = 0; i < n; ++i) t->decode_one(ids[i], s);
    if (out && cap > 0) memcpy(out, s.data(), std::min((size_t)cap, s.size()));
    return (int)s.size();
}

JIEYU_API int jyt_tok_add_special(jyt_tokenizer* t, const char* piece, int len) {
    if (!t || !piece || len < 0) return -1;
    return t->add_special(std::string(piece, (size_t)len));
}

JIEYU_API int jyt_model_dir_probe(const char* dir, int max_seq, int* out13, char* err, int cap) {
    if (!dir || !out13) return -1;
    try {
        BoundDir b;
        bind_dir(dir, max_seq, b);
        const jyc_model_desc& d = b.d;
        const int v[13] = {d.num_layers, d.hidden, d.num_heads, d.num_kv_heads, d.head_dim, d.intermediate,
                           d.vocab_size, d.max_seq, b.bias, b.tied, (int)b.kinds, b.theta,
                           (d.lm_head.q ? 1 : 0) | (d.embed.q ? 2 : 0)};
        memcpy(out13, v, sizeof v);
        if (err && cap > 0) err[0] = '\0';
        return 0;
    } catch (const std::exception& e) {
        if (err && cap > 0) set_text(err, (size_t)cap, e.what());
        return -1;
    }
}

JIEYU_API int jyt_tok_info(const jyt_tokenizer* t, int* out6) {
    if (!t || !out6) return -1;
    out6[0] = (int)t->piece_to_id.size();
    out6[1] = t->bos_id;
    out6[2] = t->eos_id;
    out6[3] = t->unk_id;
    out6[4] = t->word_end_id;
    out6[5] = (int)t->merge_result.size();
    return 0;
}

}  // extern "C"
