// bpe_tokenizer.cpp - see bpe_tokenizer.h.
#include "bpe_tokenizer.h"

#include <algorithm>
#include <cstring>
#include <deque>
#include <queue>
#include <string_view>

#include "gguf_reader.h"
#include "unicode_classes.h"

namespace bnn {

namespace {

enum : uint8_t { kLetter = 1, kNumber = 2, kSpace = 4 };
constexpr uint32_t kDead = 0xffffffffu;  // symbol of a node merged into its left neighbour

// Class bits of every code point, expanded once from the generated runs.
const uint8_t* class_table() {
    static const std::vector<uint8_t> table = [] {
        std::vector<uint8_t> t(0x110000, 0);
        for (const unicode::ClassRun& r : unicode::kRuns)
            for (uint32_t cp = r.first; cp <= r.last; ++cp)
                t[cp] = r.cls;
        for (uint32_t cp : unicode::kWhiteSpace)
            t[cp] |= kSpace;
        return t;
    }();
    return table.data();
}

// One code point of s[0..n) (n > 0) under RFC 3629: its length, or 0 for an
// invalid, truncated, overlong, surrogate or out-of-range sequence.
size_t utf8_next(const uint8_t* s, size_t n, uint32_t* cp) {
    const uint8_t b = s[0];
    if (b < 0x80) {
        *cp = b;
        return 1;
    }
    size_t len;
    uint32_t v, least;
    if (b >= 0xC2 && b <= 0xDF) {
        len = 2, v = b & 0x1Fu, least = 0x80;
    } else if (b >= 0xE0 && b <= 0xEF) {
        len = 3, v = b & 0x0Fu, least = 0x800;
    } else if (b >= 0xF0 && b <= 0xF4) {
        len = 4, v = b & 0x07u, least = 0x10000;
    } else {
        return 0;
    }
    if (n < len)
        return 0;
    for (size_t i = 1; i < len; ++i) {
        if ((s[i] & 0xC0u) != 0x80u)
            return 0;
        v = v << 6 | (s[i] & 0x3Fu);
    }
    if (v < least || v > 0x10FFFF || (v >= 0xD800 && v <= 0xDFFF))
        return 0;
    *cp = v;
    return len;
}

void utf8_append(uint32_t cp, std::string* out) {
    if (cp < 0x80) {
        out->push_back((char)cp);
    } else if (cp < 0x800) {
        out->push_back((char)(0xC0 | cp >> 6));
        out->push_back((char)(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
        out->push_back((char)(0xE0 | cp >> 12));
        out->push_back((char)(0x80 | (cp >> 6 & 0x3F)));
        out->push_back((char)(0x80 | (cp & 0x3F)));
    } else {
        out->push_back((char)(0xF0 | cp >> 18));
        out->push_back((char)(0x80 | (cp >> 12 & 0x3F)));
        out->push_back((char)(0x80 | (cp >> 6 & 0x3F)));
        out->push_back((char)(0x80 | (cp & 0x3F)));
    }
}

// GPT-2's byte-to-code-point table (tokenizer-bpe.c:718-733): printable bytes
// keep their value, the rest take 256, 257, ... in byte order.
void byte_code_points(uint32_t cp[256]) {
    uint32_t extra = 0;
    for (uint32_t b = 0; b < 256; ++b) {
        const bool keep = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || b >= 174;
        cp[b] = keep ? b : 256 + extra++;
    }
}

struct Cp {
    uint32_t cp;
    uint8_t cls;
    size_t off;  // byte offset in the segment
};

uint32_t ascii_lower(uint32_t c) { return c >= 'A' && c <= 'Z' ? c + 32 : c; }
bool is_newline(uint32_t c) { return c == '\r' || c == '\n'; }

// End (exclusive) of the pre-tokenizer chunk that starts at s[pos]: the
// Qwen2 split pattern's alternatives tried in order (tokenizer-bpe.c:418-538)
//   '(s|t|re|ve|m|ll|d)  case-insensitive contractions
//   [^\r\n\p{L}\p{N}]?\p{L}+
//   \p{N}
//   ' '?[^\s\p{L}\p{N}]+[\r\n]*
//   \s*[\r\n]+ | \s+(?!\S) | \s+
// and a single code point when none applies.
size_t chunk_end(const Cp* s, size_t n, size_t pos) {
    const uint32_t c = s[pos].cp;
    const uint8_t k = s[pos].cls;
    if (c == '\'' && pos + 1 < n) {
        const uint32_t a = ascii_lower(s[pos + 1].cp);
        if (a == 's' || a == 't' || a == 'm' || a == 'd')
            return pos + 2;
        if (pos + 2 < n) {
            const uint32_t b = ascii_lower(s[pos + 2].cp);
            if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l'))
                return pos + 3;
        }
    }
    if (!is_newline(c) && !(k & kNumber) && ((k & kLetter) || (pos + 1 < n && (s[pos + 1].cls & kLetter)))) {
        size_t e = pos + 1;
        while (e < n && (s[e].cls & kLetter))
            ++e;
        return e;
    }
    if (k & kNumber)
        return pos + 1;
    constexpr uint8_t kWord = kSpace | kLetter | kNumber;
    const size_t body = c == ' ' ? pos + 1 : pos;
    if (body >= n || !(s[body].cls & kWord)) {
        size_t e = body;
        while (e < n && !(s[e].cls & kWord))
            ++e;
        while (e < n && is_newline(s[e].cp))
            ++e;
        return e;
    }
    size_t run = 0, after_newline = 0;
    while (pos + run < n && (s[pos + run].cls & kSpace)) {
        if (is_newline(s[pos + run].cp))
            after_newline = pos + run + 1;
        ++run;
    }
    if (after_newline)
        return after_newline;
    if (run > 1 && pos + run < n)
        return pos + run - 1;  // the last blank goes with the word after it
    if (run)
        return pos + run;
    return pos + 1;
}

struct Pair {
    uint32_t rank, left, right, lsym, rsym, result;
    bool operator>(const Pair& o) const { return rank != o.rank ? rank > o.rank : left > o.left; }
};

uint64_t pair_key(uint32_t l, uint32_t r) { return (uint64_t)l << 32 | r; }

}  // namespace

struct BpeTokenizer::Scratch {
    int32_t* ids;
    uint32_t cap, count = 0;
    bool overflow = false;
    std::vector<Cp> cps;
    std::vector<uint32_t> sym, next, prev;
    std::vector<Pair> heap;

    void push(int32_t id) {
        if (count < cap)
            ids[count++] = id;
        else
            overflow = true;
    }
};

TokStatus BpeTokenizer::build(const GgufFile& g, std::string* why) {
    std::vector<std::string_view> toks, merge_lines;
    if (!g.get_str_array("tokenizer.ggml.tokens", &toks) || toks.empty()) {
        *why = "tokenizer has no vocabulary";
        return TokStatus::kFormat;
    }
    if (toks.size() > 0xffffffffull) {
        *why = "tokenizer vocabulary is too large";
        return TokStatus::kRange;
    }
    std::vector<uint32_t> types;
    if (g.has("tokenizer.ggml.token_type") && !g.get_u32_array("tokenizer.ggml.token_type", &types)) {
        *why = "tokenizer.ggml.token_type is not an int32/uint32 array";
        return TokStatus::kFormat;
    }
    if (g.has("tokenizer.ggml.merges") && !g.get_str_array("tokenizer.ggml.merges", &merge_lines)) {
        *why = "tokenizer.ggml.merges is not a string array";
        return TokStatus::kFormat;
    }
    n_tokens_ = (uint32_t)toks.size();
    auto type_of = [&](uint32_t i) { return i < types.size() ? types[i] : 1u; };

    vocab_off_.assign(n_tokens_ + 1, 0);
    size_t total = 0;
    for (uint32_t i = 0; i < n_tokens_; ++i)
        total += toks[i].size();
    vocab_.reserve(total);
    for (uint32_t i = 0; i < n_tokens_; ++i) {
        vocab_off_[i] = (uint32_t)vocab_.size();
        vocab_.append(toks[i]);
    }
    vocab_off_[n_tokens_] = (uint32_t)vocab_.size();
    if (total > 0xffffffffull) {
        *why = "tokenizer vocabulary is too large";
        return TokStatus::kRange;
    }
    auto text = [&](uint32_t i) {
        return std::string_view(vocab_.data() + vocab_off_[i], vocab_off_[i + 1] - vocab_off_[i]);
    };

    // Symbols: every token string, merge side and merge result, interned.
    std::unordered_map<std::string_view, uint32_t> index;
    std::deque<std::string> made;  // merge results that are no token (the views need a home)
    index.reserve(2 * (size_t)n_tokens_ + merge_lines.size());
    sym_token_.clear();
    auto intern = [&](std::string_view s) {
        auto it = index.find(s);
        if (it != index.end())
            return it->second;
        const uint32_t id = (uint32_t)sym_token_.size();
        sym_token_.push_back(-1);
        index.emplace(s, id);
        return id;
    };
    for (uint32_t i = 0; i < n_tokens_; ++i)
        sym_token_[intern(text(i))] = (int32_t)i;  // a later duplicate takes over the string
    merges_.clear();
    merges_.reserve(merge_lines.size());
    std::string joined;
    for (size_t i = 0; i < merge_lines.size(); ++i) {
        const std::string_view m = merge_lines[i];
        const size_t sp = m.size() > 1 ? m.find(' ', 1) : std::string_view::npos;
        if (sp == std::string_view::npos || sp + 1 >= m.size())
            continue;
        const std::string_view left = m.substr(0, sp), right = m.substr(sp + 1);
        const uint32_t l = intern(left), r = intern(right);
        if (merges_.count(pair_key(l, r)))
            continue;  // the first rank of a repeated pair stands
        joined.assign(left);
        joined.append(right);
        uint32_t res;
        auto it = index.find(joined);
        if (it != index.end()) {
            res = it->second;
        } else {
            made.push_back(joined);
            res = intern(made.back());
        }
        merges_.emplace(pair_key(l, r), Merge{(uint32_t)i, res});
    }

    uint32_t byte_cp[256];
    byte_code_points(byte_cp);
    int32_t cp_byte[324];
    std::fill(cp_byte, cp_byte + 324, -1);
    std::string enc;
    for (uint32_t b = 0; b < 256; ++b) {
        cp_byte[byte_cp[b]] = (int32_t)b;
        enc.clear();
        utf8_append(byte_cp[b], &enc);
        auto it = index.find(enc);
        if (it == index.end() || sym_token_[it->second] < 0) {
            *why = "vocabulary is missing a byte token";
            return TokStatus::kFormat;
        }
        byte_sym_[b] = it->second;
        byte_token_[b] = sym_token_[it->second];
    }

    // Pieces: control (3) and user-defined (4) tokens verbatim, the others
    // mapped back through the byte table; code points outside it, and bytes
    // that do not decode, are copied as they are.
    pieces_.clear();
    pieces_.reserve(total + n_tokens_);
    piece_off_.assign(n_tokens_ + 1, 0);
    for (uint32_t i = 0; i < n_tokens_; ++i) {
        piece_off_[i] = (uint32_t)pieces_.size();
        const std::string_view t = text(i);
        const uint32_t ty = type_of(i);
        if (ty == 3 || ty == 4) {
            pieces_.append(t);
        } else {
            const uint8_t* s = reinterpret_cast<const uint8_t*>(t.data());
            size_t p = 0;
            while (p < t.size()) {
                uint32_t cp = 0;
                const size_t k = utf8_next(s + p, t.size() - p, &cp);
                if (k && cp < 324 && cp_byte[cp] >= 0) {
                    pieces_.push_back((char)cp_byte[cp]);
                    p += k;
                } else {
                    const size_t raw = k ? k : 1;
                    pieces_.append(t.data() + p, raw);
                    p += raw;
                }
            }
        }
        pieces_.push_back('\0');
    }
    piece_off_[n_tokens_] = (uint32_t)pieces_.size();

    specials_.clear();
    empty_special_ = -1;
    for (auto& v : special_by_byte_)
        v.clear();
    for (uint32_t i = 0; i < n_tokens_; ++i) {
        const uint32_t ty = type_of(i);
        if (ty != 3 && ty != 4)
            continue;
        const uint32_t k = (uint32_t)specials_.size();
        specials_.push_back(Special{i, vocab_off_[i], vocab_off_[i + 1] - vocab_off_[i]});
        if (specials_[k].len == 0) {
            if (empty_special_ < 0)
                empty_special_ = (int32_t)k;
        } else {
            special_by_byte_[(uint8_t)vocab_[vocab_off_[i]]].push_back(k);
        }
    }
    for (auto& v : special_by_byte_)  // longest first; id order among equal lengths
        std::stable_sort(v.begin(), v.end(),
                         [&](uint32_t a, uint32_t b) { return specials_[a].len > specials_[b].len; });

    n_eog_ = 0;
    auto add_eog = [&](uint32_t id) {
        if (n_eog_ == 8)
            return;
        for (uint32_t j = 0; j < n_eog_; ++j)
            if (eog_[j] == id)
                return;
        eog_[n_eog_++] = id;
    };
    uint64_t eos = 0;
    if (g.get_u64("tokenizer.ggml.eos_token_id", &eos) && (uint32_t)eos < n_tokens_)
        add_eog((uint32_t)eos);
    for (uint32_t i = 0; i < n_tokens_; ++i)
        if (text(i) == "<|endoftext|>" || text(i) == "<|im_end|>")
            add_eog(i);
    class_table();  // expand the class table now rather than inside the first encode
    return TokStatus::kOk;
}

const BpeTokenizer::Special* BpeTokenizer::match_special(const uint8_t* text, size_t left) const {
    for (uint32_t k : special_by_byte_[text[0]]) {
        const Special& s = specials_[k];
        if (s.len <= left && std::memcmp(vocab_.data() + s.off, text, s.len) == 0)
            return &s;
    }
    return empty_special_ >= 0 ? &specials_[empty_special_] : nullptr;
}

void BpeTokenizer::encode_chunk(const uint8_t* bytes, size_t n, Scratch& w) const {
    if (n == 1) {
        w.push(byte_token_[bytes[0]]);
        return;
    }
    std::vector<uint32_t>& sym = w.sym;
    std::vector<uint32_t>& next = w.next;
    std::vector<uint32_t>& prev = w.prev;
    sym.resize(n);
    next.resize(n);
    prev.resize(n);
    for (size_t i = 0; i < n; ++i) {
        sym[i] = byte_sym_[bytes[i]];
        next[i] = (uint32_t)(i + 1);
        prev[i] = (uint32_t)i - 1;  // kDead for the first node
    }
    std::vector<Pair>& heap = w.heap;
    heap.clear();
    const auto later = std::greater<Pair>();
    auto consider = [&](uint32_t l) {
        const uint32_t r = next[l];
        if (r >= n)
            return;
        auto it = merges_.find(pair_key(sym[l], sym[r]));
        if (it == merges_.end())
            return;
        heap.push_back(Pair{it->second.rank, l, r, sym[l], sym[r], it->second.result});
        std::push_heap(heap.begin(), heap.end(), later);
    };
    for (uint32_t i = 0; i + 1 < n; ++i)
        consider(i);
    while (!heap.empty()) {
        std::pop_heap(heap.begin(), heap.end(), later);
        const Pair p = heap.back();
        heap.pop_back();
        // stale when either side has changed since the pair was seen
        if (sym[p.left] != p.lsym || next[p.left] != p.right || sym[p.right] != p.rsym)
            continue;
        sym[p.left] = p.result;
        sym[p.right] = kDead;
        next[p.left] = next[p.right];
        if (next[p.left] < n)
            prev[next[p.left]] = p.left;
        if (prev[p.left] != kDead)
            consider(prev[p.left]);
        consider(p.left);
    }
    for (uint32_t i = 0; i < n && !w.overflow; i = next[i]) {
        const int32_t tok = sym_token_[sym[i]];
        if (tok >= 0) {
            w.push(tok);
        } else {
            for (uint32_t b = i; b < next[i]; ++b)
                w.push(byte_token_[bytes[b]]);
        }
    }
}

bool BpeTokenizer::encode_segment(const uint8_t* text, size_t len, Scratch& w) const {
    if (!len)
        return true;
    const uint8_t* cls = class_table();
    w.cps.clear();
    for (size_t off = 0; off < len;) {
        uint32_t cp = 0;
        const size_t k = utf8_next(text + off, len - off, &cp);
        if (!k)
            return false;
        w.cps.push_back(Cp{cp, cls[cp], off});
        off += k;
    }
    const size_t n = w.cps.size();
    for (size_t pos = 0; pos < n;) {
        const size_t end = chunk_end(w.cps.data(), n, pos);
        const size_t b0 = w.cps[pos].off, b1 = end < n ? w.cps[end].off : len;
        encode_chunk(text + b0, b1 - b0, w);
        if (w.overflow)
            return false;
        pos = end;
    }
    return true;
}

TokStatus BpeTokenizer::encode(const char* text, size_t len, bool parse_special, int32_t* ids, uint32_t capacity,
                               uint32_t* count) const {
    Scratch w;
    w.ids = ids;
    w.cap = capacity;
    const uint8_t* t = reinterpret_cast<const uint8_t*>(text);
    bool ok = true;
    if (!parse_special) {
        ok = encode_segment(t, len, w);
    } else {
        size_t seg = 0, pos = 0;
        while (pos < len) {
            const Special* sp = match_special(t + pos, len - pos);
            if (!sp) {
                ++pos;
                continue;
            }
            if (pos > seg && !encode_segment(t + seg, pos - seg, w)) {
                ok = false;
                break;
            }
            w.push((int32_t)sp->id);
            if (w.overflow) {
                ok = false;
                break;
            }
            pos += sp->len;
            seg = pos;
        }
        if (ok && len > seg)
            ok = encode_segment(t + seg, len - seg, w);
    }
    *count = w.count;
    if (ok && !w.overflow)
        return TokStatus::kOk;
    return w.overflow ? TokStatus::kRange : TokStatus::kInvalid;
}

TokStatus BpeTokenizer::piece(int32_t id, const char** bytes, size_t* len) const {
    if (id < 0 || (uint32_t)id >= n_tokens_)
        return TokStatus::kRange;
    *bytes = pieces_.data() + piece_off_[id];
    *len = piece_off_[id + 1] - piece_off_[id] - 1;
    return TokStatus::kOk;
}

bool BpeTokenizer::is_eog(int32_t id) const {
    if (id < 0 || (uint32_t)id >= n_tokens_)
        return false;
    for (uint32_t j = 0; j < n_eog_; ++j)
        if (eog_[j] == (uint32_t)id)
            return true;
    return false;
}

}  // namespace bnn
