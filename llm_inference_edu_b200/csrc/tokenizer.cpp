// The Qwen2 tokenizer and chat template (src/tokenizer.rs), host code.
//
// The reference wraps HF `tokenizers` 0.21.4 (Cargo.toml, not vendored)
// loaded from the checkpoint's tokenizer.json.  This file restates the
// pipeline that file configures for Qwen2, from the library's published
// behaviour:
//   added tokens  split out of the raw text first (leftmost, then longest;
//                 Qwen2's are all unnormalized and unstripped);
//   normalizer    NFC;
//   pre-tokenizer the Qwen2 split pattern (Isolated), then ByteLevel
//                 (no prefix space, no regex): each piece's UTF-8 bytes as
//                 the GPT-2 byte alphabet;
//   model         BPE: the piece's symbols merged pair by pair, lowest merge
//                 rank first (leftmost among equals; a heap of candidate
//                 pairs), then looked up;
//   decoder       ByteLevel: tokens back to bytes, then lossy UTF-8;
//   stream        step_decode_stream: text is emitted only when the decoded
//                 suffix no longer ends in U+FFFD.
// Unicode classes and NFC data come from unicode_tables.inc
// (gen_unicode_tables.py).
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <memory>
#include <mutex>
#include <queue>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/qwen_b200.h"
#include "common.cuh"
#include "json.h"

namespace qb {
namespace {

#include "unicode_tables.inc"

// ------------------------------------------------------------- Unicode ----

template <size_t N>
bool in_ranges(const uint32_t (&r)[N][2], uint32_t c) {
    size_t lo = 0, hi = N;
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (c < r[mid][0]) hi = mid;
        else if (c > r[mid][1]) lo = mid + 1;
        else return true;
    }
    return false;
}

bool is_letter(uint32_t c) { return in_ranges(kLetterRanges, c); }
bool is_number(uint32_t c) { return in_ranges(kNumberRanges, c); }
bool is_space(uint32_t c) { return std::binary_search(std::begin(kWhiteSpace), std::end(kWhiteSpace), c); }

uint32_t ccc(uint32_t c) {
    size_t lo = 0, hi = sizeof(kCombiningClass) / sizeof(kCombiningClass[0]);
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (c < kCombiningClass[mid][0]) hi = mid;
        else if (c > kCombiningClass[mid][0]) lo = mid + 1;
        else return kCombiningClass[mid][1];
    }
    return 0;
}

constexpr uint32_t SBase = 0xAC00, LBase = 0x1100, VBase = 0x1161, TBase = 0x11A7;
constexpr uint32_t LCount = 19, VCount = 21, TCount = 28, NCount = VCount * TCount, SCount = LCount * NCount;

void decompose(uint32_t c, std::vector<uint32_t> &out) {
    if (c >= SBase && c < SBase + SCount) {
        const uint32_t s = c - SBase;
        out.push_back(LBase + s / NCount);
        out.push_back(VBase + (s % NCount) / TCount);
        if (s % TCount) out.push_back(TBase + s % TCount);
        return;
    }
    size_t lo = 0, hi = sizeof(kDecompIndex) / sizeof(kDecompIndex[0]);
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (c < kDecompIndex[mid][0]) hi = mid;
        else if (c > kDecompIndex[mid][0]) lo = mid + 1;
        else {
            out.insert(out.end(), kDecompData + kDecompIndex[mid][1],
                       kDecompData + kDecompIndex[mid][1] + kDecompIndex[mid][2]);
            return;
        }
    }
    out.push_back(c);
}

// The primary composite of (a, b), or 0.
uint32_t compose(uint32_t a, uint32_t b) {
    if (a >= LBase && a < LBase + LCount && b >= VBase && b < VBase + VCount)
        return SBase + ((a - LBase) * VCount + (b - VBase)) * TCount;
    if (a >= SBase && a < SBase + SCount && (a - SBase) % TCount == 0 && b > TBase && b < TBase + TCount)
        return a + (b - TBase);
    size_t lo = 0, hi = sizeof(kCompositions) / sizeof(kCompositions[0]);
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        const uint32_t *e = kCompositions[mid];
        if (a < e[0] || (a == e[0] && b < e[1])) hi = mid;
        else if (a > e[0] || (a == e[0] && b > e[1])) lo = mid + 1;
        else return e[2];
    }
    return 0;
}

// NFC (UAX #15): full canonical decomposition, canonical ordering, then
// canonical composition of every unblocked pair.
std::vector<uint32_t> nfc(const std::vector<uint32_t> &in) {
    bool plain = true;
    for (uint32_t c : in) plain = plain && c < 0x300;
    if (plain) return in;  // no decompositions and no combining marks below U+0300
    std::vector<uint32_t> d;
    d.reserve(in.size() + 8);
    for (uint32_t c : in) decompose(c, d);
    // Canonical ordering: each run of non-starters stably sorted by class.
    for (size_t i = 0; i < d.size();) {
        if (ccc(d[i]) == 0) {
            ++i;
            continue;
        }
        size_t j = i;
        while (j < d.size() && ccc(d[j]) != 0) ++j;
        if (j - i > 1)
            std::stable_sort(d.begin() + (long)i, d.begin() + (long)j,
                             [](uint32_t a, uint32_t b) { return ccc(a) < ccc(b); });
        i = j;
    }
    std::vector<uint32_t> out;
    out.reserve(d.size());
    long starter = -1;
    uint32_t last_cc = 0;
    for (uint32_t c : d) {
        const uint32_t cc = ccc(c);
        if (starter >= 0) {
            const bool adjacent = out.size() - 1 == (size_t)starter;
            const bool blocked = !adjacent && (last_cc == 0 || last_cc >= cc);
            if (!blocked) {
                const uint32_t p = compose(out[(size_t)starter], c);
                if (p) {
                    out[(size_t)starter] = p;
                    continue;
                }
            }
        }
        if (cc == 0) starter = (long)out.size();
        out.push_back(c);
        last_cc = cc;
    }
    return out;
}

// UTF-8 (already validated) to code points, and back.
std::vector<uint32_t> utf8_decode(const std::string &s) {
    std::vector<uint32_t> out;
    out.reserve(s.size());
    for (size_t i = 0; i < s.size();) {
        const uint8_t c = (uint8_t)s[i];
        int len = c < 0x80 ? 1 : c < 0xe0 ? 2 : c < 0xf0 ? 3 : 4;
        uint32_t cp = len == 1 ? c : len == 2 ? (c & 0x1f) : len == 3 ? (c & 0x0f) : (c & 0x07);
        for (int k = 1; k < len && i + (size_t)k < s.size(); ++k) cp = (cp << 6) | ((uint8_t)s[i + k] & 0x3f);
        out.push_back(cp);
        i += (size_t)len;
    }
    return out;
}

void utf8_append(std::string &s, uint32_t c) {
    if (c < 0x80) s += (char)c;
    else if (c < 0x800) { s += (char)(0xc0 | (c >> 6)); s += (char)(0x80 | (c & 0x3f)); }
    else if (c < 0x10000) {
        s += (char)(0xe0 | (c >> 12)); s += (char)(0x80 | ((c >> 6) & 0x3f)); s += (char)(0x80 | (c & 0x3f));
    } else {
        s += (char)(0xf0 | (c >> 18)); s += (char)(0x80 | ((c >> 12) & 0x3f));
        s += (char)(0x80 | ((c >> 6) & 0x3f)); s += (char)(0x80 | (c & 0x3f));
    }
}

bool valid_utf8(const uint8_t *s, size_t n) {
    size_t i = 0;
    while (i < n) {
        const uint8_t c = s[i];
        if (c < 0x80) { ++i; continue; }
        int len;
        uint32_t cp;
        if ((c & 0xe0) == 0xc0) { len = 2; cp = c & 0x1f; }
        else if ((c & 0xf0) == 0xe0) { len = 3; cp = c & 0x0f; }
        else if ((c & 0xf8) == 0xf0) { len = 4; cp = c & 0x07; }
        else return false;
        if (i + (size_t)len > n) return false;
        for (int k = 1; k < len; ++k) {
            if ((s[i + k] & 0xc0) != 0x80) return false;
            cp = (cp << 6) | (s[i + k] & 0x3f);
        }
        if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) || cp > 0x10ffff ||
            (cp >= 0xd800 && cp <= 0xdfff))
            return false;
        i += (size_t)len;
    }
    return true;
}

// String::from_utf8_lossy: each maximal ill-formed subsequence becomes one
// U+FFFD.
std::string utf8_lossy(const std::string &b) {
    std::string out;
    const size_t n = b.size();
    size_t i = 0;
    while (i < n) {
        const uint8_t c = (uint8_t)b[i];
        if (c < 0x80) { out += (char)c; ++i; continue; }
        int need;
        uint8_t lo = 0x80, hi = 0xbf;
        if (c >= 0xc2 && c <= 0xdf) need = 1;
        else if (c >= 0xe0 && c <= 0xef) {
            need = 2;
            if (c == 0xe0) lo = 0xa0;
            if (c == 0xed) hi = 0x9f;
        } else if (c >= 0xf0 && c <= 0xf4) {
            need = 3;
            if (c == 0xf0) lo = 0x90;
            if (c == 0xf4) hi = 0x8f;
        } else {
            out += "\xef\xbf\xbd";
            ++i;
            continue;
        }
        size_t j = i + 1;
        int got = 0;
        while (got < need && j < n) {
            const uint8_t x = (uint8_t)b[j];
            const uint8_t l = got == 0 ? lo : 0x80, h = got == 0 ? hi : 0xbf;
            if (x < l || x > h) break;
            ++j;
            ++got;
        }
        if (got == need) out.append(b, i, j - i);
        else out += "\xef\xbf\xbd";
        i = j;
    }
    return out;
}

// ------------------------------------------------------- pre-tokenizer ----
// The Qwen2 split pattern
//   (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}
//   | ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+
// matched by hand, alternatives in order at each position as a
// backtracking engine tries them; the match's end is returned (0: none).

bool fold_is(uint32_t c, char lower) {
    if (lower == 's' && c == 0x17f) return true;  // LATIN SMALL LETTER LONG S folds to s
    return c == (uint32_t)lower || c == (uint32_t)(lower - 'a' + 'A');
}

size_t match_at(const std::vector<uint32_t> &s, size_t p) {
    const size_t n = s.size();
    const uint32_t c = s[p];
    auto nl = [](uint32_t x) { return x == '\r' || x == '\n'; };
    // 1. contractions
    if (c == '\'' && p + 1 < n) {
        const uint32_t a = s[p + 1];
        if (fold_is(a, 's') || fold_is(a, 't') || fold_is(a, 'm') || fold_is(a, 'd')) return p + 2;
        if (p + 2 < n) {
            const uint32_t b = s[p + 2];
            if ((fold_is(a, 'r') && fold_is(b, 'e')) || (fold_is(a, 'v') && fold_is(b, 'e')) ||
                (fold_is(a, 'l') && fold_is(b, 'l')))
                return p + 3;
        }
    }
    // 2. an optional non-letter, non-number, non-newline, then letters
    {
        size_t q = p;
        if (!nl(c) && !is_letter(c) && !is_number(c)) q = p + 1;
        if (q < n && is_letter(s[q])) {
            while (q < n && is_letter(s[q])) ++q;
            return q;
        }
        if (is_letter(c)) {  // the optional part empty
            q = p;
            while (q < n && is_letter(s[q])) ++q;
            return q;
        }
    }
    // 3. one number
    if (is_number(c)) return p + 1;
    // 4. an optional space, symbols, then newlines
    {
        auto sym = [&](uint32_t x) { return !is_space(x) && !is_letter(x) && !is_number(x); };
        size_t q = p;
        if (c == ' ' && p + 1 < n && sym(s[p + 1])) q = p + 1;
        if (q < n && sym(s[q])) {
            while (q < n && sym(s[q])) ++q;
            while (q < n && nl(s[q])) ++q;
            return q;
        }
    }
    if (!is_space(c)) return 0;
    size_t run = p;
    while (run < n && is_space(s[run])) ++run;
    // 5. whitespace up to and including the run's last newline
    for (size_t j = run; j > p; --j)
        if (nl(s[j - 1])) return j;
    // 6. whitespace not followed by a non-space (the run, less its last
    //    character unless the run ends the text)
    if (run == n) return run;
    if (run - p >= 2) return run - 1;
    // 7. whitespace
    return run;
}

// Isolated split: matches and the gaps between them are pieces.
std::vector<std::pair<size_t, size_t>> split_pieces(const std::vector<uint32_t> &s) {
    std::vector<std::pair<size_t, size_t>> out;
    size_t gap = 0, p = 0;
    while (p < s.size()) {
        const size_t e = match_at(s, p);
        if (e > p) {
            if (gap < p) out.emplace_back(gap, p);
            out.emplace_back(p, e);
            p = e;
            gap = p;
        } else {
            ++p;
        }
    }
    if (gap < s.size()) out.emplace_back(gap, s.size());
    return out;
}

// The GPT-2 byte alphabet: printable bytes stand for themselves, the others
// for 256 + their rank among them.
struct ByteAlphabet {
    uint32_t to_cp[256];
    std::unordered_map<uint32_t, uint8_t> to_byte;
    ByteAlphabet() {
        int n = 0;
        for (int b = 0; b < 256; ++b) {
            const bool keep = (b >= '!' && b <= '~') || (b >= 0xa1 && b <= 0xac) || (b >= 0xae && b <= 0xff);
            to_cp[b] = keep ? (uint32_t)b : (uint32_t)(256 + n++);
            to_byte[to_cp[b]] = (uint8_t)b;
        }
    }
};
const ByteAlphabet &alphabet() {
    static const ByteAlphabet a;
    return a;
}

// ----------------------------------------------------------- tokenizer ----

struct AddedTok {
    uint32_t id;
    std::string content;
    bool special;
};

struct Tokenizer {
    std::unordered_map<std::string, uint32_t> vocab;
    std::vector<std::string> id_to_tok;  // "" where no token
    std::vector<uint8_t> has_tok;
    std::unordered_map<uint64_t, std::pair<uint32_t, uint32_t>> merges;  // (a, b) -> (rank, merged id)
    std::vector<AddedTok> added;                                          // longest first
    std::unordered_map<uint32_t, size_t> added_by_id;
    bool nfc_norm = false, ignore_merges = false;
    std::vector<uint32_t> stop_tokens;  // the chat tokenizer's
    std::vector<uint32_t> special_ids;

    bool known(uint32_t id) const {
        return (id < has_tok.size() && has_tok[id]) || added_by_id.count(id) != 0;
    }
    void set_token(uint32_t id, const std::string &t) {
        if (id >= id_to_tok.size()) {
            id_to_tok.resize((size_t)id + 1);
            has_tok.resize((size_t)id + 1, 0);
        }
        id_to_tok[id] = t;
        has_tok[id] = 1;
    }

    // BPE of one byte-level piece (its characters in the byte alphabet).
    uint32_t bpe(const std::string &piece, std::vector<uint32_t> &ids) const {
        if (ignore_merges) {
            auto it = vocab.find(piece);
            if (it != vocab.end()) {
                ids.push_back(it->second);
                return QB_OK;
            }
        }
        std::vector<uint32_t> sym;
        const std::vector<uint32_t> cps = utf8_decode(piece);
        for (uint32_t c : cps) {
            std::string one;
            utf8_append(one, c);
            auto it = vocab.find(one);
            if (it == vocab.end()) return QB_TOKENIZER_ENCODING;  // no unknown token in this model
            sym.push_back(it->second);
        }
        // Merges in (rank, position) order through a min-heap of candidate
        // pairs over a linked list of symbols; an entry whose pair has
        // changed since it was pushed is skipped.  Positions are the left
        // symbols' original indices, so "lowest position" is "leftmost".
        const size_t n = sym.size();
        std::vector<long> prev(n), next(n);
        std::vector<uint8_t> alive(n, 1);
        for (size_t i = 0; i < n; ++i) {
            prev[i] = (long)i - 1;
            next[i] = i + 1 < n ? (long)i + 1 : -1;
        }
        struct Cand {
            uint32_t rank, new_id;
            size_t pos;
            bool operator>(const Cand &o) const { return rank != o.rank ? rank > o.rank : pos > o.pos; }
        };
        std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> q;
        auto push = [&](size_t i) {
            if (next[i] < 0) return;
            auto it = merges.find((uint64_t)sym[i] << 32 | sym[(size_t)next[i]]);
            if (it != merges.end()) q.push(Cand{it->second.first, it->second.second, i});
        };
        for (size_t i = 0; i + 1 < n; ++i) push(i);
        while (!q.empty()) {
            const Cand c = q.top();
            q.pop();
            if (!alive[c.pos] || next[c.pos] < 0) continue;
            const size_t r = (size_t)next[c.pos];
            auto it = merges.find((uint64_t)sym[c.pos] << 32 | sym[r]);
            if (it == merges.end() || it->second.second != c.new_id) continue;  // stale entry
            sym[c.pos] = c.new_id;
            alive[r] = 0;
            next[c.pos] = next[r];
            if (next[r] >= 0) prev[(size_t)next[r]] = (long)c.pos;
            if (prev[c.pos] >= 0) push((size_t)prev[c.pos]);
            push(c.pos);
        }
        for (size_t i = 0; i < n; ++i)
            if (alive[i]) ids.push_back(sym[i]);
        return QB_OK;
    }

    // Normalization, pre-tokenization and BPE of text without added tokens.
    uint32_t encode_plain(const std::string &text, std::vector<uint32_t> &ids) const {
        std::vector<uint32_t> cps = utf8_decode(text);
        if (nfc_norm) cps = nfc(cps);
        const ByteAlphabet &ab = alphabet();
        for (auto &pc : split_pieces(cps)) {
            std::string bytes;
            for (size_t i = pc.first; i < pc.second; ++i) utf8_append(bytes, cps[i]);
            std::string mapped;
            for (unsigned char b : bytes) utf8_append(mapped, ab.to_cp[b]);
            const uint32_t st = bpe(mapped, ids);
            if (st) return st;
        }
        return QB_OK;
    }

    // Tokenizer::encode(text, false): added tokens first (leftmost, longest).
    uint32_t encode(const std::string &text, std::vector<uint32_t> &ids) const {
        size_t seg = 0, p = 0;
        while (p < text.size()) {
            const AddedTok *hit = nullptr;
            for (const AddedTok &a : added)
                if (!a.content.empty() && text.compare(p, a.content.size(), a.content) == 0) {
                    hit = &a;
                    break;  // longest first
                }
            if (!hit) {
                ++p;
                continue;
            }
            if (seg < p) {
                const uint32_t st = encode_plain(text.substr(seg, p - seg), ids);
                if (st) return st;
            }
            ids.push_back(hit->id);
            p += hit->content.size();
            seg = p;
        }
        if (seg < text.size()) return encode_plain(text.substr(seg), ids);
        return QB_OK;
    }

    // Tokenizer::decode with the ByteLevel decoder.
    std::string decode(const std::vector<uint32_t> &ids, bool skip_special) const {
        const ByteAlphabet &ab = alphabet();
        std::string bytes;
        for (uint32_t id : ids) {
            auto ai = added_by_id.find(id);
            const std::string *tok;
            if (ai != added_by_id.end()) {
                if (skip_special && added[ai->second].special) continue;
                tok = &added[ai->second].content;
            } else {
                tok = &id_to_tok[id];
            }
            // Every character in the byte alphabet maps back to its byte; a
            // token with any other character is kept as its UTF-8.
            const std::vector<uint32_t> cps = utf8_decode(*tok);
            std::string b;
            bool all = true;
            for (uint32_t c : cps) {
                auto it = ab.to_byte.find(c);
                if (it == ab.to_byte.end()) {
                    all = false;
                    break;
                }
                b += (char)it->second;
            }
            bytes += all ? b : *tok;
        }
        return utf8_lossy(bytes);
    }
};

// Tokenizer::from_bytes for the Qwen2 configuration: a BPE model with the
// byte-level pre-tokenizer and decoder, optional NFC.  Anything else is
// QB_TOKENIZER_UNSUPPORTED_ASSETS; malformed JSON QB_TOKENIZER_JSON.
uint32_t load_tokenizer_json(const uint8_t *data, size_t len, Tokenizer &t) {
    JVal root;
    if (!parse_json((const char *)data, len, root) || root.t != JVal::OBJ) return QB_TOKENIZER_JSON;
    const JVal *model = root.get("model");
    if (!model || model->t != JVal::OBJ) return QB_TOKENIZER_JSON;
    const JVal *type = model->get("type");
    if (type && (type->t != JVal::STR || type->s != "BPE")) return QB_TOKENIZER_UNSUPPORTED_ASSETS;
    auto flag = [](const JVal *v) { return v && v->t == JVal::BOOL && v->b; };
    auto nonempty_str = [](const JVal *v) { return v && v->t == JVal::STR && !v->s.empty(); };
    if (flag(model->get("byte_fallback")) || nonempty_str(model->get("continuing_subword_prefix")) ||
        nonempty_str(model->get("end_of_word_suffix")))
        return QB_TOKENIZER_UNSUPPORTED_ASSETS;
    if (const JVal *d = model->get("dropout"))
        if (d->t != JVal::NUL) return QB_TOKENIZER_UNSUPPORTED_ASSETS;
    t.ignore_merges = flag(model->get("ignore_merges"));
    const JVal *vocab = model->get("vocab"), *merges = model->get("merges");
    if (!vocab || vocab->t != JVal::OBJ || !merges || merges->t != JVal::ARR) return QB_TOKENIZER_JSON;
    t.vocab.reserve(vocab->o.size() * 2);
    for (auto &kv : vocab->o) {
        if (kv.second.t != JVal::NUM || !kv.second.integer) return QB_TOKENIZER_JSON;
        const unsigned long long id = strtoull(kv.second.s.c_str(), nullptr, 10);
        if (id > 0xfffffffeull) return QB_TOKENIZER_JSON;
        t.vocab[kv.first] = (uint32_t)id;
        t.set_token((uint32_t)id, kv.first);
    }
    uint32_t rank = 0;
    for (auto &m : merges->a) {
        std::string a, b;
        if (m.t == JVal::STR) {
            const size_t sp = m.s.find(' ');
            if (sp == std::string::npos) return QB_TOKENIZER_JSON;
            a = m.s.substr(0, sp);
            b = m.s.substr(sp + 1);
        } else if (m.t == JVal::ARR && m.a.size() == 2 && m.a[0].t == JVal::STR && m.a[1].t == JVal::STR) {
            a = m.a[0].s;
            b = m.a[1].s;
        } else {
            return QB_TOKENIZER_JSON;
        }
        auto ia = t.vocab.find(a), ib = t.vocab.find(b), im = t.vocab.find(a + b);
        if (ia == t.vocab.end() || ib == t.vocab.end() || im == t.vocab.end()) return QB_TOKENIZER_JSON;
        t.merges.emplace((uint64_t)ia->second << 32 | ib->second, std::make_pair(rank++, im->second));
    }
    // Normalizer: none or NFC.
    if (const JVal *nz = root.get("normalizer")) {
        if (nz->t == JVal::OBJ) {
            const JVal *ty = nz->get("type");
            if (!ty || ty->t != JVal::STR || ty->s != "NFC") return QB_TOKENIZER_UNSUPPORTED_ASSETS;
            t.nfc_norm = true;
        } else if (nz->t != JVal::NUL) {
            return QB_TOKENIZER_UNSUPPORTED_ASSETS;
        }
    }
    // Pre-tokenizer: the Qwen2 split (Isolated) then ByteLevel without a
    // prefix space or its own regex.
    {
        const JVal *pt = root.get("pre_tokenizer");
        const JVal *seq = pt && pt->t == JVal::OBJ ? pt->get("pretokenizers") : nullptr;
        if (!seq || seq->t != JVal::ARR || seq->a.size() != 2) return QB_TOKENIZER_UNSUPPORTED_ASSETS;
        const JVal &sp = seq->a[0], &bl = seq->a[1];
        const JVal *pat = sp.t == JVal::OBJ ? sp.get("pattern") : nullptr;
        const JVal *rx = pat && pat->t == JVal::OBJ ? pat->get("Regex") : nullptr;
        static const char *kPattern =
            "(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}| ?[^\\s\\p{L}\\p{N}]+[\\r\\n]*|"
            "\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+";
        const JVal *beh = sp.t == JVal::OBJ ? sp.get("behavior") : nullptr;
        const JVal *bt = bl.t == JVal::OBJ ? bl.get("type") : nullptr;
        if (!rx || rx->t != JVal::STR || rx->s != kPattern || !beh || beh->t != JVal::STR ||
            beh->s != "Isolated" || flag(sp.get("invert")) || !bt || bt->t != JVal::STR || bt->s != "ByteLevel" ||
            flag(bl.get("add_prefix_space")) || flag(bl.get("use_regex")))
            return QB_TOKENIZER_UNSUPPORTED_ASSETS;
    }
    if (const JVal *dec = root.get("decoder")) {
        const JVal *ty = dec->t == JVal::OBJ ? dec->get("type") : nullptr;
        if (!ty || ty->t != JVal::STR || ty->s != "ByteLevel") return QB_TOKENIZER_UNSUPPORTED_ASSETS;
    } else {
        return QB_TOKENIZER_UNSUPPORTED_ASSETS;
    }
    // Added tokens: whole-content matches on the raw text.  As the library
    // re-adds them when it reads the file, a token's id is its vocabulary id
    // when the model has its content, else the next id past the vocabulary
    // and the earlier added tokens (the ids written in the file are not
    // used; the Qwen2 file's agree with this rule).
    if (const JVal *at = root.get("added_tokens")) {
        if (at->t != JVal::ARR) return QB_TOKENIZER_JSON;
        uint64_t next = t.vocab.size();
        for (auto &a : at->a) {
            const JVal *content = a.get("content");
            if (a.t != JVal::OBJ || !content || content->t != JVal::STR) return QB_TOKENIZER_JSON;
            if (flag(a.get("lstrip")) || flag(a.get("rstrip")) || flag(a.get("single_word")) ||
                flag(a.get("normalized")))
                return QB_TOKENIZER_UNSUPPORTED_ASSETS;
            uint32_t idv;
            auto in_vocab = t.vocab.find(content->s);
            if (in_vocab != t.vocab.end()) {
                idv = in_vocab->second;
            } else {
                for (auto &x : t.added) next = std::max<uint64_t>(next, (uint64_t)x.id + 1);
                if (next > 0xfffffffeull) return QB_TOKENIZER_JSON;
                idv = (uint32_t)next++;
            }
            AddedTok tok{idv, content->s, flag(a.get("special"))};
            t.added.push_back(tok);
            if (tok.special) t.special_ids.push_back(tok.id);
        }
        std::stable_sort(t.added.begin(), t.added.end(),
                         [](const AddedTok &x, const AddedTok &y) { return x.content.size() > y.content.size(); });
        for (size_t i = 0; i < t.added.size(); ++i) t.added_by_id[t.added[i].id] = i;
    }
    return QB_OK;
}

// step_decode_stream (tokenizers 0.21): the stream's ids since the last
// emitted prefix, the decoded prefix and its index.
struct Stream {
    std::shared_ptr<Tokenizer> tok;
    std::vector<uint32_t> ids;
    std::string prefix;
    size_t prefix_index = 0;
    bool valid = true;
};

std::mutex g_tok_mu;
uint64_t g_tok_next = 1;
std::map<uint64_t, std::shared_ptr<Tokenizer>> g_toks;
std::map<uint64_t, std::shared_ptr<Stream>> g_streams;

std::shared_ptr<Tokenizer> find_tok(uint64_t h) {
    std::lock_guard<std::mutex> lk(g_tok_mu);
    auto it = g_toks.find(h);
    return it == g_toks.end() ? nullptr : it->second;
}

uint32_t copy_out(const std::string &s, char *out, size_t cap, size_t *len) {
    if (len) *len = s.size();
    if ((!out && !s.empty()) || cap < s.size()) return QB_INVALID_OUTPUT_LENGTH;
    if (!s.empty()) memcpy(out, s.data(), s.size());
    return QB_OK;
}

uint32_t register_tok(std::shared_ptr<Tokenizer> t, uint64_t *out) {
    std::lock_guard<std::mutex> lk(g_tok_mu);
    const uint64_t id = g_tok_next++;
    g_toks[id] = std::move(t);
    *out = id;
    return QB_OK;
}

}  // namespace
}  // namespace qb

using namespace qb;

extern "C" {

uint32_t qb_tokenizer_from_json(const uint8_t *json, size_t len, uint64_t *out) {
    if (!out || (len && !json)) return QB_INVALID_PARAMETERS;
    auto t = std::make_shared<Tokenizer>();
    const uint32_t st = load_tokenizer_json(json, len, *t);
    if (st) return st;
    return register_tok(std::move(t), out);
}

uint32_t qb_tokenizer_load_chat(const uint8_t *tokenizer_json, size_t tokenizer_len, const uint8_t *config_json,
                                size_t config_len, const uint8_t *generation_json, size_t generation_len,
                                uint64_t *out) {
    if (!out || !tokenizer_json || !config_json || !generation_json) return QB_INVALID_PARAMETERS;
    // ChatTokenizer::load, src/tokenizer.rs:68-124: the tokenizer_config.json
    // checks, then generation_config.json's stop ids, then the file itself
    // and its three special ids.
    JVal cfg, gen;
    if (!parse_json((const char *)config_json, config_len, cfg)) return QB_TOKENIZER_JSON;
    const JVal *cls = cfg.get("tokenizer_class"), *bos_add = cfg.get("add_bos_token"), *bos = cfg.get("bos_token"),
               *eos = cfg.get("eos_token");
    if (cfg.t != JVal::OBJ || !cls || cls->t != JVal::STR || cls->s != "Qwen2Tokenizer" || !bos_add ||
        bos_add->t != JVal::BOOL || bos_add->b || (bos && bos->t != JVal::NUL) || !eos || eos->t != JVal::STR ||
        eos->s != "<|im_end|>")
        return QB_TOKENIZER_UNSUPPORTED_ASSETS;
    if (!parse_json((const char *)generation_json, generation_len, gen)) return QB_TOKENIZER_JSON;
    const JVal *eid = gen.t == JVal::OBJ ? gen.get("eos_token_id") : nullptr;
    if (!eid || eid->t != JVal::ARR) return QB_TOKENIZER_UNSUPPORTED_ASSETS;
    std::vector<uint32_t> stops;
    for (auto &v : eid->a) {
        if (v.t != JVal::NUM || !v.integer) return QB_TOKENIZER_UNSUPPORTED_ASSETS;
        stops.push_back((uint32_t)strtoull(v.s.c_str(), nullptr, 10));
    }
    if (stops != std::vector<uint32_t>{151645, 151643}) return QB_TOKENIZER_UNSUPPORTED_ASSETS;
    auto t = std::make_shared<Tokenizer>();
    const uint32_t st = load_tokenizer_json(tokenizer_json, tokenizer_len, *t);
    if (st) return st;
    const struct { const char *text; uint32_t id; } req[] = {
        {"<|im_start|>", 151644}, {"<|im_end|>", 151645}, {"<|endoftext|>", 151643}};
    for (auto &r : req) {
        bool found = false;
        for (auto &a : t->added) found = found || (a.content == r.text && a.id == r.id);
        if (!found) return QB_TOKENIZER_UNSUPPORTED_ASSETS;
    }
    t->stop_tokens = stops;
    return register_tok(std::move(t), out);
}

uint32_t qb_tokenizer_encode(uint64_t h, const uint8_t *text, size_t len, uint32_t *ids, size_t cap,
                             size_t *count) {
    auto t = find_tok(h);
    if (!t) return QB_INVALID_HANDLE;
    if (len && !text) return QB_INVALID_PARAMETERS;
    if (len && !valid_utf8(text, len)) return QB_TOKENIZER_ENCODING;
    std::vector<uint32_t> out;
    const uint32_t st = t->encode(len ? std::string((const char *)text, len) : std::string(), out);
    if (st) return st;
    if (count) *count = out.size();
    if (out.size() > cap || (!ids && !out.empty())) return QB_INVALID_OUTPUT_LENGTH;
    if (!out.empty()) memcpy(ids, out.data(), out.size() * 4);
    return QB_OK;
}

uint32_t qb_tokenizer_decode(uint64_t h, const uint32_t *ids, size_t count, int32_t skip_special, char *out,
                             size_t cap, size_t *len) {
    auto t = find_tok(h);
    if (!t) return QB_INVALID_HANDLE;
    if (count && !ids) return QB_INVALID_PARAMETERS;
    std::vector<uint32_t> v(ids, ids + count);
    for (size_t i = 0; i < count; ++i)
        if (!t->known(v[i])) {
            set_detail(0, 0, v[i]);
            return QB_TOKENIZER_INVALID_TOKEN;
        }
    return copy_out(t->decode(v, skip_special != 0), out, cap, len);
}

uint32_t qb_tokenizer_stop_tokens(uint64_t h, uint32_t *ids, size_t cap, size_t *count) {
    auto t = find_tok(h);
    if (!t) return QB_INVALID_HANDLE;
    if (count) *count = t->stop_tokens.size();
    if (t->stop_tokens.size() > cap || (!ids && !t->stop_tokens.empty())) return QB_INVALID_OUTPUT_LENGTH;
    if (!t->stop_tokens.empty()) memcpy(ids, t->stop_tokens.data(), t->stop_tokens.size() * 4);
    return QB_OK;
}

uint32_t qb_tokenizer_free(uint64_t h) {
    std::lock_guard<std::mutex> lk(g_tok_mu);
    return g_toks.erase(h) ? QB_OK : QB_INVALID_HANDLE;
}

uint32_t qb_tokenizer_stream_create(uint64_t h, uint64_t *out) {
    auto t = find_tok(h);
    if (!t) return QB_INVALID_HANDLE;
    if (!out) return QB_INVALID_PARAMETERS;
    auto s = std::make_shared<Stream>();
    s->tok = t;
    std::lock_guard<std::mutex> lk(g_tok_mu);
    const uint64_t id = g_tok_next++;
    g_streams[id] = s;
    *out = id;
    return QB_OK;
}

uint32_t qb_tokenizer_stream_push(uint64_t stream, uint32_t id, char *out, size_t cap, size_t *len,
                                  int32_t *has_text) {
    std::shared_ptr<Stream> s;
    {
        std::lock_guard<std::mutex> lk(g_tok_mu);
        auto it = g_streams.find(stream);
        if (it == g_streams.end()) return QB_INVALID_HANDLE;
        s = it->second;
    }
    if (has_text) *has_text = 0;
    if (len) *len = 0;
    // TextStream::push, src/tokenizer.rs:181-207.
    if (!s->valid) return QB_TOKENIZER_INVALID_STREAM;
    const Tokenizer &t = *s->tok;
    if (!t.known(id)) {
        set_detail(0, 0, id);
        return QB_TOKENIZER_INVALID_TOKEN;
    }
    if (std::find(t.special_ids.begin(), t.special_ids.end(), id) != t.special_ids.end()) return QB_OK;
    s->ids.push_back(id);
    const std::string text = t.decode(s->ids, true);
    const bool replacement = text.size() >= 3 && text.compare(text.size() - 3, 3, "\xef\xbf\xbd") == 0;
    if (text.size() > s->prefix.size() && !replacement) {
        if (text.compare(0, s->prefix.size(), s->prefix) != 0) {
            s->valid = false;
            return QB_TOKENIZER_ENCODING;
        }
        const std::string fresh = text.substr(s->prefix.size());
        if (!out || cap < fresh.size()) {
            s->ids.pop_back();  // nothing consumed: the caller may retry with room
            if (len) *len = fresh.size();
            return QB_INVALID_OUTPUT_LENGTH;
        }
        const size_t new_index = s->ids.size() - s->prefix_index;
        s->ids.erase(s->ids.begin(), s->ids.begin() + (long)s->prefix_index);
        s->prefix = t.decode(s->ids, true);
        s->prefix_index = new_index;
        memcpy(out, fresh.data(), fresh.size());
        if (len) *len = fresh.size();
        if (has_text) *has_text = 1;
    }
    return QB_OK;
}

uint32_t qb_tokenizer_stream_pending(uint64_t stream, size_t *pending) {
    std::lock_guard<std::mutex> lk(g_tok_mu);
    auto it = g_streams.find(stream);
    if (it == g_streams.end()) return QB_INVALID_HANDLE;
    const Stream &s = *it->second;
    if (pending) *pending = s.ids.size() > s.prefix_index ? s.ids.size() - s.prefix_index : 0;
    return QB_OK;
}

uint32_t qb_tokenizer_stream_free(uint64_t stream) {
    std::lock_guard<std::mutex> lk(g_tok_mu);
    return g_streams.erase(stream) ? QB_OK : QB_INVALID_HANDLE;
}

// render_chat, src/tokenizer.rs:40-63.
uint32_t qb_render_chat(const uint32_t *roles, const uint8_t *const *contents, const size_t *lengths, size_t count,
                        int32_t generation_prompt, char *out, size_t cap, size_t *len) {
    if (count == 0) return QB_TOKENIZER_EMPTY_MESSAGES;
    if (!roles || !contents || !lengths) return QB_INVALID_PARAMETERS;
    static const char *kRole[] = {"system", "user", "assistant"};
    std::string text;
    if (roles[0] != QB_ROLE_SYSTEM)
        text += "<|im_start|>system\nYou are Qwen, created by Alibaba Cloud. You are a helpful assistant.<|im_end|>\n";
    for (size_t i = 0; i < count; ++i) {
        if (roles[i] > QB_ROLE_ASSISTANT || (lengths[i] && !contents[i])) return QB_INVALID_PARAMETERS;
        if (lengths[i] && !valid_utf8(contents[i], lengths[i])) return QB_TOKENIZER_ENCODING;
        text += "<|im_start|>";
        text += kRole[roles[i]];
        text += '\n';
        if (lengths[i]) text.append((const char *)contents[i], lengths[i]);
        text += "<|im_end|>\n";
    }
    if (generation_prompt) text += "<|im_start|>assistant\n";
    return copy_out(text, out, cap, len);
}

}  // extern "C"
