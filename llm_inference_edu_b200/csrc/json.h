// A small JSON value reader (objects, arrays, strings, numbers, literals)
// for the host-side loaders: the tiny model file, config.json and the
// tokenizer files.  Duplicate object keys and trailing content are errors.
#pragma once
#include <stdlib.h>
#include <string.h>

#include <string>
#include <unordered_set>
#include <utility>
#include <vector>

namespace qb {

struct JVal {
    enum Type { NUL, BOOL, NUM, STR, ARR, OBJ } t = NUL;
    bool b = false;
    double n = 0.0;
    bool integer = false;  // a number written without fraction, exponent or sign
    std::string s;
    std::vector<JVal> a;
    std::vector<std::pair<std::string, JVal>> o;
    const JVal *get(const char *k) const {
        for (auto &kv : o)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JParse {
    const char *p, *e;
    int depth = 0;
    void ws() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
    bool lit(const char *w) {
        const size_t n = strlen(w);
        if ((size_t)(e - p) < n || memcmp(p, w, n) != 0) return false;
        p += n;
        return true;
    }
    bool str(std::string &out) {
        if (p >= e || *p != '"') return false;
        ++p;
        out.clear();
        while (p < e && *p != '"') {
            const char c = *p++;
            if ((unsigned char)c < 0x20) return false;
            if (c != '\\') { out += c; continue; }
            if (p >= e) return false;
            const char x = *p++;
            switch (x) {
            case '"': out += '"'; break;
            case '\\': out += '\\'; break;
            case '/': out += '/'; break;
            case 'b': out += '\b'; break;
            case 'f': out += '\f'; break;
            case 'n': out += '\n'; break;
            case 'r': out += '\r'; break;
            case 't': out += '\t'; break;
            case 'u': {
                if (e - p < 4) return false;
                unsigned v = 0;
                for (int i = 0; i < 4; ++i) {
                    const char h = *p++;
                    v <<= 4;
                    if (h >= '0' && h <= '9') v |= (unsigned)(h - '0');
                    else if (h >= 'a' && h <= 'f') v |= (unsigned)(h - 'a' + 10);
                    else if (h >= 'A' && h <= 'F') v |= (unsigned)(h - 'A' + 10);
                    else return false;
                }
                if (v < 0x80) out += (char)v;
                else if (v < 0x800) { out += (char)(0xc0 | (v >> 6)); out += (char)(0x80 | (v & 0x3f)); }
                else { out += (char)(0xe0 | (v >> 12)); out += (char)(0x80 | ((v >> 6) & 0x3f));
                       out += (char)(0x80 | (v & 0x3f)); }
                break;
            }
            default: return false;
            }
        }
        if (p >= e) return false;
        ++p;
        return true;
    }
    bool num(JVal &v) {
        const char *s = p;
        bool frac = false;
        if (p < e && *p == '-') ++p;
        if (p >= e || *p < '0' || *p > '9') return false;
        if (*p == '0') ++p;
        else while (p < e && *p >= '0' && *p <= '9') ++p;
        if (p < e && *p == '.') {
            frac = true;
            ++p;
            if (p >= e || *p < '0' || *p > '9') return false;
            while (p < e && *p >= '0' && *p <= '9') ++p;
        }
        if (p < e && (*p == 'e' || *p == 'E')) {
            frac = true;
            ++p;
            if (p < e && (*p == '+' || *p == '-')) ++p;
            if (p >= e || *p < '0' || *p > '9') return false;
            while (p < e && *p >= '0' && *p <= '9') ++p;
        }
        const std::string tok(s, p);
        v.t = JVal::NUM;
        v.n = strtod(tok.c_str(), nullptr);
        v.integer = !frac && tok[0] != '-';
        if (v.integer) v.s = tok;  // exact digits for integer fields
        return true;
    }
    bool value(JVal &v) {
        ws();
        if (p >= e || ++depth > 64) return false;
        bool ok = true;
        if (*p == '{') {
            ++p;
            v.t = JVal::OBJ;
            std::unordered_set<std::string> seen;
            ws();
            if (p < e && *p == '}') {
                ++p;
            } else {
                for (;;) {
                    ws();
                    std::string k;
                    if (!str(k)) { ok = false; break; }
                    ws();
                    if (p >= e || *p++ != ':') { ok = false; break; }
                    // duplicate field (a hash set once the object is large)
                    if (v.o.size() < 16) {
                        for (auto &kv : v.o)
                            if (kv.first == k) ok = false;
                    } else {
                        if (seen.empty())
                            for (auto &kv : v.o) seen.insert(kv.first);
                        ok = seen.insert(k).second;
                    }
                    if (!ok) break;
                    v.o.emplace_back(k, JVal());
                    if (!value(v.o.back().second)) { ok = false; break; }
                    ws();
                    if (p < e && *p == ',') { ++p; continue; }
                    if (p < e && *p == '}') { ++p; break; }
                    ok = false;
                    break;
                }
            }
        } else if (*p == '[') {
            ++p;
            v.t = JVal::ARR;
            ws();
            if (p < e && *p == ']') {
                ++p;
            } else {
                for (;;) {
                    v.a.emplace_back();
                    if (!value(v.a.back())) { ok = false; break; }
                    ws();
                    if (p < e && *p == ',') { ++p; continue; }
                    if (p < e && *p == ']') { ++p; break; }
                    ok = false;
                    break;
                }
            }
        } else if (*p == '"') {
            v.t = JVal::STR;
            ok = str(v.s);
        } else if (lit("true")) {
            v.t = JVal::BOOL;
            v.b = true;
        } else if (lit("false")) {
            v.t = JVal::BOOL;
        } else if (lit("null")) {
            v.t = JVal::NUL;
        } else {
            ok = num(v);
        }
        --depth;
        return ok;
    }
};

inline bool parse_json(const char *data, size_t len, JVal &out) {
    JParse jp{data, data + len};
    if (!jp.value(out)) return false;
    jp.ws();
    return jp.p == jp.e;
}

}  // namespace qb
