// Checkpoint loading behind the C ABI: the reference's validated safetensors
// path (src/weights.rs:89-264) -- the config checks of tensor_shapes, the
// inventory checks of inspect_qwen and the exact BF16 decode of decode_qwen
// -- ending in a device model instead of host FP32 buffers.  Host code only.
//
// The file format is the safetensors layout (the reference pins crate
// safetensors 0.6.2, not vendored here): an 8-byte little-endian header
// length N, N bytes of a JSON object {name: {"dtype", "shape",
// "data_offsets": [begin, end]}, optional "__metadata__"}, then the data
// section, in which the tensors' byte ranges must lie back to back from 0
// to its end with sizes equal to shape x dtype width.
#include <ctype.h>
#include <math.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <string>
#include <vector>

#include "../../include/qwen_b200.h"
#include "common.cuh"

namespace qb {
namespace {

constexpr uint64_t kMaxHeader = 100000000ull;   // the format's header bound
constexpr uint64_t kBudget = 6ull << 30;        // the reference's 6 GiB load budget

struct TensorInfo {
    std::string dtype;
    std::vector<uint64_t> shape;
    uint64_t begin = 0, end = 0;
};

// A JSON reader for the header: objects, arrays, strings, non-negative
// integers, and (inside "__metadata__" or unknown fields) any value.
struct Json {
    const char *p, *e;
    bool ok = true;
    void ws() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
    bool eat(char c) {
        ws();
        if (p < e && *p == c) { ++p; return true; }
        return false;
    }
    bool str(std::string &out) {
        ws();
        if (p >= e || *p != '"') return ok = false;
        ++p;
        out.clear();
        while (p < e && *p != '"') {
            char c = *p++;
            if (c == '\\') {
                if (p >= e) return ok = false;
                char x = *p++;
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
                    if (e - p < 4) return ok = false;
                    unsigned v = 0;
                    for (int i = 0; i < 4; ++i) {
                        char h = *p++;
                        v <<= 4;
                        if (h >= '0' && h <= '9') v |= (unsigned)(h - '0');
                        else if (h >= 'a' && h <= 'f') v |= (unsigned)(h - 'a' + 10);
                        else if (h >= 'A' && h <= 'F') v |= (unsigned)(h - 'A' + 10);
                        else return ok = false;
                    }
                    // BMP code points as UTF-8 (names are ASCII in practice)
                    if (v < 0x80) out += (char)v;
                    else if (v < 0x800) { out += (char)(0xc0 | (v >> 6)); out += (char)(0x80 | (v & 0x3f)); }
                    else { out += (char)(0xe0 | (v >> 12)); out += (char)(0x80 | ((v >> 6) & 0x3f));
                           out += (char)(0x80 | (v & 0x3f)); }
                    break;
                }
                default: return ok = false;
                }
            } else if ((unsigned char)c < 0x20) {
                return ok = false;
            } else {
                out += c;
            }
        }
        if (p >= e) return ok = false;
        ++p;
        return true;
    }
    bool u64(uint64_t &v) {
        ws();
        if (p >= e || *p < '0' || *p > '9') return ok = false;
        v = 0;
        while (p < e && *p >= '0' && *p <= '9') {
            if (v > (~0ull - 9) / 10) return ok = false;
            v = v * 10 + (uint64_t)(*p++ - '0');
        }
        if (p < e && (*p == '.' || *p == 'e' || *p == 'E')) return ok = false;
        return true;
    }
    bool skip() {  // any value
        ws();
        if (p >= e) return ok = false;
        if (*p == '"') { std::string s; return str(s); }
        if (*p == '{') {
            ++p;
            if (eat('}')) return true;
            do {
                std::string k;
                if (!str(k) || !eat(':') || !skip()) return ok = false;
            } while (eat(','));
            if (!eat('}')) ok = false;
            return ok;
        }
        if (*p == '[') {
            ++p;
            if (eat(']')) return true;
            do {
                if (!skip()) return ok = false;
            } while (eat(','));
            if (!eat(']')) ok = false;
            return ok;
        }
        const char *s = p;
        while (p < e && (isalnum((unsigned char)*p) || *p == '-' || *p == '+' || *p == '.')) ++p;
        if (p == s) ok = false;
        return ok;
    }
    bool u64_array(std::vector<uint64_t> &v) {
        v.clear();
        if (!eat('[')) return ok = false;
        if (eat(']')) return true;
        do {
            uint64_t x;
            if (!u64(x)) return false;
            v.push_back(x);
        } while (eat(','));
        if (!eat(']')) ok = false;
        return ok;
    }
};

size_t dtype_width(const std::string &d) {
    if (d == "BOOL" || d == "U8" || d == "I8" || d == "F8_E5M2" || d == "F8_E4M3") return 1;
    if (d == "I16" || d == "U16" || d == "F16" || d == "BF16") return 2;
    if (d == "I32" || d == "U32" || d == "F32") return 4;
    if (d == "I64" || d == "U64" || d == "F64") return 8;
    return 0;
}

bool mul(uint64_t a, uint64_t b, uint64_t *o) { return !__builtin_mul_overflow(a, b, o); }
bool add(uint64_t a, uint64_t b, uint64_t *o) { return !__builtin_add_overflow(a, b, o); }

// The file's header: tensors in header order; false = not a valid file
// (the format's HeaderTooSmall/TooLarge, InvalidHeader*, InvalidOffset,
// TensorInvalidInfo, MetadataIncompleteBuffer: QB_LOAD_FORMAT).
bool parse_file(const uint8_t *data, size_t len, std::vector<std::pair<std::string, TensorInfo>> &out,
                uint64_t *data_start) {
    out.clear();
    if (len < 8) return false;
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | data[i];
    uint64_t stop;
    if (n > kMaxHeader || !add(n, 8, &stop) || stop > len) return false;
    Json j{(const char *)data + 8, (const char *)data + stop};
    if (j.p >= j.e || *j.p != '{') return false;  // the header starts with '{' (padding only after it)
    ++j.p;
    if (!j.eat('}')) {
        do {
            std::string key;
            if (!j.str(key) || !j.eat(':')) return false;
            if (key == "__metadata__") {
                if (!j.skip()) return false;
                continue;
            }
            TensorInfo t;
            bool have_d = false, have_s = false, have_o = false;
            if (!j.eat('{')) return false;
            if (!j.eat('}')) {
                do {
                    std::string f;
                    if (!j.str(f) || !j.eat(':')) return false;
                    if (f == "dtype") { if (!j.str(t.dtype)) return false; have_d = true; }
                    else if (f == "shape") { if (!j.u64_array(t.shape)) return false; have_s = true; }
                    else if (f == "data_offsets") {
                        std::vector<uint64_t> o;
                        if (!j.u64_array(o) || o.size() != 2) return false;
                        t.begin = o[0];
                        t.end = o[1];
                        have_o = true;
                    } else if (!j.skip()) return false;
                } while (j.eat(','));
                if (!j.eat('}')) return false;
            }
            if (!have_d || !have_s || !have_o || !dtype_width(t.dtype)) return false;
            // a later duplicate of a name replaces the earlier one
            auto it = std::find_if(out.begin(), out.end(), [&](const auto &x) { return x.first == key; });
            if (it != out.end()) it->second = t;
            else out.emplace_back(key, t);
        } while (j.eat(','));
        if (!j.eat('}')) return false;
    }
    j.ws();
    if (!j.ok || j.p != j.e) return false;
    // Byte ranges back to back from 0, each of its shape's size, ending at
    // the end of the buffer.
    std::vector<const TensorInfo *> byoff;
    for (auto &x : out) byoff.push_back(&x.second);
    std::sort(byoff.begin(), byoff.end(), [](const TensorInfo *a, const TensorInfo *b) {
        return a->begin != b->begin ? a->begin < b->begin : a->end < b->end;
    });
    uint64_t at = 0;
    for (const TensorInfo *t : byoff) {
        if (t->begin != at || t->end < t->begin) return false;
        uint64_t el = 1, bytes;
        for (uint64_t d : t->shape)
            if (!mul(el, d, &el)) return false;
        if (!mul(el, dtype_width(t->dtype), &bytes) || t->end - t->begin != bytes) return false;
        at = t->end;
    }
    uint64_t total;
    if (!add(at, stop, &total) || total != len) return false;
    *data_start = stop;
    return true;
}

// `count` of src/weights.rs:81-88: zero dimensions are an unsupported config.
uint32_t count(const std::vector<uint64_t> &shape, uint64_t *out) {
    for (uint64_t d : shape)
        if (d == 0) return QB_LOAD_UNSUPPORTED_CONFIG;
    uint64_t n = 1;
    for (uint64_t d : shape)
        if (!mul(n, d, &n)) return QB_DIMENSION_OVERFLOW;
    *out = n;
    return QB_OK;
}

// tensor_shapes, src/weights.rs:96-187 (the expected names in sorted order).
uint32_t tensor_shapes(const qb_qwen_config &c, std::map<std::string, std::vector<uint64_t>> &out) {
    out.clear();
    auto is = [](const char *s, const char *want) { return s && strcmp(s, want) == 0; };
    const bool arch = c.architectures_count == 1 && c.architectures && is(c.architectures[0], "Qwen2ForCausalLM");
    if (!is(c.model_type, "qwen2") || !arch || !is(c.hidden_act, "silu") || !c.tie_word_embeddings ||
        !is(c.torch_dtype, "bfloat16") || c.use_sliding_window || c.has_rope_scaling || !c.vocab_size ||
        !c.hidden_size || !c.intermediate_size || !c.num_hidden_layers || !c.num_attention_heads ||
        !c.num_key_value_heads || !c.max_position_embeddings || c.hidden_size % c.num_attention_heads ||
        c.num_attention_heads % c.num_key_value_heads || (c.hidden_size / c.num_attention_heads) % 2 ||
        !isfinite(c.rms_norm_eps) || c.rms_norm_eps <= 0.0f || !isfinite(c.rope_theta) || c.rope_theta <= 0.0f)
        return QB_LOAD_UNSUPPORTED_CONFIG;
    const uint64_t h = c.hidden_size, ffd = c.intermediate_size, L = c.num_hidden_layers;
    uint64_t kv, t, square, kvw, ff, per, tmp, emb, elements;
    if (!mul(c.num_key_value_heads, h / c.num_attention_heads, &kv)) return QB_DIMENSION_OVERFLOW;
    if (!mul(L, 12, &t) || !add(t, 2, &t)) return QB_DIMENSION_OVERFLOW;
    uint32_t s;
    if ((s = count({h, h}, &square)) || (s = count({kv, h}, &kvw)) || (s = count({ffd, h}, &ff))) return s;
    if (!mul(square, 2, &per) || !mul(kvw, 2, &tmp) || !add(per, tmp, &per) || !mul(ff, 3, &tmp) ||
        !add(per, tmp, &per) || !mul(h, 3, &tmp) || !add(per, tmp, &per) || !mul(kv, 2, &tmp) ||
        !add(per, tmp, &per))
        return QB_DIMENSION_OVERFLOW;
    if ((s = count({c.vocab_size, h}, &emb))) return s;
    if (!add(emb, h, &elements) || !mul(per, L, &tmp) || !add(elements, tmp, &elements)) return QB_DIMENSION_OVERFLOW;
    if (!mul(elements, 6, &tmp)) return QB_DIMENSION_OVERFLOW;
    if (tmp > kBudget) return QB_RESOURCE_BUDGET;
    out["model.embed_tokens.weight"] = {c.vocab_size, h};
    out["model.norm.weight"] = {h};
    for (uint64_t l = 0; l < L; ++l) {
        const std::string pre = "model.layers." + std::to_string(l) + ".";
        out[pre + "input_layernorm.weight"] = {h};
        out[pre + "post_attention_layernorm.weight"] = {h};
        out[pre + "self_attn.q_proj.weight"] = {h, h};
        out[pre + "self_attn.q_proj.bias"] = {h};
        out[pre + "self_attn.k_proj.weight"] = {kv, h};
        out[pre + "self_attn.k_proj.bias"] = {kv};
        out[pre + "self_attn.v_proj.weight"] = {kv, h};
        out[pre + "self_attn.v_proj.bias"] = {kv};
        out[pre + "self_attn.o_proj.weight"] = {h, h};
        out[pre + "mlp.gate_proj.weight"] = {ffd, h};
        out[pre + "mlp.up_proj.weight"] = {ffd, h};
        out[pre + "mlp.down_proj.weight"] = {h, ffd};
    }
    for (auto &x : out) {
        uint64_t n, b;
        if ((s = count(x.second, &n))) return s;
        if (!mul(n, 4, &b)) return QB_DIMENSION_OVERFLOW;
    }
    return QB_OK;
}

struct Record {
    std::string name;
    uint64_t offset, elements;  // byte offset in the whole buffer
};

// inspect_qwen, src/weights.rs:189-221.
uint32_t inspect(const uint8_t *data, size_t len, const qb_qwen_config &c, std::vector<Record> &recs) {
    std::map<std::string, std::vector<uint64_t>> expected;
    uint32_t s = tensor_shapes(c, expected);
    if (s) return s;
    std::vector<std::pair<std::string, TensorInfo>> file;
    uint64_t start = 0;
    if (!parse_file(data, len, file, &start)) return QB_LOAD_FORMAT;
    for (size_t i = 0; i < file.size(); ++i)
        if (!expected.count(file[i].first)) {
            set_detail(0, 0, 0, i);
            return QB_LOAD_UNEXPECTED_TENSOR;
        }
    std::map<std::string, const TensorInfo *> byname;
    for (auto &x : file) byname[x.first] = &x.second;
    recs.clear();
    size_t idx = 0;
    for (auto &x : expected) {
        auto it = byname.find(x.first);
        if (it == byname.end()) { set_detail(0, 0, 0, idx); return QB_LOAD_MISSING_TENSOR; }
        const TensorInfo &t = *it->second;
        if (t.shape != x.second) { set_detail(0, 0, 0, idx); return QB_INVALID_SHAPE; }
        if (t.dtype != "BF16") { set_detail(0, 0, 0, idx); return QB_LOAD_INVALID_DTYPE; }
        uint64_t el = 1, bytes;
        for (uint64_t d : x.second) el *= d;  // checked by tensor_shapes
        if (!mul(el, 2, &bytes)) return QB_DIMENSION_OVERFLOW;
        if (t.end - t.begin != bytes) { set_detail(0, 0, 0, idx); return QB_INVALID_SHAPE; }
        recs.push_back(Record{x.first, start + t.begin, el});
        ++idx;
    }
    return QB_OK;
}

// The library's tensor id and layer of a checkpoint name.
bool tensor_id(const std::string &name, int64_t *layer, uint32_t *id) {
    if (name == "model.embed_tokens.weight") { *layer = -1; *id = QB_T_EMBEDDING; return true; }
    if (name == "model.norm.weight") { *layer = -1; *id = QB_T_FINAL_NORM; return true; }
    const std::string pre = "model.layers.";
    if (name.compare(0, pre.size(), pre) != 0) return false;
    size_t dot = name.find('.', pre.size());
    if (dot == std::string::npos) return false;
    *layer = std::stoll(name.substr(pre.size(), dot - pre.size()));
    static const std::map<std::string, uint32_t> ids = {
        {"input_layernorm.weight", QB_T_ATTN_NORM}, {"post_attention_layernorm.weight", QB_T_FFN_NORM},
        {"self_attn.q_proj.weight", QB_T_Q}, {"self_attn.q_proj.bias", QB_T_Q_BIAS},
        {"self_attn.k_proj.weight", QB_T_K}, {"self_attn.k_proj.bias", QB_T_K_BIAS},
        {"self_attn.v_proj.weight", QB_T_V}, {"self_attn.v_proj.bias", QB_T_V_BIAS},
        {"self_attn.o_proj.weight", QB_T_O}, {"mlp.gate_proj.weight", QB_T_GATE},
        {"mlp.up_proj.weight", QB_T_UP}, {"mlp.down_proj.weight", QB_T_DOWN}};
    auto it = ids.find(name.substr(dot + 1));
    if (it == ids.end()) return false;
    *id = it->second;
    return true;
}

}  // namespace
}  // namespace qb

using namespace qb;

extern "C" {

uint32_t qb_qwen_tensor_count(const qb_qwen_config *config, size_t *count) {
    clear_detail();
    if (!config || !count) return QB_INVALID_PARAMETERS;
    std::map<std::string, std::vector<uint64_t>> expected;
    uint32_t s = tensor_shapes(*config, expected);
    if (s) return s;
    *count = expected.size();
    return QB_OK;
}

uint32_t qb_safetensors_inspect(const uint8_t *data, size_t len, const qb_qwen_config *config, size_t *tensor_count) {
    clear_detail();
    if (!config || (!data && len)) return QB_INVALID_PARAMETERS;
    std::vector<Record> recs;
    uint32_t s = inspect(data, len, *config, recs);
    if (s) return s;
    if (tensor_count) *tensor_count = recs.size();
    return QB_OK;
}

uint32_t qb_model_load_safetensors(const uint8_t *data, size_t len, const qb_qwen_config *config,
                                   uint32_t linear_format, uint32_t table_format, int device, uint64_t *out_model) {
    clear_detail();
    if (!config || !out_model || (!data && len)) return QB_INVALID_PARAMETERS;
    std::vector<Record> recs;
    uint32_t s = inspect(data, len, *config, recs);
    if (s) return s;
    uint64_t elements = 0, logical, total;
    for (auto &r : recs)
        if (!add(elements, r.elements, &elements)) return QB_DIMENSION_OVERFLOW;
    if (!mul(elements, 4, &logical)) return QB_DIMENSION_OVERFLOW;
    if (!add(logical, len, &total)) return QB_DIMENSION_OVERFLOW;
    if (total > kBudget) return QB_RESOURCE_BUDGET;
    // Every value finite before any device work (BF16 exponent all ones =
    // infinity or NaN).
    for (size_t i = 0; i < recs.size(); ++i) {
        const uint8_t *p = data + recs[i].offset;
        for (uint64_t k = 0; k < recs[i].elements; ++k) {
            const uint16_t b = (uint16_t)(p[2 * k] | (p[2 * k + 1] << 8));
            if ((b & 0x7f80u) == 0x7f80u) {
                set_detail(0, 0, (size_t)k, i);
                return QB_NONFINITE;
            }
        }
    }
    const qb_qwen_config &c = *config;
    qb_model_config mc;
    mc.vocab_size = c.vocab_size;
    mc.layers = c.num_hidden_layers;
    mc.hidden_dim = c.hidden_size;
    mc.query_heads = c.num_attention_heads;
    mc.kv_heads = c.num_key_value_heads;
    mc.head_dim = c.hidden_size / c.num_attention_heads;
    mc.ff_dim = c.intermediate_size;
    mc.max_tokens = c.max_position_embeddings;
    mc.rope_base = c.rope_theta;
    mc.norm_epsilon = c.rms_norm_eps;
    uint64_t m = 0;
    if ((s = qb_model_create(&mc, linear_format, table_format, device, &m))) return s;
    std::vector<uint16_t> buf;
    for (auto &r : recs) {
        int64_t layer;
        uint32_t id;
        if (!tensor_id(r.name, &layer, &id)) { qb_model_free(m); return QB_LOAD_UNEXPECTED_TENSOR; }
        // The payload may sit at an odd address; copy it aligned.
        buf.resize(r.elements);
        memcpy(buf.data(), data + r.offset, r.elements * 2);
        if ((s = qb_model_set_tensor(m, layer, id, QB_HOST_BF16, buf.data(), r.elements))) {
            qb_model_free(m);
            return s;
        }
    }
    if ((s = qb_model_finalize(m))) {
        qb_model_free(m);
        return s;
    }
    *out_model = m;
    return QB_OK;
}

}  // extern "C"
