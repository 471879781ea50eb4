// The poll bridge (apple/cpu_bridge: src/lib.rs, src/worker.rs) over the
// device token loop.  Host code only: one worker thread owns the model and
// the generation state (qb_generation_* on the GPU); the caller's thread
// only copies inputs, hands over one command at a time and collects one
// event per command.  The protocol, codes and event contents follow the
// reference bridge; see include/qwen_b200_bridge.h.
#include <cuda_runtime.h>
#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <condition_variable>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/qwen_b200.h"
#include "../../include/qwen_b200_bridge.h"
#include "json.h"

namespace {

using qb::JVal;
using qb::parse_json;

constexpr size_t kMaxText = 4096;          // src/lib.rs:7
constexpr size_t kTinyLimit = 8u << 20;    // src/lib.rs:186
constexpr size_t kPathLimit = 4096;        // src/lib.rs:187
constexpr size_t kBridgeContext = 32;      // src/worker.rs:92,109
constexpr size_t kBridgeVocab = 151936;    // src/worker.rs:109
constexpr size_t kQwenAdmitted = 8;        // src/worker.rs:128
constexpr size_t kBudget = 128u << 20;     // CachedSession's default budget (src/kv_cache.rs:184-190)

// An object whose keys are all in `allowed` (serde's deny_unknown_fields)
// and hold every key in `required`.
bool keys_ok(const JVal &v, std::initializer_list<const char *> required,
             std::initializer_list<const char *> optional = {}) {
    if (v.t != JVal::OBJ) return false;
    for (auto &kv : v.o) {
        bool known = false;
        for (const char *k : required) known = known || kv.first == k;
        for (const char *k : optional) known = known || kv.first == k;
        if (!known) return false;
    }
    for (const char *k : required)
        if (!v.get(k)) return false;
    return true;
}

bool as_size(const JVal *v, size_t &out) {
    if (!v || v->t != JVal::NUM || !v->integer) return false;
    errno = 0;
    char *end = nullptr;
    const unsigned long long x = strtoull(v->s.c_str(), &end, 10);
    if (errno != 0 || *end != '\0') return false;
    out = (size_t)x;
    return true;
}

bool as_f32(const JVal *v, float &out) {
    if (!v || v->t != JVal::NUM) return false;
    out = (float)v->n;
    return true;
}

bool as_f32_vec(const JVal *v, std::vector<float> &out) {
    if (!v || v->t != JVal::ARR) return false;
    out.resize(v->a.size());
    for (size_t i = 0; i < v->a.size(); ++i)
        if (!as_f32(&v->a[i], out[i])) return false;
    return true;
}

// ------------------------------------------------------------- sources ----

struct ModelHandle {
    uint64_t h = 0;
    ~ModelHandle() {
        if (h) qb_model_free(h);
    }
};

// Decoder::from_json (src/model.rs:185-189) as an FP32 device model.
bool load_tiny(const std::vector<uint8_t> &bytes, int device, ModelHandle &m, qb_model_config &c) {
    JVal root;
    if (!parse_json((const char *)bytes.data(), bytes.size(), root)) return false;
    if (!keys_ok(root, {"config", "weights"})) return false;
    const JVal &cf = *root.get("config"), &wt = *root.get("weights");
    if (!keys_ok(cf, {"vocab_size", "layers", "hidden_dim", "query_heads", "kv_heads", "head_dim", "ff_dim",
                      "max_tokens", "rope_base", "norm_epsilon"}))
        return false;
    if (!as_size(cf.get("vocab_size"), c.vocab_size) || !as_size(cf.get("layers"), c.layers) ||
        !as_size(cf.get("hidden_dim"), c.hidden_dim) || !as_size(cf.get("query_heads"), c.query_heads) ||
        !as_size(cf.get("kv_heads"), c.kv_heads) || !as_size(cf.get("head_dim"), c.head_dim) ||
        !as_size(cf.get("ff_dim"), c.ff_dim) || !as_size(cf.get("max_tokens"), c.max_tokens) ||
        !as_f32(cf.get("rope_base"), c.rope_base) || !as_f32(cf.get("norm_epsilon"), c.norm_epsilon))
        return false;
    if (!keys_ok(wt, {"embedding", "layers", "final_norm"})) return false;
    const JVal &layers = *wt.get("layers");
    if (layers.t != JVal::ARR) return false;
    for (auto &l : layers.a)
        if (!keys_ok(l, {"attention_norm", "query", "key", "value", "attention_output", "ffn_norm", "gate", "up",
                         "down"},
                     {"query_bias", "key_bias", "value_bias"}))
            return false;
    if (qb_model_create(&c, QB_LINEAR_F32, QB_TABLE_F32, device, &m.h) != QB_OK) return false;
    std::vector<float> v;
    auto put = [&](int64_t layer, uint32_t id, const JVal *src) {
        return as_f32_vec(src, v) &&
               qb_model_set_tensor(m.h, layer, id, QB_HOST_F32, v.empty() ? nullptr : v.data(), v.size()) == QB_OK;
    };
    if (!put(-1, QB_T_EMBEDDING, wt.get("embedding")) || !put(-1, QB_T_FINAL_NORM, wt.get("final_norm")))
        return false;
    for (size_t i = 0; i < layers.a.size(); ++i) {
        const JVal &l = layers.a[i];
        const struct { const char *k; uint32_t id; } f[] = {
            {"attention_norm", QB_T_ATTN_NORM}, {"query", QB_T_Q}, {"key", QB_T_K}, {"value", QB_T_V},
            {"attention_output", QB_T_O}, {"ffn_norm", QB_T_FFN_NORM}, {"gate", QB_T_GATE}, {"up", QB_T_UP},
            {"down", QB_T_DOWN}, {"query_bias", QB_T_Q_BIAS}, {"key_bias", QB_T_K_BIAS},
            {"value_bias", QB_T_V_BIAS}};
        for (auto &x : f) {
            const JVal *src = l.get(x.k);
            if (!src || src->t == JVal::NUL) continue;  // absent or null optional bias
            if (!put((int64_t)i, x.id, src)) return false;
        }
    }
    // The layer count (ModelError::InvalidLayerCount) and completeness are
    // checked by finalize.
    return qb_model_finalize(m.h) == QB_OK;
}

bool read_file(const std::string &path, std::vector<uint8_t> &out) {
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    bool ok = fseek(f, 0, SEEK_END) == 0;
    const long n = ok ? ftell(f) : -1;
    ok = ok && n >= 0 && fseek(f, 0, SEEK_SET) == 0;
    if (ok) {
        out.resize((size_t)n);
        ok = n == 0 || fread(out.data(), 1, (size_t)n, f) == (size_t)n;
    }
    fclose(f);
    return ok;
}

struct TokHandle {
    uint64_t h = 0;
    ~TokHandle() {
        if (h) qb_tokenizer_free(h);
    }
};
struct StreamHandle {
    uint64_t h = 0;
    ~StreamHandle() { reset(0); }
    void reset(uint64_t nh) {
        if (h) qb_tokenizer_stream_free(h);
        h = nh;
    }
};

// load_qwen + Decoder::from_qwen(weights, 32) + ChatTokenizer::load
// (src/worker.rs:85-99): the directory's config.json and model.safetensors
// through the checkpoint loader (a 32-position context, FP32 linears and
// table), then tokenizer.json, tokenizer_config.json and
// generation_config.json through the chat tokenizer's checks.
bool load_qwen_dir(const std::string &dir, int device, ModelHandle &m, qb_model_config &c, TokHandle &tok) {
    std::vector<uint8_t> cfg_bytes, st;
    if (!read_file(dir + "/config.json", cfg_bytes)) return false;
    JVal cfg;
    if (!parse_json((const char *)cfg_bytes.data(), cfg_bytes.size(), cfg) || cfg.t != JVal::OBJ) return false;
    auto str_of = [&](const char *k) {
        const JVal *v = cfg.get(k);
        return v && v->t == JVal::STR ? v->s : std::string();
    };
    auto size_of_key = [&](const char *k) {
        size_t x = 0;
        return as_size(cfg.get(k), x) ? x : (size_t)0;
    };
    auto f32_of = [&](const char *k) {
        float x = 0.0f;
        return as_f32(cfg.get(k), x) ? x : 0.0f;
    };
    auto bool_of = [&](const char *k) {
        const JVal *v = cfg.get(k);
        return v && v->t == JVal::BOOL && v->b ? 1 : 0;
    };
    const std::string model_type = str_of("model_type"), act = str_of("hidden_act"), dtype = str_of("torch_dtype");
    std::vector<std::string> arch_s;
    if (const JVal *a = cfg.get("architectures"))
        if (a->t == JVal::ARR)
            for (auto &x : a->a)
                if (x.t == JVal::STR) arch_s.push_back(x.s);
    std::vector<const char *> archs;
    for (auto &s : arch_s) archs.push_back(s.c_str());
    qb_qwen_config q{};
    q.model_type = model_type.c_str();
    q.hidden_act = act.c_str();
    q.torch_dtype = dtype.c_str();
    q.architectures = archs.empty() ? nullptr : archs.data();
    q.architectures_count = archs.size();
    q.vocab_size = size_of_key("vocab_size");
    q.hidden_size = size_of_key("hidden_size");
    q.intermediate_size = size_of_key("intermediate_size");
    q.num_hidden_layers = size_of_key("num_hidden_layers");
    q.num_attention_heads = size_of_key("num_attention_heads");
    q.num_key_value_heads = size_of_key("num_key_value_heads");
    q.max_position_embeddings = size_of_key("max_position_embeddings");
    q.rms_norm_eps = f32_of("rms_norm_eps");
    q.rope_theta = f32_of("rope_theta");
    q.tie_word_embeddings = bool_of("tie_word_embeddings");
    q.use_sliding_window = bool_of("use_sliding_window");
    const JVal *rs = cfg.get("rope_scaling");
    q.has_rope_scaling = rs && rs->t != JVal::NUL ? 1 : 0;
    size_t count = 0;
    if (qb_qwen_tensor_count(&q, &count) != QB_OK) return false;  // the config's own checks first
    if (q.max_position_embeddings > kBridgeContext) q.max_position_embeddings = kBridgeContext;
    if (!read_file(dir + "/model.safetensors", st)) return false;
    if (qb_model_load_safetensors(st.data(), st.size(), &q, QB_LINEAR_F32, QB_TABLE_F32, device, &m.h) != QB_OK)
        return false;
    c = qb_model_config{};
    c.vocab_size = q.vocab_size;
    c.max_tokens = q.max_position_embeddings;
    std::vector<uint8_t> tj, tc, gc;
    if (!read_file(dir + "/tokenizer.json", tj) || !read_file(dir + "/tokenizer_config.json", tc) ||
        !read_file(dir + "/generation_config.json", gc))
        return false;
    return qb_tokenizer_load_chat(tj.data(), tj.size(), tc.data(), tc.size(), gc.data(), gc.size(), &tok.h) ==
           QB_OK;
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

// ------------------------------------------------------------- engine ----

enum class Cmd { BeginIds, BeginText, Next, Reset };
struct Command {
    Cmd kind = Cmd::Next;
    std::vector<uint32_t> ids;
    std::string text;
    size_t max_new = 0;
};
struct Delivery {
    AieEvent event{};
    std::string text;
};

// The two one-slot channels between the caller and the worker
// (sync_channel(1) each in src/lib.rs:98-99), the cancel flag read by the
// generation at token boundaries, and the admission flags.
struct Engine {
    std::mutex mu;
    std::condition_variable cmd_cv, ev_cv;
    bool has_cmd = false, has_ev = false;
    bool closed = false;       // the caller side is gone (aie_close)
    bool worker_done = false;  // the worker side is gone
    Command cmd;
    Delivery ev;
    volatile int32_t cancel = 0;
    std::atomic<bool> fatal{false}, busy{true};
};

std::mutex g_reg_mu;
std::map<uint64_t, std::shared_ptr<Engine>> g_reg;
std::atomic<uint64_t> g_next_id{1};
std::atomic<bool> g_worker_active{false};

std::shared_ptr<Engine> engine(uint64_t h) {
    std::lock_guard<std::mutex> lk(g_reg_mu);
    auto it = g_reg.find(h);
    return it == g_reg.end() ? nullptr : it->second;
}

void set_cancel(Engine &e, bool on) { __atomic_store_n(&e.cancel, on ? 1 : 0, __ATOMIC_RELEASE); }

// Blocking send of one event; false once the caller side is gone.
bool deliver(Engine &e, const AieEvent &ev, std::string text) {
    std::unique_lock<std::mutex> lk(e.mu);
    e.ev_cv.wait(lk, [&] { return !e.has_ev || e.closed; });
    if (e.closed) return false;
    e.ev.event = ev;
    e.ev.text = std::move(text);
    e.has_ev = true;
    return true;
}

// The generation handle a worker owns (GenerationSession in src/worker.rs).
struct GenHandle {
    uint64_t h = 0;
    ~GenHandle() { reset(0); }
    void reset(uint64_t nh) {
        if (h) qb_generation_free(h);
        h = nh;
    }
};

AieEvent snapshot(const GenHandle *g, uint32_t kind, uint32_t code, int64_t token) {
    AieEvent ev{kind, code, token < 0 ? 0xffffffffu : (uint32_t)token, 0, 0};
    qb_generation_info info{};
    if (g && g->h && qb_generation_info_get(g->h, &info) == QB_OK) {
        ev.processed = (uint32_t)info.processed;
        ev.history = (uint32_t)info.history_len;
    }
    return ev;
}

// StateError to the bridge's codes (src/worker.rs:47-66).
AieEvent failure(const GenHandle *g, uint32_t status) {
    uint32_t code = AIE_EXECUTION_FAILED;
    if (status == QB_CANCELLED) code = AIE_CANCELLED;
    else if (status == QB_INVALID_PARAMETERS || status == QB_NOT_STARTED || status == QB_ALREADY_STARTED)
        code = AIE_INVALID_INPUT;
    return snapshot(g, code == AIE_CANCELLED ? AIE_CANCEL_EVENT : AIE_ERROR, code, -1);
}

struct Source {
    uint32_t kind;
    std::vector<uint8_t> bytes;
};

// worker::run (src/worker.rs:68-243).
void run(const Source &src, Engine &e, int device) {
    ModelHandle model;
    TokHandle tok;
    qb_model_config c{};
    const bool loaded = src.kind == 0 ? load_tiny(src.bytes, device, model, c)
                                      : load_qwen_dir(std::string(src.bytes.begin(), src.bytes.end()), device,
                                                      model, c, tok);
    if (!loaded || c.max_tokens > kBridgeContext || c.vocab_size > kBridgeVocab) {
        e.fatal.store(true);
        deliver(e, snapshot(nullptr, AIE_ERROR, AIE_MODEL_FAILED, -1), std::string());
        return;
    }
    if (!deliver(e, snapshot(nullptr, AIE_READY, AIE_OK, -1), std::string())) return;
    GenHandle gen;
    StreamHandle stream;
    const bool has_tokenizer = tok.h != 0;
    const size_t admitted = has_tokenizer ? kQwenAdmitted : c.max_tokens;
    const size_t capacity = c.max_tokens;
    uint32_t stop_ids[8];
    size_t nstops = 0;
    if (has_tokenizer && qb_tokenizer_stop_tokens(tok.h, stop_ids, 8, &nstops) != QB_OK) nstops = 0;
    auto new_stream = [&]() {
        uint64_t sh = 0;
        if (has_tokenizer && qb_tokenizer_stream_create(tok.h, &sh) != QB_OK) sh = 0;
        stream.reset(sh);
    };
    new_stream();
    for (;;) {
        Command cmd;
        {
            std::unique_lock<std::mutex> lk(e.mu);
            e.cmd_cv.wait(lk, [&] { return e.has_cmd || e.closed; });
            if (e.closed) return;
            cmd = std::move(e.cmd);
            e.has_cmd = false;
        }
        std::string text;
        AieEvent ev{};
        const volatile int32_t *cancel = &e.cancel;
        if (cmd.kind == Cmd::BeginIds || cmd.kind == Cmd::BeginText) {
            qb_generation_info info{};
            const bool started = gen.h && qb_generation_info_get(gen.h, &info) == QB_OK && info.history_len > 0;
            bool ok = !started;
            std::vector<uint32_t> ids;
            if (ok) {
                if (cmd.kind == Cmd::BeginIds) {
                    ids = cmd.ids;
                } else if (!has_tokenizer) {
                    ok = false;
                } else {
                    // ChatTokenizer::encode of the plain text on the worker.
                    size_t n = 0;
                    const uint8_t *tb = (const uint8_t *)cmd.text.data();
                    uint32_t st = qb_tokenizer_encode(tok.h, tb, cmd.text.size(), nullptr, 0, &n);
                    if (st == QB_INVALID_OUTPUT_LENGTH || st == QB_OK) {
                        ids.resize(n);
                        st = qb_tokenizer_encode(tok.h, tb, cmd.text.size(), ids.data(), n, &n);
                    }
                    ok = st == QB_OK;
                }
            }
            if (ok) {
                ok = !ids.empty() && ids.size() <= admitted && cmd.max_new <= admitted - ids.size();
                for (uint32_t id : ids) ok = ok && id < c.vocab_size;
            }
            if (!ok) {
                ev = snapshot(&gen, AIE_ERROR, AIE_INVALID_INPUT, -1);
            } else {
                uint64_t cand = 0;
                const uint32_t st = qb_generation_create(model.h, capacity, nstops ? stop_ids : nullptr, nstops,
                                                         cmd.max_new, QB_KV_F32, kBudget, &cand);
                if (st != QB_OK) {
                    ev = failure(&gen, st);
                } else {
                    const uint32_t r = qb_generation_start(cand, ids.data(), ids.size(), cancel);
                    // A prompt admitted into history is kept (a cancelled or
                    // failed evaluation resumes or reports from it); one
                    // refused before admission leaves the previous state.
                    qb_generation_info ci{};
                    if (qb_generation_info_get(cand, &ci) == QB_OK && ci.history_len > 0) {
                        gen.reset(cand);
                        new_stream();
                    } else {
                        qb_generation_free(cand);
                    }
                    ev = r == QB_OK ? snapshot(&gen, AIE_STARTED, AIE_OK, -1) : failure(&gen, r);
                }
            }
        } else if (cmd.kind == Cmd::Next) {
            if (!gen.h) {
                ev = snapshot(nullptr, AIE_ERROR, AIE_INVALID_INPUT, -1);
            } else {
                uint32_t tid = 0;
                int32_t has = 0;
                const uint32_t r = qb_generation_next_token(gen.h, cancel, &tid, &has);
                if (r != QB_OK) {
                    ev = failure(&gen, r);
                } else if (has) {
                    bool decoded = true;
                    if (stream.h) {
                        // TextStream::push: the newly completed text (or none yet).
                        char buf[kMaxText];
                        size_t n = 0;
                        int32_t has_text = 0;
                        decoded = qb_tokenizer_stream_push(stream.h, tid, buf, kMaxText, &n, &has_text) == QB_OK;
                        if (decoded && has_text) text.assign(buf, n);
                    } else {
                        text = std::to_string(tid) + " ";  // ids, as the reference emits without a tokenizer
                    }
                    if (decoded) {
                        ev = snapshot(&gen, AIE_TOKEN, AIE_OK, tid);
                    } else {
                        ev = snapshot(&gen, AIE_ERROR, AIE_EXECUTION_FAILED, -1);
                        ev.processed = 0;  // terminal: no valid cache is exposed
                    }
                } else {
                    ev = snapshot(&gen, AIE_STOPPED, AIE_OK, -1);
                }
            }
        } else {  // Reset
            if (gen.h) qb_generation_reset(gen.h);
            new_stream();
            set_cancel(e, false);
            ev = snapshot(&gen, AIE_RESET_EVENT, AIE_OK, -1);
        }
        if (ev.code == AIE_EXECUTION_FAILED) {
            // No recovery and no valid cache after an execution failure.
            e.fatal.store(true);
            deliver(e, ev, std::move(text));
            return;
        }
        if (!deliver(e, ev, std::move(text))) return;
    }
}

// The worker thread: runs the source, contains exceptions as a PANIC event,
// frees the model and generation (inside run) before it releases the
// single-worker reservation.
void worker_main(Source src, std::shared_ptr<Engine> e, int device) {
    try {
        run(src, *e, device);
    } catch (...) {
        e->fatal.store(true);
        try {
            deliver(*e, AieEvent{AIE_ERROR, AIE_PANIC, 0xffffffffu, 0, 0}, std::string());
        } catch (...) {
        }
    }
    {
        std::lock_guard<std::mutex> lk(e->mu);
        e->worker_done = true;
    }
    e->ev_cv.notify_all();
    g_worker_active.store(false, std::memory_order_release);
}

// submit (src/lib.rs:139-157).
uint32_t submit(uint64_t h, Command cmd) {
    auto e = engine(h);
    if (!e) return AIE_INVALID_HANDLE;
    if (e->fatal.load()) return AIE_EXECUTION_FAILED;
    bool expected = false;
    if (!e->busy.compare_exchange_strong(expected, true)) return AIE_BUSY;
    {
        std::lock_guard<std::mutex> lk(e->mu);
        if (e->worker_done || e->has_cmd) {
            e->busy.store(false);
            return AIE_CLOSED;
        }
        e->cmd = std::move(cmd);
        e->has_cmd = true;
    }
    e->cmd_cv.notify_one();
    return AIE_OK;
}

template <class T> bool aligned(const T *p) { return p && ((uintptr_t)p % alignof(T)) == 0; }

template <class F> uint32_t boundary(F &&f) {
    try {
        return f();
    } catch (...) {
        return AIE_PANIC;
    }
}

// One event out of the channel, or PENDING / CLOSED.
uint32_t take(uint64_t h, Delivery &out) {
    auto e = engine(h);
    if (!e) return AIE_INVALID_HANDLE;
    {
        std::lock_guard<std::mutex> lk(e->mu);
        if (!e->has_ev) return e->worker_done ? AIE_CLOSED : AIE_PENDING;
        out = std::move(e->ev);
        e->has_ev = false;
    }
    e->ev_cv.notify_all();
    e->busy.store(false);
    return AIE_OK;
}

}  // namespace

extern "C" {

uint32_t aie_abi_version(void) { return 2; }

uint32_t aie_open(uint32_t kind, const uint8_t *bytes, size_t length, uint64_t *out_handle) {
    return boundary([&]() -> uint32_t {
        size_t limit;
        if (kind == 0) limit = kTinyLimit;
        else if (kind == 1) limit = kPathLimit;
        else return AIE_INVALID_INPUT;
        if (!aligned(out_handle) || !bytes || length == 0 || length > limit) return AIE_INVALID_INPUT;
        Source src{kind, std::vector<uint8_t>(bytes, bytes + length)};
        if (kind == 1 && (!valid_utf8(src.bytes.data(), length) || memchr(bytes, 0, length)))
            return AIE_INVALID_INPUT;
        int device = 0;
        if (cudaGetDevice(&device) != cudaSuccess) {
            cudaGetLastError();
            device = 0;
        }
        std::lock_guard<std::mutex> lk(g_reg_mu);
        bool expected = false;
        if (!g_reg.empty() || !g_worker_active.compare_exchange_strong(expected, true)) return AIE_BUSY;
        const uint64_t id = g_next_id.fetch_add(1);
        if (id == 0) {
            g_worker_active.store(false);
            return AIE_CLOSED;
        }
        auto e = std::make_shared<Engine>();
        try {
            std::thread(worker_main, std::move(src), e, device).detach();
        } catch (...) {
            g_worker_active.store(false);
            return AIE_EXECUTION_FAILED;
        }
        g_reg[id] = e;
        *out_handle = id;
        return AIE_OK;
    });
}

uint32_t aie_begin_ids(uint64_t handle, const uint32_t *ids, size_t count, uint32_t max_new) {
    return boundary([&]() -> uint32_t {
        if (!aligned(ids) || count == 0 || count > 32 || max_new == 0 || max_new >= 32) return AIE_INVALID_INPUT;
        Command c;
        c.kind = Cmd::BeginIds;
        c.ids.assign(ids, ids + count);
        c.max_new = max_new;
        return submit(handle, std::move(c));
    });
}

uint32_t aie_begin_text(uint64_t handle, const uint8_t *bytes, size_t length, uint32_t max_new) {
    return boundary([&]() -> uint32_t {
        if (!bytes || length == 0 || length > 65536 || max_new == 0 || max_new >= 32) return AIE_INVALID_INPUT;
        if (!valid_utf8(bytes, length)) return AIE_INVALID_INPUT;
        Command c;
        c.kind = Cmd::BeginText;
        c.text.assign((const char *)bytes, length);
        c.max_new = max_new;
        return submit(handle, std::move(c));
    });
}

uint32_t aie_next(uint64_t handle) {
    return boundary([&]() -> uint32_t { return submit(handle, Command{Cmd::Next, {}, {}, 0}); });
}

uint32_t aie_reset(uint64_t handle) {
    return boundary([&]() -> uint32_t { return submit(handle, Command{Cmd::Reset, {}, {}, 0}); });
}

uint32_t aie_set_cancel(uint64_t handle, uint32_t enabled) {
    return boundary([&]() -> uint32_t {
        if (enabled > 1) return AIE_INVALID_INPUT;
        auto e = engine(handle);
        if (!e) return AIE_INVALID_HANDLE;
        set_cancel(*e, enabled == 1);
        return AIE_OK;
    });
}

uint32_t aie_poll(uint64_t handle, AieEvent *out_event) {
    return boundary([&]() -> uint32_t {
        if (!aligned(out_event)) return AIE_INVALID_INPUT;
        Delivery d;
        const uint32_t st = take(handle, d);
        if (st == AIE_OK) *out_event = d.event;
        return st;
    });
}

uint32_t aie_poll_text(uint64_t handle, AieEvent *out_event, uint8_t *text, size_t capacity, size_t *out_length) {
    return boundary([&]() -> uint32_t {
        if (!aligned(out_event) || !aligned(out_length) || !text || capacity != kMaxText) return AIE_INVALID_INPUT;
        Delivery d;
        const uint32_t st = take(handle, d);
        if (st != AIE_OK) return st;
        const size_t n = d.text.size() < kMaxText ? d.text.size() : kMaxText;  // bounded by the producer
        memcpy(text, d.text.data(), n);
        *out_event = d.event;
        *out_length = n;
        return AIE_OK;
    });
}

uint32_t aie_close(uint64_t handle) {
    return boundary([&]() -> uint32_t {
        std::shared_ptr<Engine> e;
        {
            std::lock_guard<std::mutex> lk(g_reg_mu);
            auto it = g_reg.find(handle);
            if (it == g_reg.end()) return AIE_INVALID_HANDLE;
            e = it->second;
            g_reg.erase(it);
        }
        set_cancel(*e, true);
        {
            std::lock_guard<std::mutex> lk(e->mu);
            e->closed = true;
        }
        e->cmd_cv.notify_all();
        e->ev_cv.notify_all();
        return AIE_OK;
    });
}

}  // extern "C"
