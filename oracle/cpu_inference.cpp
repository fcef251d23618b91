// CPU ORACLE — test infrastructure only. Nothing in the product links or calls this file; only
// tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load liboracle_cpu.so, as the
// checker, never as the thing measured for the GPU engine.
//
// A line-by-line C++ restatement of the reference CPU engine,
// metal_infrence_engine/src/cpu_inference.rs (the reference's correctness spec: its Metal
// shaders say "every kernel mirrors a function in cpu_inference.rs", inference.metal:7).
// The reference is Rust and cannot be built here (no cargo/rustc, no crates), so this port is the
// oracle. Parity status: UNPINNED against the reference's own golden vectors — they need the
// real Qwen3-0.6B checkpoint (tests/metal_parity.rs:13 "Paris" = 12095, mlx_baseline/bench.py:48),
// which is absent. The port is cross-checked instead against Hugging Face transformers' Qwen3 on
// the same seeded random weights (tests/golden/make_golden.py).
//
// Numerics follow Rust semantics: IEEE f32 throughout, no FMA contraction (build with
// -ffp-contract=off, never -ffast-math), sequential sums in the reference's order, libm
// expf/powf/sinf/cosf/sqrtf (what Rust's f32 methods lower to on Linux).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <thread>
#include <unistd.h>
#include <unordered_map>
#include <vector>

namespace {

// ---------------------------------------------------------------------------------------------
// Minimal JSON reader (what serde_json does for the header and config.json in the reference)
// ---------------------------------------------------------------------------------------------
struct JVal {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    double num = 0;
    bool b = false;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal* get(const std::string& k) const {
        for (auto& kv : obj) if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const char* p;
    const char* e;
    void ws() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++; }
    [[noreturn]] void fail(const char* m) { throw std::runtime_error(std::string("json: ") + m); }
    JVal parse() {
        ws();
        if (p >= e) fail("unexpected end");
        JVal v;
        char c = *p;
        if (c == '{') {
            v.kind = JVal::Obj; p++; ws();
            if (p < e && *p == '}') { p++; return v; }
            for (;;) {
                ws(); if (p >= e || *p != '"') fail("expected key");
                std::string k = pstr(); ws();
                if (p >= e || *p != ':') fail("expected ':'");
                p++;
                v.obj.emplace_back(k, parse()); ws();
                if (p < e && *p == ',') { p++; continue; }
                if (p < e && *p == '}') { p++; return v; }
                fail("expected ',' or '}'");
            }
        } else if (c == '[') {
            v.kind = JVal::Arr; p++; ws();
            if (p < e && *p == ']') { p++; return v; }
            for (;;) {
                v.arr.push_back(parse()); ws();
                if (p < e && *p == ',') { p++; continue; }
                if (p < e && *p == ']') { p++; return v; }
                fail("expected ',' or ']'");
            }
        } else if (c == '"') {
            v.kind = JVal::Str; v.str = pstr();
        } else if (c == 't' && e - p >= 4 && !strncmp(p, "true", 4)) { v.kind = JVal::Bool; v.b = true; p += 4; }
        else if (c == 'f' && e - p >= 5 && !strncmp(p, "false", 5)) { v.kind = JVal::Bool; p += 5; }
        else if (c == 'n' && e - p >= 4 && !strncmp(p, "null", 4)) { p += 4; }
        else {
            char* end = nullptr;
            std::string tmp(p, std::min<size_t>(64, e - p));
            v.num = strtod(tmp.c_str(), &end);
            if (end == tmp.c_str()) fail("bad value");
            v.kind = JVal::Num; p += end - tmp.c_str();
        }
        return v;
    }
    std::string pstr() {
        p++;
        std::string s;
        while (p < e && *p != '"') {
            if (*p == '\\') { p++; if (p >= e) fail("bad escape"); s += (*p == 'n' ? '\n' : *p == 't' ? '\t' : *p); p++; }
            else s += *p++;
        }
        if (p >= e) fail("unterminated string");
        p++;
        return s;
    }
};

JVal parse_json(const char* b, size_t n) { JParser jp{b, b + n}; return jp.parse(); }

// ---------------------------------------------------------------------------------------------
// cpu_inference.rs:11-33  Tensor / Config
// ---------------------------------------------------------------------------------------------
struct Tensor {
    std::string name, dtype;
    std::vector<int32_t> shape;
    std::vector<int32_t> data_offsets;  // i32 in the reference (cpu_inference.rs:17)
};

struct Config {
    size_t hidden_size, intermediate_size, num_hidden_layers, num_attention_heads, num_key_value_heads,
        head_dim, vocab_size;
    float rms_norm_eps, rope_theta;
    uint32_t eos_token_id;
};

}  // namespace

struct OracleModel {
    void* map = nullptr;
    size_t map_len = 0;
    std::vector<Tensor> tensors;
    Config config{};
    std::unordered_map<std::string, size_t> index;
    const uint8_t* raw_weights = nullptr;
    ~OracleModel() { if (map) munmap(map, map_len); }

    // cpu_inference.rs:87-96  bf16 weights viewed straight out of the mmap
    const uint16_t* weight(const std::string& name, size_t* numel_out = nullptr) const {
        auto it = index.find(name);
        if (it == index.end()) throw std::runtime_error("missing tensor " + name);
        const Tensor& t = tensors[it->second];
        if (t.dtype != "BF16") throw std::runtime_error(name + ": only BF16 is supported");
        size_t start = (size_t)t.data_offsets[0], end = (size_t)t.data_offsets[1];
        size_t numel = 1;
        for (int32_t d : t.shape) numel *= (size_t)d;
        if ((end - start) / 2 != numel) throw std::runtime_error(name + ": size mismatch");
        if (numel_out) *numel_out = numel;
        return reinterpret_cast<const uint16_t*>(raw_weights + start);
    }
};

// cpu_inference.rs:44-55  per-layer K/V history, [t][kv_heads*head_dim] per position
struct OracleCache {
    std::vector<std::vector<float>> k, v;
};

namespace {

int g_threads = 0;  // 0: std::thread::hardware_concurrency(), like available_parallelism()

// cpu_inference.rs:183
inline float bf16_to_f32(uint16_t x) { uint32_t u = (uint32_t)x << 16; float f; std::memcpy(&f, &u, 4); return f; }

// cpu_inference.rs:185  a.iter().zip(b).map(|(x, y)| x * y).sum()
float dot(const float* a, const float* b, size_t n) {
    float s = -0.0f;
    for (size_t i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

// cpu_inference.rs:187
inline float silu(float x) { return x / (1.0f + expf(-x)); }

// cpu_inference.rs:189-194
void rmsnorm(float* out, const float* x, const uint16_t* w, size_t n, float eps) {
    float ss = -0.0f;
    for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
    float ms = ss / (float)n;
    float s = 1.0f / sqrtf(ms + eps);
    for (size_t i = 0; i < n; i++) out[i] = x[i] * s * bf16_to_f32(w[i]);
}

// cpu_inference.rs:196-201
void rmsnorm_inplace(float* x, const uint16_t* w, size_t n, float eps) {
    float ss = -0.0f;
    for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
    float ms = ss / (float)n;
    float s = 1.0f / sqrtf(ms + eps);
    for (size_t i = 0; i < n; i++) x[i] = x[i] * s * bf16_to_f32(w[i]);
}

// cpu_inference.rs:203-215  HF rotate_half: element i pairs with i + head_dim/2
void rope(float* x, size_t len, size_t pos, float theta) {
    size_t half = len / 2;
    for (size_t i = 0; i < half; i++) {
        float freq = powf(theta, -2.0f * (float)i / (float)len);
        float ang = (float)pos * freq;
        float sn = sinf(ang), cs = cosf(ang);
        float a = x[i], b = x[i + half];
        x[i] = a * cs - b * sn;
        x[i + half] = b * cs + a * sn;
    }
}

// cpu_inference.rs:217-223
void softmax(float* x, size_t n) {
    float mx = -INFINITY;
    for (size_t i = 0; i < n; i++) mx = fmaxf(mx, x[i]);  // f32::max ignores NaN like fmaxf
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    for (size_t i = 0; i < n; i++) x[i] /= sum;
}

// cpu_inference.rs:243-257  8 interleaved accumulators, sequential sum, then the remainder
float dot_bf16(const uint16_t* w, const float* x, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t full = n / 8 * 8;
    for (size_t c = 0; c < full; c += 8)
        for (int i = 0; i < 8; i++) acc[i] += bf16_to_f32(w[c + i]) * x[c + i];
    float s = -0.0f;
    for (int i = 0; i < 8; i++) s += acc[i];
    for (size_t c = full; c < n; c++) s += bf16_to_f32(w[c]) * x[c];
    return s;
}

// cpu_inference.rs:225-241  rows split into contiguous blocks over the host threads
void matvec(float* out, size_t rows, const uint16_t* w, const float* x, size_t cols) {
    size_t threads = g_threads > 0 ? (size_t)g_threads : std::max(1u, std::thread::hardware_concurrency());
    size_t rows_per = (rows + threads - 1) / threads;
    std::vector<std::thread> th;
    for (size_t r0 = 0; r0 < rows; r0 += rows_per) {
        size_t r1 = std::min(rows, r0 + rows_per);
        th.emplace_back([=] {
            for (size_t r = r0; r < r1; r++) out[r] = dot_bf16(w + r * cols, x, cols);
        });
    }
    for (auto& t : th) t.join();
}

thread_local std::string g_err;

size_t cfg_usize(const JVal& c, const char* k) {
    const JVal* v = c.get(k);
    if (!v || v->kind != JVal::Num || v->num < 0) throw std::runtime_error(std::string("config.json: missing ") + k);
    return (size_t)v->num;
}
float cfg_f32(const JVal& c, const char* k) {
    const JVal* v = c.get(k);
    if (!v || v->kind != JVal::Num) throw std::runtime_error(std::string("config.json: missing ") + k);
    return (float)v->num;
}

std::string read_file(const std::string& path) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) throw std::runtime_error("cannot open " + path);
    std::string s;
    char buf[65536];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) s.append(buf, n);
    fclose(f);
    return s;
}

}  // namespace

extern "C" {

const char* oracle_last_error() { return g_err.c_str(); }
void oracle_set_threads(int n) { g_threads = n; }
int oracle_threads() { return g_threads > 0 ? g_threads : (int)std::max(1u, std::thread::hardware_concurrency()); }

// cpu_inference.rs:58-84  Model::load_model
int oracle_load(const char* file, OracleModel** out) {
    *out = nullptr;
    try {
        auto m = std::make_unique<OracleModel>();
        int fd = open(file, O_RDONLY);
        if (fd < 0) throw std::runtime_error(std::string("cannot open ") + file);
        struct stat st;
        fstat(fd, &st);
        m->map_len = (size_t)st.st_size;
        if (m->map_len < 8) { close(fd); throw std::runtime_error("file too short"); }
        m->map = mmap(nullptr, m->map_len, PROT_READ, MAP_PRIVATE, fd, 0);
        close(fd);
        if (m->map == MAP_FAILED) { m->map = nullptr; throw std::runtime_error("mmap failed"); }
        const uint8_t* b = (const uint8_t*)m->map;
        uint64_t header_length = 0;
        for (int i = 0; i < 8; i++) header_length |= (uint64_t)b[i] << (8 * i);
        if (header_length + 8 > m->map_len) throw std::runtime_error("header length beyond end of file");
        JVal parsed = parse_json((const char*)b + 8, header_length);
        if (parsed.kind != JVal::Obj) throw std::runtime_error("header is not a JSON object");
        for (auto& kv : parsed.obj) {
            if (kv.first == "__metadata__") continue;
            Tensor t;
            t.name = kv.first;
            const JVal* dt = kv.second.get("dtype");
            const JVal* sh = kv.second.get("shape");
            const JVal* of = kv.second.get("data_offsets");
            if (!dt || !sh || !of || dt->kind != JVal::Str || sh->kind != JVal::Arr || of->kind != JVal::Arr)
                throw std::runtime_error("bad tensor entry " + kv.first);
            t.dtype = dt->str;
            for (auto& d : sh->arr) t.shape.push_back((int32_t)d.num);
            for (auto& d : of->arr) t.data_offsets.push_back((int32_t)d.num);
            if (t.data_offsets.size() != 2) throw std::runtime_error("bad data_offsets " + kv.first);
            if ((uint64_t)t.data_offsets[1] + 8 + header_length > m->map_len)
                throw std::runtime_error("tensor " + kv.first + " extends past end of file");
            m->tensors.push_back(std::move(t));
        }
        m->raw_weights = b + 8 + header_length;
        if ((uintptr_t)m->raw_weights % 2 != 0) throw std::runtime_error("safetensors data section is not 2-byte aligned");
        for (size_t i = 0; i < m->tensors.size(); i++) m->index[m->tensors[i].name] = i;

        std::string fs(file);
        size_t slash = fs.find_last_of('/');
        std::string cfg_path = (slash == std::string::npos ? std::string() : fs.substr(0, slash + 1)) + "config.json";
        std::string cs = read_file(cfg_path);
        JVal c = parse_json(cs.data(), cs.size());
        Config& cf = m->config;
        cf.hidden_size = cfg_usize(c, "hidden_size");
        cf.intermediate_size = cfg_usize(c, "intermediate_size");
        cf.num_hidden_layers = cfg_usize(c, "num_hidden_layers");
        cf.num_attention_heads = cfg_usize(c, "num_attention_heads");
        cf.num_key_value_heads = cfg_usize(c, "num_key_value_heads");
        cf.head_dim = cfg_usize(c, "head_dim");
        cf.vocab_size = cfg_usize(c, "vocab_size");
        cf.rms_norm_eps = cfg_f32(c, "rms_norm_eps");
        cf.rope_theta = cfg_f32(c, "rope_theta");
        cf.eos_token_id = (uint32_t)cfg_usize(c, "eos_token_id");
        *out = m.release();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

void oracle_free(OracleModel* m) { delete m; }

// fields: hidden, inter, layers, heads, kv_heads, head_dim, vocab
void oracle_config(const OracleModel* m, uint64_t* fields, float* eps, float* theta, uint32_t* eos) {
    const Config& c = m->config;
    uint64_t f[7] = {c.hidden_size, c.intermediate_size, c.num_hidden_layers, c.num_attention_heads,
                     c.num_key_value_heads, c.head_dim, c.vocab_size};
    std::memcpy(fields, f, sizeof f);
    *eps = c.rms_norm_eps;
    *theta = c.rope_theta;
    *eos = c.eos_token_id;
}

// tests/mbu.rs:19-30: every tensor except the embedding table, plus one bf16 embedding row
uint64_t oracle_weight_bytes_per_token(const OracleModel* m) {
    uint64_t bytes = 0;
    for (auto& t : m->tensors) {
        if (t.name == "model.embed_tokens.weight") continue;
        bytes += (uint64_t)(t.data_offsets[1] - t.data_offsets[0]);
    }
    return bytes + m->config.hidden_size * 2;
}

// cpu_inference.rs:51-54  KVCache::new
OracleCache* oracle_cache_new(const OracleModel* m) {
    auto* c = new OracleCache;
    c->k.resize(m->config.num_hidden_layers);
    c->v.resize(m->config.num_hidden_layers);
    return c;
}
void oracle_cache_free(OracleCache* c) { delete c; }

size_t oracle_cache_len(const OracleModel* m, const OracleCache* c) {
    size_t kv_dim = m->config.num_key_value_heads * m->config.head_dim;
    return c->k.empty() ? 0 : c->k[0].size() / kv_dim;
}

// copies layer `layer`'s K and V history, [len][kv_dim] each
int oracle_cache_read(const OracleCache* c, size_t layer, float* k_out, float* v_out) {
    if (layer >= c->k.size()) { g_err = "layer out of range"; return -1; }
    std::memcpy(k_out, c->k[layer].data(), c->k[layer].size() * 4);
    std::memcpy(v_out, c->v[layer].data(), c->v[layer].size() * 4);
    return 0;
}

// appends `npos` positions of deterministic filler values to every layer (CPU-baseline timing
// only: it lets a timed decode start at a deep position without an untimed token-by-token prefill)
int oracle_cache_fill(const OracleModel* m, OracleCache* c, size_t npos, uint64_t seed) {
    size_t kv_dim = m->config.num_key_value_heads * m->config.head_dim;
    uint64_t s = seed * 6364136223846793005ull + 1442695040888963407ull;
    for (size_t l = 0; l < c->k.size(); l++) {
        for (size_t i = 0; i < npos * kv_dim; i++) {
            s = s * 6364136223846793005ull + 1442695040888963407ull;
            c->k[l].push_back((float)((int32_t)(s >> 40) - (1 << 23)) / (float)(1 << 23));
            s = s * 6364136223846793005ull + 1442695040888963407ull;
            c->v[l].push_back((float)((int32_t)(s >> 40) - (1 << 23)) / (float)(1 << 23));
        }
    }
    return 0;
}

// cpu_inference.rs:100-179  Model::forward: one token at `pos`, appends its K/V, returns logits
int oracle_forward(const OracleModel* m, OracleCache* cache, uint32_t token, size_t pos, float* logits_out) {
    try {
        const Config& c = m->config;
        const size_t hd = c.head_dim;
        const size_t q_dim = c.num_attention_heads * hd;
        const size_t kv_dim = c.num_key_value_heads * hd;
        const size_t group = c.num_attention_heads / c.num_key_value_heads;
        const float eps = c.rms_norm_eps;

        size_t embed_n = 0;
        const uint16_t* embed = m->weight("model.embed_tokens.weight", &embed_n);
        size_t row = (size_t)token * c.hidden_size;
        if (row + c.hidden_size > embed_n) throw std::runtime_error("token id out of range");
        std::vector<float> x(c.hidden_size);
        for (size_t i = 0; i < c.hidden_size; i++) x[i] = bf16_to_f32(embed[row + i]);

        std::vector<float> xn(c.hidden_size), q(q_dim), k(kv_dim), v(kv_dim), att(q_dim),
            proj(c.hidden_size), gate(c.intermediate_size), up(c.intermediate_size), scores(pos + 1);

        for (size_t l = 0; l < c.num_hidden_layers; l++) {
            std::string p = "model.layers." + std::to_string(l) + ".";
            auto w = [&](const char* n) { return m->weight(p + n); };

            // attention
            rmsnorm(xn.data(), x.data(), w("input_layernorm.weight"), c.hidden_size, eps);
            matvec(q.data(), q_dim, w("self_attn.q_proj.weight"), xn.data(), c.hidden_size);
            matvec(k.data(), kv_dim, w("self_attn.k_proj.weight"), xn.data(), c.hidden_size);
            matvec(v.data(), kv_dim, w("self_attn.v_proj.weight"), xn.data(), c.hidden_size);

            // qwen3 normalizes each q/k head before rope
            const uint16_t* q_norm = w("self_attn.q_norm.weight");
            const uint16_t* k_norm = w("self_attn.k_norm.weight");
            for (size_t h = 0; h < q_dim; h += hd) { rmsnorm_inplace(&q[h], q_norm, hd, eps); rope(&q[h], hd, pos, c.rope_theta); }
            for (size_t h = 0; h < kv_dim; h += hd) { rmsnorm_inplace(&k[h], k_norm, hd, eps); rope(&k[h], hd, pos, c.rope_theta); }

            cache->k[l].insert(cache->k[l].end(), k.begin(), k.end());
            cache->v[l].insert(cache->v[l].end(), v.begin(), v.end());
            const std::vector<float>& kc = cache->k[l];
            const std::vector<float>& vc = cache->v[l];
            // the reference slices kc[t*kv_dim ..] for t in 0..=pos and panics past the end
            if ((pos + 1) * kv_dim > kc.size()) throw std::runtime_error("pos beyond the cache length");

            const float scale = 1.0f / sqrtf((float)hd);
            for (size_t h = 0; h < c.num_attention_heads; h++) {
                const float* qh = &q[h * hd];
                size_t kv_off = (h / group) * hd;
                for (size_t t = 0; t <= pos; t++) scores[t] = dot(qh, &kc[t * kv_dim + kv_off], hd) * scale;
                softmax(scores.data(), pos + 1);
                float* o = &att[h * hd];
                std::fill(o, o + hd, 0.0f);
                for (size_t t = 0; t <= pos; t++) {
                    const float* vt = &vc[t * kv_dim + kv_off];
                    for (size_t i = 0; i < hd; i++) o[i] += scores[t] * vt[i];
                }
            }
            matvec(proj.data(), c.hidden_size, w("self_attn.o_proj.weight"), att.data(), q_dim);
            for (size_t i = 0; i < c.hidden_size; i++) x[i] += proj[i];

            // swiglu mlp
            rmsnorm(xn.data(), x.data(), w("post_attention_layernorm.weight"), c.hidden_size, eps);
            matvec(gate.data(), c.intermediate_size, w("mlp.gate_proj.weight"), xn.data(), c.hidden_size);
            matvec(up.data(), c.intermediate_size, w("mlp.up_proj.weight"), xn.data(), c.hidden_size);
            for (size_t i = 0; i < c.intermediate_size; i++) gate[i] = silu(gate[i]) * up[i];
            matvec(proj.data(), c.hidden_size, w("mlp.down_proj.weight"), gate.data(), c.intermediate_size);
            for (size_t i = 0; i < c.hidden_size; i++) x[i] += proj[i];
        }

        rmsnorm(xn.data(), x.data(), m->weight("model.norm.weight"), c.hidden_size, eps);
        matvec(logits_out, c.vocab_size, m->weight("lm_head.weight"), xn.data(), c.hidden_size);
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// Model::forward (cpu_inference.rs:100-179) for n consecutive tokens at positions start_pos ..
// start_pos + n - 1, computed layer by layer over all n positions instead of token by token. Every
// value goes through the same functions in the same order as n calls of oracle_forward: a
// position's projections are dot_bf16 of the same row and input, and its attention reads only
// positions <= its own, whose K/V this layer has already appended. So the cache and the logits are
// bit-identical to the token-by-token loop (tests/test_oracle.py checks this), while each weight row
// is read once per block of positions rather than once per token: a 2048-token prompt on the
// Qwen3-0.6B geometry takes seconds instead of minutes. That is the only reason it exists.
// Logits are written for the positions listed in out_idx (indices into 0..n-1), row k of
// logits_out for out_idx[k]; the cache must hold exactly start_pos positions.
int oracle_forward_seq(const OracleModel* m, OracleCache* cache, const uint32_t* tokens, size_t n, size_t start_pos,
                       const size_t* out_idx, size_t n_out, float* logits_out) {
    try {
        const Config& c = m->config;
        const size_t H = c.hidden_size, I = c.intermediate_size, hd = c.head_dim;
        const size_t q_dim = c.num_attention_heads * hd, kv_dim = c.num_key_value_heads * hd;
        const size_t group = c.num_attention_heads / c.num_key_value_heads;
        const float eps = c.rms_norm_eps;
        if (oracle_cache_len(m, cache) != start_pos) throw std::runtime_error("cache length differs from start_pos");
        for (size_t k = 0; k < n_out; k++)
            if (out_idx[k] >= n) throw std::runtime_error("out_idx beyond n");
        size_t embed_n = 0;
        const uint16_t* embed = m->weight("model.embed_tokens.weight", &embed_n);
        std::vector<float> x(n * H), xn(n * H), q(n * q_dim), kk(n * kv_dim), vv(n * kv_dim), att(n * q_dim),
            proj(n * H), gate(n * I), up(n * I);
        for (size_t t = 0; t < n; t++) {
            const size_t row = (size_t)tokens[t] * H;
            if (row + H > embed_n) throw std::runtime_error("token id out of range");
            for (size_t i = 0; i < H; i++) x[t * H + i] = bf16_to_f32(embed[row + i]);
        }
        const size_t threads = g_threads > 0 ? (size_t)g_threads : std::max(1u, std::thread::hardware_concurrency());
        // out[t][r] = dot_bf16(w row r, in[t]) for t < n: rows split over the threads, positions
        // taken in blocks so a block's inputs stay cached while the thread walks its rows
        auto seq_matvec = [&](float* out, size_t rows, const uint16_t* w, const float* in, size_t cols,
                              const std::vector<size_t>* pick) {
            const size_t np = pick ? pick->size() : n;
            const size_t rows_per = (rows + threads - 1) / threads;
            std::vector<std::thread> th;
            for (size_t r0 = 0; r0 < rows; r0 += rows_per) {
                const size_t r1 = std::min(rows, r0 + rows_per);
                th.emplace_back([=] {
                    for (size_t b0 = 0; b0 < np; b0 += 16) {
                        const size_t b1 = std::min(np, b0 + 16);
                        for (size_t r = r0; r < r1; r++)
                            for (size_t b = b0; b < b1; b++) {
                                const size_t t = pick ? (*pick)[b] : b;
                                out[b * rows + r] = dot_bf16(w + r * cols, in + t * cols, cols);
                            }
                    }
                });
            }
            for (auto& t : th) t.join();
        };
        auto parallel = [&](size_t count, const std::function<void(size_t)>& fn) {
            std::vector<std::thread> th;
            const size_t per = (count + threads - 1) / threads;
            for (size_t a0 = 0; a0 < count; a0 += per) {
                const size_t a1 = std::min(count, a0 + per);
                th.emplace_back([=, &fn] { for (size_t a = a0; a < a1; a++) fn(a); });
            }
            for (auto& t : th) t.join();
        };
        const float scale = 1.0f / sqrtf((float)hd);
        for (size_t l = 0; l < c.num_hidden_layers; l++) {
            std::string p = "model.layers." + std::to_string(l) + ".";
            auto w = [&](const char* nm) { return m->weight(p + nm); };
            const uint16_t* ln1 = w("input_layernorm.weight");
            for (size_t t = 0; t < n; t++) rmsnorm(&xn[t * H], &x[t * H], ln1, H, eps);
            seq_matvec(q.data(), q_dim, w("self_attn.q_proj.weight"), xn.data(), H, nullptr);
            seq_matvec(kk.data(), kv_dim, w("self_attn.k_proj.weight"), xn.data(), H, nullptr);
            seq_matvec(vv.data(), kv_dim, w("self_attn.v_proj.weight"), xn.data(), H, nullptr);
            const uint16_t* q_norm = w("self_attn.q_norm.weight");
            const uint16_t* k_norm = w("self_attn.k_norm.weight");
            for (size_t t = 0; t < n; t++) {
                const size_t pos = start_pos + t;
                for (size_t h = 0; h < q_dim; h += hd) { rmsnorm_inplace(&q[t * q_dim + h], q_norm, hd, eps); rope(&q[t * q_dim + h], hd, pos, c.rope_theta); }
                for (size_t h = 0; h < kv_dim; h += hd) { rmsnorm_inplace(&kk[t * kv_dim + h], k_norm, hd, eps); rope(&kk[t * kv_dim + h], hd, pos, c.rope_theta); }
                cache->k[l].insert(cache->k[l].end(), kk.begin() + t * kv_dim, kk.begin() + (t + 1) * kv_dim);
                cache->v[l].insert(cache->v[l].end(), vv.begin() + t * kv_dim, vv.begin() + (t + 1) * kv_dim);
            }
            const std::vector<float>& kc = cache->k[l];
            const std::vector<float>& vc = cache->v[l];
            parallel(n * c.num_attention_heads, [&](size_t job) {
                const size_t t = job / c.num_attention_heads, h = job % c.num_attention_heads;
                const size_t pos = start_pos + t;
                std::vector<float> scores(pos + 1);
                const float* qh = &q[t * q_dim + h * hd];
                const size_t kv_off = (h / group) * hd;
                for (size_t s = 0; s <= pos; s++) scores[s] = dot(qh, &kc[s * kv_dim + kv_off], hd) * scale;
                softmax(scores.data(), pos + 1);
                float* o = &att[t * q_dim + h * hd];
                std::fill(o, o + hd, 0.0f);
                for (size_t s = 0; s <= pos; s++) {
                    const float* vt = &vc[s * kv_dim + kv_off];
                    for (size_t i = 0; i < hd; i++) o[i] += scores[s] * vt[i];
                }
            });
            seq_matvec(proj.data(), H, w("self_attn.o_proj.weight"), att.data(), q_dim, nullptr);
            for (size_t i = 0; i < n * H; i++) x[i] += proj[i];
            const uint16_t* ln2 = w("post_attention_layernorm.weight");
            for (size_t t = 0; t < n; t++) rmsnorm(&xn[t * H], &x[t * H], ln2, H, eps);
            seq_matvec(gate.data(), I, w("mlp.gate_proj.weight"), xn.data(), H, nullptr);
            seq_matvec(up.data(), I, w("mlp.up_proj.weight"), xn.data(), H, nullptr);
            for (size_t i = 0; i < n * I; i++) gate[i] = silu(gate[i]) * up[i];
            seq_matvec(proj.data(), H, w("mlp.down_proj.weight"), gate.data(), I, nullptr);
            for (size_t i = 0; i < n * H; i++) x[i] += proj[i];
        }
        if (n_out) {
            const uint16_t* fn = m->weight("model.norm.weight");
            std::vector<size_t> pick(out_idx, out_idx + n_out);
            for (size_t k = 0; k < n_out; k++) rmsnorm(&xn[pick[k] * H], &x[pick[k] * H], fn, H, eps);
            seq_matvec(logits_out, c.vocab_size, m->weight("lm_head.weight"), xn.data(), H, &pick);
        }
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// cpu_inference.rs:225-257  the reference's matvec on its own (bf16 weights [rows][cols], f32 x),
// rows split over the host threads: the CPU side of the isolated GEMV microbenchmark
void oracle_matvec(const uint16_t* w, const float* x, float* out, size_t rows, size_t cols) {
    matvec(out, rows, w, x, cols);
}

// tests/common/mod.rs:17-22 (also bench.rs:99-104, main.rs:37-42): first strict maximum
uint32_t oracle_argmax(const float* x, size_t n) {
    size_t best = 0;
    for (size_t i = 1; i < n; i++) if (x[i] > x[best]) best = i;
    return (uint32_t)best;
}

}  // extern "C"
