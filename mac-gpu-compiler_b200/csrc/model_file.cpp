// Safetensors + config.json reader (see model_file.h).
#include "model_file.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "../../include/cuda_inference.h"

namespace qw {
namespace {

// ---- a small strict JSON reader: objects, arrays, strings, numbers, true/false/null ----
struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
    const Json* at(const char* key) const {
        for (auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class JsonReader {
public:
    JsonReader(const char* b, size_t n) : p_(b), e_(b + n) {}
    bool parse(Json& out, std::string& err) {
        if (!value(out, 0)) { err = err_; return false; }
        skip();
        if (p_ != e_) { err = "trailing characters after JSON value"; return false; }
        return true;
    }

private:
    const char* p_;
    const char* e_;
    std::string err_;
    bool fail(const char* m) { if (err_.empty()) err_ = m; return false; }
    void skip() { while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_; }
    bool lit(const char* s) {
        size_t n = std::strlen(s);
        if ((size_t)(e_ - p_) < n || std::memcmp(p_, s, n) != 0) return false;
        p_ += n;
        return true;
    }
    bool string(std::string& s) {
        if (p_ >= e_ || *p_ != '"') return fail("expected string");
        ++p_;
        while (p_ < e_ && *p_ != '"') {
            char c = *p_++;
            if (c == '\\') {
                if (p_ >= e_) return fail("bad escape");
                char x = *p_++;
                switch (x) {
                    case 'n': s += '\n'; break;
                    case 't': s += '\t'; break;
                    case 'r': s += '\r'; break;
                    case 'b': s += '\b'; break;
                    case 'f': s += '\f'; break;
                    case 'u':
                        if (e_ - p_ < 4) return fail("bad \\u escape");
                        s += '?';  // tensor names and config keys are ASCII
                        p_ += 4;
                        break;
                    default: s += x;
                }
            } else {
                s += c;
            }
        }
        if (p_ >= e_) return fail("unterminated string");
        ++p_;
        return true;
    }
    bool value(Json& v, int depth) {
        if (depth > 64) return fail("JSON nested too deeply");
        skip();
        if (p_ >= e_) return fail("unexpected end of JSON");
        char c = *p_;
        if (c == '{') {
            v.kind = Json::Obj;
            ++p_;
            skip();
            if (p_ < e_ && *p_ == '}') { ++p_; return true; }
            for (;;) {
                skip();
                std::string k;
                if (!string(k)) return false;
                skip();
                if (p_ >= e_ || *p_ != ':') return fail("expected ':'");
                ++p_;
                v.obj.emplace_back(std::move(k), Json());
                if (!value(v.obj.back().second, depth + 1)) return false;
                skip();
                if (p_ < e_ && *p_ == ',') { ++p_; continue; }
                if (p_ < e_ && *p_ == '}') { ++p_; return true; }
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = Json::Arr;
            ++p_;
            skip();
            if (p_ < e_ && *p_ == ']') { ++p_; return true; }
            for (;;) {
                v.arr.emplace_back();
                if (!value(v.arr.back(), depth + 1)) return false;
                skip();
                if (p_ < e_ && *p_ == ',') { ++p_; continue; }
                if (p_ < e_ && *p_ == ']') { ++p_; return true; }
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') { v.kind = Json::Str; return string(v.str); }
        if (lit("true")) { v.kind = Json::Bool; v.num = 1; return true; }
        if (lit("false")) { v.kind = Json::Bool; return true; }
        if (lit("null")) { v.kind = Json::Null; return true; }
        char buf[64];
        size_t n = 0;
        while (p_ + n < e_ && n < sizeof(buf) - 1 && std::strchr("+-0123456789.eE", p_[n])) { buf[n] = p_[n]; ++n; }
        buf[n] = 0;
        if (n == 0) return fail("bad JSON value");
        char* end = nullptr;
        v.num = std::strtod(buf, &end);
        if (end != buf + n) return fail("bad number");
        v.kind = Json::Num;
        p_ += n;
        return true;
    }
};

bool read_text(const std::string& path, std::string& out) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return false;
    char buf[1 << 16];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, n);
    std::fclose(f);
    return true;
}

bool get_uint(const Json& o, const char* k, uint64_t& out, std::string& msg) {
    const Json* v = o.at(k);
    if (!v || v->kind != Json::Num || v->num < 0 || v->num != (double)(uint64_t)v->num) {
        msg = std::string("config.json: missing or invalid integer field '") + k + "'";
        return false;
    }
    out = (uint64_t)v->num;
    return true;
}

bool get_float(const Json& o, const char* k, float& out, std::string& msg) {
    const Json* v = o.at(k);
    if (!v || v->kind != Json::Num) {
        msg = std::string("config.json: missing or invalid number field '") + k + "'";
        return false;
    }
    out = (float)v->num;
    return true;
}

}  // namespace

ModelFile::~ModelFile() {
    if (map_) munmap(map_, map_len_);
}

int ModelFile::open(const std::string& path, std::string& msg) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) { msg = "cannot open " + path; return QW_ERR_IO; }
    struct stat st;
    if (fstat(fd, &st) != 0) { ::close(fd); msg = "cannot stat " + path; return QW_ERR_IO; }
    map_len_ = (size_t)st.st_size;
    if (map_len_ < 8) { ::close(fd); msg = path + ": file shorter than the 8-byte header length"; return QW_ERR_FORMAT; }
    map_ = mmap(nullptr, map_len_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map_ == MAP_FAILED) { map_ = nullptr; msg = "mmap failed for " + path; return QW_ERR_IO; }
    const uint8_t* b = static_cast<const uint8_t*>(map_);
    uint64_t hl = 0;
    for (int i = 0; i < 8; i++) hl |= (uint64_t)b[i] << (8 * i);
    if (hl > map_len_ - 8) { msg = path + ": header length points past the end of the file"; return QW_ERR_FORMAT; }
    Json hdr;
    std::string jerr;
    if (!JsonReader(reinterpret_cast<const char*>(b + 8), (size_t)hl).parse(hdr, jerr)) {
        msg = path + ": bad safetensors header: " + jerr;
        return QW_ERR_FORMAT;
    }
    if (hdr.kind != Json::Obj) { msg = path + ": safetensors header is not a JSON object"; return QW_ERR_FORMAT; }
    data_ = b + 8 + hl;
    const uint64_t data_len = map_len_ - 8 - hl;
    for (auto& kv : hdr.obj) {
        if (kv.first == "__metadata__") continue;
        const Json& t = kv.second;
        const Json* dt = t.at("dtype");
        const Json* sh = t.at("shape");
        const Json* of = t.at("data_offsets");
        if (t.kind != Json::Obj || !dt || dt->kind != Json::Str || !sh || sh->kind != Json::Arr || !of ||
            of->kind != Json::Arr || of->arr.size() != 2) {
            msg = "tensor '" + kv.first + "': malformed header entry";
            return QW_ERR_FORMAT;
        }
        TensorView v;
        v.dtype = dt->str;
        for (auto& d : sh->arr) {
            if (d.kind != Json::Num || d.num < 0) { msg = "tensor '" + kv.first + "': bad shape"; return QW_ERR_FORMAT; }
            v.shape.push_back((int64_t)d.num);
        }
        if (of->arr[0].kind != Json::Num || of->arr[1].kind != Json::Num || of->arr[0].num < 0 ||
            of->arr[1].num < of->arr[0].num) {
            msg = "tensor '" + kv.first + "': bad data_offsets";
            return QW_ERR_FORMAT;
        }
        v.begin = (uint64_t)of->arr[0].num;
        v.end = (uint64_t)of->arr[1].num;
        if (v.end > data_len) { msg = "tensor '" + kv.first + "': data extends past the end of the file (truncated?)"; return QW_ERR_FORMAT; }
        tensors_[kv.first] = std::move(v);
    }

    std::string cpath = path;
    size_t slash = cpath.find_last_of('/');
    cpath = (slash == std::string::npos ? std::string() : cpath.substr(0, slash + 1)) + "config.json";
    std::string ctext;
    if (!read_text(cpath, ctext)) { msg = "cannot read " + cpath; return QW_ERR_IO; }
    Json cj;
    if (!JsonReader(ctext.data(), ctext.size()).parse(cj, jerr) || cj.kind != Json::Obj) {
        msg = cpath + ": bad JSON: " + jerr;
        return QW_ERR_FORMAT;
    }
    uint64_t eos = 0;
    if (!get_uint(cj, "hidden_size", cfg_.hidden, msg) || !get_uint(cj, "intermediate_size", cfg_.inter, msg) ||
        !get_uint(cj, "num_hidden_layers", cfg_.layers, msg) || !get_uint(cj, "num_attention_heads", cfg_.heads, msg) ||
        !get_uint(cj, "num_key_value_heads", cfg_.kv_heads, msg) || !get_uint(cj, "head_dim", cfg_.head_dim, msg) ||
        !get_uint(cj, "vocab_size", cfg_.vocab, msg) || !get_float(cj, "rms_norm_eps", cfg_.eps, msg) ||
        !get_float(cj, "rope_theta", cfg_.theta, msg) || !get_uint(cj, "eos_token_id", eos, msg))
        return QW_ERR_FORMAT;
    cfg_.eos = (uint32_t)eos;
    return validate(msg);
}

int ModelFile::validate(std::string& msg) {
    const ModelConfig& c = cfg_;
    auto need = [&](const std::string& name, std::vector<int64_t> shape) -> int {
        auto it = tensors_.find(name);
        if (it == tensors_.end()) { msg = "missing tensor " + name; return QW_ERR_FORMAT; }
        const TensorView& t = it->second;
        // the reference accepts only BF16 (cpu_inference.rs:90, metal_inference.rs:244)
        if (t.dtype != "BF16") { msg = name + ": only BF16 is supported, got " + t.dtype; return QW_ERR_UNSUPPORTED; }
        if (t.shape != shape) { msg = name + ": unexpected shape"; return QW_ERR_FORMAT; }
        uint64_t numel = 1;
        for (auto d : shape) numel *= (uint64_t)d;
        if (t.end - t.begin != numel * 2) { msg = name + ": byte size does not match its shape"; return QW_ERR_FORMAT; }
        // weights are read in place as u16 (cpu_inference.rs:75-76); keep every tensor 2-byte aligned
        if (((uintptr_t)(data_ + t.begin)) % 2 != 0) { msg = name + ": data is not 2-byte aligned"; return QW_ERR_FORMAT; }
        return 0;
    };
    const int64_t H = (int64_t)c.hidden, I = (int64_t)c.inter, D = (int64_t)c.head_dim;
    const int64_t QD = (int64_t)c.heads * D, KVD = (int64_t)c.kv_heads * D, V = (int64_t)c.vocab;
    int rc;
    if ((rc = need("model.embed_tokens.weight", {V, H}))) return rc;
    if ((rc = need("lm_head.weight", {V, H}))) return rc;
    if ((rc = need("model.norm.weight", {H}))) return rc;
    for (uint64_t l = 0; l < c.layers; l++) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        if ((rc = need(p + "input_layernorm.weight", {H})) || (rc = need(p + "post_attention_layernorm.weight", {H})) ||
            (rc = need(p + "self_attn.q_proj.weight", {QD, H})) || (rc = need(p + "self_attn.k_proj.weight", {KVD, H})) ||
            (rc = need(p + "self_attn.v_proj.weight", {KVD, H})) || (rc = need(p + "self_attn.o_proj.weight", {H, QD})) ||
            (rc = need(p + "self_attn.q_norm.weight", {D})) || (rc = need(p + "self_attn.k_norm.weight", {D})) ||
            (rc = need(p + "mlp.gate_proj.weight", {I, H})) || (rc = need(p + "mlp.up_proj.weight", {I, H})) ||
            (rc = need(p + "mlp.down_proj.weight", {H, I})))
            return rc;
    }
    return check_supported(c, msg);
}

const TensorView* ModelFile::find(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

const uint8_t* ModelFile::data(const std::string& name) const {
    const TensorView* t = find(name);
    return t ? data_ + t->begin : nullptr;
}

uint64_t ModelFile::weight_bytes_per_token() const {
    uint64_t bytes = 0;
    for (auto& kv : tensors_)
        if (kv.first != "model.embed_tokens.weight") bytes += kv.second.end - kv.second.begin;
    return bytes + cfg_.hidden * 2;
}

int check_supported(const ModelConfig& c, std::string& msg) {
    // a GEMV width K is supported when it is a multiple of 256 and at most 1024 (one segment), or a
    // multiple of 1024 whose 1024-column segment count divides the decode kernel's 12 consumer
    // warps (seg_count in decode_kernel.cuh)
    auto seg_ok = [](uint64_t K) {
        if (K == 0 || K % 256 != 0) return false;
        if (K <= 1024) return true;
        return K % 1024 == 0 && 12 % (K / 1024) == 0;
    };
    if (c.layers == 0 || c.vocab == 0 || c.heads == 0 || c.kv_heads == 0) { msg = "config: zero-sized dimension"; return QW_ERR_FORMAT; }
    if (c.head_dim != 128) { msg = "unsupported head_dim (the kernels fix it at 128, like inference.metal's attention)"; return QW_ERR_UNSUPPORTED; }
    if (c.heads % c.kv_heads != 0) { msg = "num_attention_heads must be a multiple of num_key_value_heads"; return QW_ERR_UNSUPPORTED; }
    if (c.heads / c.kv_heads > 3) { msg = "more than 3 query heads per KV head is not supported"; return QW_ERR_UNSUPPORTED; }
    if (!seg_ok(c.hidden) || !seg_ok(c.inter) || !seg_ok(c.heads * c.head_dim)) {
        msg = "hidden_size, intermediate_size and heads*head_dim must be multiples of 256 up to 1024, or split into 1, 2, 3, 4, 6 or 12 segments of 1024 columns";
        return QW_ERR_UNSUPPORTED;
    }
    if (c.vocab >= (1ull << 31)) { msg = "vocab_size too large"; return QW_ERR_UNSUPPORTED; }
    if (!(c.eps > 0.f) || !(c.theta > 0.f)) { msg = "rms_norm_eps and rope_theta must be positive"; return QW_ERR_FORMAT; }
    return 0;
}

}  // namespace qw
