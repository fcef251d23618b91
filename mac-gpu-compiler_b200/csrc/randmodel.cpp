// Seeded random-init Qwen3 checkpoint writer.
//
// Writes a safetensors file with the Hugging Face Qwen3 tensor names and shapes, the same set
// the reference engine reads (metal_infrence_engine/src/cpu_inference.rs:109-177), so that the
// reference loader, its bytes-per-token rule (tests/mbu.rs:19-30) and this repo's engine all
// apply unchanged. Values: linear weights and the embedding ~ N(0, 0.02), RMSNorm gains
// 1 + N(0, 0.01), all rounded to bf16 (round-to-nearest-even). `lm_head.weight` is a byte copy
// of `model.embed_tokens.weight` (Qwen3-0.6B ties them) stored under its own name.
//
// The normal deviates come from a counter-based generator (splitmix64 of (seed, tensor, index)
// followed by Box-Muller in double), so the file is identical for any thread count and fast to
// produce: about 1.5 GB for the full 0.6B geometry in a few seconds.
//
// Host-only C++; built into librandmodel.so. Not part of the CUDA engine.

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace {

struct Spec {
    uint32_t hidden, inter, layers, heads, kv_heads, head_dim, vocab;
};

struct TensorDesc {
    std::string name;
    std::vector<uint64_t> shape;
    double mean, std;   // value = mean + std * N(0,1)
    int copy_of;        // >= 0: byte copy of that tensor (tied lm_head)
    uint64_t offset;    // into the data section
    uint64_t numel() const { uint64_t n = 1; for (auto d : shape) n *= d; return n; }
};

inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// element pair k of tensor `ti`: two independent standard normals
inline void normal_pair(uint64_t key, uint64_t k, double* z0, double* z1) {
    uint64_t h1 = splitmix64(key ^ (2 * k));
    uint64_t h2 = splitmix64(key ^ (2 * k + 1) ^ 0xD1B54A32D192ED03ull);
    double u1 = ((double)(h1 >> 11) + 0.5) * (1.0 / 9007199254740992.0);  // (0, 1)
    double u2 = (double)(h2 >> 11) * (1.0 / 9007199254740992.0);          // [0, 1)
    double r = std::sqrt(-2.0 * std::log(u1));
    double a = 6.283185307179586 * u2;
    *z0 = r * std::cos(a);
    *z1 = r * std::sin(a);
}

void fill_tensor(uint16_t* dst, const TensorDesc& t, uint64_t seed, int ti, int nthreads) {
    const uint64_t n = t.numel();
    const uint64_t key = splitmix64(seed * 0x100000001B3ull + 0x51ED27ull) ^ splitmix64(0xA5A5ull + (uint64_t)ti);
    const uint64_t pairs = (n + 1) / 2;
    auto work = [&](uint64_t p0, uint64_t p1) {
        const float mean = (float)t.mean, sd = (float)t.std;
        for (uint64_t k = p0; k < p1; k++) {
            double z0, z1;
            normal_pair(key, k, &z0, &z1);
            uint64_t i = 2 * k;
            dst[i] = f32_to_bf16_rne(mean + sd * (float)z0);
            if (i + 1 < n) dst[i + 1] = f32_to_bf16_rne(mean + sd * (float)z1);
        }
    };
    if (pairs < (1u << 16) || nthreads <= 1) { work(0, pairs); return; }
    std::vector<std::thread> th;
    uint64_t per = (pairs + nthreads - 1) / nthreads;
    for (int i = 0; i < nthreads; i++) {
        uint64_t a = (uint64_t)i * per, b = std::min(pairs, a + per);
        if (a < b) th.emplace_back(work, a, b);
    }
    for (auto& x : th) x.join();
}

std::vector<TensorDesc> tensor_list(const Spec& s) {
    std::vector<TensorDesc> v;
    const double W = 0.02, G = 0.01;
    auto add = [&](std::string name, std::vector<uint64_t> shape, double mean, double sd, int copy = -1) {
        v.push_back(TensorDesc{std::move(name), std::move(shape), mean, sd, copy, 0});
    };
    add("model.embed_tokens.weight", {s.vocab, s.hidden}, 0.0, W);
    const uint64_t qd = (uint64_t)s.heads * s.head_dim, kvd = (uint64_t)s.kv_heads * s.head_dim;
    for (uint32_t l = 0; l < s.layers; l++) {
        std::string p = "model.layers." + std::to_string(l) + ".";
        add(p + "input_layernorm.weight", {s.hidden}, 1.0, G);
        add(p + "self_attn.q_proj.weight", {qd, s.hidden}, 0.0, W);
        add(p + "self_attn.k_proj.weight", {kvd, s.hidden}, 0.0, W);
        add(p + "self_attn.v_proj.weight", {kvd, s.hidden}, 0.0, W);
        add(p + "self_attn.o_proj.weight", {s.hidden, qd}, 0.0, W);
        add(p + "self_attn.q_norm.weight", {s.head_dim}, 1.0, G);
        add(p + "self_attn.k_norm.weight", {s.head_dim}, 1.0, G);
        add(p + "post_attention_layernorm.weight", {s.hidden}, 1.0, G);
        add(p + "mlp.gate_proj.weight", {s.inter, s.hidden}, 0.0, W);
        add(p + "mlp.up_proj.weight", {s.inter, s.hidden}, 0.0, W);
        add(p + "mlp.down_proj.weight", {s.hidden, s.inter}, 0.0, W);
    }
    add("model.norm.weight", {s.hidden}, 1.0, G);
    add("lm_head.weight", {s.vocab, s.hidden}, 0.0, 0.0, 0);
    return v;
}

}  // namespace

extern "C" {

// Writes `path` (a .safetensors file). Returns 0 on success, -1 on I/O or size errors.
// The caller writes config.json beside it.
int rm_write_model(const char* path, uint32_t hidden, uint32_t inter, uint32_t layers, uint32_t heads,
                   uint32_t kv_heads, uint32_t head_dim, uint32_t vocab, uint64_t seed, int nthreads) {
    Spec s{hidden, inter, layers, heads, kv_heads, head_dim, vocab};
    if (nthreads <= 0) nthreads = (int)std::max(1u, std::thread::hardware_concurrency());
    auto ts = tensor_list(s);
    uint64_t off = 0;
    for (auto& t : ts) { t.offset = off; off += t.numel() * 2; }
    // the reference stores data_offsets as i32 (cpu_inference.rs:17): keep files under 2 GiB
    if (off >= (1ull << 31)) return -1;

    std::string hdr = "{\"__metadata__\":{\"format\":\"pt\"}";
    for (auto& t : ts) {
        hdr += ",\"" + t.name + "\":{\"dtype\":\"BF16\",\"shape\":[";
        for (size_t i = 0; i < t.shape.size(); i++) hdr += (i ? "," : "") + std::to_string(t.shape[i]);
        hdr += "],\"data_offsets\":[" + std::to_string(t.offset) + "," + std::to_string(t.offset + t.numel() * 2) + "]}";
    }
    hdr += "}";
    while ((8 + hdr.size()) % 16 != 0) hdr += ' ';  // data section starts 16-byte aligned

    std::vector<uint16_t> data(off / 2);
    for (size_t ti = 0; ti < ts.size(); ti++) {
        auto& t = ts[ti];
        uint16_t* dst = data.data() + t.offset / 2;
        if (t.copy_of >= 0) {
            auto& src = ts[t.copy_of];
            std::memcpy(dst, data.data() + src.offset / 2, src.numel() * 2);
        } else {
            fill_tensor(dst, t, seed, (int)ti, nthreads);
        }
    }
    FILE* f = std::fopen(path, "wb");
    if (!f) return -1;
    uint64_t hl = hdr.size();
    unsigned char lenb[8];
    for (int i = 0; i < 8; i++) lenb[i] = (unsigned char)(hl >> (8 * i));
    bool ok = std::fwrite(lenb, 1, 8, f) == 8 && std::fwrite(hdr.data(), 1, hl, f) == hl &&
              std::fwrite(data.data(), 2, data.size(), f) == data.size();
    ok = (std::fclose(f) == 0) && ok;
    return ok ? 0 : -1;
}

}  // extern "C"
