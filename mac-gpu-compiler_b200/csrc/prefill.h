// Batched prefill interface between the engine (which owns the model and cache) and prefill.cu.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>

#include <cuda_runtime.h>

namespace qw {
namespace pf {

// device weights in the engine's repacked layout (see engine.cu: per layer q|k|v, o, gate/up
// interleaved by row, down; norms per layer: input, post-attention, q_norm, k_norm)
struct Weights {
    const uint16_t* layer_w;
    const uint16_t* layer_n;
    const uint16_t* final_norm;
    const uint16_t* embed;
    const uint16_t* lm_head;
    long long layer_stride, norm_stride;
    int H, I, L, NQ, NKV, V;
    float eps;
};

// the KV cache: K and V [layer][kv_head][max_seq][128] f32, RoPE table [max_seq][64] (cos, sin)
struct CacheView {
    float* k;
    float* v;
    const float2* rope;
    int max_seq;
};

// most K splits of one GEMM; each split writes its own [n][H] slice of Scratch::Y
constexpr int KSPLIT_MAX = 4;

// device scratch for n tokens
struct Scratch {
    float* X = nullptr;        // [n][H] residual stream
    float* Y = nullptr;        // [n][max(QKVR, 2I, KSPLIT_MAX * H)] GEMM outputs
    float* Q = nullptr;        // [n][QD] normed, rotated queries
    float* att = nullptr;      // [n][QD] attention outputs
    uint16_t* ahi = nullptr;   // [n][max(H, QD, I)] GEMM input, high bf16 halves
    uint16_t* alo = nullptr;   // ... low halves
    int cap = 0;               // tokens the buffers hold
    float* attp = nullptr;     // attention partials of split query tiles
    size_t attp_cap = 0;       // floats attp holds
};

// floats of attention partials a pass over n tokens from position `start` needs
size_t attention_partial_floats(int n, int start, int NQ, int NKV);

// One forward pass over n tokens d_ids (device) at positions start .. start+n-1: writes their K/V
// into the cache and, with d_logits ([n][V] device), every position's logits. Stream-ordered.
int run(const Weights& w, const CacheView& c, const uint32_t* d_ids, int n, int start, float* d_logits, Scratch& sc,
        int* err_word, cudaStream_t s, std::string& err);

}  // namespace pf
}  // namespace qw
