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

// most K splits of one GEMM; split z writes its own [n][N] slice of Scratch::Y
constexpr int KSPLIT_MAX = 16;

// most rows of one row-mode step (the skinny GEMM's activation rows)
constexpr int ROWS_MAX = 16;

// K splits of an [M x N] x K GEMM: enough to come near one CTA per SM when the output tiles alone
// would leave SMs idle, at most KSPLIT_MAX and K / 64
int ksplit_for(int M, int N, int K);

// One row of a row-mode step (a decode batch): sequence b's cache and position. Lives in device
// memory; the step's argmax advances `pos`, so a captured step replays without host writes.
struct RowView {
    float* k;                  // cache K [layer][kv_head][max_seq][128]
    float* v;                  // cache V, same layout
    const float2* rope;        // cache RoPE table [max_seq][64]
    int max_seq;
    int pos;                   // position of the row's input token this step
    int start;                 // position of the row's first decode input (output index = pos - start)
    int pad;
};

// device scratch for n tokens
struct Scratch {
    float* X = nullptr;        // [n][H] residual stream
    float* Y = nullptr;        // GEMM outputs, ycap floats: [ksplit][n][N] for the widest use
    float* Q = nullptr;        // [n][QD] normed, rotated queries
    float* att = nullptr;      // [n][QD] attention outputs
    uint16_t* ahi = nullptr;   // [n][max(H, QD, I)] GEMM input, high bf16 halves
    uint16_t* alo = nullptr;   // ... low halves
    int cap = 0;               // tokens the buffers hold
    float* attp = nullptr;     // attention partials of split query tiles
    size_t attp_cap = 0;       // floats attp holds
    size_t ycap = 0;           // floats Y holds
    unsigned* att_tickets = nullptr;  // row mode: [ROWS_MAX][NKV] split arrivals, zero between launches
    float* row_ssq = nullptr;  // row mode: [2][ROWS_MAX][NORM_BLOCKS_MAX] per-block sums of squares of the norms
};

// row mode: the most 128-column blocks a hidden row splits into for the block-parallel norm
constexpr int NORM_BLOCKS_MAX = 64;

// floats of Scratch::Y a pass over n rows needs (largest ksplit x n x N over the four GEMMs)
size_t y_floats(int n, int H, int I, int NQ, int NKV);

// floats of attention partials a pass over n tokens from position `start` needs
size_t attention_partial_floats(int n, int start, int NQ, int NKV);

// One forward pass over n tokens d_ids (device) at positions start .. start+n-1: writes their K/V
// into the cache and, with d_logits ([n][V] device), every position's logits. Stream-ordered.
int run(const Weights& w, const CacheView& c, const uint32_t* d_ids, int n, int start, float* d_logits, Scratch& sc,
        int* err_word, cudaStream_t s, std::string& err);

// Positions per attention split of a row-mode step
constexpr int ROW_SPLIT = 64;

// floats of attention partials a row-mode step over B rows with `splits` position splits needs
size_t row_partial_floats(int B, int NQ, int splits);

// One row-mode step over B rows (B <= ROWS_MAX): row b feeds d_tok[b] at d_rows[b].pos into its
// own cache and, with d_logits ([B][V]), gets its logits. `splits` position splits of ROW_SPLIT
// cover every row's positions (pos < splits * ROW_SPLIT). distinct_caches: no two rows share a
// cache, so each attention CTA may form its own row's q, k and v (no separate qkv_post pass); rows
// that share a cache (a lookup verify pass) need every row's K/V written before any attention.
// Stream-ordered; capturable.
int run_rows(const Weights& w, const RowView* d_rows, int B, int splits, bool distinct_caches, const uint32_t* d_tok,
             float* d_logits, Scratch& sc, int* err_word, cudaStream_t s, std::string& err);

// device scratch of the row argmax: per row, the best (value, index) of each of its AR_PARTS
// blocks and an arrival ticket (zero between launches)
constexpr int AR_PARTS = 16;
struct ArgmaxScratch {
    float val[ROWS_MAX][AR_PARTS];
    unsigned idx[ROWS_MAX][AR_PARTS];
    unsigned ticket[ROWS_MAX];
};

// Greedy step end for B rows: d_tok[b] = argmax(d_logits[b]) (the reference CPU rule),
// d_out[(pos - start) * B + b] = the same token, then pos += 1. Stream-ordered; capturable.
int argmax_rows(const float* d_logits, int V, int B, RowView* d_rows, uint32_t* d_tok, uint32_t* d_out, ArgmaxScratch* sc,
                cudaStream_t s, std::string& err);

// d_out[t] = argmax(d_logits[t]) for t < n <= ROWS_MAX (the reference CPU rule). Stream-ordered.
int argmax_each(const float* d_logits, int V, int n, uint32_t* d_out, ArgmaxScratch* sc, cudaStream_t s, std::string& err);

}  // namespace pf
}  // namespace qw
