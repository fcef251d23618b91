// Persistent weight-streaming decode kernel for batch-1 Qwen3 (sm_100a).
//
// One cooperative launch runs `steps` whole tokens: embed -> L x [rmsnorm, q|k|v GEMV, per-head
// q/k RMSNorm + RoPE, KV append, GQA attention, o GEMV + residual, rmsnorm, gate|up GEMV + SiLU*up,
// down GEMV + residual] -> final rmsnorm -> lm_head GEMV -> argmax -> next token's embed.
// It is the same math as the reference CPU engine (metal_infrence_engine/src/cpu_inference.rs:
// 100-179) and replaces its Metal twin (metal_inference.rs:320-387, inference.metal:98-346).
//
// Layout of the work (one CTA per SM, grid = SM count, all CTAs co-resident):
//   * warp 12 (one elected lane) is the PRODUCER. It walks the CTA's static schedule and streams
//     every weight tile and every cached K/V tile the CTA will need, in order, into an 8-slot x
//     24 KB shared-memory ring with 1-D TMA bulk copies (cp.async.bulk, no multicast). None of
//     those bytes depends on the token being decoded, so the producer runs ahead of the math by
//     up to 192 KB per SM across phase, layer and token boundaries: HBM keeps streaming while
//     the consumers wait for their inputs.
//   * warps 0..11 are CONSUMERS. Each GEMV phase gives every CTA a contiguous block of output
//     rows; a ring slot holds whole rows, and a (row, 1024-column segment) unit is one warp's dot
//     product against the activation vector it holds in registers. Epilogues are fused: q|k|v
//     rows are written raw; o/down add the residual (each CTA keeps its residual rows in shared
//     memory); gate/up rows are interleaved so the SiLU*up product is formed in the CTA; lm_head
//     rows feed a per-CTA argmax partial.
//   * Hand-off between phases uses TAGGED WORDS: every activation element crosses CTAs as one
//     64-bit word {f32 value, 32-bit tag}, the tag naming the launch (epoch) and the phase that
//     wrote it. 8-byte stores are single-copy atomic, so a consumer that reads the tag it expects
//     has the value that goes with it: polling the input IS the synchronisation, with no fence and
//     no separate flag round trip. A buffer is rewritten only after every CTA has consumed the
//     previous contents (each phase needs all of the previous phase's outputs), so tags never
//     race with a reader.
//   * Attention: each KV head's positions are split into up to S contiguous chunks, one CTA per
//     (kv head, chunk). A CTA applies q_norm/k_norm + RoPE itself; the CTA whose chunk holds `pos`
//     also writes the new K/V into the cache; each CTA publishes an online-softmax partial for its
//     G query heads as tagged words, and the chunk-0 CTA merges them in chunk order
//     (deterministic) into the attention output.
//   * One grid barrier per token (after lm_head: the argmax needs every CTA's partial, and the next
//     token's K/V reads need the previous token's K/V writes) built from per-CTA release flags.
//
// Every wait is bounded in time; on expiry the kernel records an error, stops waiting anywhere
// (fast-forwards to the end without blocking), waits (bounded) for its own bulk copies in flight
// and returns. The host reports the error.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "ptx.cuh"

namespace qw {

constexpr int NCW = 12;                       // consumer warps
constexpr int NCT = NCW * 32;                 // consumer threads
constexpr int NTHREADS = NCT + 32;            // + producer warp
constexpr int NSLOT = 8;                      // ring slots
constexpr int SLOT_BYTES = 24 * 1024;         // bytes per slot
constexpr int HD = 128;                       // head_dim (the reference's attention kernel also fixes it)
constexpr int ATT_P = SLOT_BYTES / (2 * HD * 4);  // cached positions per attention ring slot (24)
constexpr int MAX_G = 3;                      // query heads per KV head
constexpr int MAX_S = 18;                     // attention chunks per KV head
constexpr int MIN_CHUNK = 48;                 // default fewest positions per attention chunk (DecodeParams::min_chunk)
constexpr uint32_t LM_PREFETCH_BYTES = 256u * 1024;  // lm_head bytes per CTA warmed into L2 ahead of use
constexpr int APART_STRIDE = HD + 4;          // words per attention partial: acc[128], m, l, pad
constexpr int ATT_WST = HD + 4;               // floats per (warp, head) softmax state staged in part: acc[128], m, l, pad
constexpr int GP = 4;
enum : int { EPI_PART = 0, EPI_STORE = 1, EPI_SILU = 2 };  // GEMV epilogues (see gemv_full_segments)                         // tagged word pairs a consumer thread polls at once
constexpr uint32_t NONE_IDX = 0xFFFFFFFFu;
// Math: the softmax / SiLU exponentials use __expf and the RMSNorm scales rsqrtf (hardware
// approximations, ~1e-6 relative error): the inline IEEE expansions of expf and 1/sqrtf would
// roughly double the code that every layer executes, which costs far more in instruction fetch
// than the accuracy is worth against the 1e-2 logit bar (results stay ~1e-5 from the CPU oracle).
// phase timeline (optional): per layer, stamps after: 0 layer start, 1 A input ready (x gathered +
// rmsnorm), 2 A rows stored, 3 B inputs ready (q/k/v gathered, norm+RoPE), 4 B chunk done,
// 5 B merged/published, 6 C input ready (att gathered), 7 C rows stored, 8 D input ready,
// 9 D rows stored, 10 E input ready (h gathered), 11 E rows stored, 12 (merging CTAs) partials
// polled, 13 (merging CTAs) attention output published; then 4 stamps for the token
// tail: lm_head input ready, lm_head done, end-of-token barrier passed, next token known
constexpr int TRACE_PER_LAYER = 14;

// error codes written to DecodeParams::err[0]
enum : int { DERR_NONE = 0, DERR_TIMEOUT_GRID = 1, DERR_TIMEOUT_FULL = 2, DERR_TIMEOUT_EMPTY = 3,
             DERR_TIMEOUT_KV = 4, DERR_BAD_TOKEN = 5, DERR_TIMEOUT_DRAIN = 6, DERR_TIMEOUT_DATA = 7,
             DERR_SHAPE = 8 };

typedef unsigned long long u64;

struct DecodeParams {
    // weights (bf16 bit patterns)
    const uint16_t* layer_w;     // per layer: qkv[QD+2*KVD][H] | o[H][QD] | gu[2I][H] (gate/up interleaved by row) | down[H][I]
    const uint16_t* layer_n;     // per layer: ln1[H] | ln2[H] | q_norm[128] | k_norm[128]
    const uint16_t* final_norm;  // [H]
    const uint16_t* embed;       // [V][H]
    const uint16_t* lm_head;     // [V][H]
    // KV cache, [L][KVH][max_seq][128] f32 each, and the RoPE table [max_seq][64] (cos, sin)
    float* kc;
    float* vc;
    const float2* rope;
    // tagged activation words {f32 value | tag << 32}
    u64* x;                      // [H] residual stream
    u64* qkv;                    // [QD + 2*KVD] raw projections
    u64* hbuf;                   // [I] SiLU(gate)*up
    u64* att;                    // [QD] attention output
    u64* apart;                  // [KVH][S][G][APART_STRIDE] attention partials
    // argmax partials and the per-token barrier
    float* am_val;               // [grid]
    unsigned* am_idx;            // [grid]
    int* nan0;                   // logits[0] is NaN (the CPU argmax then returns 0)
    u64* flags;                  // [grid] barrier flags: epoch << 32 | tokens finished
    int* err;                    // [4] code, cta, where, detail
    float* logits;               // [V] or null (decode skips it)
    u64* trace;                  // [grid][TRACE_PER_LAYER * L + 4] globaltimer stamps of step 0, or null
    // tokens
    const uint32_t* tok_in;      // step 0 input token (device memory)
    uint32_t* tok_out;           // [steps + 1] or null: tok_out[i + 1] = argmax of step i
    uint32_t* host_tok;          // mapped pinned host memory [steps + 1] or null
    unsigned* host_count;        // mapped pinned host counter or null
    long long layer_stride;      // elements between layers in layer_w
    long long norm_stride;       // elements between layers in layer_n
    int H, I, L, NQ, NKV, V, max_seq;
    int start_pos, steps;
    unsigned epoch;
    float eps, scale;
    int S;                       // attention chunks per KV head (<= MAX_S)
    int part_cap;                // floats in the shared partial-sum buffer
    int xs_cap;                  // floats in the shared activation buffer
    int xloc_cap;                // floats in the shared residual-rows buffer
    long long timeout_ns;
    int poll_ns;                 // back-off between unsuccessful polling rounds of tagged words (0 = none)
    int min_chunk;               // fewest positions per attention chunk (larger: fewer chunk CTAs to merge)
    int stall_cta;               // test hook (-1: off): this CTA never raises its first end-of-token flag,
                                 // so every CTA's bounded barrier wait runs out and the launch reports it
};

// static row partition of a GEMV phase for one CTA
struct GemvGeo {
    int r0, r1;       // output rows [r0, r1)
    int K;            // columns
    int rpp;          // rows per ring slot
    int segs;         // column segments per row (K / segw), see seg_count
    int segw;         // columns per segment (<= 1024)
    int cpl;          // 16-byte chunks per lane per segment (segw / 256)
    long long woff;   // element offset of the matrix inside a layer block
};

// Column segments per row: rows of up to 1024 columns are one segment; wider rows split into
// 1024-column segments, and their count must divide the 12 consumer warps (so that each warp keeps
// one fixed segment of x in registers).
__host__ __device__ inline int seg_count(int K) {
    if (K <= 0 || K % 256 != 0) return 0;
    if (K <= 1024) return 1;
    return (K % 1024 == 0 && 12 % (K / 1024) == 0) ? K / 1024 : 0;
}

// Shared-memory layout of a GEMV input vector: within each block of 256 columns, lane l's two
// float4 of columns 8l .. 8l+3 and 8l+4 .. 8l+7 are stored at float4 slots l and 32 + l, so the
// warp-wide float4 loads of a 1024-column segment are contiguous 512-byte accesses (no bank
// conflicts). Consecutive even/odd columns stay adjacent.
__host__ __device__ inline int xperm(int c) {
    return (c & ~255) | ((c & 4) << 5) | (((c >> 3) & 31) << 2) | (c & 3);
}

// per consumer warp, per GEMV phase: what the warp does in each ring piece
struct WarpGeo {
    int npieces;      // ring pieces of the phase
    int myseg;        // the column segment this warp holds in registers
    int rl;           // the row of each piece this warp works on
    int wbyte;        // byte offset of that row's segment within a piece
};

// `unit` (dividing the outputs) makes every CTA's share of outputs a whole number of units, so a
// unit of 8 gives each CTA whole 64-byte blocks of the 8-byte hand-off words it publishes. Blocks
// written by one CTA alone hand off faster: where CTAs' ranges share sectors, their stores and the
// other CTAs' polls of those sectors contend (one all-CTA hand-off round of a 1024-word vector
// measured 1.5 us with shared sectors, 0.9 us with one 64-byte block per CTA). Some CTAs may then
// own no rows of a phase.
__device__ inline GemvGeo make_geo(long long rows, int K, int cta, int n, long long woff, int pair, int unit = 1) {
    GemvGeo g;
    if (pair) {  // gate/up: partition pairs so each CTA owns whole (gate_i, up_i) row pairs
        long long U = rows / 2 / unit;
        g.r0 = (int)(2 * unit * (U * cta / n));
        g.r1 = (int)(2 * unit * (U * (cta + 1) / n));
    } else {
        long long U = rows / unit;
        g.r0 = (int)(unit * (U * cta / n));
        g.r1 = (int)(unit * (U * (cta + 1) / n));
    }
    g.K = K;
    g.rpp = SLOT_BYTES / (2 * K);
    g.segs = seg_count(K);
    g.segw = K / g.segs;
    g.cpl = g.segw / 256;
    g.woff = woff;
    return g;
}

__device__ inline WarpGeo make_warp_geo(const GemvGeo& g, int w) {
    WarpGeo wg;
    wg.npieces = (g.r1 - g.r0 + g.rpp - 1) / g.rpp;
    wg.myseg = g.segs ? w % g.segs : 0;
    wg.rl = g.segs ? w / g.segs : 0;
    wg.wbyte = (wg.rl * g.K + wg.myseg * g.segw) * 2;
    return wg;
}

// attention work item of a CTA at a given position (same answer in producer and consumers)
struct AttnItem {
    int g, s, t0, t1, S_eff;
    bool active, has_cur;
};

__device__ inline AttnItem attn_item(const DecodeParams& p, int cta, int pos) {
    AttnItem a;
    const int n_t = pos + 1;
    int chunk = (n_t + p.S - 1) / p.S;
    if (chunk < p.min_chunk) chunk = p.min_chunk;
    a.S_eff = (n_t + chunk - 1) / chunk;
    a.g = cta / p.S;
    a.s = cta % p.S;
    a.active = (cta < p.NKV * p.S) && (a.s < a.S_eff);
    a.t0 = a.s * chunk;
    a.t1 = min(n_t, a.t0 + chunk);
    a.has_cur = a.active && (a.t1 == n_t);
    return a;
}

struct LoopState {
    int step;        // token of the launch being decoded
    int l;           // layer
    unsigned token;  // input token of the current step (consumers)
};

struct Smem {
    // qs / ks / vs are accessed as float4: keep them 16-byte aligned
    __align__(16) float qs[MAX_G][HD];
    __align__(16) float ks[HD];
    __align__(16) float vs[HD];
    GemvGeo geo[5];              // this CTA's rows of phases A (q|k|v), C (o), D (gate|up), E (down), F (lm_head)
    WarpGeo wgeo[5][NCW];        // per phase and consumer warp (see WarpGeo)
    float ml[MAX_S][MAX_G][2];   // attention partials' (m, l) gathered by the merging CTA
    float red[64];
    float ssq[NCW];              // per consumer warp: sum of squares of the last RMSNorm input
    float redv[NCW];
    unsigned redi[NCW];
    uint64_t full[NSLOT];
    uint64_t empty[NSLOT];
    DecodeParams prm;              // the launch's parameters (read by every phase routine)
    uint32_t ring_it[NCW + 1];     // per warp: ring pieces consumed (consumers) or walked (producer)
    uint32_t n_issued;             // producer: pieces whose copies were issued
    LoopState loop[NCW + 1];       // per warp: token/layer loop state (see Decoder::ls)
    uint32_t progress;   // tokens whose end-of-token barrier this CTA's consumers have passed
    int abort;           // set once any wait expired
    unsigned token;
};

static_assert(offsetof(Smem, qs) % 16 == 0 && offsetof(Smem, ks) % 16 == 0 && offsetof(Smem, vs) % 16 == 0,
              "float4-accessed shared arrays must be 16-byte aligned");
static_assert(offsetof(Smem, full) % 8 == 0 && offsetof(Smem, empty) % 8 == 0, "mbarriers must be 8-byte aligned");

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

__device__ __forceinline__ float dot8(uint4 w, const float* x) {
    float a = bf16_lo(w.x) * x[0];
    float b = bf16_hi(w.x) * x[1];
    a = fmaf(bf16_lo(w.y), x[2], a);
    b = fmaf(bf16_hi(w.y), x[3], b);
    a = fmaf(bf16_lo(w.z), x[4], a);
    b = fmaf(bf16_hi(w.z), x[5], b);
    a = fmaf(bf16_lo(w.w), x[6], a);
    b = fmaf(bf16_hi(w.w), x[7], b);
    return a + b;
}

// Packed-f32 form of dot8 (Blackwell's two-lane FFMA2): the 8 products are accumulated into
// (acc.x, acc.y) in place, so a 16-byte chunk costs 8 bf16 conversions and 4 FMA instructions.
__device__ __forceinline__ float2 dot8_acc2(uint4 w, const float* x, float2 acc) {
    acc = __ffma2_rn(make_float2(bf16_lo(w.x), bf16_hi(w.x)), make_float2(x[0], x[1]), acc);
    acc = __ffma2_rn(make_float2(bf16_lo(w.y), bf16_hi(w.y)), make_float2(x[2], x[3]), acc);
    acc = __ffma2_rn(make_float2(bf16_lo(w.z), bf16_hi(w.z)), make_float2(x[4], x[5]), acc);
    acc = __ffma2_rn(make_float2(bf16_lo(w.w), bf16_hi(w.w)), make_float2(x[6], x[7]), acc);
    return acc;
}

// argmax ordering: larger value wins, ties to the lower index, NaN never wins (NONE_IDX = empty)
__device__ __forceinline__ bool am_better(float av, unsigned ai, float bv, unsigned bi) {
    if (ai == NONE_IDX) return false;
    if (bi == NONE_IDX) return true;
    return av > bv || (av == bv && ai < bi);
}

__device__ __forceinline__ uint32_t word_tag(u64 w) { return (uint32_t)(w >> 32); }
__device__ __forceinline__ float word_val(u64 w) { return __uint_as_float((uint32_t)w); }
__device__ __forceinline__ u64 tagged(float v, uint32_t tag) { return ((u64)tag << 32) | __float_as_uint(v); }

// the kernels' shared memory: fixed-size state, then (dynamic) ring | xs | part | xloc
__shared__ Smem qw_sm;
extern __shared__ __align__(128) uint8_t qw_dyn[];

// The decoder has no per-thread object state: the launch parameters (copied into shared memory at
// launch), the ring counters and the phase geometry live at fixed shared-memory addresses, and
// everything else is re-derived from special registers. With no object whose address the
// out-of-line phase routines need, nothing sits in local memory, which on this kernel is backed
// by an L1 of only ~24 KB (shared memory takes the rest) and would miss to L2 on the critical
// path. It also keeps the kernel within the 128 registers a 13-warp CTA can have per thread.
//
// Two compile-time switches leave code out of the kernel that a launch does not need: kTrace, the
// phase-timeline stamps (qw_set_trace), and kGeneric, the GEMV routine for phases whose rows do not
// split into whole 1024-column segments (the Qwen3-0.6B shapes never need it). The kernel's speed
// depends on its code size as well as on the instructions it executes: without both, the 130 + 128
// token decode ran 2% faster (same-box A/B, 1,972 -> 2,012 tok/s). The effect is one of layout as much
// as of size: instantiating only the 2-head attention routine in this variant made it 2% slower again.
template <bool kTrace, bool kGeneric>
class DecoderT {
public:
    __device__ __forceinline__ static int tid() { return (int)threadIdx.x; }
    __device__ __forceinline__ static int warp() { return (int)(threadIdx.x >> 5); }
    __device__ __forceinline__ static int lane() { return (int)(threadIdx.x & 31); }
    __device__ __forceinline__ static int cta() { return (int)blockIdx.x; }
    __device__ __forceinline__ static int nctas() { return (int)gridDim.x; }
    __device__ __forceinline__ static uint8_t* ring() { return qw_dyn; }
    __device__ __forceinline__ static float* xs() { return reinterpret_cast<float*>(qw_dyn + NSLOT * SLOT_BYTES); }
    // ring pieces this warp has consumed (consumer warps) or walked (the producer)
    __device__ __forceinline__ static uint32_t& ring_pos() { return qw_sm.ring_it[threadIdx.x >> 5]; }
    __device__ __forceinline__ static float* part() { return xs() + qw_sm.prm.xs_cap; }
    __device__ __forceinline__ static float* xloc() { return part() + qw_sm.prm.part_cap; }
    __device__ __forceinline__ static int QD() { return qw_sm.prm.NQ * HD; }
    __device__ __forceinline__ static int KVD() { return qw_sm.prm.NKV * HD; }
    __device__ __forceinline__ static int G() { return qw_sm.prm.NQ / qw_sm.prm.NKV; }
    __device__ __forceinline__ static int QKVR() { return QD() + 2 * KVD(); }
    // this CTA's static row partition of phases A (q|k|v), C (o), D (gate|up), E (down), F (lm_head)
    __device__ __forceinline__ static const GemvGeo& gA() { return qw_sm.geo[0]; }
    __device__ __forceinline__ static const GemvGeo& gC() { return qw_sm.geo[1]; }
    __device__ __forceinline__ static const GemvGeo& gD() { return qw_sm.geo[2]; }
    __device__ __forceinline__ static const GemvGeo& gE() { return qw_sm.geo[3]; }
    __device__ __forceinline__ static const GemvGeo& gF() { return qw_sm.geo[4]; }

    // one thread, before the CTA-wide barrier that follows mbarrier initialisation
    __device__ static void init_geometry(const DecodeParams& p) {
        const int c = blockIdx.x, nc = gridDim.x;
        const long long qd = (long long)p.NQ * HD, kvd = (long long)p.NKV * HD, qkvr = qd + 2 * kvd;
        const long long offC = qkvr * p.H;
        const long long offD = offC + (long long)p.H * qd;
        const long long offE = offD + 2LL * p.I * p.H;
        qw_sm.geo[0] = make_geo(qkvr, p.H, c, nc, 0, 0, qkvr % 8 == 0 && qkvr / 8 >= nc ? 8 : 1);
        // q|k|v rows (A), x rows (C, E) and h values (D) in 64-byte units where the widths allow (see
        // make_geo). Every CTA still owns rows of phase A (q|k|v units only when there are at least as
        // many units as CTAs): the buffer-reuse argument (every phase's input is complete only after
        // every CTA has read the previous contents) runs through phase A
        const int ux = p.H % 8 == 0 ? 8 : 1, uh = p.I % 8 == 0 ? 8 : 1;
        qw_sm.geo[1] = make_geo(p.H, (int)qd, c, nc, offC, 0, ux);
        qw_sm.geo[2] = make_geo(2LL * p.I, p.H, c, nc, offD, 1, uh);
        qw_sm.geo[3] = make_geo(p.H, p.I, c, nc, offE, 0, ux);
        qw_sm.geo[4] = make_geo(p.V, p.H, c, nc, 0, 0);
        for (int k = 0; k < 5; k++)
            for (int w = 0; w < NCW; w++) qw_sm.wgeo[k][w] = make_warp_geo(qw_sm.geo[k], w);
        if constexpr (!kGeneric) {  // the host picked the variant without the generic routine: confirm it
            const bool part[5] = {false, true, false, true, true};  // EPI of A, C, D, E, F
            for (int k = 0; k < 5; k++)
                if (!full_segments(qw_sm.geo[k], part[k])) fail(DERR_SHAPE, k);
        }
    }

    // phase sequence numbers within the launch -> tags (12 bits of epoch, 20 bits of sequence)
    __device__ static uint32_t seq(int step, int l, int ph) {  // ph: 1 A, 2 B, 3 C, 4 D, 5 E
        const volatile DecodeParams& p = qw_sm.prm;
        return (uint32_t)step * (uint32_t)(5 * p.L + 1) + (uint32_t)(5 * l + ph);
    }
    __device__ static uint32_t tag(uint32_t sq) {
        const volatile DecodeParams& p = qw_sm.prm;
        return ((p.epoch & 0xFFFu) << 20) | (sq & 0xFFFFFu);
    }

    __device__ __forceinline__ static void stamp(int step, int idx) {
        const volatile DecodeParams& p = qw_sm.prm;
        if constexpr (kTrace) {
            if (p.trace != nullptr && step == 0 && tid() == 0)
                p.trace[(size_t)cta() * (TRACE_PER_LAYER * p.L + 4) + idx] = globaltimer_ns();
        } else {
            (void)p;
            (void)step;
            (void)idx;
        }
    }


    // ------------------------------------------------------------------ errors and waits
    __device__ static bool aborted() { return *reinterpret_cast<volatile const int*>(&qw_sm.abort) != 0; }

    __device__ __noinline__ static void fail(int code, int where) {
        const DecodeParams& p = qw_sm.prm;
        *reinterpret_cast<volatile int*>(&qw_sm.abort) = 1;
        if (atomicCAS(&p.err[0], 0, code) == 0) {
            p.err[1] = cta();
            p.err[2] = where;
            __threadfence();
        }
    }

    // Called between unsuccessful polls; returns true when the caller must stop waiting. Inline and
    // nearly free on the fast path: only every 32nd call goes out of line to read the timer, the
    // CTA's abort flag and (after 50 us) the global error word. Arguments pass by value: an
    // out-of-line call per polling round, or references to the loop counters, would move the
    // polling state through the stack on every round.
    __device__ __forceinline__ static bool wait_expired(uint32_t& spins, uint64_t& t0, int code, int where) {
        if ((++spins & 31) != 0) return false;
        t0 = wait_check(spins, t0, code, where);
        return t0 == ~0ull;
    }

    // returns the (possibly started) wait start time, or ~0 when the wait must end
    __device__ __noinline__ static uint64_t wait_check(uint32_t spins, uint64_t t0, int code, int where) {
        const DecodeParams& p = qw_sm.prm;
        if (aborted()) return ~0ull;
        const uint64_t now = globaltimer_ns();
        if (spins == 32) return now;
        const uint64_t waited = now - t0;
        if (waited > 50000 && (spins & 1023) == 0 && ld_volatile_s32(p.err) != 0) {
            *reinterpret_cast<volatile int*>(&qw_sm.abort) = 1;
            return ~0ull;
        }
        if (waited > (uint64_t)p.timeout_ns) {
            fail(code, where);
            return ~0ull;
        }
        return t0;
    }

    __device__ __forceinline__ static bool wait_mbar(uint64_t* bar, uint32_t parity, int code) {
        if (mbar_try_wait(bar, parity)) return true;  // fast path: the phase already completed
        return wait_mbar_slow(bar, parity, code);
    }

    __device__ __noinline__ static bool wait_mbar_slow(uint64_t* bar, uint32_t parity, int code) {
        uint32_t& it = ring_pos();
        if (aborted()) return false;
        uint32_t spins = 0;
        uint64_t t0 = 0;
        while (!mbar_try_wait(bar, parity))
            if (wait_expired(spins, t0, code, (int)it)) return false;
        return true;
    }

    // Waits for ring pieces pc .. pc+n-1 (n <= 32) with lane j waiting on piece pc + j, so the
    // mbarrier probes of a group run side by side instead of one after another. Returns (to every
    // lane) whether all of them landed; the __syncwarp orders the lanes' later reads of every
    // piece after the probe that saw it land.
    __device__ __forceinline__ static bool wait_pieces(uint32_t pc, int n) {
        bool mine = true;
        if (lane() < n) mine = wait_mbar(&qw_sm.full[(pc + lane()) % NSLOT], ((pc + lane()) / NSLOT) & 1, DERR_TIMEOUT_FULL);
        const bool ok = __all_sync(0xFFFFFFFFu, mine);
        __syncwarp();
        return ok;
    }

    // xs[0..K) <- values of the tagged words src[0..K) once each carries `tg` (K even, src 16-byte aligned)
    //
    // With `gain` (an RMSNorm input): xs holds x * gain, and each warp's sum of x^2 goes to
    // ssq[warp]; the GEMV that follows applies the scale rsqrt(mean(x^2) + eps) to its row outputs
    // (norm_scale), which is the same product regrouped. The gains of a thread's pairs are fetched
    // before it starts polling, and the squares are summed in a fixed order (arrival order varies).
    __device__ __noinline__ static void gather(const u64* src, int K, uint32_t tg, const uint16_t* gain = nullptr) {
        const DecodeParams& p = qw_sm.prm;
        const int npairs = K >> 1;
        float ss = 0.f;
        for (int base = 0; base < npairs; base += NCT * GP) {
            unsigned pending = 0;
            uint32_t g2[GP];
            float sq[GP];
#pragma unroll
            for (int j = 0; j < GP; j++) {
                sq[j] = 0.f;
                g2[j] = 0x3F803F80u;  // (1.0, 1.0) in bf16
                if (base + tid() + j * NCT < npairs) {
                    pending |= 1u << j;
                    if (gain) g2[j] = __ldg(reinterpret_cast<const uint32_t*>(gain) + base + tid() + j * NCT);
                }
            }
            uint32_t spins = 0;
            uint64_t t0 = 0;
            while (pending && !aborted()) {
                ulonglong2 w[GP];
#pragma unroll
                for (int j = 0; j < GP; j++)
                    if (pending & (1u << j)) w[j] = ld_relaxed_v2u64(src + 2 * (base + tid() + j * NCT));
#pragma unroll
                for (int j = 0; j < GP; j++) {
                    if ((pending & (1u << j)) && word_tag(w[j].x) == tg && word_tag(w[j].y) == tg) {
                        const int i = 2 * (base + tid() + j * NCT);
                        const float a = word_val(w[j].x), b = word_val(w[j].y);
                        sq[j] = fmaf(a, a, b * b);
                        *reinterpret_cast<float2*>(xs() + xperm(i)) = make_float2(a * bf16_lo(g2[j]), b * bf16_hi(g2[j]));
                        pending &= ~(1u << j);
                    }
                }
                if (pending) {
                    if (wait_expired(spins, t0, DERR_TIMEOUT_DATA, (int)tg)) break;
                    if (p.poll_ns) __nanosleep(p.poll_ns);
                }
            }
#pragma unroll
            for (int j = 0; j < GP; j++) ss += sq[j];
        }
        if (gain) {
            ss = warp_sum(ss);
            if (lane() == 0) qw_sm.ssq[warp()] = ss;
        }
        named_bar_sync(1, NCT);
    }

    // one end-of-token grid barrier: every CTA has published `done` finished tokens
    __device__ __noinline__ static void token_barrier(uint32_t done) {
        const DecodeParams& p = qw_sm.prm;
        named_bar_sync(1, NCT);
        const u64 target = ((u64)p.epoch << 32) | done;
        if (tid() == 0 && !(cta() == p.stall_cta && done == 1)) {
            fence_acq_rel_gpu();
            st_relaxed_u64(p.flags + cta(), target);
        }
        if (warp() == 0 && !aborted()) {
            uint32_t spins = 0;
            uint64_t t0 = 0;
            for (;;) {
                bool ok = true;
                u64 v[8];
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const int j = lane() + 32 * k;
                    v[k] = j < nctas() ? ld_relaxed_u64(p.flags + j) : target;
                }
#pragma unroll
                for (int k = 0; k < 8; k++) ok &= v[k] >= target;
                for (int j = lane() + 256; j < nctas(); j += 32) ok &= ld_relaxed_u64(p.flags + j) >= target;
                if (__all_sync(0xFFFFFFFFu, ok)) break;
                int stop = 0;
                if (lane() == 0) stop = wait_expired(spins, t0, DERR_TIMEOUT_GRID, (int)done);
                if (__shfl_sync(0xFFFFFFFFu, stop, 0)) break;
            }
            fence_acq_rel_gpu();
        }
        named_bar_sync(1, NCT);
        if (tid() == 0) st_release_cta_shared(&qw_sm.progress, done);
    }

    // ------------------------------------------------------------------ consumer helpers
    // RMSNorm input of a GEMV phase (cpu_inference.rs:189-194): xs <- x * w and ssq <- the warps'
    // sums of x^2; the phase's epilogue multiplies its row outputs by norm_scale(). x is the tagged
    // residual stream, or (from_embed) the embedding row of `token`, in which case the CTA also
    // initialises its own residual rows xloc from that row.
    __device__ __noinline__ static void norm_prologue(const uint16_t* w, bool from_embed, unsigned token, uint32_t tg) {
        const DecodeParams& p = qw_sm.prm;
        if (!from_embed) {
            gather(p.x, p.H, tg, w);
            return;
        }
        const int H = p.H;
        const uint16_t* erow = p.embed + (size_t)token * H;
        float ss = 0.f;
        #pragma unroll 1
        for (int i = tid(); i < H; i += NCT) {
            const float v = bf16_to_f32(__ldg(erow + i));
            ss = fmaf(v, v, ss);
            xs()[xperm(i)] = v * bf16_to_f32(__ldg(w + i));
            if (i >= gC().r0 && i < gC().r1) xloc()[i - gC().r0] = v;
        }
        ss = warp_sum(ss);
        if (lane() == 0) qw_sm.ssq[warp()] = ss;
        named_bar_sync(1, NCT);
    }

    // 1 / sqrt(mean(x^2) + eps) of the last RMSNorm input (valid after the barrier closing its gather)
    __device__ __forceinline__ static float norm_scale() {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < NCW; w++) t += qw_sm.ssq[w];
        return rsqrtf(t / (float)qw_sm.prm.H + qw_sm.prm.eps);
    }

    // All ring pieces of one GEMV phase: part[(row - r0) * segs + seg] = partial dot product.
    // Unit u = (row u / segs, segment u % segs) of a piece goes to warp u % 12; since segs divides
    // 12 a warp always works on the same segment, whose x values it holds in registers. Lane l
    // reads 16-byte chunks l, l + 32, ... of the segment, so each shared-memory load is one
    // contiguous 512-byte warp access.
    // When a piece holds at most one unit per warp (every Qwen3-0.6B phase), pieces are taken in
    // groups of up to four: wait for all of them, issue all their loads, run the independent FMA
    // chains, release the slots, then reduce the group's rows together with one transposing
    // butterfly (6 shuffles for 4 rows). A layer phase (2-4 pieces, resident in shared memory by
    // the time its input arrives) is then one group: its cost is the shared-memory traffic, not a
    // per-piece chain of load, FMA and shuffle latencies.
    __device__ __noinline__ static void gemv_generic(const GemvGeo& gs) {
        uint32_t& it = ring_pos();
        const GemvGeo g = gs;  // loop-invariant: keep the phase geometry in registers
        const int w = warp(), ln = lane();
        const int myseg = w % g.segs;
        float xr[32];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            if (i < g.cpl) {
                const float4* xp = reinterpret_cast<const float4*>(xs() + myseg * g.segw) + i * 64 + ln;
                float4 a = xp[0], b = xp[32];
                xr[i * 8 + 0] = a.x; xr[i * 8 + 1] = a.y; xr[i * 8 + 2] = a.z; xr[i * 8 + 3] = a.w;
                xr[i * 8 + 4] = b.x; xr[i * 8 + 5] = b.y; xr[i * 8 + 6] = b.z; xr[i * 8 + 7] = b.w;
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) xr[i * 8 + j] = 0.f;
            }
        }
        float* const prt = part();
        const int npieces = (g.r1 - g.r0 + g.rpp - 1) / g.rpp;
        uint32_t pc = it;
        if (g.rpp * g.segs <= NCW) {
            for (int q0 = 0; q0 < npieces; q0 += 4) {
                const int n = min(4, npieces - q0);
                bool ok = true;
                for (int j = 0; j < n; j++)
                    ok = wait_mbar(&qw_sm.full[(pc + j) % NSLOT], ((pc + j) / NSLOT) & 1, DERR_TIMEOUT_FULL) && ok;
                float v[4] = {0.f, 0.f, 0.f, 0.f};
                int dst[4] = {-1, -1, -1, -1};
                if (ok) {
                    uint4 wv[4][4];
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int r = g.r0 + (q0 + j) * g.rpp;
                        const bool have = j < n && w < min(g.rpp, g.r1 - r) * g.segs;
                        const int rl = w / g.segs;
                        if (have) dst[j] = (r - g.r0 + rl) * g.segs + myseg;
                        const uint4* wp = reinterpret_cast<const uint4*>(
                            ring() + ((pc + j) % NSLOT) * SLOT_BYTES + ((size_t)rl * g.K + (size_t)myseg * g.segw) * 2);
#pragma unroll
                        for (int i = 0; i < 4; i++) wv[j][i] = (have && i < g.cpl) ? wp[i * 32 + ln] : make_uint4(0, 0, 0, 0);
                    }
#pragma unroll
                    for (int j = 0; j < 4; j++)
#pragma unroll
                        for (int i = 0; i < 4; i++) v[j] += dot8(wv[j][i], xr + i * 8);
                }
                __syncwarp();
                if (ln == 0 && ok)  // a slot is released only after its data landed
                    for (int j = 0; j < n; j++) mbar_arrive(&qw_sm.empty[(pc + j) % NSLOT]);
                pc += n;
                // transposing butterfly: afterwards lanes 0, 8, 16, 24 hold the totals of rows 0..3
                const bool hi16 = ln & 16, hi8 = ln & 8;
                float k0 = hi16 ? v[2] : v[0], k1 = hi16 ? v[3] : v[1];
                k0 += __shfl_xor_sync(0xFFFFFFFFu, hi16 ? v[0] : v[2], 16);
                k1 += __shfl_xor_sync(0xFFFFFFFFu, hi16 ? v[1] : v[3], 16);
                float t = hi8 ? k1 : k0;
                t += __shfl_xor_sync(0xFFFFFFFFu, hi8 ? k0 : k1, 8);
                t += __shfl_xor_sync(0xFFFFFFFFu, t, 4);
                t += __shfl_xor_sync(0xFFFFFFFFu, t, 2);
                t += __shfl_xor_sync(0xFFFFFFFFu, t, 1);
                const int jj = (hi16 ? 2 : 0) + (hi8 ? 1 : 0);
                int d = dst[0];
                if (jj == 1) d = dst[1];
                if (jj == 2) d = dst[2];
                if (jj == 3) d = dst[3];
                if ((ln & 7) == 0 && d >= 0) prt[d] = t;
            }
        } else {
            // small K: several units per warp per piece
            for (int r = g.r0; r < g.r1; r += g.rpp, ++pc) {
                const int slot = pc % NSLOT;
                const bool ok = wait_mbar(&qw_sm.full[slot], (pc / NSLOT) & 1, DERR_TIMEOUT_FULL);
                if (ok) {
                    const int units = min(g.rpp, g.r1 - r) * g.segs;
                    const uint8_t* base = ring() + slot * SLOT_BYTES + (size_t)myseg * g.segw * 2;
                    for (int u = w; u < units; u += NCW) {
                        const int rl = u / g.segs;
                        const uint4* wp = reinterpret_cast<const uint4*>(base + (size_t)rl * g.K * 2);
                        float acc = 0.f;
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            if (i < g.cpl) acc += dot8(wp[i * 32 + ln], xr + i * 8);
                        acc = warp_sum(acc);
                        if (ln == 0) prt[(r - g.r0 + rl) * g.segs + myseg] = acc;
                    }
                }
                __syncwarp();
                if (ln == 0 && ok) mbar_arrive(&qw_sm.empty[slot]);
            }
        }
        it = pc;
        named_bar_sync(1, NCT);
    }

    // The Qwen3-0.6B case of gemv_generic, with everything static: 1024-column segments (4 chunks of
    // 16 bytes per lane) and at most one unit per warp per piece.
    //
    // Epilogue EPI: EPI_PART leaves the row sums in part() for a later pass; EPI_STORE (segs == 1)
    // has the lane holding a row's total store it at once, times the RMSNorm scale, as a tagged
    // word out[row]; EPI_SILU (segs == 1, 12 rows per piece, interleaved gate/up rows) gives each
    // warp whole (gate, up) row pairs - warp w takes pair w % 6 of pieces w / 6 and w / 6 + 2 of a
    // group - and stores silu(gate) * up as out[row / 2]. The fused epilogues write their results
    // before the phase's closing barrier, so the hand-off to other CTAs starts earlier.
    // whether gemv_full_segments covers phase g: whole 1024-column segments, at most one unit per warp
    // per piece, and (outputs stored from the reduction lanes) one segment of 12 rows per piece
    __host__ __device__ static bool full_segments(const GemvGeo& g, bool part) {
        return g.cpl == 4 && g.rpp * g.segs <= NCW && (part || (g.segs == 1 && g.rpp == 12));
    }

    template <int EPI>
    __device__ __noinline__ static void gemv_full_segments(const GemvGeo& gs, u64* out, uint32_t tg) {
        uint32_t& it = ring_pos();
        const GemvGeo g = gs;
        const int w = warp(), ln = lane();
        const WarpGeo wgo = qw_sm.wgeo[&gs - qw_sm.geo][w];
        const int myseg = wgo.myseg, rl = wgo.rl;
        const float sc = EPI == EPI_PART ? 1.f : norm_scale();
        float xr[32];
        {
            const float4* xp = reinterpret_cast<const float4*>(xs() + myseg * 1024) + ln;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float4 a = xp[i * 64], b = xp[i * 64 + 32];
                xr[i * 8 + 0] = a.x; xr[i * 8 + 1] = a.y; xr[i * 8 + 2] = a.z; xr[i * 8 + 3] = a.w;
                xr[i * 8 + 4] = b.x; xr[i * 8 + 5] = b.y; xr[i * 8 + 6] = b.z; xr[i * 8 + 7] = b.w;
            }
        }
        float* const prt = part();
        const int npieces = wgo.npieces;
        const int woff = wgo.wbyte + ln * 16;
        uint32_t pc = it;
        // a phase whose pieces all fit in the ring releases them once, after the phase's closing
        // barrier below; a longer one (lm_head) releases each group as soon as it is read
        const bool release_here = npieces > NSLOT;
        for (int q0 = 0; q0 < npieces; q0 += 4) {
            const int n = min(4, npieces - q0);
            const bool ok = wait_pieces(pc, n);
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            int dst[4] = {-1, -1, -1, -1};
            if (ok) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    // unit j of this warp: EPI_SILU -> row 2 * (w % 6) + (j & 1) of piece w / 6 + (j & 2);
                    // otherwise -> row rl of piece j
                    const int pj = EPI == EPI_SILU ? w / 6 + (j & 2) : j;
                    const int r = g.r0 + (q0 + pj) * g.rpp;
                    const int rr = EPI == EPI_SILU ? 2 * (w % 6) + (j & 1) : rl;
                    const bool have = EPI == EPI_SILU ? (pj < n && rr < g.r1 - r) : (j < n && w < min(g.rpp, g.r1 - r) * g.segs);
                    if (have) {
                        dst[j] = (r - g.r0 + rr) * g.segs + myseg;
                        const uint4* wp = reinterpret_cast<const uint4*>(
                            ring() + ((pc + pj) % NSLOT) * SLOT_BYTES + (EPI == EPI_SILU ? rr * 2048 + ln * 16 : woff));
                        uint4 wv[4];
#pragma unroll
                        for (int i = 0; i < 4; i++) wv[i] = wp[i * 32];
                        // two packed accumulators (chunks 0, 2 and 1, 3): 8 dependent FFMA2 each
                        float2 e = make_float2(0.f, 0.f), o = e;
                        e = dot8_acc2(wv[0], xr + 0, e);
                        o = dot8_acc2(wv[1], xr + 8, o);
                        e = dot8_acc2(wv[2], xr + 16, e);
                        o = dot8_acc2(wv[3], xr + 24, o);
                        v[j] = (e.x + e.y) + (o.x + o.y);
                    }
                }
            }
            if (release_here) {
                __syncwarp();
                if (ln == 0 && ok)  // a slot is released only after its data landed
                    for (int j = 0; j < n; j++) mbar_arrive(&qw_sm.empty[(pc + j) % NSLOT]);
            }
            pc += n;
            const bool hi16 = ln & 16, hi8 = ln & 8;
            float k0 = hi16 ? v[2] : v[0], k1 = hi16 ? v[3] : v[1];
            k0 += __shfl_xor_sync(0xFFFFFFFFu, hi16 ? v[0] : v[2], 16);
            k1 += __shfl_xor_sync(0xFFFFFFFFu, hi16 ? v[1] : v[3], 16);
            float t = hi8 ? k1 : k0;
            t += __shfl_xor_sync(0xFFFFFFFFu, hi8 ? k0 : k1, 8);
            t += __shfl_xor_sync(0xFFFFFFFFu, t, 4);
            t += __shfl_xor_sync(0xFFFFFFFFu, t, 2);
            t += __shfl_xor_sync(0xFFFFFFFFu, t, 1);
            const int jj = (hi16 ? 2 : 0) + (hi8 ? 1 : 0);
            int d = dst[0];
            if (jj == 1) d = dst[1];
            if (jj == 2) d = dst[2];
            if (jj == 3) d = dst[3];
            if (EPI == EPI_PART) {
                if ((ln & 7) == 0 && d >= 0) prt[d] = t;
            } else if (EPI == EPI_STORE) {
                if ((ln & 7) == 0 && d >= 0) st_relaxed_u64(out + g.r0 + d, tagged(t * sc, tg));
            } else {
                // lanes 0 and 16 hold a gate row total, lanes 8 and 24 the matching up row total
                const float up = __shfl_down_sync(0xFFFFFFFFu, t, 8);
                if ((ln & 15) == 0 && d >= 0) {
                    const float gt = t * sc, u = up * sc;
                    st_relaxed_u64(out + (g.r0 + d) / 2, tagged(gt / (1.0f + __expf(-gt)) * u, tg));
                }
            }
        }
        it = pc;
        named_bar_sync(1, NCT);
        // every warp has read the phase's pieces: one lane per slot releases it for all 12 warps
        if (!release_here && warp() == 0 && lane() < npieces && !aborted())
            mbar_arrive_cnt(&qw_sm.empty[(pc - npieces + lane()) % NSLOT], NCW);
    }

    // one GEMV phase of the CTA; returns after a CTA-wide barrier (part() then holds every row's sums)
    // EPI_STORE and EPI_SILU write their outputs (out, tagged tg) themselves; EPI_PART leaves the
    // row sums in part() for residual_rows / lm_epilogue
    template <int EPI>
    __device__ __forceinline__ static void gemv_consume(const GemvGeo& g, u64* out = nullptr, uint32_t tg = 0) {
        if constexpr (kGeneric) {
            if (full_segments(g, EPI == EPI_PART)) {
                gemv_full_segments<EPI>(g, out, tg);
            } else {
                gemv_generic(g);
                if (EPI == EPI_STORE) store_rows(out, g, tg);
                if (EPI == EPI_SILU) silu_rows(tg);
            }
        } else {
            gemv_full_segments<EPI>(g, out, tg);  // init_geometry checked every phase's shape
        }
    }

    __device__ __forceinline__ static float row_value(const GemvGeo& g, int rl) {
        float y = 0.f;
        for (int sgi = 0; sgi < g.segs; sgi++) y += part()[rl * g.segs + sgi];
        return y;
    }

    // ------------------------------------------------------------------ attention (phase B)
    // one warp: gather a tagged 128-vector, per-head RMSNorm (q_norm/k_norm), rotate-half RoPE
    // (cpu_inference.rs:134-138, :196-215; the table is the one MetalKVCache builds, :141-154)
    __device__ __forceinline__ static float4 gather_head(const u64* src, uint32_t tg) {
        const DecodeParams& p = qw_sm.prm;
        uint32_t spins = 0;
        uint64_t t0 = 0;
        ulonglong2 a = make_ulonglong2(0, 0), b = make_ulonglong2(0, 0);
        bool ok = false;
        while (!aborted()) {
            a = ld_relaxed_v2u64(src + lane() * 4);
            b = ld_relaxed_v2u64(src + lane() * 4 + 2);
            ok = word_tag(a.x) == tg && word_tag(a.y) == tg && word_tag(b.x) == tg && word_tag(b.y) == tg;
            if (__all_sync(0xFFFFFFFFu, ok)) break;
            int stop = 0;
            if (lane() == 0) stop = wait_expired(spins, t0, DERR_TIMEOUT_DATA, (int)tg);
            if (__shfl_sync(0xFFFFFFFFu, stop, 0)) break;
            if (p.poll_ns) __nanosleep(p.poll_ns);
        }
        return make_float4(word_val(a.x), word_val(a.y), word_val(b.x), word_val(b.y));
    }

    __device__ __forceinline__ static void head_norm_rope(float4 v, const uint16_t* nw, const float2* rrow, float* dst) {
        const DecodeParams& p = qw_sm.prm;
        float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        ss = warp_sum(ss);
        const float s = rsqrtf(ss / (float)HD + p.eps);
        const int d0 = lane() * 4;
        float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; j++) e[j] = e[j] * s * bf16_to_f32(__ldg(nw + d0 + j));
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float other = __shfl_xor_sync(0xFFFFFFFFu, e[j], 16);  // element d +- 64
            const float2 cs = rrow[(d0 + j) & 63];
            if (lane() < 16) o[j] = e[j] * cs.x - other * cs.y;   // x[i]      = a*cos - b*sin
            else o[j] = e[j] * cs.x + other * cs.y;             // x[i+half] = b*cos + a*sin
        }
        reinterpret_cast<float4*>(dst)[lane()] = make_float4(o[0], o[1], o[2], o[3]);
    }

    // Running softmax state of one warp for up to MAX_G query heads: every lane holds the same
    // (m, l) per head and its own 4 of the 128 accumulator dimensions.
    struct WarpSoftmax {
        float m[MAX_G], l[MAX_G];
        float4 acc[MAX_G];
    };

    // Up to two cached positions (K and V rows of 128 f32 in shared memory; the second may be
    // absent) into a warp's running softmax (cpu_inference.rs:144-161: scores q.k / sqrt(128),
    // softmax, sum of p * v). The warp scores both positions against its Gh query heads with
    // butterfly sums, so every lane holds every score; the 2 x Gh sums are independent, so their
    // shuffle chains overlap. Then each head's state is rescaled once for the pair.
    template <int GQ>
    __device__ __forceinline__ static void attn_pair(const float* K0, const float* V0, const float* K1, const float* V1,
                                                     bool has1, const float4* q4, WarpSoftmax& ws, float scale) {
        const float4 k0 = reinterpret_cast<const float4*>(K0)[lane()];
        const float4 v0 = reinterpret_cast<const float4*>(V0)[lane()];
        float4 k1 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = k1;
        if (has1) {
            k1 = reinterpret_cast<const float4*>(K1)[lane()];
            v1 = reinterpret_cast<const float4*>(V1)[lane()];
        }
        float s0[MAX_G], s1[MAX_G];
#pragma unroll
        for (int h = 0; h < GQ; h++) {
            s0[h] = q4[h].x * k0.x + q4[h].y * k0.y + q4[h].z * k0.z + q4[h].w * k0.w;
            s1[h] = q4[h].x * k1.x + q4[h].y * k1.y + q4[h].z * k1.z + q4[h].w * k1.w;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int h = 0; h < GQ; h++) {
                {
                    s0[h] += __shfl_xor_sync(0xFFFFFFFFu, s0[h], o);
                    s1[h] += __shfl_xor_sync(0xFFFFFFFFu, s1[h], o);
                }
            }
        }
#pragma unroll
        for (int h = 0; h < GQ; h++) {
            {
                const float a0 = s0[h] * scale, a1 = has1 ? s1[h] * scale : -INFINITY;
                const float mn = fmaxf(ws.m[h], fmaxf(a0, a1));
                const float corr = __expf(ws.m[h] - mn);  // 0 while m is still -inf
                const float p0 = __expf(a0 - mn), p1 = __expf(a1 - mn);  // p1 = 0 without a second position
                ws.l[h] = fmaf(ws.l[h], corr, p0 + p1);
                ws.acc[h].x = fmaf(ws.acc[h].x, corr, fmaf(p0, v0.x, p1 * v1.x));
                ws.acc[h].y = fmaf(ws.acc[h].y, corr, fmaf(p0, v0.y, p1 * v1.y));
                ws.acc[h].z = fmaf(ws.acc[h].z, corr, fmaf(p0, v0.z, p1 * v1.z));
                ws.acc[h].w = fmaf(ws.acc[h].w, corr, fmaf(p0, v0.w, p1 * v1.w));
                ws.m[h] = mn;
            }
        }
    }

    // phase B for GQ query heads per KV head (a compile-time count: with a runtime count the
    // per-position code roughly doubles in length)
    template <int GQ>
    __device__ __noinline__ static void attention_g(int step, int l, int pos) {
        const DecodeParams& p = qw_sm.prm;
        uint32_t& it = ring_pos();
        const AttnItem a = attn_item(p, cta(), pos);
        if (!a.active) return;   // uniform over the CTA
        const uint16_t* nrm = p.layer_n + (size_t)l * p.norm_stride;
        const uint16_t* qn = nrm + 2 * p.H;
        const uint16_t* kn = qn + HD;
        const float2* rrow = p.rope + (size_t)pos * (HD / 2);
        const uint32_t tgA = tag(seq(step, l, 1)), tgB = tag(seq(step, l, 2));
        // q heads g*G .. g*G+G-1, and (last chunk) this position's k and v
        if (warp() < GQ) head_norm_rope(gather_head(p.qkv + (size_t)(a.g * GQ + warp()) * HD, tgA), qn, rrow, qw_sm.qs[warp()]);
        if (a.has_cur) {
            if (warp() == GQ) head_norm_rope(gather_head(p.qkv + QD() + (size_t)a.g * HD, tgA), kn, rrow, qw_sm.ks);
            if (warp() == GQ + 1)
                reinterpret_cast<float4*>(qw_sm.vs)[lane()] = gather_head(p.qkv + QD() + KVD() + (size_t)a.g * HD, tgA);
        }
        named_bar_sync(1, NCT);
        stamp(step, l * TRACE_PER_LAYER + 3);
        if (a.has_cur && tid() < 2 * HD) {  // append K/V at slot `pos` (cpu_inference.rs:140-141)
            const size_t off = (((size_t)l * p.NKV + a.g) * p.max_seq + pos) * HD;
            if (tid() < HD) p.kc[off + tid()] = qw_sm.ks[tid()];
            else p.vc[off + tid() - HD] = qw_sm.vs[tid() - HD];
        }
        float4 q4[GQ];
#pragma unroll
        for (int h = 0; h < GQ; h++)
            q4[h] = reinterpret_cast<const float4*>(qw_sm.qs[h])[lane()];
        // Each warp takes the chunk's positions j = warp, warp + 12, ... (j counted from t0), two per
        // call, and keeps its own running softmax: no CTA-wide barrier per ring piece. A piece holds
        // ATT_P = 24 = 2 x 12 positions, so position pp of a piece is chunk position j with
        // j % 12 == pp % 12.
        WarpSoftmax ws;
        const float scale = p.scale;
#pragma unroll
        for (int h = 0; h < GQ; h++) {
            ws.m[h] = -INFINITY;
            ws.l[h] = 0.f;
            ws.acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const int tc1 = a.has_cur ? pos : a.t1;  // cached positions [t0, tc1)
        const int npieces = tc1 > a.t0 ? (tc1 - a.t0 + ATT_P - 1) / ATT_P : 0;
        for (int q0 = 0; q0 < npieces; q0 += 4) {  // up to four pieces waited for side by side
            const int n = min(4, npieces - q0);
            const uint32_t pc = it;
            const bool ok = wait_pieces(pc, n);
            for (int j = 0; j < n; j++) {
                const int np = min(ATT_P, tc1 - (a.t0 + (q0 + j) * ATT_P));
                const float* Kb = reinterpret_cast<const float*>(ring() + ((pc + j) % NSLOT) * SLOT_BYTES);
                const float* Vb = Kb + ATT_P * HD;
                if (ok)
                    for (int pp = warp(); pp < np; pp += 2 * NCW)
                        attn_pair<GQ>(Kb + pp * HD, Vb + pp * HD, Kb + (pp + NCW) * HD, Vb + (pp + NCW) * HD, pp + NCW < np, q4,
                                  ws, scale);
            }
            __syncwarp();
            if (lane() == 0 && ok)
                for (int j = 0; j < n; j++) mbar_arrive(&qw_sm.empty[(pc + j) % NSLOT]);
            it = pc + n;
        }
        if (a.has_cur && warp() == (tc1 - a.t0) % NCW) attn_pair<GQ>(qw_sm.ks, qw_sm.vs, nullptr, nullptr, false, q4, ws, scale);
        // combine the 12 warps' states in warp order (deterministic): stage [warp][h < G][acc 128 | m | l | pad]
        float* const wst = part();
        constexpr int WST = ATT_WST;
#pragma unroll
        for (int h = 0; h < GQ; h++) {
            if (h < GQ) {
                float* d = wst + (warp() * GQ + h) * WST;
                reinterpret_cast<float4*>(d)[lane()] = ws.acc[h];
                if (lane() == 0) {
                    d[HD] = ws.m[h];
                    d[HD + 1] = ws.l[h];
                }
            }
        }
        named_bar_sync(1, NCT);
        float m = -INFINITY, lsum = 0.f, acc = 0.f;
        if (tid() < GQ * HD) {
            const int h = tid() >> 7, d = tid() & (HD - 1);
#pragma unroll
            for (int w = 0; w < NCW; w++) m = fmaxf(m, wst[(w * GQ + h) * WST + HD]);
#pragma unroll
            for (int w = 0; w < NCW; w++) {
                const float* src = wst + (w * GQ + h) * WST;
                const float e = src[HD] == -INFINITY ? 0.f : __expf(src[HD] - m);  // a warp without positions adds nothing
                lsum = fmaf(e, src[HD + 1], lsum);
                acc = fmaf(e, src[d], acc);
            }
        }
        named_bar_sync(1, NCT);  // the warp states in part are dead: the merge below may reuse part
        stamp(step, l * TRACE_PER_LAYER + 4);
        const size_t head_base = (size_t)a.g * p.S * GQ;  // partial (s, h) at apart[((head_base + s*G + h) * APART_STRIDE]
        if (a.s != 0) {
            // publish this chunk's partial as tagged words for the chunk-0 CTA of this KV head
            if (tid() < GQ * HD) {
                const int h = tid() >> 7, d = tid() & (HD - 1);
                u64* dst = p.apart + (head_base + (size_t)a.s * GQ + h) * APART_STRIDE;
                st_relaxed_u64(dst + d, tagged(acc, tgB));
                if (d == 0) {
                    st_relaxed_u64(dst + HD, tagged(m, tgB));
                    st_relaxed_u64(dst + HD + 1, tagged(lsum, tgB));
                }
            }
            return;
        }
        // chunk 0 merges the partials of chunks 0..S_eff-1 in chunk order: an accumulator thread
        // (h, d) polls word d of chunks 1.. (four chunks in flight per round) into the shared stage,
        // and the first (S_eff-1)*G*2 threads also poll one (m or l) word each.
        if (tid() < GQ * HD && (tid() & (HD - 1)) == 0) {
            qw_sm.ml[0][tid() >> 7][0] = m;
            qw_sm.ml[0][tid() >> 7][1] = lsum;
        }
        float* stage = part();  // chunk s >= 1 partial words, [s - 1][G * HD] (part is free during phase B)
        {
            const int h = tid() >> 7, d = tid() & (HD - 1);
            const u64* mlsrc = nullptr;
            float* mldst = nullptr;
            if (tid() < (a.S_eff - 1) * GQ * 2) {  // the first (S_eff-1)*G*2 threads also fetch one (m or l) word
                const int s = 1 + tid() / (2 * GQ), hh = (tid() >> 1) % GQ, which = tid() & 1;
                mlsrc = p.apart + (head_base + (size_t)s * GQ + hh) * APART_STRIDE + HD + which;
                mldst = &qw_sm.ml[s][hh][which];
            }
            // up to four chunks' words (bits 0-3) and the (m, l) word (bit 4) in flight per round
            for (int s0 = 1; s0 < a.S_eff || mlsrc; s0 += 4) {
                uint32_t pending = mlsrc ? 16u : 0u;  // the (m, l) word is polled in the first round only
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (tid() < GQ * HD && s0 + j < a.S_eff) pending |= 1u << j;
                uint32_t spins = 0;
                uint64_t t0 = 0;
                while (pending && !aborted()) {
                    u64 w[5];
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        if (pending & (1u << j)) w[j] = ld_relaxed_u64(p.apart + (head_base + (size_t)(s0 + j) * GQ + h) * APART_STRIDE + d);
                    if (pending & 16u) w[4] = ld_relaxed_u64(mlsrc);
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        if ((pending & (1u << j)) && word_tag(w[j]) == tgB) {
                            stage[(s0 + j - 1) * (GQ * HD) + tid()] = word_val(w[j]);
                            pending &= ~(1u << j);
                        }
                    if ((pending & 16u) && word_tag(w[4]) == tgB) {
                        *mldst = word_val(w[4]);
                        pending &= ~16u;
                    }
                    if (pending) {
                        if (wait_expired(spins, t0, DERR_TIMEOUT_DATA, (int)tgB)) break;
                        if (p.poll_ns) __nanosleep(p.poll_ns);
                    }
                }
                mlsrc = nullptr;
            }
        }
        stamp(step, l * TRACE_PER_LAYER + 12);
        named_bar_sync(1, NCT);
        if (tid() < GQ * HD) {
            const int h = tid() >> 7, d = tid() & (HD - 1);
            float M = qw_sm.ml[0][h][0];
#pragma unroll 4
            for (int s = 1; s < a.S_eff; s++) M = fmaxf(M, qw_sm.ml[s][h][0]);
            const float w0 = __expf(qw_sm.ml[0][h][0] - M);
            float Lt = w0 * qw_sm.ml[0][h][1], O = w0 * acc;
#pragma unroll 4
            for (int s = 1; s < a.S_eff; s++) {
                const float w = __expf(qw_sm.ml[s][h][0] - M);
                Lt = fmaf(w, qw_sm.ml[s][h][1], Lt);
                O = fmaf(w, stage[(s - 1) * (GQ * HD) + tid()], O);
            }
            st_relaxed_u64(p.att + (size_t)(a.g * GQ + h) * HD + d, tagged(O / Lt, tgB));
        }
        stamp(step, l * TRACE_PER_LAYER + 13);
        named_bar_sync(1, NCT);  // the stage lives in part, which the next phase's GEMV overwrites
    }

    __device__ __noinline__ static void attention_consume(int step, int l, int pos) {
        switch (G()) {
            case 1: attention_g<1>(step, l, pos); break;
            case 2: attention_g<2>(step, l, pos); break;
            default: attention_g<3>(step, l, pos); break;
        }
    }

    // ------------------------------------------------------------------ lm_head + argmax
    __device__ __noinline__ static void lm_epilogue() {
        const DecodeParams& p = qw_sm.prm;
        const float sc = norm_scale();
        const GemvGeo& g = gF();
        const int nloc = g.r1 - g.r0;
        float bv = -INFINITY;
        unsigned bi = NONE_IDX;
        #pragma unroll 1
        for (int i = tid(); i < nloc; i += NCT) {
            const float y = row_value(g, i) * sc;
            const unsigned row = (unsigned)(g.r0 + i);
            if (p.logits) __stcg(p.logits + row, y);
            if (!isnan(y) && am_better(y, row, bv, bi)) { bv = y; bi = row; }
            if (row == 0) __stcg(p.nan0, isnan(y) ? 1 : 0);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
            const unsigned oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
            if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane() == 0) { qw_sm.redv[warp()] = bv; qw_sm.redi[warp()] = bi; }
        named_bar_sync(1, NCT);
        if (tid() == 0) {
            for (int w = 1; w < NCW; w++)
                if (am_better(qw_sm.redv[w], qw_sm.redi[w], bv, bi)) { bv = qw_sm.redv[w]; bi = qw_sm.redi[w]; }
            __stcg(p.am_val + cta(), bv);
            __stcg(p.am_idx + cta(), bi);
        }
    }

    // after the end-of-token barrier: every CTA reduces the partials to the same next token
    __device__ __noinline__ static unsigned argmax_combine() {
        const DecodeParams& p = qw_sm.prm;
        if (warp() == 0) {
            float bv = -INFINITY;
            unsigned bi = NONE_IDX;
            for (int j = lane(); j < nctas(); j += 32) {
                const float v = __ldcg(p.am_val + j);
                const unsigned i = __ldcg(p.am_idx + j);
                if (am_better(v, i, bv, bi)) { bv = v; bi = i; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
                const unsigned oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
                if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
            }
            if (lane() == 0) {
                unsigned t = bi;
                if (__ldcg(p.nan0) != 0 || t == NONE_IDX || t >= (unsigned)p.V) t = 0;  // first-strict-max rule
                qw_sm.token = t;
            }
        }
        named_bar_sync(1, NCT);
        return qw_sm.token;
    }

    // q|k|v rows (phase A), with the RMSNorm scale of the phase's input
    __device__ __noinline__ static void store_rows(u64* dst, const GemvGeo& g, uint32_t tg) {
        const float sc = norm_scale();
        #pragma unroll 1
        for (int i = tid(); i < g.r1 - g.r0; i += NCT) st_relaxed_u64(dst + g.r0 + i, tagged(row_value(g, i) * sc, tg));
    }

    // x[r] += y[r] on this CTA's rows (cpu_inference.rs:163-164, :171-172)
    __device__ __noinline__ static void residual_rows(const GemvGeo& g, uint32_t tg) {
        const DecodeParams& p = qw_sm.prm;
        #pragma unroll 1
        for (int i = tid(); i < g.r1 - g.r0; i += NCT) {
            const float v = xloc()[i] + row_value(g, i);
            xloc()[i] = v;
            st_relaxed_u64(p.x + g.r0 + i, tagged(v, tg));
        }
    }

    // ------------------------------------------------------------------ consumer main loop
    // Loop state of the token/layer loops, per warp in shared memory. The loops call out-of-line
    // phase routines that may use every register; a loop counter held in a register across such a
    // call would be spilled to local memory. Reading the state back from shared memory after each
    // call (volatile: the compiler may not keep a copy) leaves no value that has to survive a call.
    // (%tid.x is read with a volatile asm so that the compiler re-reads it instead of keeping the
    // derived address live across the calls)
    __device__ __forceinline__ static volatile LoopState& ls() {
        uint32_t t;
        asm volatile("mov.u32 %0, %%tid.x;" : "=r"(t));
        return qw_sm.loop[t >> 5];
    }
    __device__ __forceinline__ static const volatile DecodeParams& vprm() { return qw_sm.prm; }
    __device__ __forceinline__ static int cur_step() { return ls().step; }
    __device__ __forceinline__ static int cur_layer() { return ls().l; }
    __device__ __forceinline__ static const uint16_t* layer_norms() {
        return vprm().layer_n + (size_t)cur_layer() * vprm().norm_stride;
    }
    __device__ __forceinline__ static uint32_t ltag(int ph) { return tag(seq(cur_step(), cur_layer(), ph)); }
    __device__ __forceinline__ static void lstamp(int k) { stamp(cur_step(), cur_layer() * TRACE_PER_LAYER + k); }
    __device__ __forceinline__ static void tstamp(int k) { stamp(cur_step(), vprm().L * TRACE_PER_LAYER + k); }

    // h[r] = silu(gate_r) * up_r on this CTA's interleaved gate/up rows (cpu_inference.rs:166-170, :187)
    __device__ __noinline__ static void silu_rows(uint32_t tg) {
        const GemvGeo& g = gD();
        u64* const h = qw_sm.prm.hbuf;
        const float sc = norm_scale();
        #pragma unroll 1
        for (int i = tid(); i < (g.r1 - g.r0) / 2; i += NCT) {
            const float gt = row_value(g, 2 * i) * sc, up = row_value(g, 2 * i + 1) * sc;
            st_relaxed_u64(h + g.r0 / 2 + i, tagged(gt / (1.0f + __expf(-gt)) * up, tg));
        }
    }

    // CTA 0 hands step `step`'s token to the device ring and the mapped host mirror
    __device__ __noinline__ static void publish_token(int step, unsigned token) {
        const DecodeParams& p = qw_sm.prm;
        if (cta() == 0 && tid() == 0 && !aborted()) {
            if (p.tok_out) p.tok_out[step + 1] = token;
            if (p.host_tok) {
                volatile uint32_t* ht = p.host_tok;
                ht[step + 1] = token;
                __threadfence_system();
                *reinterpret_cast<volatile unsigned*>(p.host_count) = (unsigned)(step + 1);
            }
        }
    }

    // one layer: A rmsnorm + q|k|v, B attention, C o + residual, D rmsnorm + gate|up + SiLU, E down + residual
    __device__ __forceinline__ static void consume_layer() {
        lstamp(0);
        norm_prologue(layer_norms(), cur_layer() == 0, ls().token, cur_layer() == 0 ? 0u : tag(seq(cur_step(), cur_layer() - 1, 5)));
        lstamp(1);
        gemv_consume<EPI_STORE>(gA(), vprm().qkv, ltag(1));
        lstamp(2);
        attention_consume(cur_step(), cur_layer(), vprm().start_pos + cur_step());
        lstamp(5);
        gather(vprm().att, QD(), ltag(2));
        lstamp(6);
        gemv_consume<EPI_PART>(gC());
        residual_rows(gC(), ltag(3));
        lstamp(7);
        norm_prologue(layer_norms() + vprm().H, false, 0, ltag(3));
        lstamp(8);
        gemv_consume<EPI_SILU>(gD(), vprm().hbuf, ltag(4));
        lstamp(9);
        gather(vprm().hbuf, vprm().I, ltag(4));
        lstamp(10);
        gemv_consume<EPI_PART>(gE());
        residual_rows(gE(), ltag(5));
        lstamp(11);
    }

    __device__ static void consume() {
        {
            const DecodeParams& p = qw_sm.prm;
            unsigned token = __ldcg(p.tok_in);
            if (token >= (unsigned)p.V) {
                if (tid() == 0) fail(DERR_BAD_TOKEN, (int)token);
                token = 0;
            }
            ls().token = token;
        }
        for (ls().step = 0; cur_step() < vprm().steps; ls().step = cur_step() + 1) {
            for (ls().l = 0; cur_layer() < vprm().L; ls().l = cur_layer() + 1) consume_layer();
            // F: final rmsnorm -> lm_head -> argmax partials -> end-of-token barrier -> next token
            norm_prologue(vprm().final_norm, false, 0, tag(seq(cur_step(), vprm().L - 1, 5)));
            tstamp(0);
            gemv_consume<EPI_PART>(gF());
            lm_epilogue();
            tstamp(1);
            token_barrier((uint32_t)cur_step() + 1);
            tstamp(2);
            ls().token = argmax_combine();
            tstamp(3);
            publish_token(cur_step(), ls().token);
        }
    }

    // ------------------------------------------------------------------ producer
    __device__ static bool slot_acquire(uint32_t& slot) {
        uint32_t& it = ring_pos();
        slot = it % NSLOT;
        const uint32_t par = ((it / NSLOT) & 1) ^ 1;
        return wait_mbar(&qw_sm.empty[slot], par, DERR_TIMEOUT_EMPTY);
    }

    __device__ __forceinline__ static const uint16_t* layer_weights(int l) {
        return vprm().layer_w + (size_t)l * vprm().layer_stride;
    }

    __device__ __noinline__ static void gemv_produce(const GemvGeo& g, const uint16_t* wbase) {
        const uint64_t pol = policy_evict_first();
        uint32_t& it = ring_pos();
        for (int r = g.r0; r < g.r1; r += g.rpp) {
            const int nr = min(g.rpp, g.r1 - r);
            uint32_t slot;
            if (slot_acquire(slot)) {
                const uint32_t bytes = (uint32_t)nr * (uint32_t)g.K * 2u;
                mbar_arrive_expect_tx(&qw_sm.full[slot], bytes);
                bulk_g2s_evict_first(ring() + slot * SLOT_BYTES, wbase + g.woff + (size_t)r * g.K, bytes, &qw_sm.full[slot], pol);
                qw_sm.n_issued = it + 1;
            }
            ++it;
        }
    }

    __device__ __noinline__ static void attn_produce(int step, int l, int pos) {
        const DecodeParams& p = qw_sm.prm;
        uint32_t& it = ring_pos();
        const AttnItem a = attn_item(p, cta(), pos);
        if (!a.active) return;
        const int tc1 = a.has_cur ? pos : a.t1;
        if (a.t0 >= tc1) return;
        // K/V rows of earlier positions may have been written by other CTAs in earlier steps of this
        // launch: wait until this CTA's consumers have passed the previous token's barrier, then order
        // the async-proxy reads after it.
        if (step > 0 && !aborted() && l == 0) {
            uint32_t spins = 0;
            uint64_t t0 = 0;
            while (ld_acquire_cta_shared(&qw_sm.progress) < (uint32_t)step) {
                if (wait_expired(spins, t0, DERR_TIMEOUT_KV, step)) break;
                __nanosleep(32);
            }
            fence_proxy_async_global();
        }
        const size_t head = ((size_t)l * p.NKV + a.g) * p.max_seq;
        for (int t = a.t0; t < tc1; t += ATT_P) {
            const int np = min(ATT_P, tc1 - t);
            uint32_t slot;
            if (slot_acquire(slot)) {
                const uint32_t bytes = (uint32_t)np * HD * 4u;
                mbar_arrive_expect_tx(&qw_sm.full[slot], 2u * bytes);
                uint8_t* dst = ring() + slot * SLOT_BYTES;
                bulk_g2s(dst, p.kc + (head + t) * HD, bytes, &qw_sm.full[slot]);
                bulk_g2s(dst + ATT_P * HD * 4, p.vc + (head + t) * HD, bytes, &qw_sm.full[slot]);
                qw_sm.n_issued = it + 1;
            }
            ++it;
        }
    }

    // warm L2 with this CTA's rows of one layer (A, C, D, E), so the ring's bulk copies of that
    // layer hit L2: the ring holds less than a layer, and without this the next layer's first
    // pieces would be fetched from HBM only once the current layer's last pieces are released
    __device__ __noinline__ static void prefetch_layer(const uint16_t* W) {
        const GemvGeo* gs[4] = {&gA(), &gC(), &gD(), &gE()};
        for (int k = 0; k < 4; k++) {
            const GemvGeo& g = *gs[k];
            const uint32_t bytes = (uint32_t)(g.r1 - g.r0) * (uint32_t)g.K * 2u;
            if (bytes) bulk_prefetch_l2(W + g.woff + (size_t)g.r0 * g.K, bytes);
        }
    }

    __device__ static void prefetch_lm_head() {
        const DecodeParams& p = qw_sm.prm;
        const GemvGeo& g = gF();
        const uint32_t all = (uint32_t)(g.r1 - g.r0) * (uint32_t)g.K * 2u;
        const uint32_t bytes = all < LM_PREFETCH_BYTES ? all : LM_PREFETCH_BYTES;
        if (bytes) bulk_prefetch_l2(p.lm_head + (size_t)g.r0 * g.K, bytes);
    }

    __device__ static void produce() {
        prefetch_layer(vprm().layer_w);
        for (ls().step = 0; cur_step() < vprm().steps; ls().step = cur_step() + 1) {
            for (ls().l = 0; cur_layer() < vprm().L; ls().l = cur_layer() + 1) {
                if (cur_layer() + 1 < vprm().L) prefetch_layer(layer_weights(cur_layer() + 1));
                else prefetch_lm_head();
                gemv_produce(gA(), layer_weights(cur_layer()));
                attn_produce(cur_step(), cur_layer(), vprm().start_pos + cur_step());
                gemv_produce(gC(), layer_weights(cur_layer()));
                gemv_produce(gD(), layer_weights(cur_layer()));
                gemv_produce(gE(), layer_weights(cur_layer()));
            }
            if (cur_step() + 1 < vprm().steps) prefetch_layer(vprm().layer_w);
            gemv_produce(gF(), vprm().lm_head);
        }
        drain();
    }

    // Normally every issued copy has been consumed by the time the producer finishes. After an
    // abort, wait (bounded) for the copies still in flight before the CTA may exit. Consumers stop
    // releasing slots once they abort, so only the last NSLOT issued pieces can be outstanding,
    // one per slot.
    __device__ __noinline__ static void drain() {
        const DecodeParams& p = qw_sm.prm;
        if (aborted()) {
            const uint32_t first = qw_sm.n_issued > NSLOT ? qw_sm.n_issued - NSLOT : 0;
            for (uint32_t j = first; j < qw_sm.n_issued; j++) {
                const int slot = j % NSLOT;
                const uint32_t par = (j / NSLOT) & 1;
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(&qw_sm.full[slot], par)) {
                    if (globaltimer_ns() - t0 > (uint64_t)p.timeout_ns) {
                        atomicCAS(&p.err[3], 0, DERR_TIMEOUT_DRAIN);
                        break;
                    }
                }
            }
        }
    }
};

// every phase of the model's shapes runs gemv_full_segments (kGeneric = false is then safe): rows of
// the lm_head, o and down in whole 1024-column segments whose count divides 12, q|k|v and gate|up
// over exactly 1024 columns
inline bool full_segment_shapes(int H, int QD, int I) {
    auto part_ok = [](int K) { return K % 1024 == 0 && K / 1024 >= 1 && 12 % (K / 1024) == 0; };
    return H == 1024 && part_ok(QD) && part_ok(I);
}

// the GEMV micro-benchmark kernel's decoder: every shape, no trace
using Decoder = DecoderT<false, true>;

}  // namespace qw
