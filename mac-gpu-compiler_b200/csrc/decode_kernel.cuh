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
//     the consumers wait on the grid-wide dependencies below.
//   * warps 0..11 are CONSUMERS. Each GEMV phase gives every CTA a contiguous block of output
//     rows; a ring slot holds whole rows, and a (row, 1024-column segment) unit is one warp's dot
//     product against the activation vector it holds in registers. Epilogues are fused: q|k|v
//     rows are written raw; o/down add the residual; gate/up rows are interleaved so the SiLU*up
//     product is formed in the CTA; lm_head rows feed a per-CTA argmax partial.
//   * Dependencies between phases (every GEMV output feeds every CTA of the next phase) are
//     grid barriers built from per-CTA release flags (flag = epoch << 32 | barrier number): a CTA
//     publishes with st.release.gpu and waits with ld.acquire.gpu polls of all flags. No atomics
//     on the barrier path, and no reset between launches (the host bumps `epoch`).
//   * Attention: each KV head's positions are split into up to S contiguous chunks, one CTA per
//     (kv head, chunk). A CTA applies q_norm/k_norm + RoPE itself, the CTA whose chunk holds `pos`
//     also writes the new K/V into the cache, each CTA keeps an online-softmax partial for its
//     G query heads, and the last CTA to finish a KV head (atomic ticket) merges the partials in
//     chunk order (deterministic) into the attention output.
//
// Every wait is bounded in time; on expiry the kernel records an error, stops waiting anywhere
// (fast-forwards to the end without blocking), waits (bounded) for its own bulk copies in flight
// and returns. The host reports the error.
#pragma once
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
constexpr int MIN_CHUNK = 8;                  // fewest positions per attention split
constexpr int APART_STRIDE = HD + 4;          // floats per attention partial: acc[128], m, l, pad
constexpr uint32_t NONE_IDX = 0xFFFFFFFFu;

// error codes written to DecodeParams::err[0]
enum : int { DERR_NONE = 0, DERR_TIMEOUT_GRID = 1, DERR_TIMEOUT_FULL = 2, DERR_TIMEOUT_EMPTY = 3,
             DERR_TIMEOUT_KV = 4, DERR_BAD_TOKEN = 5, DERR_TIMEOUT_DRAIN = 6 };

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
    // scratch
    float* x;                    // [H] residual stream
    float* qkv;                  // [QD + 2*KVD] raw projections
    float* att;                  // [QD] attention output
    float* hbuf;                 // [I] SiLU(gate)*up
    float* apart;                // [KVH][S][G][APART_STRIDE]
    unsigned* acount;            // [KVH] arrival tickets (returned to 0 by the last arriver)
    float* am_val;               // [grid] argmax partials
    unsigned* am_idx;            // [grid]
    int* nan0;                   // logits[0] is NaN (the CPU argmax then returns 0)
    unsigned long long* flags;   // [grid] barrier flags
    int* err;                    // [4] code, cta, barrier/piece, detail
    float* logits;               // [V] or null (decode skips it)
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
    int S;                       // attention splits per KV head
    int part_cap;                // floats in the shared partial-sum buffer
    int xs_cap;                  // floats in the shared activation buffer
    long long timeout_ns;
};

// static row partition of a GEMV phase for one CTA
struct GemvGeo {
    int r0, r1;       // output rows [r0, r1)
    int K;            // columns
    int rpp;          // rows per ring slot
    int segs;         // 1024-column segments per row (K / segw)
    int segw;         // columns per segment
    int cpl;          // 16-byte chunks per lane per segment (segw / 256)
    long long woff;   // element offset of the matrix inside a layer block
};

__host__ __device__ inline int seg_count(int K) { return K <= 1024 ? 1 : K / 1024; }

__device__ inline GemvGeo make_geo(long long rows, int K, int cta, int n, long long woff, int pair) {
    GemvGeo g;
    if (pair) {  // gate/up: partition pairs so each CTA owns whole (gate_i, up_i) row pairs
        long long P = rows / 2;
        g.r0 = (int)(2 * (P * cta / n));
        g.r1 = (int)(2 * (P * (cta + 1) / n));
    } else {
        g.r0 = (int)(rows * cta / n);
        g.r1 = (int)(rows * (cta + 1) / n);
    }
    g.K = K;
    g.rpp = SLOT_BYTES / (2 * K);
    g.segs = seg_count(K);
    g.segw = K / g.segs;
    g.cpl = g.segw / 256;
    g.woff = woff;
    return g;
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
    if (chunk < MIN_CHUNK) chunk = MIN_CHUNK;
    a.S_eff = (n_t + chunk - 1) / chunk;
    a.g = cta / p.S;
    a.s = cta % p.S;
    a.active = (cta < p.NKV * p.S) && (a.s < a.S_eff);
    a.t0 = a.s * chunk;
    a.t1 = min(n_t, a.t0 + chunk);
    a.has_cur = a.active && (a.t1 == n_t);
    return a;
}

struct Smem {
    float qs[MAX_G][HD];
    float ks[HD];
    float vs[HD];
    float sc[2][MAX_G][ATT_P];
    float red[64];
    float redv[NCW];
    unsigned redi[NCW];
    uint64_t full[NSLOT];
    uint64_t empty[NSLOT];
    uint32_t progress;   // grid barriers passed by this CTA's consumers
    int abort;           // set once any wait expired
    unsigned token;
    int is_last;
};

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

// argmax ordering: larger value wins, ties to the lower index, NaN never wins (NONE_IDX = empty)
__device__ __forceinline__ bool am_better(float av, unsigned ai, float bv, unsigned bi) {
    if (ai == NONE_IDX) return false;
    if (bi == NONE_IDX) return true;
    return av > bv || (av == bv && ai < bi);
}

class Decoder {
public:
    const DecodeParams& p;
    Smem& sm;
    uint8_t* ring;
    float* xs;
    float* part;
    int cta, n, warp, lane, tid;
    int QD, KVD, G, QKVR;
    GemvGeo gA, gC, gD, gE, gF;
    uint32_t bar_no = 0;   // grid barriers passed / published so far in this launch
    uint32_t it = 0;       // ring pieces consumed (consumer) or walked (producer)
    uint32_t n_issued = 0; // producer: pieces whose copies were issued (all before any abort)

    __device__ Decoder(const DecodeParams& p_, Smem& sm_, uint8_t* dyn)
        : p(p_), sm(sm_) {
        ring = dyn;
        xs = reinterpret_cast<float*>(dyn + NSLOT * SLOT_BYTES);
        part = xs + p.xs_cap;
        cta = blockIdx.x;
        n = gridDim.x;
        tid = threadIdx.x;
        warp = tid >> 5;
        lane = tid & 31;
        QD = p.NQ * HD;
        KVD = p.NKV * HD;
        G = p.NQ / p.NKV;
        QKVR = QD + 2 * KVD;
        const long long offC = (long long)QKVR * p.H;
        const long long offD = offC + (long long)p.H * QD;
        const long long offE = offD + 2LL * p.I * p.H;
        gA = make_geo(QKVR, p.H, cta, n, 0, 0);
        gC = make_geo(p.H, QD, cta, n, offC, 0);
        gD = make_geo(2LL * p.I, p.H, cta, n, offD, 1);
        gE = make_geo(p.H, p.I, cta, n, offE, 0);
        gF = make_geo(p.V, p.H, cta, n, 0, 0);
    }

    // ------------------------------------------------------------------ errors and waits
    __device__ bool aborted() const { return *reinterpret_cast<volatile const int*>(&sm.abort) != 0; }

    __device__ void fail(int code, int where) {
        *reinterpret_cast<volatile int*>(&sm.abort) = 1;
        if (atomicCAS(&p.err[0], 0, code) == 0) {
            p.err[1] = cta;
            p.err[2] = where;
            __threadfence();
        }
    }

    __device__ bool wait_mbar(uint64_t* bar, uint32_t parity, int code) {
        if (aborted()) return false;
        uint32_t spins = 0;
        uint64_t t0 = 0;
        while (!mbar_try_wait(bar, parity)) {
            ++spins;
            if (spins == 16) t0 = globaltimer_ns();
            else if (spins > 16 && (spins & 63) == 0) {
                if (aborted()) return false;
                if (ld_volatile_s32(p.err) != 0) { *reinterpret_cast<volatile int*>(&sm.abort) = 1; return false; }
                if (globaltimer_ns() - t0 > (uint64_t)p.timeout_ns) { fail(code, (int)it); return false; }
            }
        }
        return true;
    }

    // consumers: wait until every CTA published barrier `b` (b >= 1), then release all consumers
    __device__ void grid_wait(uint32_t b) {
        if (warp == 0 && !aborted()) {
            const unsigned long long target = ((unsigned long long)p.epoch << 32) | b;
            uint32_t spins = 0;
            uint64_t t0 = 0;
            for (;;) {
                bool ok = true;
                for (int j = lane; j < n; j += 32) ok &= ld_acquire_gpu(p.flags + j) >= target;
                if (__all_sync(0xFFFFFFFFu, ok)) break;
                ++spins;
                if (spins == 64) t0 = globaltimer_ns();
                if (spins > 64 && (spins & 31) == 0) {
                    int bad = 0;
                    if (lane == 0) {
                        if (ld_volatile_s32(p.err) != 0) bad = 1;
                        else if (globaltimer_ns() - t0 > (uint64_t)p.timeout_ns) bad = 2;
                    }
                    bad = __shfl_sync(0xFFFFFFFFu, bad, 0);
                    if (bad) {
                        if (lane == 0) {
                            if (bad == 2) fail(DERR_TIMEOUT_GRID, (int)b);
                            else *reinterpret_cast<volatile int*>(&sm.abort) = 1;
                        }
                        break;
                    }
                }
            }
        }
        named_bar_sync(1, NCT);
        // after the barrier every poller's acquire is ordered before this release
        if (tid == 0) st_release_cta_shared(&sm.progress, b);
    }

    // consumers: all epilogue writes done -> publish barrier number ++bar_no
    __device__ void grid_arrive() {
        named_bar_sync(1, NCT);
        ++bar_no;
        if (tid == 0) {
            __threadfence();
            st_release_gpu(p.flags + cta, ((unsigned long long)p.epoch << 32) | bar_no);
        }
    }

    // ------------------------------------------------------------------ consumer helpers
    __device__ float block_sum(float v) {
        v = warp_sum(v);
        if (lane == 0) sm.red[warp] = v;
        named_bar_sync(1, NCT);
        if (warp == 0) {
            float t = lane < NCW ? sm.red[lane] : 0.f;
            t = warp_sum(t);
            if (lane == 0) sm.red[32] = t;
        }
        named_bar_sync(1, NCT);
        return sm.red[32];
    }

    // xs[i] = src[i] * (1/sqrt(mean(src^2) + eps)) * w[i]   (cpu_inference.rs:189-194)
    // src is the residual stream x, or (from_embed) the embedding row of `token`, in which case the
    // CTA also initialises its own rows [x_r0, x_r1) of the global residual stream.
    __device__ void norm_prologue(const uint16_t* w, bool from_embed, unsigned token) {
        const int H = p.H;
        float ss = 0.f;
        const uint16_t* erow = p.embed + (size_t)token * H;
        for (int i = tid; i < H; i += NCT) {
            float v = from_embed ? bf16_to_f32(__ldg(erow + i)) : __ldcg(p.x + i);
            xs[i] = v;
            ss = fmaf(v, v, ss);
            if (from_embed && i >= gC.r0 && i < gC.r1) __stcg(p.x + i, v);
        }
        const float tot = block_sum(ss);
        const float s = 1.0f / sqrtf(tot / (float)H + p.eps);
        for (int i = tid; i < H; i += NCT) xs[i] = xs[i] * s * bf16_to_f32(__ldg(w + i));
        named_bar_sync(1, NCT);
    }

    __device__ void load_prologue(const float* src, int K) {
        for (int i = tid; i < K; i += NCT) xs[i] = __ldcg(src + i);
        named_bar_sync(1, NCT);
    }

    // all ring pieces of one GEMV phase: part[(row - r0) * segs + seg] = partial dot product
    __device__ void gemv_consume(const GemvGeo& g) {
        const int myseg = warp % g.segs;
        float xr[32];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            if (i < g.cpl) {
                const float4* xp = reinterpret_cast<const float4*>(xs + myseg * g.segw + (i * 32 + lane) * 8);
                float4 a = xp[0], b = xp[1];
                xr[i * 8 + 0] = a.x; xr[i * 8 + 1] = a.y; xr[i * 8 + 2] = a.z; xr[i * 8 + 3] = a.w;
                xr[i * 8 + 4] = b.x; xr[i * 8 + 5] = b.y; xr[i * 8 + 6] = b.z; xr[i * 8 + 7] = b.w;
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) xr[i * 8 + j] = 0.f;
            }
        }
        for (int r = g.r0; r < g.r1; r += g.rpp) {
            const int nr = min(g.rpp, g.r1 - r);
            const int units = nr * g.segs;
            const int slot = it % NSLOT;
            const uint32_t par = (it / NSLOT) & 1;
            const bool ok = wait_mbar(&sm.full[slot], par, DERR_TIMEOUT_FULL);
            if (ok) {
                const uint8_t* base = ring + slot * SLOT_BYTES;
                for (int u = warp; u < units; u += NCW) {
                    const int rl = u / g.segs;  // u % segs == myseg because NCW % segs == 0
                    const uint4* wp = reinterpret_cast<const uint4*>(base + ((size_t)rl * g.K + (size_t)myseg * g.segw) * 2);
                    float acc = 0.f;
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        if (i < g.cpl) acc += dot8(wp[i * 32 + lane], xr + i * 8);
                    acc = warp_sum(acc);
                    if (lane == 0) part[(r - g.r0 + rl) * g.segs + myseg] = acc;
                }
            }
            __syncwarp();
            if (lane == 0 && ok) mbar_arrive(&sm.empty[slot]);  // a slot is released only after its data landed
            ++it;
        }
        named_bar_sync(1, NCT);
    }

    __device__ __forceinline__ float row_value(const GemvGeo& g, int rl) const {
        float y = 0.f;
        for (int sgi = 0; sgi < g.segs; sgi++) y += part[rl * g.segs + sgi];
        return y;
    }

    // ------------------------------------------------------------------ attention (phase B)
    // per-head RMSNorm (q_norm/k_norm) then rotate-half RoPE, one warp per 128-vector
    // (cpu_inference.rs:134-138, :196-215; the table is the one MetalKVCache builds, :141-154)
    __device__ void head_norm_rope(const float* src, const uint16_t* nw, const float2* rrow, float* dst) {
        float4 v = __ldcg(reinterpret_cast<const float4*>(src) + lane);
        float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        ss = warp_sum(ss);
        const float s = 1.0f / sqrtf(ss / (float)HD + p.eps);
        const int d0 = lane * 4;
        float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; j++) e[j] = e[j] * s * bf16_to_f32(__ldg(nw + d0 + j));
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float other = __shfl_xor_sync(0xFFFFFFFFu, e[j], 16);  // element d +- 64
            const float2 cs = rrow[(d0 + j) & 63];
            if (lane < 16) o[j] = e[j] * cs.x - other * cs.y;   // x[i]      = a*cos - b*sin
            else o[j] = e[j] * cs.x + other * cs.y;             // x[i+half] = b*cos + a*sin
        }
        reinterpret_cast<float4*>(dst)[lane] = make_float4(o[0], o[1], o[2], o[3]);
    }

    // online-softmax update over np positions whose K/V rows (128 f32 each) are in shared memory
    __device__ void attn_block(const float* Kb, const float* Vb, int np, int buf, const float4* q4,
                               float& m, float& l, float& acc) {
        for (int pp = warp; pp < np; pp += NCW) {
            const float4 k4 = reinterpret_cast<const float4*>(Kb + pp * HD)[lane];
            for (int h = 0; h < G; h++) {
                float d = q4[h].x * k4.x + q4[h].y * k4.y + q4[h].z * k4.z + q4[h].w * k4.w;
                d = warp_sum(d);
                if (lane == 0) sm.sc[buf][h][pp] = d * p.scale;
            }
        }
        named_bar_sync(1, NCT);
        if (tid < G * HD) {
            const int h = tid >> 7, d = tid & (HD - 1);
            float mp = -INFINITY;
            for (int pp = 0; pp < np; pp++) mp = fmaxf(mp, sm.sc[buf][h][pp]);
            const float mn = fmaxf(m, mp);
            const float corr = (m == -INFINITY) ? 0.f : expf(m - mn);
            l *= corr;
            acc *= corr;
            for (int pp = 0; pp < np; pp++) {
                const float e = expf(sm.sc[buf][h][pp] - mn);
                l += e;
                acc = fmaf(e, Vb[pp * HD + d], acc);
            }
            m = mn;
        }
    }

    __device__ void attention_consume(int l, int pos) {
        const AttnItem a = attn_item(p, cta, pos);
        if (!a.active) return;   // uniform over the CTA
        const uint16_t* nrm = p.layer_n + (size_t)l * p.norm_stride;
        const uint16_t* qn = nrm + 2 * p.H;
        const uint16_t* kn = qn + HD;
        const float2* rrow = p.rope + (size_t)pos * (HD / 2);
        // q heads g*G .. g*G+G-1, and (last chunk) this position's k and v
        if (warp < G) head_norm_rope(p.qkv + (size_t)(a.g * G + warp) * HD, qn, rrow, sm.qs[warp]);
        if (a.has_cur) {
            if (warp == G) head_norm_rope(p.qkv + QD + (size_t)a.g * HD, kn, rrow, sm.ks);
            if (warp == G + 1) reinterpret_cast<float4*>(sm.vs)[lane] =
                __ldcg(reinterpret_cast<const float4*>(p.qkv + QD + KVD + (size_t)a.g * HD) + lane);
        }
        named_bar_sync(1, NCT);
        if (a.has_cur && tid < 2 * HD) {  // append K/V at slot `pos` (cpu_inference.rs:140-141)
            const size_t off = (((size_t)l * p.NKV + a.g) * p.max_seq + pos) * HD;
            if (tid < HD) __stcg(p.kc + off + tid, sm.ks[tid]);
            else __stcg(p.vc + off + tid - HD, sm.vs[tid - HD]);
        }
        float4 q4[MAX_G];
        for (int h = 0; h < MAX_G; h++)
            q4[h] = h < G ? reinterpret_cast<const float4*>(sm.qs[h])[lane] : make_float4(0, 0, 0, 0);
        float m = -INFINITY, lsum = 0.f, acc = 0.f;
        int buf = 0;
        const int tc1 = a.has_cur ? pos : a.t1;  // cached positions [t0, tc1)
        for (int t = a.t0; t < tc1; t += ATT_P) {
            const int np = min(ATT_P, tc1 - t);
            const int slot = it % NSLOT;
            const uint32_t par = (it / NSLOT) & 1;
            const bool ok = wait_mbar(&sm.full[slot], par, DERR_TIMEOUT_FULL);
            const float* Kb = reinterpret_cast<const float*>(ring + slot * SLOT_BYTES);
            const float* Vb = Kb + ATT_P * HD;
            attn_block(Kb, Vb, np, buf, q4, m, lsum, acc);
            __syncwarp();
            if (lane == 0 && ok) mbar_arrive(&sm.empty[slot]);
            ++it;
            buf ^= 1;
        }
        if (a.has_cur) {
            attn_block(sm.ks, sm.vs, 1, buf, q4, m, lsum, acc);
            buf ^= 1;
        }
        // publish this chunk's partial, then the last chunk of the KV head merges them
        if (tid < G * HD) {
            const int h = tid >> 7, d = tid & (HD - 1);
            float* dst = p.apart + ((size_t)(a.g * p.S + a.s) * G + h) * APART_STRIDE;
            __stcg(dst + d, acc);
            if (d == 0) { __stcg(dst + HD, m); __stcg(dst + HD + 1, lsum); }
        }
        named_bar_sync(1, NCT);
        if (tid == 0) {
            __threadfence();
            const unsigned old = atomicAdd(p.acount + a.g, 1u);
            const int last = (old == (unsigned)(a.S_eff - 1));
            if (last) {
                p.acount[a.g] = 0u;
                __threadfence();
            }
            sm.is_last = last;
        }
        named_bar_sync(1, NCT);
        if (sm.is_last && tid < G * HD) {
            const int h = tid >> 7, d = tid & (HD - 1);
            float M = -INFINITY;
            for (int s = 0; s < a.S_eff; s++)
                M = fmaxf(M, __ldcg(p.apart + ((size_t)(a.g * p.S + s) * G + h) * APART_STRIDE + HD));
            float Lt = 0.f, O = 0.f;
            for (int s = 0; s < a.S_eff; s++) {
                const float* src = p.apart + ((size_t)(a.g * p.S + s) * G + h) * APART_STRIDE;
                const float w = expf(__ldcg(src + HD) - M);
                Lt = fmaf(w, __ldcg(src + HD + 1), Lt);
                O = fmaf(w, __ldcg(src + d), O);
            }
            __stcg(p.att + (size_t)(a.g * G + h) * HD + d, O / Lt);
        }
    }

    // ------------------------------------------------------------------ lm_head + argmax
    __device__ void lm_epilogue() {
        const GemvGeo& g = gF;
        const int nloc = g.r1 - g.r0;
        float bv = -INFINITY;
        unsigned bi = NONE_IDX;
        for (int i = tid; i < nloc; i += NCT) {
            const float y = row_value(g, i);
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
        if (lane == 0) { sm.redv[warp] = bv; sm.redi[warp] = bi; }
        named_bar_sync(1, NCT);
        if (tid == 0) {
            for (int w = 1; w < NCW; w++)
                if (am_better(sm.redv[w], sm.redi[w], bv, bi)) { bv = sm.redv[w]; bi = sm.redi[w]; }
            __stcg(p.am_val + cta, bv);
            __stcg(p.am_idx + cta, bi);
        }
    }

    // after the lm_head barrier: every CTA reduces the partials to the same next token
    __device__ unsigned argmax_combine() {
        if (warp == 0) {
            float bv = -INFINITY;
            unsigned bi = NONE_IDX;
            for (int j = lane; j < n; j += 32) {
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
            if (lane == 0) {
                unsigned t = bi;
                if (__ldcg(p.nan0) != 0 || t == NONE_IDX || t >= (unsigned)p.V) t = 0;  // first-strict-max rule
                sm.token = t;
            }
        }
        named_bar_sync(1, NCT);
        return sm.token;
    }

    // ------------------------------------------------------------------ consumer main loop
    __device__ void consume() {
        unsigned token = __ldcg(p.tok_in);
        if (token >= (unsigned)p.V) {
            if (tid == 0) fail(DERR_BAD_TOKEN, (int)token);
            token = 0;
        }
        for (int step = 0; step < p.steps; step++) {
            const int pos = p.start_pos + step;
            for (int l = 0; l < p.L; l++) {
                const uint16_t* nrm = p.layer_n + (size_t)l * p.norm_stride;
                // A: rmsnorm -> q|k|v
                if (l > 0) grid_wait(bar_no);
                norm_prologue(nrm, l == 0, token);
                gemv_consume(gA);
                for (int i = tid; i < gA.r1 - gA.r0; i += NCT) __stcg(p.qkv + gA.r0 + i, row_value(gA, i));
                grid_arrive();
                // B: q/k norm + rope, KV append, attention
                grid_wait(bar_no);
                attention_consume(l, pos);
                grid_arrive();
                // C: o_proj + residual
                grid_wait(bar_no);
                load_prologue(p.att, QD);
                gemv_consume(gC);
                for (int i = tid; i < gC.r1 - gC.r0; i += NCT)
                    __stcg(p.x + gC.r0 + i, __ldcg(p.x + gC.r0 + i) + row_value(gC, i));
                grid_arrive();
                // D: rmsnorm -> gate|up -> silu(gate) * up
                grid_wait(bar_no);
                norm_prologue(nrm + p.H, false, 0);
                gemv_consume(gD);
                for (int i = tid; i < (gD.r1 - gD.r0) / 2; i += NCT) {
                    const float gt = row_value(gD, 2 * i), up = row_value(gD, 2 * i + 1);
                    __stcg(p.hbuf + gD.r0 / 2 + i, gt / (1.0f + expf(-gt)) * up);
                }
                grid_arrive();
                // E: down_proj + residual
                grid_wait(bar_no);
                load_prologue(p.hbuf, p.I);
                gemv_consume(gE);
                for (int i = tid; i < gE.r1 - gE.r0; i += NCT)
                    __stcg(p.x + gE.r0 + i, __ldcg(p.x + gE.r0 + i) + row_value(gE, i));
                grid_arrive();
            }
            // F: final rmsnorm -> lm_head -> argmax partials
            grid_wait(bar_no);
            norm_prologue(p.final_norm, false, 0);
            gemv_consume(gF);
            lm_epilogue();
            grid_arrive();
            grid_wait(bar_no);
            token = argmax_combine();
            if (cta == 0 && tid == 0 && !aborted()) {
                if (p.tok_out) p.tok_out[step + 1] = token;
                if (p.host_tok) {
                    volatile uint32_t* ht = p.host_tok;
                    ht[step + 1] = token;
                    __threadfence_system();
                    *reinterpret_cast<volatile unsigned*>(p.host_count) = (unsigned)(step + 1);
                }
            }
        }
    }

    // ------------------------------------------------------------------ producer
    __device__ bool slot_acquire(uint32_t& slot) {
        slot = it % NSLOT;
        const uint32_t par = ((it / NSLOT) & 1) ^ 1;
        return wait_mbar(&sm.empty[slot], par, DERR_TIMEOUT_EMPTY);
    }

    __device__ void gemv_produce(const GemvGeo& g, const uint16_t* wbase, uint64_t pol) {
        for (int r = g.r0; r < g.r1; r += g.rpp) {
            const int nr = min(g.rpp, g.r1 - r);
            uint32_t slot;
            if (slot_acquire(slot)) {
                const uint32_t bytes = (uint32_t)nr * (uint32_t)g.K * 2u;
                mbar_arrive_expect_tx(&sm.full[slot], bytes);
                bulk_g2s_evict_first(ring + slot * SLOT_BYTES, wbase + g.woff + (size_t)r * g.K, bytes, &sm.full[slot], pol);
                n_issued = it + 1;
            }
            ++it;
        }
    }

    // barrier number after which step `step`'s attention of layer `l` is globally complete
    __device__ uint32_t attn_barrier(int step, int l) const {
        return (uint32_t)step * (uint32_t)(5 * p.L + 1) + (uint32_t)(5 * l + 2);
    }

    __device__ void attn_produce(int step, int l, int pos) {
        const AttnItem a = attn_item(p, cta, pos);
        if (!a.active) return;
        const int tc1 = a.has_cur ? pos : a.t1;
        if (a.t0 >= tc1) return;
        // K/V rows up to pos-1 are written by other CTAs in earlier steps of this launch: wait until
        // this CTA's consumers have seen that step's attention barrier, then order the async-proxy
        // reads after it.
        if (step > 0 && !aborted()) {
            const uint32_t need = attn_barrier(step - 1, l);
            uint64_t t0 = globaltimer_ns();
            while (ld_acquire_cta_shared(&sm.progress) < need) {
                if (aborted()) break;
                if (globaltimer_ns() - t0 > (uint64_t)p.timeout_ns) { fail(DERR_TIMEOUT_KV, (int)need); break; }
                __nanosleep(64);
            }
            fence_proxy_async_global();
        }
        const size_t head = ((size_t)l * p.NKV + a.g) * p.max_seq;
        for (int t = a.t0; t < tc1; t += ATT_P) {
            const int np = min(ATT_P, tc1 - t);
            uint32_t slot;
            if (slot_acquire(slot)) {
                const uint32_t bytes = (uint32_t)np * HD * 4u;
                mbar_arrive_expect_tx(&sm.full[slot], 2u * bytes);
                uint8_t* dst = ring + slot * SLOT_BYTES;
                bulk_g2s(dst, p.kc + (head + t) * HD, bytes, &sm.full[slot]);
                bulk_g2s(dst + ATT_P * HD * 4, p.vc + (head + t) * HD, bytes, &sm.full[slot]);
                n_issued = it + 1;
            }
            ++it;
        }
    }

    __device__ void produce() {
        const uint64_t pol = policy_evict_first();
        for (int step = 0; step < p.steps; step++) {
            const int pos = p.start_pos + step;
            for (int l = 0; l < p.L; l++) {
                const uint16_t* W = p.layer_w + (size_t)l * p.layer_stride;
                gemv_produce(gA, W, pol);
                attn_produce(step, l, pos);
                gemv_produce(gC, W, pol);
                gemv_produce(gD, W, pol);
                gemv_produce(gE, W, pol);
            }
            gemv_produce(gF, p.lm_head, pol);
        }
        drain();
    }

    // Normally every issued copy has been consumed by the time the producer finishes. After an
    // abort, wait (bounded) for the copies still in flight before the CTA may exit. Consumers stop
    // releasing slots once they abort, so only the last NSLOT issued pieces can be outstanding,
    // one per slot.
    __device__ void drain() {
        if (aborted()) {
            const uint32_t first = n_issued > NSLOT ? n_issued - NSLOT : 0;
            for (uint32_t j = first; j < n_issued; j++) {
                const int slot = j % NSLOT;
                const uint32_t par = (j / NSLOT) & 1;
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(&sm.full[slot], par)) {
                    if (globaltimer_ns() - t0 > (uint64_t)p.timeout_ns) {
                        atomicCAS(&p.err[3], 0, DERR_TIMEOUT_DRAIN);
                        break;
                    }
                }
            }
        }
    }
};

}  // namespace qw
