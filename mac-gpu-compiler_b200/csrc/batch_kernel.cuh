// Persistent weight-streaming decode kernel for a batch of up to 8 sequences (sm_100a).
//
// The batch form of decode_kernel.cuh: one cooperative launch runs `steps` greedy steps for nb <= 8
// independent sequences (each with its own KV cache and position), streaming every weight byte
// once per step for all of them. The reference decodes one sequence per engine
// (metal_inference.rs:286-387); this is the per-GPU batch of the box workload.
//
// Same skeleton as the batch-1 kernel (148 CTAs, 12 consumer warps + one producer lane, TMA bulk
// ring of weight and K/V pieces, tagged-word hand-offs, one grid barrier per step), with these
// differences:
//   * every hand-off buffer holds nb rows ([row][width] tagged words), and every RMSNorm has one
//     scale per row;
//   * GEMV: the CTA's weight rows meet all nb activation rows. Lane l of warp w owns column chunk
//     (w % 4) * 32 + l (8 columns) of a 1024-column block and holds those 8 columns of all nb rows
//     in registers (64 floats); warp group w / 4 takes every third weight row. Per weight row a
//     lane reads 16 bytes of weights and does 64 FMAs; the 8 row sums are reduced across the warp
//     by a transposing butterfly (9 shuffles) and across the group's 4 warps in shared memory.
//     Inputs wider than 1024 columns (o: 2048, down: 3072) are gathered and multiplied one
//     1024-column block at a time, so the staging buffer holds nb x 1024 floats;
//   * attention: one CTA per (row, KV head, chunk) item, each row over its own cache;
//   * lm_head: per weight-row piece, each warp group combines its 4 warps' sums through a
//     double-buffered shared-memory stage and keeps a running argmax per row.
//
// Measured on B200 (Qwen3-0.6B geometry, 8 rows): 1.7 ms per step against 0.99 ms for the row-mode
// graph, so qw_decode_batch runs it only when asked (QW_BATCH_DECODER=persistent). Its GEMV
// phases take as long for one row as for eight: each weight row costs about 100 instructions per
// warp (the 64 FMAs per lane and the 9-shuffle reduction), which bounds the phase, not its bytes.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "decode_kernel.cuh"
#include "ptx.cuh"

namespace qw {
namespace bk {

constexpr int NB = 8;                          // most rows of one launch
constexpr int NCW = 12;                        // consumer warps
constexpr int NCT = NCW * 32;
constexpr int NTHREADS = NCT + 32;             // + producer warp
constexpr int NSLOT = 6;                       // ring slots (144 KB)
constexpr int SLOT_BYTES = 24 * 1024;
constexpr int HD = 128;
constexpr int KBLK = 1024;                     // GEMV input columns staged at a time
constexpr int ATT_P = SLOT_BYTES / (2 * HD * 4);  // cached positions per attention ring slot (24)
constexpr int MAX_G = 3;
constexpr int MAX_S = 4;                       // attention chunks per (row, KV head)
constexpr int MAX_ROWS = 64;                   // weight rows of a layer phase per CTA
constexpr int APART = HD + 4;                  // words per attention partial: acc[128], m, l, pad
constexpr int ATT_WST = HD + 4;

// dynamic shared memory (floats after the ring)
constexpr int XS_FLOATS = NB * KBLK;                   // staged GEMV input block [row][1024]
constexpr int PG_FLOATS = MAX_ROWS * NB * 4;           // per (weight row, batch row, column warp) sums
constexpr int ACC_FLOATS = MAX_ROWS * NB;              // per (weight row, batch row) sums over blocks
constexpr int XLOC_FLOATS = MAX_ROWS * NB;             // residual rows [row][b] of phases C and E
constexpr int AST_FLOATS = NCW * MAX_G * ATT_WST;      // attention warp states
constexpr int STAGE_FLOATS = (MAX_S - 1) * MAX_G * HD; // merge stage of the other chunks' partials
constexpr int LMP_FLOATS = 2 * 3 * 4 * NB * 4;         // lm_head stage [buffer][group][row][b][column warp]
constexpr size_t DYN_BYTES = (size_t)NSLOT * SLOT_BYTES +
                             4u * (XS_FLOATS + PG_FLOATS + ACC_FLOATS + XLOC_FLOATS + AST_FLOATS + STAGE_FLOATS + LMP_FLOATS);

enum : int { BERR_NONE = 0, BERR_TIMEOUT_GRID = 1, BERR_TIMEOUT_FULL = 2, BERR_TIMEOUT_EMPTY = 3,
             BERR_TIMEOUT_KV = 4, BERR_BAD_TOKEN = 5, BERR_TIMEOUT_DRAIN = 6, BERR_TIMEOUT_DATA = 7,
             BERR_SHAPE = 8 };

struct BParams {
    const uint16_t* layer_w;     // as DecodeParams (q|k|v, o, gate/up interleaved, down per layer)
    const uint16_t* layer_n;
    const uint16_t* final_norm;
    const uint16_t* embed;
    const uint16_t* lm_head;
    // per row: its cache (K, V [L][KVH][max_seq][128] f32, RoPE table) and first position
    float* kc[NB];
    float* vc[NB];
    const float2* rope[NB];
    int max_seq[NB];
    int pos0[NB];
    // tagged words, nb rows each: x [H], q|k|v [QD + 2 KVD], h [I], att [QD], attention partials
    u64* x;
    u64* qkv;
    u64* hbuf;
    u64* att;
    u64* apart;                  // [row][KVH][S][G][APART]
    float* am_val;               // [grid][NB]
    unsigned* am_idx;            // [grid][NB]
    int* nan0;                   // [NB]: logits[row][0] is NaN
    u64* flags;                  // [grid] barrier flags: epoch << 32 | steps finished
    int* err;                    // [4] code, cta, where, detail
    const uint32_t* tok_in;      // [nb] first tokens (device)
    uint32_t* tok_out;           // [steps][nb]
    long long layer_stride, norm_stride;
    int H, I, L, NQ, NKV, V, nb, steps;
    unsigned epoch;
    float eps, scale;
    int S, min_chunk;
    long long timeout_ns;
    u64* trace;                  // [grid][14 L + 4] globaltimer stamps of step 0 (the decode kernel's layout), or null
    int stall_cta;               // test hook (-1: off): this CTA never raises its first end-of-step flag,
                                 // so every CTA's bounded barrier wait runs out and the launch reports it
};

struct BLoop {
    int step, l;
};

struct BSmem {
    __align__(16) float qs[MAX_G][HD];
    __align__(16) float ks[HD];
    __align__(16) float vs[HD];
    GemvGeo geo[5];              // A (q|k|v), C (o), D (gate|up), E (down), F (lm_head)
    float ml[MAX_S][MAX_G][2];
    float ssq[NCW][NB];          // per warp and row: sum of squares of the last RMSNorm input
    float redv[NCW][NB];
    unsigned redi[NCW][NB];
    uint64_t full[NSLOT];
    uint64_t empty[NSLOT];
    BParams prm;
    uint32_t ring_it[NCW + 1];
    uint32_t n_issued;
    BLoop loop[NCW + 1];
    unsigned tokens[NB];
    uint32_t progress;
    int abort;
};

__shared__ BSmem bk_sm;

// one attention work item: (row b, KV head g, chunk s) of CTA `cta` at the rows' positions
struct BItem {
    int b, g, s, t0, t1, S_eff, pos;
    bool active, has_cur;
};

__device__ inline BItem bitem(const BParams& p, int cta, int step) {
    BItem a;
    const int per_row = p.NKV * p.S;
    a.b = cta / per_row;
    a.g = (cta / p.S) % p.NKV;
    a.s = cta % p.S;
    a.active = cta < p.nb * per_row;
    a.pos = a.active ? p.pos0[a.b] + step : 0;
    const int n_t = a.pos + 1;
    int chunk = (n_t + p.S - 1) / p.S;
    if (chunk < p.min_chunk) chunk = p.min_chunk;
    a.S_eff = (n_t + chunk - 1) / chunk;
    a.active = a.active && a.s < a.S_eff;
    a.t0 = a.s * chunk;
    a.t1 = min(n_t, a.t0 + chunk);
    a.has_cur = a.active && a.t1 == n_t;
    return a;
}

class BDecoder {
public:
    __device__ __forceinline__ static int tid() { return (int)threadIdx.x; }
    __device__ __forceinline__ static int warp() { return (int)(threadIdx.x >> 5); }
    __device__ __forceinline__ static int lane() { return (int)(threadIdx.x & 31); }
    __device__ __forceinline__ static int cta() { return (int)blockIdx.x; }
    __device__ __forceinline__ static int nctas() { return (int)gridDim.x; }
    __device__ __forceinline__ static uint8_t* ring() { return qw_dyn; }
    __device__ __forceinline__ static float* xs() { return reinterpret_cast<float*>(qw_dyn + NSLOT * SLOT_BYTES); }
    __device__ __forceinline__ static float* pg() { return xs() + XS_FLOATS; }
    __device__ __forceinline__ static float* racc() { return pg() + PG_FLOATS; }
    __device__ __forceinline__ static float* xloc() { return racc() + ACC_FLOATS; }
    __device__ __forceinline__ static float* ast() { return xloc() + XLOC_FLOATS; }
    __device__ __forceinline__ static float* stage() { return ast() + AST_FLOATS; }
    __device__ __forceinline__ static float* lmp() { return stage() + STAGE_FLOATS; }
    __device__ __forceinline__ static uint32_t& ring_pos() { return bk_sm.ring_it[threadIdx.x >> 5]; }
    __device__ __forceinline__ static int QD() { return bk_sm.prm.NQ * HD; }
    __device__ __forceinline__ static int KVD() { return bk_sm.prm.NKV * HD; }
    __device__ __forceinline__ static int QKVR() { return QD() + 2 * KVD(); }
    __device__ __forceinline__ static int G() { return bk_sm.prm.NQ / bk_sm.prm.NKV; }
    __device__ __forceinline__ static const GemvGeo& gA() { return bk_sm.geo[0]; }
    __device__ __forceinline__ static const GemvGeo& gC() { return bk_sm.geo[1]; }
    __device__ __forceinline__ static const GemvGeo& gD() { return bk_sm.geo[2]; }
    __device__ __forceinline__ static const GemvGeo& gE() { return bk_sm.geo[3]; }
    __device__ __forceinline__ static const GemvGeo& gF() { return bk_sm.geo[4]; }

    // one thread, before the barrier that follows mbarrier initialisation: the batch-1 kernel's row
    // partition, and the shape checks this kernel relies on
    __device__ static void init_geometry(const BParams& p) {
        const int c = blockIdx.x, nc = gridDim.x;
        const long long qd = (long long)p.NQ * HD, kvd = (long long)p.NKV * HD, qkvr = qd + 2 * kvd;
        const long long offC = qkvr * p.H;
        const long long offD = offC + (long long)p.H * qd;
        const long long offE = offD + 2LL * p.I * p.H;
        bk_sm.geo[0] = make_geo(qkvr, p.H, c, nc, 0, 0, qkvr % 8 == 0 && qkvr / 8 >= nc ? 8 : 1);
        const int ux = p.H % 8 == 0 ? 8 : 1, uh = p.I % 8 == 0 ? 8 : 1;
        bk_sm.geo[1] = make_geo(p.H, (int)qd, c, nc, offC, 0, ux);
        bk_sm.geo[2] = make_geo(2LL * p.I, p.H, c, nc, offD, 1, uh);
        bk_sm.geo[3] = make_geo(p.H, p.I, c, nc, offE, 0, ux);
        bk_sm.geo[4] = make_geo(p.V, p.H, c, nc, 0, 0);
        bool ok = p.H == KBLK && qd % KBLK == 0 && p.I % KBLK == 0 && p.nb >= 1 && p.nb <= NB && p.NQ % p.NKV == 0 &&
                  p.NQ / p.NKV <= MAX_G && p.S >= 1 && p.S <= MAX_S;
        for (int k = 0; k < 4; k++) {
            const GemvGeo& g = bk_sm.geo[k];
            const int rows = g.r1 - g.r0;
            ok = ok && rows <= MAX_ROWS && (rows + g.rpp - 1) / g.rpp <= NSLOT;
        }
        if (!ok) fail(BERR_SHAPE, 0);
    }

    // ---------------------------------------------------------------- errors and bounded waits
    __device__ static bool aborted() { return *reinterpret_cast<volatile const int*>(&bk_sm.abort) != 0; }

    __device__ __noinline__ static void fail(int code, int where) {
        const BParams& p = bk_sm.prm;
        *reinterpret_cast<volatile int*>(&bk_sm.abort) = 1;
        if (atomicCAS(&p.err[0], 0, code) == 0) {
            p.err[1] = cta();
            p.err[2] = where;
            __threadfence();
        }
    }

    __device__ __forceinline__ static bool wait_expired(uint32_t& spins, uint64_t& t0, int code, int where) {
        if ((++spins & 31) != 0) return false;
        t0 = wait_check(spins, t0, code, where);
        return t0 == ~0ull;
    }

    __device__ __noinline__ static uint64_t wait_check(uint32_t spins, uint64_t t0, int code, int where) {
        const BParams& p = bk_sm.prm;
        if (aborted()) return ~0ull;
        const uint64_t now = globaltimer_ns();
        if (spins == 32) return now;
        const uint64_t waited = now - t0;
        if (waited > 50000 && (spins & 1023) == 0 && ld_volatile_s32(p.err) != 0) {
            *reinterpret_cast<volatile int*>(&bk_sm.abort) = 1;
            return ~0ull;
        }
        if (waited > (uint64_t)p.timeout_ns) {
            fail(code, where);
            return ~0ull;
        }
        return t0;
    }

    __device__ __forceinline__ static bool wait_mbar(uint64_t* bar, uint32_t parity, int code) {
        if (mbar_try_wait(bar, parity)) return true;
        if (aborted()) return false;
        uint32_t spins = 0;
        uint64_t t0 = 0;
        while (!mbar_try_wait(bar, parity))
            if (wait_expired(spins, t0, code, (int)ring_pos())) return false;
        return true;
    }

    // ring pieces pc .. pc+n-1 (n <= 32): lane j waits on piece pc + j
    __device__ __forceinline__ static bool wait_pieces(uint32_t pc, int n) {
        bool mine = true;
        if (lane() < n) mine = wait_mbar(&bk_sm.full[(pc + lane()) % NSLOT], ((pc + lane()) / NSLOT) & 1, BERR_TIMEOUT_FULL);
        const bool ok = __all_sync(0xFFFFFFFFu, mine);
        __syncwarp();
        return ok;
    }

    // phase timeline of step 0 (qw_set_trace): CTA thread 0's %globaltimer at point k of layer l
    // (k < 14), or of the step's tail (l = L)
    __device__ __forceinline__ static void stamp(int l, int k) {
        const volatile BParams& p = bk_sm.prm;
        if (p.trace != nullptr && bk_sm.loop[0].step == 0 && tid() == 0)
            p.trace[(size_t)cta() * (14 * p.L + 4) + l * 14 + k] = globaltimer_ns();
    }

    // phase tags: 12 bits of epoch, 20 bits of sequence (seq = step (5L + 1) + 5 l + phase)
    __device__ static uint32_t tag(int step, int l, int ph) {
        const volatile BParams& p = bk_sm.prm;
        const uint32_t sq = (uint32_t)step * (uint32_t)(5 * p.L + 1) + (uint32_t)(5 * l + ph);
        return ((p.epoch & 0xFFFu) << 20) | (sq & 0xFFFFFu);
    }

    // ---------------------------------------------------------------- inputs of a GEMV phase
    // xs[b][0..1024) <- the tagged words src[b * ld + col0 .. + 1024) of rows b < nb once each carries
    // `tg`; with `gain` (an RMSNorm input: col0 = 0, the row is the whole 1024-wide x) xs holds
    // x * gain and ssq[warp][b] the warp's sum of x^2 per row (the epilogues apply the scale).
    __device__ __noinline__ static void gather_rows(const u64* src, int ld, int col0, uint32_t tg, const uint16_t* gain) {
        const BParams& p = bk_sm.prm;
        constexpr int PAIRS = KBLK / 2;
        const int total = p.nb * PAIRS;
        float ss[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) ss[b] = 0.f;
        for (int base = 0; base < total; base += NCT * 4) {
            unsigned pending = 0;
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (base + tid() + j * NCT < total) pending |= 1u << j;
            uint32_t spins = 0;
            uint64_t t0 = 0;
            while (pending && !aborted()) {
                ulonglong2 w[4];
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (pending & (1u << j)) {
                        const int q = base + tid() + j * NCT, b = q / PAIRS, i = (q - b * PAIRS) * 2;
                        w[j] = ld_relaxed_v2u64(src + (size_t)b * ld + col0 + i);
                    }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if ((pending & (1u << j)) && word_tag(w[j].x) == tg && word_tag(w[j].y) == tg) {
                        const int q = base + tid() + j * NCT, b = q / PAIRS, i = (q - b * PAIRS) * 2;
                        float a = word_val(w[j].x), c = word_val(w[j].y);
                        if (gain) {
                            const uint32_t g2 = __ldg(reinterpret_cast<const uint32_t*>(gain) + (i >> 1));
#pragma unroll
                            for (int bb = 0; bb < NB; bb++)
                                if (bb == b) ss[bb] += fmaf(a, a, c * c);
                            a *= bf16_lo(g2);
                            c *= bf16_hi(g2);
                        }
                        *reinterpret_cast<float2*>(xs() + b * KBLK + i) = make_float2(a, c);
                        pending &= ~(1u << j);
                    }
                }
                if (pending && wait_expired(spins, t0, BERR_TIMEOUT_DATA, (int)tg)) break;
            }
        }
        if (gain) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
                const float t = warp_sum(ss[b]);
                if (lane() == 0) bk_sm.ssq[warp()][b] = t;
            }
        }
        named_bar_sync(1, NCT);
    }

    // layer 0 of a step: x = the embedding rows of the rows' tokens (xs <- x * gain, ssq), and the
    // CTA's residual rows xloc <- x
    __device__ __noinline__ static void embed_input(const uint16_t* gain) {
        const BParams& p = bk_sm.prm;
        float ss[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) ss[b] = 0.f;
        const int r0 = gC().r0, r1 = gC().r1;
        for (int q = tid(); q < p.nb * (KBLK / 2); q += NCT) {
            const int b = q / (KBLK / 2), i = (q - b * (KBLK / 2)) * 2;
            const uint32_t e = __ldg(reinterpret_cast<const uint32_t*>(p.embed + (size_t)bk_sm.tokens[b] * KBLK) + (i >> 1));
            const uint32_t g2 = __ldg(reinterpret_cast<const uint32_t*>(gain) + (i >> 1));
            const float a = bf16_lo(e), c = bf16_hi(e);
#pragma unroll
            for (int bb = 0; bb < NB; bb++)
                if (bb == b) ss[bb] += fmaf(a, a, c * c);
            *reinterpret_cast<float2*>(xs() + b * KBLK + i) = make_float2(a * bf16_lo(g2), c * bf16_hi(g2));
            if (i >= r0 && i < r1) xloc()[(i - r0) * NB + b] = a;
            if (i + 1 >= r0 && i + 1 < r1) xloc()[(i + 1 - r0) * NB + b] = c;
        }
#pragma unroll
        for (int b = 0; b < NB; b++) {
            const float t = warp_sum(ss[b]);
            if (lane() == 0) bk_sm.ssq[warp()][b] = t;
        }
        named_bar_sync(1, NCT);
    }

    // 1 / sqrt(mean(x^2) + eps) of row b's last RMSNorm input (after the gather's closing barrier)
    __device__ __forceinline__ static float norm_scale(int b) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < NCW; w++) t += bk_sm.ssq[w][b];
        return rsqrtf(t / (float)bk_sm.prm.H + bk_sm.prm.eps);
    }

    // this lane's 8 columns (chunk (warp % 4) * 32 + lane of the staged block) of every row
    __device__ __forceinline__ static void load_x(float (&xr)[NB][8]) {
        const int c = (warp() & 3) * 32 + lane();
#pragma unroll
        for (int b = 0; b < NB; b++) {
            const float4 u = reinterpret_cast<const float4*>(xs() + b * KBLK + c * 8)[0];
            const float4 v = reinterpret_cast<const float4*>(xs() + b * KBLK + c * 8)[1];
            xr[b][0] = u.x; xr[b][1] = u.y; xr[b][2] = u.z; xr[b][3] = u.w;
            xr[b][4] = v.x; xr[b][5] = v.y; xr[b][6] = v.z; xr[b][7] = v.w;
        }
    }

    // one weight row's 16-byte chunk against the lane's 8 columns of all rows, then the warp sum per
    // row by a transposing butterfly: afterwards lane l (l % 4 == 0) holds row l / 4's total
    __device__ __forceinline__ static float row_dot(uint4 w, const float (&xr)[NB][8]) {
        const float2 w0 = make_float2(bf16_lo(w.x), bf16_hi(w.x)), w1 = make_float2(bf16_lo(w.y), bf16_hi(w.y));
        const float2 w2 = make_float2(bf16_lo(w.z), bf16_hi(w.z)), w3 = make_float2(bf16_lo(w.w), bf16_hi(w.w));
        float v[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float2 a = __fmul2_rn(w0, make_float2(xr[b][0], xr[b][1]));
            float2 c = __fmul2_rn(w1, make_float2(xr[b][2], xr[b][3]));
            a = __ffma2_rn(w2, make_float2(xr[b][4], xr[b][5]), a);
            c = __ffma2_rn(w3, make_float2(xr[b][6], xr[b][7]), c);
            v[b] = (a.x + a.y) + (c.x + c.y);
        }
        const bool h16 = lane() & 16, h8 = lane() & 8, h4 = lane() & 4;
        float u[4];
#pragma unroll
        for (int i = 0; i < 4; i++) u[i] = (h16 ? v[i + 4] : v[i]) + __shfl_xor_sync(0xFFFFFFFFu, h16 ? v[i] : v[i + 4], 16);
        float t[2];
#pragma unroll
        for (int i = 0; i < 2; i++) t[i] = (h8 ? u[i + 2] : u[i]) + __shfl_xor_sync(0xFFFFFFFFu, h8 ? u[i] : u[i + 2], 8);
        float s = (h4 ? t[1] : t[0]) + __shfl_xor_sync(0xFFFFFFFFu, h4 ? t[0] : t[1], 4);
        s += __shfl_xor_sync(0xFFFFFFFFu, s, 2);
        s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
        return s;
    }

    // ---------------------------------------------------------------- GEMV phases
    // One layer phase over its K / 1024 input blocks. Block 0's input is staged by the caller; block
    // kb > 0 is gathered here from src (rows of width ld, tagged tg_in). For each block the warps of
    // group warp / 4 multiply every third weight row of the CTA (ring pieces, all resident: a phase's
    // pieces fit in the ring) and the group's 4 column warps' sums meet in pg; racc[row][b] adds the
    // blocks in order. The pieces are released after the last block.
    __device__ __noinline__ static void gemv_phase(const GemvGeo& gs, const u64* src, int ld, uint32_t tg_in) {
        uint32_t& it = ring_pos();
        const GemvGeo g = gs;
        const uint32_t pc = it;
        const int nrows = g.r1 - g.r0, nkb = g.K / KBLK, npieces = (nrows + g.rpp - 1) / g.rpp;
        const int grp = warp() >> 2, cw = warp() & 3, c = cw * 32 + lane();
        bool ok = true;
        for (int kb = 0; kb < nkb; kb++) {
            if (kb > 0) gather_rows(src, ld, kb * KBLK, tg_in, nullptr);
            float xr[NB][8];
            load_x(xr);
            if (kb == 0) ok = wait_pieces(pc, npieces);
            if (ok) {
                #pragma unroll 1
                for (int r = grp; r < nrows; r += 3) {
                    const int pce = r / g.rpp;
                    const uint4 w = *reinterpret_cast<const uint4*>(ring() + ((pc + pce) % NSLOT) * SLOT_BYTES +
                                                                    (size_t)(r - pce * g.rpp) * g.K * 2 +
                                                                    (size_t)(kb * KBLK + c * 8) * 2);
                    const float s = row_dot(w, xr);
                    if ((lane() & 3) == 0) pg()[(r * NB + (lane() >> 2)) * 4 + cw] = s;
                }
            }
            named_bar_sync(1, NCT);
            for (int i = tid(); i < nrows * NB; i += NCT) {
                const float* q = pg() + i * 4;
                const float s = (q[0] + q[1]) + (q[2] + q[3]);
                racc()[i] = kb == 0 ? s : racc()[i] + s;
            }
            named_bar_sync(1, NCT);
        }
        it = pc + npieces;
        // every warp has read the phase's pieces: one lane per slot releases it for all 12 warps
        if (warp() == 0 && lane() < npieces && !aborted()) mbar_arrive_cnt(&bk_sm.empty[(pc + lane()) % NSLOT], NCW);
    }

    // phase A's outputs: q|k|v[b][row] = sum * the row's input RMSNorm scale
    __device__ __noinline__ static void store_qkv(uint32_t tg) {
        const BParams& p = bk_sm.prm;
        const GemvGeo& g = gA();
        const int nrows = g.r1 - g.r0, w = QKVR();
        for (int i = tid(); i < nrows * NB; i += NCT) {
            const int r = i / NB, b = i - r * NB;
            if (b < p.nb) st_relaxed_u64(p.qkv + (size_t)b * w + g.r0 + r, tagged(racc()[i] * norm_scale(b), tg));
        }
    }

    // phase D's outputs: h[b][i] = silu(gate_i) * up_i over the CTA's interleaved gate/up rows
    __device__ __noinline__ static void silu_rows(uint32_t tg) {
        const BParams& p = bk_sm.prm;
        const GemvGeo& g = gD();
        const int npair = (g.r1 - g.r0) / 2;
        for (int i = tid(); i < npair * NB; i += NCT) {
            const int q = i / NB, b = i - q * NB;
            if (b < p.nb) {
                const float sc = norm_scale(b);
                const float gt = racc()[(2 * q) * NB + b] * sc, up = racc()[(2 * q + 1) * NB + b] * sc;
                st_relaxed_u64(p.hbuf + (size_t)b * p.I + g.r0 / 2 + q, tagged(gt / (1.0f + __expf(-gt)) * up, tg));
            }
        }
    }

    // phases C and E: x[b][row] += sum on the CTA's residual rows (cpu_inference.rs:163-164, :171-172)
    __device__ __noinline__ static void residual_rows(const GemvGeo& g, uint32_t tg) {
        const BParams& p = bk_sm.prm;
        const int nrows = g.r1 - g.r0;
        for (int i = tid(); i < nrows * NB; i += NCT) {
            const int r = i / NB, b = i - r * NB;
            if (b < p.nb) {
                const float v = xloc()[i] + racc()[i];
                xloc()[i] = v;
                st_relaxed_u64(p.x + (size_t)b * p.H + g.r0 + r, tagged(v, tg));
            }
        }
    }

    // phase F: the CTA's lm_head rows streamed piece by piece (each warp releases a piece once read);
    // per piece each warp group's 4 column warps meet in a double-buffered stage, and group thread
    // t < 32 keeps a running argmax of row b = t % 8 over piece rows j = t / 8 (the reference rule:
    // first strict max, NaN never wins, common/mod.rs:17-22). The CTA's best per row goes to am_*.
    __device__ __noinline__ static void lm_head_argmax() {
        const BParams& p = bk_sm.prm;
        const GemvGeo g = gF();
        uint32_t& it = ring_pos();
        const int nrows = g.r1 - g.r0, npieces = (nrows + g.rpp - 1) / g.rpp;
        const int grp = warp() >> 2, cw = warp() & 3, c = cw * 32 + lane(), gt = tid() - grp * 128;
        const int mb = gt & 7, mj = gt >> 3;
        const float sc = mb < p.nb ? norm_scale(mb) : 1.f;
        float xr[NB][8];
        load_x(xr);
        float bv = -INFINITY;
        unsigned bi = NONE_IDX;
        #pragma unroll 1
        for (int q = 0; q < npieces; q++) {
            const uint32_t pc = it;
            const bool ok = wait_pieces(pc, 1);
            const int prow0 = q * g.rpp, pn = min(g.rpp, nrows - prow0);
            float* st = lmp() + ((q & 1) * 3 + grp) * (4 * NB * 4);
            if (ok) {
                #pragma unroll 1
                for (int j = 0; j < 4; j++) {
                    const int r = grp + 3 * j;
                    if (r < pn) {
                        const uint4 w = *reinterpret_cast<const uint4*>(ring() + (pc % NSLOT) * SLOT_BYTES + (size_t)r * g.K * 2 +
                                                                        (size_t)c * 16);
                        const float s = row_dot(w, xr);
                        if ((lane() & 3) == 0) st[(j * NB + (lane() >> 2)) * 4 + cw] = s;
                    }
                }
            }
            __syncwarp();
            if (lane() == 0 && ok) mbar_arrive(&bk_sm.empty[pc % NSLOT]);
            it = pc + 1;
            named_bar_sync(2 + grp, 128);
            if (gt < 32 && mb < p.nb && ok) {
                const int r = grp + 3 * mj;
                if (r < pn) {
                    const float* v = st + (mj * NB + mb) * 4;
                    const float y = ((v[0] + v[1]) + (v[2] + v[3])) * sc;
                    const unsigned row = (unsigned)(g.r0 + prow0 + r);
                    if (!isnan(y) && am_better(y, row, bv, bi)) {
                        bv = y;
                        bi = row;
                    }
                    if (row == 0) __stcg(p.nan0 + mb, isnan(y) ? 1 : 0);
                }
            }
        }
        if (gt < 32) {
            bk_sm.redv[grp * 4 + mj][mb] = bv;
            bk_sm.redi[grp * 4 + mj][mb] = bi;
        }
        named_bar_sync(1, NCT);
        if (tid() < p.nb) {
            const int b = tid();
            float v = -INFINITY;
            unsigned ix = NONE_IDX;
            for (int k = 0; k < NCW; k++)
                if (am_better(bk_sm.redv[k][b], bk_sm.redi[k][b], v, ix)) {
                    v = bk_sm.redv[k][b];
                    ix = bk_sm.redi[k][b];
                }
            __stcg(p.am_val + (size_t)cta() * NB + b, v);
            __stcg(p.am_idx + (size_t)cta() * NB + b, ix);
        }
    }

    // ---------------------------------------------------------------- end of a step
    __device__ __noinline__ static void step_barrier(uint32_t done) {
        const BParams& p = bk_sm.prm;
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
                for (int j = lane(); j < nctas(); j += 32) ok &= ld_relaxed_u64(p.flags + j) >= target;
                if (__all_sync(0xFFFFFFFFu, ok)) break;
                int stop = 0;
                if (lane() == 0) stop = wait_expired(spins, t0, BERR_TIMEOUT_GRID, (int)done);
                if (__shfl_sync(0xFFFFFFFFu, stop, 0)) break;
            }
            fence_acq_rel_gpu();
        }
        named_bar_sync(1, NCT);
        if (tid() == 0) st_release_cta_shared(&bk_sm.progress, done);
    }

    // after the barrier: every CTA reduces the partials to the same next token per row
    __device__ __noinline__ static void argmax_combine() {
        const BParams& p = bk_sm.prm;
        if (warp() < p.nb) {
            const int b = warp();
            float bv = -INFINITY;
            unsigned bi = NONE_IDX;
            for (int j = lane(); j < nctas(); j += 32) {
                const float v = __ldcg(p.am_val + (size_t)j * NB + b);
                const unsigned i = __ldcg(p.am_idx + (size_t)j * NB + b);
                if (am_better(v, i, bv, bi)) {
                    bv = v;
                    bi = i;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
                const unsigned oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
                if (am_better(ov, oi, bv, bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (lane() == 0) {
                unsigned t = bi;
                if (__ldcg(p.nan0 + b) != 0 || t == NONE_IDX || t >= (unsigned)p.V) t = 0;  // first-strict-max rule
                bk_sm.tokens[b] = t;
            }
        }
        named_bar_sync(1, NCT);
    }

    // ---------------------------------------------------------------- attention (phase B)
    // one warp: a tagged 128-vector (4 words per lane)
    __device__ __forceinline__ static float4 gather_head(const u64* src, uint32_t tg) {
        uint32_t spins = 0;
        uint64_t t0 = 0;
        ulonglong2 a = make_ulonglong2(0, 0), b = make_ulonglong2(0, 0);
        while (!aborted()) {
            a = ld_relaxed_v2u64(src + lane() * 4);
            b = ld_relaxed_v2u64(src + lane() * 4 + 2);
            const bool ok = word_tag(a.x) == tg && word_tag(a.y) == tg && word_tag(b.x) == tg && word_tag(b.y) == tg;
            if (__all_sync(0xFFFFFFFFu, ok)) break;
            int stop = 0;
            if (lane() == 0) stop = wait_expired(spins, t0, BERR_TIMEOUT_DATA, (int)tg);
            if (__shfl_sync(0xFFFFFFFFu, stop, 0)) break;
        }
        return make_float4(word_val(a.x), word_val(a.y), word_val(b.x), word_val(b.y));
    }

    // per-head RMSNorm (q_norm / k_norm gains nw) and rotate-half RoPE (cpu_inference.rs:134-138,
    // :196-215) of one warp's head into dst
    __device__ __forceinline__ static void head_norm_rope(float4 v, const uint16_t* nw, const float2* rrow, float* dst) {
        float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        ss = warp_sum(ss);
        const float s = rsqrtf(ss / (float)HD + bk_sm.prm.eps);
        const int d0 = lane() * 4;
        float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; j++) e[j] = e[j] * s * bf16_to_f32(__ldg(nw + d0 + j));
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float other = __shfl_xor_sync(0xFFFFFFFFu, e[j], 16);
            const float2 cs = rrow[(d0 + j) & 63];
            o[j] = lane() < 16 ? e[j] * cs.x - other * cs.y : e[j] * cs.x + other * cs.y;
        }
        reinterpret_cast<float4*>(dst)[lane()] = make_float4(o[0], o[1], o[2], o[3]);
    }

    struct WarpSoftmax {
        float m[MAX_G], l[MAX_G];
        float4 acc[MAX_G];
    };

    // up to two cached positions into a warp's running softmax (cpu_inference.rs:144-161)
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
                s0[h] += __shfl_xor_sync(0xFFFFFFFFu, s0[h], o);
                s1[h] += __shfl_xor_sync(0xFFFFFFFFu, s1[h], o);
            }
        }
#pragma unroll
        for (int h = 0; h < GQ; h++) {
            const float a0 = s0[h] * scale, a1 = has1 ? s1[h] * scale : -INFINITY;
            const float mn = fmaxf(ws.m[h], fmaxf(a0, a1));
            const float corr = __expf(ws.m[h] - mn);
            const float p0 = __expf(a0 - mn), p1 = __expf(a1 - mn);
            ws.l[h] = fmaf(ws.l[h], corr, p0 + p1);
            ws.acc[h].x = fmaf(ws.acc[h].x, corr, fmaf(p0, v0.x, p1 * v1.x));
            ws.acc[h].y = fmaf(ws.acc[h].y, corr, fmaf(p0, v0.y, p1 * v1.y));
            ws.acc[h].z = fmaf(ws.acc[h].z, corr, fmaf(p0, v0.z, p1 * v1.z));
            ws.acc[h].w = fmaf(ws.acc[h].w, corr, fmaf(p0, v0.w, p1 * v1.w));
            ws.m[h] = mn;
        }
    }

    // item (row b, KV head g, chunk s): q/k norm + RoPE, K/V append (the chunk with the row's
    // position), the chunk's online softmax over ring pieces, a partial per query head for the
    // chunk-0 CTA, which merges the chunks in order into att[b]
    template <int GQ>
    __device__ __noinline__ static void attention_g(int step, int l) {
        const BParams& p = bk_sm.prm;
        uint32_t& it = ring_pos();
        const BItem a = bitem(p, cta(), step);
        if (!a.active) return;  // uniform over the CTA
        const int b = a.b, pos = a.pos;
        const uint16_t* qn = p.layer_n + (size_t)l * p.norm_stride + 2 * p.H;
        const uint16_t* kn = qn + HD;
        const float2* rrow = p.rope[b] + (size_t)pos * (HD / 2);
        const uint32_t tgA = tag(step, l, 1), tgB = tag(step, l, 2);
        const u64* qkv = p.qkv + (size_t)b * QKVR();
        if (warp() < GQ) head_norm_rope(gather_head(qkv + (size_t)(a.g * GQ + warp()) * HD, tgA), qn, rrow, bk_sm.qs[warp()]);
        if (a.has_cur) {
            if (warp() == GQ) head_norm_rope(gather_head(qkv + QD() + (size_t)a.g * HD, tgA), kn, rrow, bk_sm.ks);
            if (warp() == GQ + 1)
                reinterpret_cast<float4*>(bk_sm.vs)[lane()] = gather_head(qkv + QD() + KVD() + (size_t)a.g * HD, tgA);
        }
        named_bar_sync(1, NCT);
        if (a.has_cur && tid() < 2 * HD) {  // append K/V at slot `pos` of row b's cache (cpu_inference.rs:140-141)
            const size_t off = (((size_t)l * p.NKV + a.g) * p.max_seq[b] + pos) * HD;
            if (tid() < HD) p.kc[b][off + tid()] = bk_sm.ks[tid()];
            else p.vc[b][off + tid() - HD] = bk_sm.vs[tid() - HD];
        }
        float4 q4[GQ];
#pragma unroll
        for (int h = 0; h < GQ; h++) q4[h] = reinterpret_cast<const float4*>(bk_sm.qs[h])[lane()];
        WarpSoftmax ws;
        const float scale = p.scale;
#pragma unroll
        for (int h = 0; h < GQ; h++) {
            ws.m[h] = -INFINITY;
            ws.l[h] = 0.f;
            ws.acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const int tc1 = a.has_cur ? pos : a.t1;
        const int npieces = tc1 > a.t0 ? (tc1 - a.t0 + ATT_P - 1) / ATT_P : 0;
        for (int q0 = 0; q0 < npieces; q0 += 4) {
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
                for (int j = 0; j < n; j++) mbar_arrive(&bk_sm.empty[(pc + j) % NSLOT]);
            it = pc + n;
        }
        if (a.has_cur && warp() == (tc1 - a.t0) % NCW) attn_pair<GQ>(bk_sm.ks, bk_sm.vs, nullptr, nullptr, false, q4, ws, scale);
        // combine the 12 warps' states in warp order
        float* const wst = ast();
#pragma unroll
        for (int h = 0; h < GQ; h++) {
            float* d = wst + (warp() * GQ + h) * ATT_WST;
            reinterpret_cast<float4*>(d)[lane()] = ws.acc[h];
            if (lane() == 0) {
                d[HD] = ws.m[h];
                d[HD + 1] = ws.l[h];
            }
        }
        named_bar_sync(1, NCT);
        float m = -INFINITY, lsum = 0.f, acc = 0.f;
        if (tid() < GQ * HD) {
            const int h = tid() >> 7, d = tid() & (HD - 1);
#pragma unroll
            for (int w = 0; w < NCW; w++) m = fmaxf(m, wst[(w * GQ + h) * ATT_WST + HD]);
#pragma unroll
            for (int w = 0; w < NCW; w++) {
                const float* src = wst + (w * GQ + h) * ATT_WST;
                const float e = src[HD] == -INFINITY ? 0.f : __expf(src[HD] - m);
                lsum = fmaf(e, src[HD + 1], lsum);
                acc = fmaf(e, src[d], acc);
            }
        }
        const size_t head_base = ((size_t)b * p.NKV + a.g) * p.S * GQ;  // partial (s, h) at apart[(head_base + s G + h) APART]
        if (a.s != 0) {
            if (tid() < GQ * HD) {
                const int h = tid() >> 7, d = tid() & (HD - 1);
                u64* dst = p.apart + (head_base + (size_t)a.s * GQ + h) * APART;
                st_relaxed_u64(dst + d, tagged(acc, tgB));
                if (d == 0) {
                    st_relaxed_u64(dst + HD, tagged(m, tgB));
                    st_relaxed_u64(dst + HD + 1, tagged(lsum, tgB));
                }
            }
            named_bar_sync(1, NCT);  // the warp states in ast are read above before any later reuse
            return;
        }
        // chunk 0: poll the other chunks' partials (word d of each, plus their (m, l)) into stage
        if (tid() < GQ * HD && (tid() & (HD - 1)) == 0) {
            bk_sm.ml[0][tid() >> 7][0] = m;
            bk_sm.ml[0][tid() >> 7][1] = lsum;
        }
        if (tid() < GQ * HD && a.S_eff > 1) {
            const int h = tid() >> 7, d = tid() & (HD - 1);
            uint32_t pending = 0;
            for (int s = 1; s < a.S_eff; s++) pending |= 1u << s;
            const bool mlt = d < 2;  // threads d = 0, 1 of each head also fetch m (d = 0) or l (d = 1)
            uint32_t mlpend = mlt ? pending : 0u;
            uint32_t spins = 0;
            uint64_t t0 = 0;
            while ((pending | mlpend) && !aborted()) {
                for (int s = 1; s < a.S_eff; s++) {
                    const u64* src = p.apart + (head_base + (size_t)s * GQ + h) * APART;
                    if (pending & (1u << s)) {
                        const u64 w = ld_relaxed_u64(src + d);
                        if (word_tag(w) == tgB) {
                            stage()[(s - 1) * (GQ * HD) + tid()] = word_val(w);
                            pending &= ~(1u << s);
                        }
                    }
                    if (mlpend & (1u << s)) {
                        const u64 w = ld_relaxed_u64(src + HD + d);
                        if (word_tag(w) == tgB) {
                            bk_sm.ml[s][h][d] = word_val(w);
                            mlpend &= ~(1u << s);
                        }
                    }
                }
                if ((pending | mlpend) && wait_expired(spins, t0, BERR_TIMEOUT_DATA, (int)tgB)) break;
            }
        }
        named_bar_sync(1, NCT);
        if (tid() < GQ * HD) {
            const int h = tid() >> 7, d = tid() & (HD - 1);
            float M = bk_sm.ml[0][h][0];
            for (int s = 1; s < a.S_eff; s++) M = fmaxf(M, bk_sm.ml[s][h][0]);
            const float w0 = __expf(bk_sm.ml[0][h][0] - M);
            float Lt = w0 * bk_sm.ml[0][h][1], O = w0 * acc;
            for (int s = 1; s < a.S_eff; s++) {
                const float w = __expf(bk_sm.ml[s][h][0] - M);
                Lt = fmaf(w, bk_sm.ml[s][h][1], Lt);
                O = fmaf(w, stage()[(s - 1) * (GQ * HD) + tid()], O);
            }
            st_relaxed_u64(p.att + (size_t)b * QD() + (size_t)(a.g * GQ + h) * HD + d, tagged(O / Lt, tgB));
        }
        named_bar_sync(1, NCT);
    }

    __device__ __noinline__ static void attention(int step, int l) {
        switch (G()) {
            case 1: attention_g<1>(step, l); break;
            case 2: attention_g<2>(step, l); break;
            default: attention_g<3>(step, l); break;
        }
    }

    // ---------------------------------------------------------------- consumer main loop
    // loop state in shared memory, re-read after every out-of-line call (see decode_kernel.cuh)
    __device__ __forceinline__ static volatile BLoop& ls() {
        uint32_t t;
        asm volatile("mov.u32 %0, %%tid.x;" : "=r"(t));
        return bk_sm.loop[t >> 5];
    }
    __device__ __forceinline__ static const volatile BParams& vprm() { return bk_sm.prm; }

    // one layer for every row: A rmsnorm + q|k|v, B attention, C o + residual, D rmsnorm + gate|up +
    // SiLU, E down + residual (cpu_inference.rs:113-173)
    __device__ __forceinline__ static void consume_layer() {
        const int step = ls().step, l = ls().l;
        const uint16_t* nrm = vprm().layer_n + (size_t)l * vprm().norm_stride;
        stamp(l, 0);
        if (l == 0) embed_input(nrm);
        else gather_rows(vprm().x, vprm().H, 0, tag(step, l - 1, 5), nrm);
        stamp(ls().l, 1);
        gemv_phase(gA(), nullptr, 0, 0);
        store_qkv(tag(ls().step, ls().l, 1));
        stamp(ls().l, 2);
        attention(ls().step, ls().l);
        stamp(ls().l, 3);
        gather_rows(vprm().att, QD(), 0, tag(ls().step, ls().l, 2), nullptr);
        stamp(ls().l, 4);
        gemv_phase(gC(), vprm().att, QD(), tag(ls().step, ls().l, 2));
        residual_rows(gC(), tag(ls().step, ls().l, 3));
        stamp(ls().l, 5);
        gather_rows(vprm().x, vprm().H, 0, tag(ls().step, ls().l, 3),
                    vprm().layer_n + (size_t)ls().l * vprm().norm_stride + vprm().H);
        stamp(ls().l, 6);
        gemv_phase(gD(), nullptr, 0, 0);
        silu_rows(tag(ls().step, ls().l, 4));
        stamp(ls().l, 7);
        gather_rows(vprm().hbuf, vprm().I, 0, tag(ls().step, ls().l, 4), nullptr);
        stamp(ls().l, 8);
        gemv_phase(gE(), vprm().hbuf, vprm().I, tag(ls().step, ls().l, 4));
        residual_rows(gE(), tag(ls().step, ls().l, 5));
        stamp(ls().l, 9);
    }

    __device__ static void consume() {
        {
            const BParams& p = bk_sm.prm;
            if (tid() < NB) {
                unsigned t = 0;
                if (tid() < p.nb) {
                    t = __ldcg(p.tok_in + tid());
                    if (t >= (unsigned)p.V) {
                        fail(BERR_BAD_TOKEN, (int)t);
                        t = 0;
                    }
                }
                bk_sm.tokens[tid()] = t;
            }
            named_bar_sync(1, NCT);
        }
        for (ls().step = 0; ls().step < vprm().steps; ls().step = ls().step + 1) {
            for (ls().l = 0; ls().l < vprm().L; ls().l = ls().l + 1) consume_layer();
            // F: final rmsnorm -> lm_head -> per-row argmax partials -> barrier -> next tokens
            gather_rows(vprm().x, vprm().H, 0, tag(ls().step, vprm().L - 1, 5), vprm().final_norm);
            stamp(vprm().L, 0);
            lm_head_argmax();
            stamp(vprm().L, 1);
            step_barrier((uint32_t)ls().step + 1);
            stamp(vprm().L, 2);
            argmax_combine();
            stamp(vprm().L, 3);
            if (cta() == 0 && tid() < vprm().nb && !aborted())
                vprm().tok_out[(size_t)ls().step * vprm().nb + tid()] = bk_sm.tokens[tid()];
        }
    }

    // ---------------------------------------------------------------- producer
    __device__ static bool slot_acquire(uint32_t& slot) {
        uint32_t& it = ring_pos();
        slot = it % NSLOT;
        const uint32_t par = ((it / NSLOT) & 1) ^ 1;
        return wait_mbar(&bk_sm.empty[slot], par, BERR_TIMEOUT_EMPTY);
    }

    __device__ __noinline__ static void gemv_produce(const GemvGeo& g, const uint16_t* wbase) {
        const uint64_t pol = policy_evict_first();
        uint32_t& it = ring_pos();
        for (int r = g.r0; r < g.r1; r += g.rpp) {
            const int nr = min(g.rpp, g.r1 - r);
            uint32_t slot;
            if (slot_acquire(slot)) {
                const uint32_t bytes = (uint32_t)nr * (uint32_t)g.K * 2u;
                mbar_arrive_expect_tx(&bk_sm.full[slot], bytes);
                bulk_g2s_evict_first(ring() + slot * SLOT_BYTES, wbase + g.woff + (size_t)r * g.K, bytes, &bk_sm.full[slot], pol);
                bk_sm.n_issued = it + 1;
            }
            ++it;
        }
    }

    // the cached K/V rows [t0, min(t1, pos)) of this CTA's attention item, ATT_P positions per piece
    __device__ __noinline__ static void attn_produce(int step, int l) {
        const BParams& p = bk_sm.prm;
        uint32_t& it = ring_pos();
        const BItem a = bitem(p, cta(), step);
        if (!a.active) return;
        const int tc1 = a.has_cur ? a.pos : a.t1;
        if (a.t0 >= tc1) return;
        // K/V rows of earlier steps were written by other CTAs: wait until this CTA's consumers have
        // passed the previous step's barrier, then order the async-proxy reads after it
        if (step > 0 && !aborted() && l == 0) {
            uint32_t spins = 0;
            uint64_t t0 = 0;
            while (ld_acquire_cta_shared(&bk_sm.progress) < (uint32_t)step) {
                if (wait_expired(spins, t0, BERR_TIMEOUT_KV, step)) break;
                __nanosleep(32);
            }
            fence_proxy_async_global();
        }
        const size_t head = ((size_t)l * p.NKV + a.g) * p.max_seq[a.b];
        for (int t = a.t0; t < tc1; t += ATT_P) {
            const int np = min(ATT_P, tc1 - t);
            uint32_t slot;
            if (slot_acquire(slot)) {
                const uint32_t bytes = (uint32_t)np * HD * 4u;
                mbar_arrive_expect_tx(&bk_sm.full[slot], 2u * bytes);
                uint8_t* dst = ring() + slot * SLOT_BYTES;
                bulk_g2s(dst, p.kc[a.b] + (head + t) * HD, bytes, &bk_sm.full[slot]);
                bulk_g2s(dst + ATT_P * HD * 4, p.vc[a.b] + (head + t) * HD, bytes, &bk_sm.full[slot]);
                bk_sm.n_issued = it + 1;
            }
            ++it;
        }
    }

    __device__ __noinline__ static void prefetch_layer(const uint16_t* W) {
        const GemvGeo* gs[4] = {&gA(), &gC(), &gD(), &gE()};
        for (int k = 0; k < 4; k++) {
            const GemvGeo& g = *gs[k];
            const uint32_t bytes = (uint32_t)(g.r1 - g.r0) * (uint32_t)g.K * 2u;
            if (bytes) bulk_prefetch_l2(W + g.woff + (size_t)g.r0 * g.K, bytes);
        }
    }

    __device__ static void produce() {
        const volatile BParams& p = bk_sm.prm;
        prefetch_layer(p.layer_w);
        for (ls().step = 0; ls().step < p.steps; ls().step = ls().step + 1) {
            for (ls().l = 0; ls().l < p.L; ls().l = ls().l + 1) {
                const uint16_t* W = p.layer_w + (size_t)ls().l * p.layer_stride;
                if (ls().l + 1 < p.L) prefetch_layer(W + p.layer_stride);
                gemv_produce(gA(), W);
                attn_produce(ls().step, ls().l);
                gemv_produce(gC(), p.layer_w + (size_t)ls().l * p.layer_stride);
                gemv_produce(gD(), p.layer_w + (size_t)ls().l * p.layer_stride);
                gemv_produce(gE(), p.layer_w + (size_t)ls().l * p.layer_stride);
            }
            if (ls().step + 1 < p.steps) prefetch_layer(p.layer_w);
            gemv_produce(gF(), p.lm_head);
        }
        drain();
    }

    // after an abort, wait (bounded) for the copies still in flight before the CTA may exit
    __device__ __noinline__ static void drain() {
        const BParams& p = bk_sm.prm;
        if (aborted()) {
            const uint32_t first = bk_sm.n_issued > NSLOT ? bk_sm.n_issued - NSLOT : 0;
            for (uint32_t j = first; j < bk_sm.n_issued; j++) {
                const int slot = j % NSLOT;
                const uint32_t par = (j / NSLOT) & 1;
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(&bk_sm.full[slot], par)) {
                    if (globaltimer_ns() - t0 > (uint64_t)p.timeout_ns) {
                        atomicCAS(&p.err[3], 0, BERR_TIMEOUT_DRAIN);
                        break;
                    }
                }
            }
        }
    }
};

// the batch decode kernel: 12 consumer warps and one producer lane per CTA, one CTA per SM
__global__ void __launch_bounds__(NTHREADS, 1) batch_decode_kernel(const __grid_constant__ BParams p) {
    if (threadIdx.x == 0) {
        for (int i = 0; i < NSLOT; i++) {
            mbar_init(&bk_sm.full[i], 1);
            mbar_init(&bk_sm.empty[i], NCW);
        }
        bk_sm.progress = 0;
        bk_sm.abort = 0;
        bk_sm.prm = p;
        for (int w = 0; w <= NCW; w++) bk_sm.ring_it[w] = 0;
        bk_sm.n_issued = 0;
        BDecoder::init_geometry(p);
        fence_mbar_init();
    }
    for (int i = threadIdx.x; i < XS_FLOATS; i += NTHREADS) BDecoder::xs()[i] = 0.f;  // rows past nb stay zero
    __syncthreads();
    if (BDecoder::aborted()) return;  // shape check failed (the host launched it for shapes it does not cover)
    if (BDecoder::warp() == NCW) {
        if (BDecoder::lane() == 0) BDecoder::produce();
        return;
    }
    BDecoder::consume();
}

}  // namespace bk
}  // namespace qw
