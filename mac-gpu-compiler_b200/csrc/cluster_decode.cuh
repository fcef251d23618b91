// Cluster decode kernel: batch-1 Qwen3 decode for the Qwen3-0.6B layer shape (hidden 1024,
// 16 query / 8 KV heads of 128, SwiGLU 3072) on sm_100a thread-block clusters.
//
// Same math as the reference CPU engine (metal_infrence_engine/src/cpu_inference.rs:100-179) and the
// persistent decode kernel of decode_kernel.cuh; what changes is the work split. The grid is one
// 8-CTA cluster per KV head (8 clusters, 64 CTAs, one per SM). Cluster g owns everything of KV
// head g: its two query heads' and its own q|k|v rows, its attention, its slice of o_proj's columns
// and one eighth of the MLP's intermediate width. (Clusters of 8 because that is what B200's GPCs
// hold eight of at one CTA per SM: the occupancy query gives 7 clusters of 16, 15 of 8.) Within a
// cluster, activations move through distributed shared memory: a CTA pushes its outputs into every
// peer's shared memory with st.async, whose bytes complete a transaction count on the peer's
// mbarrier, so the peer's wait on that mbarrier both synchronises and delivers (a one-way hand-off). Only the two reductions of the
// residual stream per layer (after o_proj and after down_proj) cross clusters, through tagged words
// in global memory, and each such word has 8 readers (one CTA per cluster) instead of every CTA.
//
// Per layer, in CTA r (0..7) of cluster g:
//   A  x*ln1 (every CTA holds it) -> 64 q|k|v rows of head group g (1024 columns); the 64 values are
//      pushed to all 8 CTAs of the cluster (E2)
//   B  per-head q/k RMSNorm + RoPE of head group g (every CTA, from the pushed 512 values); the CTA
//      whose position range holds `pos` appends K/V; each CTA scores its 1/8 of the positions and
//      pushes its online-softmax partial (m, l, sum p.v for both query heads) to all 8 (E3); every
//      CTA merges the 8 partials in rank order into the head group's 256 attention outputs
//   C  o_proj rows [128r, 128r+128) over the head group's 256 columns -> a partial residual update,
//      published as tagged words po[g][row]
//   G1 CTA r of every cluster sums po[0..7][128r..128r+128) in cluster order into its residual rows,
//      then pushes its 128 values of x*ln2 and its sum of squares to all 8 CTAs (E4)
//   D  gate|up rows of h[384g + 48r, +48) (interleaved), SiLU(gate)*up -> pushed to all 8 (E5)
//   E  down_proj rows [128r, 128r+128) over the cluster's 384 h columns -> pd[g][row]
//   G2 as G1 with pd, pushing x*ln1 of the next layer (or the final norm's gain) (E1)
// After the layers: lm_head rows [V*c/64, V*(c+1)/64) of CTA c, per-CTA argmax partials, one
// grid barrier per token, and every CTA combines the partials into the next token.
//
// Weights stream through an 8-slot shared-memory ring filled by one producer lane with 1-D TMA bulk
// copies (no multicast); the next layer's rows of each CTA are warmed into L2 at the start of a layer.
// Each CTA moves 480 KB per layer through its 192 KB ring, so the GEMVs release every ring piece as
// soon as its data is in registers: the producer refills the ring while the phase still computes.
// Every wait is bounded in time; on expiry the kernel records an error and stops waiting. A CTA
// leaves only after a cluster barrier, so no peer can still be writing into its shared memory.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "decode_kernel.cuh"
#include "ptx.cuh"

namespace qw {
namespace cl {

constexpr int CL = 8;                           // CTAs per cluster
constexpr int NCW = 12;                         // consumer warps
constexpr int NCT = NCW * 32;
constexpr int NTHREADS = NCT + 32;              // + producer warp
constexpr int NSLOT = 8;
constexpr int SLOT_BYTES = 24 * 1024;
constexpr int HD = 128, H = 1024, NQ = 16, NKV = 8, G = 2, I = 3072;
constexpr int QD = NQ * HD, KVD = NKV * HD, QKVR = QD + 2 * KVD;
constexpr int A_ROWS = (G + 2) * HD / CL;       // 64 q|k|v rows per CTA
constexpr int XO = H / CL;                      // 128 residual rows per CTA
constexpr int HO = I / NKV / CL;                // 48 h values per CTA
constexpr int OK = G * HD;                      // 256 o_proj columns per cluster
constexpr int DK = I / NKV;                     // 384 down_proj columns per cluster
constexpr int ATT_P = SLOT_BYTES / (2 * HD * 4);  // 24 cached positions per ring slot
constexpr int APW = 2 * HD + 8;                 // floats per attention partial: acc[2][128], m[2], l[2], pad
constexpr int WST = HD + 4;                     // floats per (warp, head) softmax state
constexpr int TRACE_PER_LAYER = 14;

static_assert(A_ROWS == 64 && XO == 128 && HO == 48 && OK == 256 && DK == 384, "Qwen3-0.6B layer shape");
static_assert(HD % A_ROWS == 0, "a CTA's q|k|v rows lie in one head");
static_assert(A_ROWS <= APW && HO <= APW && XO <= APW && XO % 32 == 0, "stage holds every pushed vector");

struct Params {
    const uint16_t* layer_w;     // the shared layout: per layer qkv[QKVR][H] | o[H][QD] | gu[2I][H] (interleaved) | down[H][I]
    const uint16_t* o_blk;       // o_proj repacked [L][NKV][CL][XO][OK]
    const uint16_t* d_blk;       // down_proj repacked [L][NKV][CL][XO][DK]
    const uint16_t* layer_n;     // per layer: ln1[H] | ln2[H] | q_norm[128] | k_norm[128]
    const uint16_t* final_norm;
    const uint16_t* embed;
    const uint16_t* lm_head;
    float* kc;
    float* vc;
    const float2* rope;
    u64* po;                     // [NKV][H] o_proj partials (tagged words)
    u64* pd;                     // [NKV][H] down_proj partials (tagged words)
    float* am_val;               // [grid]
    unsigned* am_idx;            // [grid]
    int* nan0;
    u64* flags;                  // [grid] epoch << 32 | tokens finished
    int* err;                    // [4]
    float* logits;               // [V] or null
    u64* trace;                  // [grid][TRACE_PER_LAYER * L + 4] or null
    const uint32_t* tok_in;
    uint32_t* tok_out;
    uint32_t* host_tok;
    unsigned* host_count;
    long long layer_stride, norm_stride;
    int L, V, max_seq, start_pos, steps;
    unsigned epoch;
    float eps, scale;
    long long timeout_ns;
    int stall_cta;               // test hook (-1: off): this CTA never raises its first end-of-token flag,
                                 // so every CTA's bounded barrier wait runs out and the launch reports it
};

struct LoopState {
    int step, l;
    unsigned token;
};

struct Smem {
    uint64_t full[NSLOT];
    uint64_t empty[NSLOT];
    uint64_t xbar, qbar, abar, hbar;   // exchange mbarriers (one transaction count per use)
    Params prm;
    uint32_t ring_it[NCW + 1];
    uint32_t n_issued;
    LoopState loop[NCW + 1];
    uint32_t progress;
    int abort;
    unsigned token;
    int g, r;                          // cluster (KV head) and rank in the cluster
    uint32_t a_row0;                   // first q|k|v row of this CTA in the layer's qkv block
    uint32_t lm_r0, lm_r1;             // lm_head rows of this CTA
    float sspart[XO / 32];
    float redv[NCW];
    unsigned redi[NCW];
    __align__(16) float qs[G][HD];
    __align__(16) float ks[HD];
    __align__(16) float vs[HD];
    __align__(16) float xown[XO];      // residual rows [XO r, XO (r+1)) (f32, as the reference keeps x)
    __align__(16) float stage[APW];    // outputs on their way to the peers
    __align__(16) float gst[NKV][XO];  // polled partial residual updates, by cluster
};

// dynamic shared memory: ring | exchange targets (written by peers) | local scratch.
// The attention's per-warp softmax states (wst) overlay xsA, xsD, qkv, hs and att: while a CTA
// combines its warps' states, it has finished reading xsA (phase A) and qkv (q/k norm + RoPE), has
// not yet written att (the merge comes after), and no peer can push into xsA, xsD or hs yet (each
// of those pushes needs this CTA's o_proj or gate|up outputs first, which come later).
struct Dyn {
    uint8_t ring[NSLOT][SLOT_BYTES];
    union {
        struct {
            float xsA[H];              // x * ln1 (or final norm) in the GEMV's permuted layout (E1)
            float xsD[H];              // x * ln2 (E4)
            float qkv[G * HD + 2 * HD];  // q0 | q1 | k | v of the head group (E2)
            float hs[DK];              // the cluster's 384 SiLU(gate)*up values (E5)
            float att[OK];             // merged attention output of the head group
        };
        float wst[NCW][G][WST];        // per-warp softmax states (local, see above)
    };
    float ssA[CL], ssD[CL];            // the CL senders' sums of squares of x
    float apr[CL][APW];                // attention partials by sender (E3)
};
static_assert(sizeof(float) * (2 * H + (G + 2) * HD + DK + OK) >= sizeof(float) * NCW * G * WST,
              "the softmax states fit in the buffers they overlay");

constexpr size_t DYN_BYTES = sizeof(Dyn);
static_assert(offsetof(Dyn, xsA) % 16 == 0 && offsetof(Dyn, qkv) % 16 == 0 && offsetof(Dyn, apr) % 16 == 0 &&
              offsetof(Dyn, hs) % 16 == 0 && offsetof(Dyn, att) % 16 == 0 && offsetof(Dyn, wst) % 16 == 0,
              "float4 targets must be 16-byte aligned");
static_assert(APW % 4 == 0 && (XO * 4) % 16 == 0, "exchange chunks are 16 bytes");

__shared__ Smem cl_sm;
extern __shared__ __align__(128) uint8_t cl_dyn[];

// bytes a receiver expects per use of each exchange from its 15 peers (a CTA's own share is written
// with plain shared-memory stores)
constexpr uint32_t TX_X = (CL - 1) * (XO * 4 + 4);
constexpr uint32_t TX_Q = (CL - 1) * A_ROWS * 4;
constexpr uint32_t TX_A = (CL - 1) * APW * 4;
constexpr uint32_t TX_H = (CL - 1) * HO * 4;

class CDecoder {
public:
    __device__ __forceinline__ static int tid() { return (int)threadIdx.x; }
    __device__ __forceinline__ static int warp() { return (int)(threadIdx.x >> 5); }
    __device__ __forceinline__ static int lane() { return (int)(threadIdx.x & 31); }
    __device__ __forceinline__ static int cta() { return (int)blockIdx.x; }
    __device__ __forceinline__ static int nctas() { return (int)gridDim.x; }
    __device__ __forceinline__ static Dyn& dyn() { return *reinterpret_cast<Dyn*>(cl_dyn); }
    __device__ __forceinline__ static uint32_t& ring_pos() { return cl_sm.ring_it[threadIdx.x >> 5]; }
    __device__ __forceinline__ static volatile LoopState& ls() {
        uint32_t t;
        asm volatile("mov.u32 %0, %%tid.x;" : "=r"(t));
        return cl_sm.loop[t >> 5];
    }
    __device__ __forceinline__ static const volatile Params& vprm() { return cl_sm.prm; }
    __device__ __forceinline__ static int cur_step() { return ls().step; }
    __device__ __forceinline__ static int cur_layer() { return ls().l; }

    // tags of the two cross-cluster hand-offs of a layer (ph 0: o_proj partials, 1: down partials)
    __device__ static uint32_t tag(int step, int l, int ph) {
        const volatile Params& p = cl_sm.prm;
        // sequence numbers start at 1: an all-zero word (tag 0) never matches, even in a launch
        // whose 12-bit epoch field is 0
        const uint32_t sq = (uint32_t)step * (uint32_t)(2 * p.L) + (uint32_t)(2 * l + ph) + 1u;
        return ((p.epoch & 0xFFFu) << 20) | (sq & 0xFFFFFu);
    }

    __device__ __forceinline__ static void stamp(int idx) {
        const volatile Params& p = cl_sm.prm;
        if (p.trace != nullptr && cur_step() == 0 && tid() == 0)
            p.trace[(size_t)cta() * (TRACE_PER_LAYER * p.L + 4) + idx] = globaltimer_ns();
    }
    __device__ __forceinline__ static void lstamp(int k) { stamp(cur_layer() * TRACE_PER_LAYER + k); }
    __device__ __forceinline__ static void tstamp(int k) { stamp(vprm().L * TRACE_PER_LAYER + k); }

    // ------------------------------------------------------------------ errors and bounded waits
    __device__ static bool aborted() { return *reinterpret_cast<volatile const int*>(&cl_sm.abort) != 0; }

    __device__ __noinline__ static void fail(int code, int where) {
        const Params& p = cl_sm.prm;
        *reinterpret_cast<volatile int*>(&cl_sm.abort) = 1;
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
        const Params& p = cl_sm.prm;
        if (aborted()) return ~0ull;
        const uint64_t now = globaltimer_ns();
        if (spins == 32) return now;
        const uint64_t waited = now - t0;
        if (waited > 50000 && (spins & 1023) == 0 && ld_volatile_s32(p.err) != 0) {
            *reinterpret_cast<volatile int*>(&cl_sm.abort) = 1;
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
        return wait_mbar_slow(bar, parity, code);
    }
    __device__ __noinline__ static bool wait_mbar_slow(uint64_t* bar, uint32_t parity, int code) {
        if (aborted()) return false;
        uint32_t spins = 0;
        uint64_t t0 = 0;
        while (!mbar_try_wait(bar, parity))
            if (wait_expired(spins, t0, code, (int)ring_pos())) return false;
        return true;
    }

    // Waits for use `use` of an exchange mbarrier (count 1: thread 0 arms it with the bytes of the 7
    // peers; their st.async bytes may arrive before or after that), then a CTA barrier, so that the
    // CTA's own share (plain shared-memory stores by its other threads) is visible too. Every
    // consumer thread returns with its reads ordered after all CL senders' writes.
    __device__ __noinline__ static void wait_exchange(uint64_t* bar, uint32_t use, uint32_t bytes) {
        // after an abort a phase may never complete: arming it again could over-arrive it
        if (!aborted()) {
            if (tid() == 0) mbar_arrive_expect_tx(bar, bytes);
            const uint32_t parity = use & 1u;
            if (!mbar_try_wait_cluster(bar, parity)) {
                uint32_t spins = 0;
                uint64_t t0 = 0;
                while (!mbar_try_wait_cluster(bar, parity))
                    if (wait_expired(spins, t0, DERR_TIMEOUT_DATA, (int)use)) break;
            }
        }
        named_bar_sync(1, NCT);
    }

    // one 16-byte chunk to CTA `dest` of the cluster: st.async into a peer, a plain store into itself
    __device__ __forceinline__ static void put4(float* dst_local, float4 v, uint64_t* bar_local, uint32_t dest) {
        if (dest == (uint32_t)cl_sm.r) *reinterpret_cast<float4*>(dst_local) = v;
        else st_async_v4(mapa_shared(smem_u32(dst_local), dest), v, mapa_shared(smem_u32(bar_local), dest));
    }

    // pushes n floats (n % 4 == 0) of stage to dst_local's counterpart in all CTAs of the cluster,
    // completing `bar` there; the threads [first, first + CL * n / 4) take a 16-byte chunk each
    __device__ __forceinline__ static void push(const float* src, int n, float* dst_local, uint64_t* bar_local,
                                                int first) {
        const int chunks = n >> 2;
        const int k = tid() - first;
        if (k < 0 || k >= CL * chunks) return;
        const uint32_t dest = (uint32_t)(k / chunks), c = (uint32_t)(k % chunks);
        const float4 v = reinterpret_cast<const float4*>(src)[c];
        put4(dst_local + 4 * c, v, bar_local, dest);
    }

    // ------------------------------------------------------------------ GEMV over K = 1024 rows
    // One ring piece holds 12 rows; warp w takes row w of each piece, holding its 1024-column input
    // in registers (32 floats in the permuted layout), so a row is 4 x 16-byte loads per lane. Pieces
    // go in groups of up to four: wait for all, load, FMA, then one transposing butterfly reduces the
    // group's (up to) four rows, after which lanes 0, 8, 16, 24 hold rows 0..3 of the group.
    // EPI 0: q|k|v rows -> stage[row] = total * sc. EPI 1: interleaved gate/up rows, warp w takes
    // pair w % 6 of pieces w / 6 and w / 6 + 2 -> stage[pair] = silu(g * sc) * u * sc. EPI 2: lm_head
    // rows -> logits (if wanted) and this CTA's argmax partial.
    template <int EPI>
    __device__ __noinline__ static void gemv_rows(int rows, const float* xs, float sc, uint32_t lm_r0) {
        uint32_t& it = ring_pos();
        const int w = warp(), ln = lane();
        float xr[32];
        {
            const float4* xp = reinterpret_cast<const float4*>(xs) + ln;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float4 a = xp[i * 64], b = xp[i * 64 + 32];
                xr[i * 8 + 0] = a.x; xr[i * 8 + 1] = a.y; xr[i * 8 + 2] = a.z; xr[i * 8 + 3] = a.w;
                xr[i * 8 + 4] = b.x; xr[i * 8 + 5] = b.y; xr[i * 8 + 6] = b.z; xr[i * 8 + 7] = b.w;
            }
        }
        const int npieces = (rows + 11) / 12;
        float bv = -INFINITY;
        unsigned bi = NONE_IDX;
        uint32_t pc = it;
        for (int q0 = 0; q0 < npieces; q0 += 4) {
            const int n = min(4, npieces - q0);
            bool ok = true;
            if (lane() < n) ok = wait_mbar(&cl_sm.full[(pc + lane()) % NSLOT], ((pc + lane()) / NSLOT) & 1, DERR_TIMEOUT_FULL);
            ok = __all_sync(0xFFFFFFFFu, ok);
            __syncwarp();
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            int dst[4] = {-1, -1, -1, -1};
            if (ok) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int pj = EPI == 1 ? w / 6 + (j & 2) : j;
                    const int rr = EPI == 1 ? 2 * (w % 6) + (j & 1) : w;
                    const int row = (q0 + pj) * 12 + rr;
                    if (pj < n && rr < 12 && row < rows) {
                        dst[j] = row;
                        const uint4* wp = reinterpret_cast<const uint4*>(dyn().ring[(pc + pj) % NSLOT] + rr * 2048 + ln * 16);
                        uint4 wv[4];
#pragma unroll
                        for (int i = 0; i < 4; i++) wv[i] = wp[i * 32];
                        float2 e = make_float2(0.f, 0.f), o = e;
                        e = dot8_acc2(wv[0], xr + 0, e);
                        o = dot8_acc2(wv[1], xr + 8, o);
                        e = dot8_acc2(wv[2], xr + 16, e);
                        o = dot8_acc2(wv[3], xr + 24, o);
                        v[j] = (e.x + e.y) + (o.x + o.y);
                    }
                }
            }
            // the group's data is in registers: hand its slots back to the producer now (every warp
            // arrives on every slot of the group; a slot is released only after its data landed)
            __syncwarp();
            if (ln == 0 && ok)
                for (int j = 0; j < n; j++) mbar_arrive(&cl_sm.empty[(pc + j) % NSLOT]);
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
            if (EPI == 0) {
                if ((ln & 7) == 0 && d >= 0) cl_sm.stage[d] = t * sc;
            } else if (EPI == 1) {
                const float up = __shfl_down_sync(0xFFFFFFFFu, t, 8);
                if ((ln & 15) == 0 && d >= 0) {
                    const float gt = t * sc, u = up * sc;
                    cl_sm.stage[d >> 1] = gt / (1.0f + __expf(-gt)) * u;
                }
            } else {
                if ((ln & 7) == 0 && d >= 0) {
                    const float y = t * sc;
                    const unsigned row = lm_r0 + (unsigned)d;
                    const Params& p = cl_sm.prm;
                    if (p.logits) __stcg(p.logits + row, y);
                    if (row == 0) __stcg(p.nan0, isnan(y) ? 1 : 0);
                    if (!isnan(y) && am_better(y, row, bv, bi)) { bv = y; bi = row; }
                }
            }
        }
        it = pc;
        if (EPI == 2) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
                const unsigned oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
                if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
            }
            if (ln == 0) { cl_sm.redv[w] = bv; cl_sm.redi[w] = bi; }
        }
        named_bar_sync(1, NCT);
    }

    // ------------------------------------------------------------------ GEMV over 4-row units, K = 256 / 384
    // A unit is 4 consecutive rows (8K bytes = K/64 x 512-byte warp loads); lane l's 16-byte chunk
    // of load i sits at byte 512 i + 16 l of the unit, i.e. row (512 i + 16 l) / 2K, column chunk
    // ((512 i + 16 l) mod 2K) / 16. Warp w takes units w and w + 12; each unit's four row totals go
    // (through the transposing butterfly) to lanes 0, 8, 16, 24, which publish them as tagged words
    // out[row] for the other clusters.
    template <int K>
    __device__ __noinline__ static void gemv_units(int units, const float* x, u64* out, uint32_t tg) {
        constexpr int NL = K / 64;                     // 16-byte loads per lane per unit
        constexpr int UPP = SLOT_BYTES / (8 * K);      // units per ring piece
        uint32_t& it = ring_pos();
        const int w = warp(), ln = lane();
        // the lane's input chunks: K = 256: chunk l of every row; K = 384: chunks l, (l < 16 ? 32 + l : l - 16), 16 + l
        float xa[8], xb[8], xc[8];
        {
            const int ca = ln, cb = K == 384 ? (ln < 16 ? 32 + ln : ln - 16) : ln, cc = K == 384 ? 16 + ln : ln;
            const float4* xp = reinterpret_cast<const float4*>(x);
            float4 t0 = xp[2 * ca], t1 = xp[2 * ca + 1];
            xa[0] = t0.x; xa[1] = t0.y; xa[2] = t0.z; xa[3] = t0.w; xa[4] = t1.x; xa[5] = t1.y; xa[6] = t1.z; xa[7] = t1.w;
            t0 = xp[2 * cb]; t1 = xp[2 * cb + 1];
            xb[0] = t0.x; xb[1] = t0.y; xb[2] = t0.z; xb[3] = t0.w; xb[4] = t1.x; xb[5] = t1.y; xb[6] = t1.z; xb[7] = t1.w;
            t0 = xp[2 * cc]; t1 = xp[2 * cc + 1];
            xc[0] = t0.x; xc[1] = t0.y; xc[2] = t0.z; xc[3] = t0.w; xc[4] = t1.x; xc[5] = t1.y; xc[6] = t1.z; xc[7] = t1.w;
        }
        const int npieces = (units + UPP - 1) / UPP;
        const uint32_t pc = it;
        int released = 0;  // lane 0: pieces [0, released) this warp has handed back to the producer
        for (int u = w; u < units; u += NCW) {
            const int pj = u / UPP;
            const bool ok = wait_mbar(&cl_sm.full[(pc + pj) % NSLOT], ((pc + pj) / NSLOT) & 1, DERR_TIMEOUT_FULL);
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            if (ok) {
                const uint4* wp = reinterpret_cast<const uint4*>(dyn().ring[(pc + pj) % NSLOT] + (u % UPP) * (8 * K)) + ln;
                uint4 wv[NL];
#pragma unroll
                for (int i = 0; i < NL; i++) wv[i] = wp[i * 32];
                // release every piece this warp has no further unit in (its data is in registers)
                const int done = u + NCW < units ? (u + NCW) / UPP : npieces;
                __syncwarp();
                if (ln == 0)
                    for (; released < done; released++) mbar_arrive(&cl_sm.empty[(pc + released) % NSLOT]);
                if (K == 256) {
#pragma unroll
                    for (int i = 0; i < 4; i++) acc[i] = dot8(wv[i], xa);
                } else {
                    const float d1 = dot8(wv[1], xb), d4 = dot8(wv[4], xb);
                    acc[0] = dot8(wv[0], xa) + (ln < 16 ? d1 : 0.f);
                    acc[1] = dot8(wv[2], xc) + (ln < 16 ? 0.f : d1);
                    acc[2] = dot8(wv[3], xa) + (ln < 16 ? d4 : 0.f);
                    acc[3] = dot8(wv[5], xc) + (ln < 16 ? 0.f : d4);
                }
            }
            const bool hi16 = ln & 16, hi8 = ln & 8;
            float k0 = hi16 ? acc[2] : acc[0], k1 = hi16 ? acc[3] : acc[1];
            k0 += __shfl_xor_sync(0xFFFFFFFFu, hi16 ? acc[0] : acc[2], 16);
            k1 += __shfl_xor_sync(0xFFFFFFFFu, hi16 ? acc[1] : acc[3], 16);
            float t = hi8 ? k1 : k0;
            t += __shfl_xor_sync(0xFFFFFFFFu, hi8 ? k0 : k1, 8);
            t += __shfl_xor_sync(0xFFFFFFFFu, t, 4);
            t += __shfl_xor_sync(0xFFFFFFFFu, t, 2);
            t += __shfl_xor_sync(0xFFFFFFFFu, t, 1);
            const int jj = (hi16 ? 2 : 0) + (hi8 ? 1 : 0);
            if ((ln & 7) == 0 && ok) st_relaxed_u64(out + 4 * u + jj, tagged(t, tg));
        }
        // pieces this warp read nothing from (after an expired wait: none, the slot stays taken)
        __syncwarp();
        if (ln == 0 && !aborted())
            for (; released < npieces; released++) mbar_arrive(&cl_sm.empty[(pc + released) % NSLOT]);
        it = pc + npieces;
        named_bar_sync(1, NCT);
    }

    // ------------------------------------------------------------------ the residual hand-off (G1, G2)
    // CTA r of every cluster polls the 8 clusters' partial updates of rows [XO r, XO (r+1)), adds them
    // in cluster order to its residual rows (cpu_inference.rs:163-164, :171-172), then pushes x * gain
    // (the next RMSNorm's input, in the GEMV's permuted layout) and its sum of x^2 to its cluster.
    __device__ __noinline__ static void residual_exchange(const u64* part, uint32_t tg, const uint16_t* gain,
                                                          float* xs_dst, float* ss_dst) {
        const int r = cl_sm.r;
        float gn = 0.f;
        if (tid() < XO) gn = bf16_to_f32(__ldg(gain + XO * r + tid()));
        // (cluster, word pair) items, two rounds for some threads; each thread keeps both of its items
        // in flight and checks their tags together
        constexpr int ITEMS = NKV * XO / 2;
        const int k0 = tid(), k1 = tid() + NCT;
        const bool has0 = k0 < ITEMS, has1 = k1 < ITEMS;
        const u64* src0 = part + (size_t)(k0 / (XO / 2)) * H + XO * r + 2 * (k0 % (XO / 2));
        const u64* src1 = has1 ? part + (size_t)(k1 / (XO / 2)) * H + XO * r + 2 * (k1 % (XO / 2)) : src0;
        static_assert(ITEMS <= 2 * NCT, "two polled items per thread at most");
        bool need0 = has0, need1 = has1;
        uint32_t spins = 0;
        uint64_t t0 = 0;
        while ((need0 || need1) && !aborted()) {
            ulonglong2 w0 = make_ulonglong2(0, 0), w1 = w0;
            if (need0) w0 = ld_relaxed_v2u64(src0);
            if (need1) w1 = ld_relaxed_v2u64(src1);
            if (need0 && word_tag(w0.x) == tg && word_tag(w0.y) == tg) {
                cl_sm.gst[k0 / (XO / 2)][2 * (k0 % (XO / 2))] = word_val(w0.x);
                cl_sm.gst[k0 / (XO / 2)][2 * (k0 % (XO / 2)) + 1] = word_val(w0.y);
                need0 = false;
            }
            if (need1 && word_tag(w1.x) == tg && word_tag(w1.y) == tg) {
                cl_sm.gst[k1 / (XO / 2)][2 * (k1 % (XO / 2))] = word_val(w1.x);
                cl_sm.gst[k1 / (XO / 2)][2 * (k1 % (XO / 2)) + 1] = word_val(w1.y);
                need1 = false;
            }
            if ((need0 || need1) && wait_expired(spins, t0, DERR_TIMEOUT_DATA, (int)tg)) break;
        }
        named_bar_sync(1, NCT);
        if (tid() < XO) {
            float s = cl_sm.xown[tid()];
            float u = 0.f;
#pragma unroll
            for (int gg = 0; gg < NKV; gg++) u += cl_sm.gst[gg][tid()];
            s += u;
            cl_sm.xown[tid()] = s;
            cl_sm.stage[tid()] = s * gn;
            const float ss = warp_sum(s * s);
            if (lane() == 0) cl_sm.sspart[warp()] = ss;
        }
        named_bar_sync(1, NCT);
        push_x(xs_dst, ss_dst);
    }

    // stage[0..XO) = x * gain of this CTA's rows, sspart = their sums of squares: push both
    __device__ __forceinline__ static void push_x(float* xs_dst, float* ss_dst) {
        static_assert(CL * XO / 4 + CL <= NCT, "one chunk per thread");
        const int r = cl_sm.r;
        const int k = tid();
        uint64_t* bar = &cl_sm.xbar;
        if (k < CL * XO / 4) {
            const uint32_t dest = (uint32_t)(k / (XO / 4)), c = (uint32_t)(k % (XO / 4));
            const float4 v = reinterpret_cast<const float4*>(cl_sm.stage)[c];
            put4(xs_dst + xperm(XO * r + 4 * (int)c), v, bar, dest);
        } else if (k < CL * XO / 4 + CL) {
            const uint32_t dest = (uint32_t)(k - CL * XO / 4);
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < XO / 32; i++) ss += cl_sm.sspart[i];
            if (dest == (uint32_t)r) ss_dst[r] = ss;
            else st_async_b32(mapa_shared(smem_u32(ss_dst + r), dest), ss, mapa_shared(smem_u32(bar), dest));
        }
    }

    // 1 / sqrt(mean(x^2) + eps) from the CL senders' sums (fixed order)
    __device__ __forceinline__ static float norm_scale(const float* ss) {
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < CL; i++) t += ss[i];
        return rsqrtf(t / (float)H + cl_sm.prm.eps);
    }

    // ------------------------------------------------------------------ attention helpers
    __device__ __forceinline__ static void head_norm_rope(float4 v, const uint16_t* nw, const float2* rrow, float* dst) {
        float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        ss = warp_sum(ss);
        const float s = rsqrtf(ss / (float)HD + cl_sm.prm.eps);
        const int d0 = lane() * 4;
        float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; j++) e[j] = e[j] * s * bf16_to_f32(__ldg(nw + d0 + j));
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float other = __shfl_xor_sync(0xFFFFFFFFu, e[j], 16);
            const float2 cs = rrow[(d0 + j) & 63];
            if (lane() < 16) o[j] = e[j] * cs.x - other * cs.y;
            else o[j] = e[j] * cs.x + other * cs.y;
        }
        reinterpret_cast<float4*>(dst)[lane()] = make_float4(o[0], o[1], o[2], o[3]);
    }

    struct WS {
        float m[G], l[G];
        float4 acc[G];
    };

    // up to two cached positions into a warp's running softmax for both query heads
    __device__ __forceinline__ static void attn_pair(const float* K0, const float* V0, const float* K1, const float* V1,
                                                     bool has1, const float4* q4, WS& ws, float scale) {
        const float4 k0 = reinterpret_cast<const float4*>(K0)[lane()];
        const float4 v0 = reinterpret_cast<const float4*>(V0)[lane()];
        float4 k1 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = k1;
        if (has1) {
            k1 = reinterpret_cast<const float4*>(K1)[lane()];
            v1 = reinterpret_cast<const float4*>(V1)[lane()];
        }
        float s0[G], s1[G];
#pragma unroll
        for (int h = 0; h < G; h++) {
            s0[h] = q4[h].x * k0.x + q4[h].y * k0.y + q4[h].z * k0.z + q4[h].w * k0.w;
            s1[h] = q4[h].x * k1.x + q4[h].y * k1.y + q4[h].z * k1.z + q4[h].w * k1.w;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int h = 0; h < G; h++) {
                s0[h] += __shfl_xor_sync(0xFFFFFFFFu, s0[h], o);
                s1[h] += __shfl_xor_sync(0xFFFFFFFFu, s1[h], o);
            }
#pragma unroll
        for (int h = 0; h < G; h++) {
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

    // position range of CTA rank s for a token at `pos`: [t0, t1) of 0..pos, CL near-equal ranges
    __device__ __forceinline__ static void chunk_of(int s, int pos, int& t0, int& t1) {
        const int n = pos + 1, c = (n + CL - 1) / CL;
        t0 = min(n, s * c);
        t1 = min(n, t0 + c);
    }

    // phase B: q/k norm + RoPE of the pushed q|k|v, K/V append, this CTA's share of the positions,
    // the CL-way partial exchange and the merge into att[256]
    __device__ __noinline__ static void attention(int step, int l, int pos) {
        const Params& p = cl_sm.prm;
        uint32_t& it = ring_pos();
        const int g = cl_sm.g, r = cl_sm.r;
        const uint16_t* nrm = p.layer_n + (size_t)l * p.norm_stride;
        const float2* rrow = p.rope + (size_t)pos * (HD / 2);
        int t0, t1;
        chunk_of(r, pos, t0, t1);
        const bool has_cur = t0 <= pos && pos < t1;
        const float* qkv = dyn().qkv;
        if (warp() < G) {
            const float4 v = reinterpret_cast<const float4*>(qkv + warp() * HD)[lane()];
            head_norm_rope(v, nrm + 2 * H, rrow, cl_sm.qs[warp()]);
        } else if (warp() == G && has_cur) {
            const float4 v = reinterpret_cast<const float4*>(qkv + G * HD)[lane()];
            head_norm_rope(v, nrm + 2 * H + HD, rrow, cl_sm.ks);
        } else if (warp() == G + 1 && has_cur) {
            reinterpret_cast<float4*>(cl_sm.vs)[lane()] = reinterpret_cast<const float4*>(qkv + (G + 1) * HD)[lane()];
        }
        named_bar_sync(1, NCT);
        lstamp(3);
        if (has_cur && tid() < 2 * HD) {  // append K/V at slot `pos` (cpu_inference.rs:140-141)
            const size_t off = (((size_t)l * NKV + g) * p.max_seq + pos) * HD;
            if (tid() < HD) p.kc[off + tid()] = cl_sm.ks[tid()];
            else p.vc[off + tid() - HD] = cl_sm.vs[tid() - HD];
        }
        float4 q4[G];
#pragma unroll
        for (int h = 0; h < G; h++) q4[h] = reinterpret_cast<const float4*>(cl_sm.qs[h])[lane()];
        WS ws;
#pragma unroll
        for (int h = 0; h < G; h++) {
            ws.m[h] = -INFINITY;
            ws.l[h] = 0.f;
            ws.acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const float scale = p.scale;
        const int tc1 = has_cur ? pos : t1;  // cached positions [t0, tc1)
        const int npieces = tc1 > t0 ? (tc1 - t0 + ATT_P - 1) / ATT_P : 0;
        for (int q0 = 0; q0 < npieces; q0 += 4) {
            const int n = min(4, npieces - q0);
            const uint32_t pc = it;
            bool ok = true;
            if (lane() < n) ok = wait_mbar(&cl_sm.full[(pc + lane()) % NSLOT], ((pc + lane()) / NSLOT) & 1, DERR_TIMEOUT_FULL);
            ok = __all_sync(0xFFFFFFFFu, ok);
            __syncwarp();
            for (int j = 0; j < n; j++) {
                const int np = min(ATT_P, tc1 - (t0 + (q0 + j) * ATT_P));
                const float* Kb = reinterpret_cast<const float*>(dyn().ring[(pc + j) % NSLOT]);
                const float* Vb = Kb + ATT_P * HD;
                if (ok)
                    for (int pp = warp(); pp < np; pp += 2 * NCW)
                        attn_pair(Kb + pp * HD, Vb + pp * HD, Kb + (pp + NCW) * HD, Vb + (pp + NCW) * HD, pp + NCW < np, q4,
                                  ws, scale);
            }
            __syncwarp();
            if (lane() == 0 && ok)
                for (int j = 0; j < n; j++) mbar_arrive(&cl_sm.empty[(pc + j) % NSLOT]);
            it = pc + n;
        }
        if (has_cur && warp() == (tc1 - t0) % NCW) attn_pair(cl_sm.ks, cl_sm.vs, nullptr, nullptr, false, q4, ws, scale);
        // combine the 12 warps' states in warp order: stage = acc[2][128] | m[2] | l[2] | pad
#pragma unroll
        for (int h = 0; h < G; h++) {
            float* d = dyn().wst[warp()][h];
            reinterpret_cast<float4*>(d)[lane()] = ws.acc[h];
            if (lane() == 0) {
                d[HD] = ws.m[h];
                d[HD + 1] = ws.l[h];
            }
        }
        named_bar_sync(1, NCT);
        if (tid() < G * HD) {
            const int h = tid() >> 7, d = tid() & (HD - 1);
            float m = -INFINITY, lsum = 0.f, acc = 0.f;
#pragma unroll
            for (int w = 0; w < NCW; w++) m = fmaxf(m, dyn().wst[w][h][HD]);
#pragma unroll
            for (int w = 0; w < NCW; w++) {
                const float* src = dyn().wst[w][h];
                const float e = src[HD] == -INFINITY ? 0.f : __expf(src[HD] - m);
                lsum = fmaf(e, src[HD + 1], lsum);
                acc = fmaf(e, src[d], acc);
            }
            cl_sm.stage[tid()] = acc;
            if (d == 0) {
                cl_sm.stage[G * HD + h] = m;
                cl_sm.stage[G * HD + G + h] = lsum;
            }
        } else if (tid() < G * HD + 4) {
            cl_sm.stage[G * HD + 2 * G + (tid() - G * HD)] = 0.f;
        }
        named_bar_sync(1, NCT);
        lstamp(4);
        // E3: this CTA's partial to the whole cluster (CL x 66 chunks over the 384 consumer threads)
        for (int k = tid(); k < CL * (APW / 4); k += NCT) {
            const uint32_t dest = (uint32_t)(k / (APW / 4)), c = (uint32_t)(k % (APW / 4));
            const float4 v = reinterpret_cast<const float4*>(cl_sm.stage)[c];
            put4(dyn().apr[r] + 4 * c, v, &cl_sm.abar, dest);
        }
        wait_exchange(&cl_sm.abar, (uint32_t)(step * p.L + l), TX_A);
        lstamp(5);
        // merge the CL partials in rank order (cpu_inference.rs:143-161: softmax over all positions)
        if (tid() < G * HD) {
            const int h = tid() >> 7, d = tid() & (HD - 1);
            float M = -INFINITY;
#pragma unroll
            for (int s = 0; s < CL; s++) M = fmaxf(M, dyn().apr[s][G * HD + h]);
            float Lt = 0.f, O = 0.f;
#pragma unroll 4
            for (int s = 0; s < CL; s++) {
                const float ms = dyn().apr[s][G * HD + h];
                const float wgt = ms == -INFINITY ? 0.f : __expf(ms - M);
                Lt = fmaf(wgt, dyn().apr[s][G * HD + G + h], Lt);
                O = fmaf(wgt, dyn().apr[s][tid()], O);
            }
            dyn().att[tid()] = O / Lt;
        }
        named_bar_sync(1, NCT);
    }

    // ------------------------------------------------------------------ lm_head, argmax, token barrier
    __device__ __noinline__ static void lm_partial() {
        const Params& p = cl_sm.prm;
        if (tid() == 0) {
            float bv = cl_sm.redv[0];
            unsigned bi = cl_sm.redi[0];
            for (int w = 1; w < NCW; w++)
                if (am_better(cl_sm.redv[w], cl_sm.redi[w], bv, bi)) { bv = cl_sm.redv[w]; bi = cl_sm.redi[w]; }
            __stcg(p.am_val + cta(), bv);
            __stcg(p.am_idx + cta(), bi);
        }
    }

    __device__ __noinline__ static void token_barrier(uint32_t done) {
        const Params& p = cl_sm.prm;
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
                if (lane() == 0) stop = wait_expired(spins, t0, DERR_TIMEOUT_GRID, (int)done);
                if (__shfl_sync(0xFFFFFFFFu, stop, 0)) break;
            }
            fence_acq_rel_gpu();
        }
        named_bar_sync(1, NCT);
        if (tid() == 0) st_release_cta_shared(&cl_sm.progress, done);
    }

    __device__ __noinline__ static unsigned argmax_combine() {
        const Params& p = cl_sm.prm;
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
                cl_sm.token = t;
            }
        }
        named_bar_sync(1, NCT);
        return cl_sm.token;
    }

    __device__ __noinline__ static void publish_token(int step, unsigned token) {
        const Params& p = cl_sm.prm;
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

    // the embedding row of `token` as layer 0's input: every CTA reads the whole row (xsA = x * ln1,
    // ssA[0] = sum of x^2, ssA[1..] = 0) and keeps its own XO rows as the residual
    __device__ __noinline__ static void embed_input(unsigned token) {
        const Params& p = cl_sm.prm;
        const uint16_t* erow = p.embed + (size_t)token * H;
        const uint16_t* g1 = p.layer_n;
        float ss = 0.f;
        for (int i = tid(); i < H; i += NCT) {
            const float v = bf16_to_f32(__ldg(erow + i));
            ss = fmaf(v, v, ss);
            dyn().xsA[xperm(i)] = v * bf16_to_f32(__ldg(g1 + i));
            const int o = i - XO * cl_sm.r;
            if (o >= 0 && o < XO) cl_sm.xown[o] = v;
        }
        ss = warp_sum(ss);
        if (lane() == 0) cl_sm.redv[warp()] = ss;
        named_bar_sync(1, NCT);
        if (tid() < CL) {
            float t = 0.f;
            if (tid() == 0)
                for (int w = 0; w < NCW; w++) t += cl_sm.redv[w];
            dyn().ssA[tid()] = t;
        }
        named_bar_sync(1, NCT);
    }

    // ------------------------------------------------------------------ consumer main loop
    __device__ __forceinline__ static uint32_t xuse(int step, int k) { return (uint32_t)(step * 2 * vprm().L + k); }

    __device__ __noinline__ static void layer() {
        const int step = cur_step(), l = cur_layer();
        const int L = vprm().L;
        const int pos = vprm().start_pos + step;
        const uint16_t* nrm = vprm().layer_n + (size_t)l * vprm().norm_stride;
        lstamp(0);
        if (l > 0) wait_exchange(&cl_sm.xbar, xuse(step, 2 * l - 1), TX_X);
        lstamp(1);
        // A: q|k|v rows, pushed to the cluster (E2)
        gemv_rows<0>(A_ROWS, dyn().xsA, norm_scale(dyn().ssA), 0);
        push(cl_sm.stage, A_ROWS, dyn().qkv + A_ROWS * cl_sm.r, &cl_sm.qbar, 0);
        wait_exchange(&cl_sm.qbar, (uint32_t)(step * L + l), TX_Q);
        lstamp(2);
        attention(step, l, pos);
        lstamp(6);
        // C: o_proj rows [64r, 64r+64) over the head group's 256 columns -> po[g]
        gemv_units<OK>(XO / 4, dyn().att, vprm().po + (size_t)cl_sm.g * H + XO * cl_sm.r, tag(step, l, 0));
        lstamp(7);
        residual_exchange(vprm().po, tag(step, l, 0), nrm + H, dyn().xsD, dyn().ssD);
        wait_exchange(&cl_sm.xbar, xuse(step, 2 * l), TX_X);
        lstamp(8);
        // D: gate|up rows of this CTA's 24 h values, SiLU * up, pushed to the cluster (E5)
        gemv_rows<1>(2 * HO, dyn().xsD, norm_scale(dyn().ssD), 0);
        push(cl_sm.stage, HO, dyn().hs + HO * cl_sm.r, &cl_sm.hbar, 0);
        wait_exchange(&cl_sm.hbar, (uint32_t)(step * L + l), TX_H);
        lstamp(9);
        // E: down_proj rows [64r, 64r+64) over the cluster's 384 columns -> pd[g]
        gemv_units<DK>(XO / 4, dyn().hs, vprm().pd + (size_t)cl_sm.g * H + XO * cl_sm.r, tag(step, l, 1));
        lstamp(10);
        const uint16_t* next_gain = l + 1 < L ? nrm + vprm().norm_stride : vprm().final_norm;
        residual_exchange(vprm().pd, tag(step, l, 1), next_gain, dyn().xsA, dyn().ssA);
        lstamp(11);
    }

    __device__ static void consume() {
        {
            const Params& p = cl_sm.prm;
            unsigned token = __ldcg(p.tok_in);
            if (token >= (unsigned)p.V) {
                if (tid() == 0) fail(DERR_BAD_TOKEN, (int)token);
                token = 0;
            }
            ls().token = token;
        }
        for (ls().step = 0; cur_step() < vprm().steps; ls().step = cur_step() + 1) {
            embed_input(ls().token);
            for (ls().l = 0; cur_layer() < vprm().L; ls().l = cur_layer() + 1) layer();
            // final norm (pushed by the last layer's residual exchange) -> lm_head -> argmax
            wait_exchange(&cl_sm.xbar, xuse(cur_step(), 2 * vprm().L - 1), TX_X);
            tstamp(0);
            gemv_rows<2>((int)(cl_sm.lm_r1 - cl_sm.lm_r0), dyn().xsA, norm_scale(dyn().ssA), cl_sm.lm_r0);
            lm_partial();
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
        return wait_mbar(&cl_sm.empty[slot], par, DERR_TIMEOUT_EMPTY);
    }

    // `bytes` of contiguous weights from `src` as pieces of at most `piece` bytes
    __device__ __noinline__ static void produce_bytes(const uint16_t* src, uint32_t bytes, uint32_t piece) {
        const uint64_t pol = policy_evict_first();
        uint32_t& it = ring_pos();
        const uint8_t* s = reinterpret_cast<const uint8_t*>(src);
        for (uint32_t off = 0; off < bytes; off += piece) {
            const uint32_t nb = min(piece, bytes - off);
            uint32_t slot;
            if (slot_acquire(slot)) {
                mbar_arrive_expect_tx(&cl_sm.full[slot], nb);
                bulk_g2s_evict_first(dyn().ring[slot], s + off, nb, &cl_sm.full[slot], pol);
                cl_sm.n_issued = it + 1;
            }
            ++it;
        }
    }

    __device__ __noinline__ static void attn_produce(int step, int l, int pos) {
        const Params& p = cl_sm.prm;
        uint32_t& it = ring_pos();
        int t0, t1;
        chunk_of(cl_sm.r, pos, t0, t1);
        const bool has_cur = t0 <= pos && pos < t1;
        const int tc1 = has_cur ? pos : t1;
        if (t0 >= tc1) return;
        // K/V of earlier positions may have been written by other CTAs in earlier steps of this
        // launch: wait until this CTA's consumers passed the previous token's barrier, then order the
        // async-proxy reads after it
        if (step > 0 && !aborted() && l == 0) {
            uint32_t spins = 0;
            uint64_t t0w = 0;
            while (ld_acquire_cta_shared(&cl_sm.progress) < (uint32_t)step) {
                if (wait_expired(spins, t0w, DERR_TIMEOUT_KV, step)) break;
                __nanosleep(32);
            }
            fence_proxy_async_global();
        }
        const size_t head = ((size_t)l * NKV + cl_sm.g) * p.max_seq;
        for (int t = t0; t < tc1; t += ATT_P) {
            const int np = min(ATT_P, tc1 - t);
            uint32_t slot;
            if (slot_acquire(slot)) {
                const uint32_t bytes = (uint32_t)np * HD * 4u;
                mbar_arrive_expect_tx(&cl_sm.full[slot], 2u * bytes);
                uint8_t* dst = dyn().ring[slot];
                bulk_g2s(dst, p.kc + (head + t) * HD, bytes, &cl_sm.full[slot]);
                bulk_g2s(dst + ATT_P * HD * 4, p.vc + (head + t) * HD, bytes, &cl_sm.full[slot]);
                cl_sm.n_issued = it + 1;
            }
            ++it;
        }
    }

    __device__ __forceinline__ static const uint16_t* a_src(int l) {
        return vprm().layer_w + (size_t)l * vprm().layer_stride + (size_t)cl_sm.a_row0 * H;
    }
    __device__ __forceinline__ static const uint16_t* c_src(int l) {
        return vprm().o_blk + (((size_t)l * NKV + cl_sm.g) * CL + cl_sm.r) * (size_t)(XO * OK);
    }
    __device__ __forceinline__ static const uint16_t* d_src(int l) {
        return vprm().layer_w + (size_t)l * vprm().layer_stride + (size_t)QKVR * H + (size_t)H * QD +
               (size_t)2 * (DK * cl_sm.g + HO * cl_sm.r) * H;
    }
    __device__ __forceinline__ static const uint16_t* e_src(int l) {
        return vprm().d_blk + (((size_t)l * NKV + cl_sm.g) * CL + cl_sm.r) * (size_t)(XO * DK);
    }

    // warm L2 with this CTA's rows of layer l and the cached K/V its attention will read for a token
    // at `pos` (the ring holds less than a layer; at long context the K/V rows are a third of it)
    __device__ __noinline__ static void prefetch_layer(int l, int pos) {
        const Params& p = cl_sm.prm;
        bulk_prefetch_l2(a_src(l), A_ROWS * H * 2);
        bulk_prefetch_l2(c_src(l), XO * OK * 2);
        bulk_prefetch_l2(d_src(l), 2 * HO * H * 2);
        bulk_prefetch_l2(e_src(l), XO * DK * 2);
        int t0, t1;
        chunk_of(cl_sm.r, pos, t0, t1);
        const int tc1 = (t0 <= pos && pos < t1) ? pos : t1;
        if (tc1 > t0) {
            const size_t row = (((size_t)l * NKV + cl_sm.g) * p.max_seq + t0) * HD;
            const uint32_t bytes = (uint32_t)(tc1 - t0) * HD * 4u;
            bulk_prefetch_l2(p.kc + row, bytes);
            bulk_prefetch_l2(p.vc + row, bytes);
        }
    }

    __device__ static void produce() {
        prefetch_layer(0, vprm().start_pos);
        for (ls().step = 0; cur_step() < vprm().steps; ls().step = cur_step() + 1) {
            const int pos = vprm().start_pos + cur_step();
            for (ls().l = 0; cur_layer() < vprm().L; ls().l = cur_layer() + 1) {
                const int l = cur_layer();
                if (l + 1 < vprm().L) prefetch_layer(l + 1, pos);
                else {
                    const uint32_t lm_bytes = (cl_sm.lm_r1 - cl_sm.lm_r0) * (uint32_t)H * 2u;
                    bulk_prefetch_l2(vprm().lm_head + (size_t)cl_sm.lm_r0 * H, min(lm_bytes, 256u * 1024u));
                }
                produce_bytes(a_src(l), A_ROWS * H * 2, 12 * H * 2);
                attn_produce(cur_step(), l, pos);
                produce_bytes(c_src(l), XO * OK * 2, SLOT_BYTES);
                produce_bytes(d_src(l), 2 * HO * H * 2, 12 * H * 2);
                produce_bytes(e_src(l), XO * DK * 2, SLOT_BYTES);
            }
            if (cur_step() + 1 < vprm().steps) prefetch_layer(0, pos + 1);
            produce_bytes(vprm().lm_head + (size_t)cl_sm.lm_r0 * H, (cl_sm.lm_r1 - cl_sm.lm_r0) * (uint32_t)H * 2u,
                          12 * H * 2);
        }
        drain();
    }

    __device__ __noinline__ static void drain() {
        const Params& p = cl_sm.prm;
        if (aborted()) {
            const uint32_t first = cl_sm.n_issued > NSLOT ? cl_sm.n_issued - NSLOT : 0;
            for (uint32_t j = first; j < cl_sm.n_issued; j++) {
                const int slot = j % NSLOT;
                const uint32_t par = (j / NSLOT) & 1;
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(&cl_sm.full[slot], par)) {
                    if (globaltimer_ns() - t0 > (uint64_t)p.timeout_ns) {
                        atomicCAS(&p.err[3], 0, DERR_TIMEOUT_DRAIN);
                        break;
                    }
                }
            }
        }
    }
};

// 13 warps, one CTA per SM, clusters of 16 (one per KV head)
__global__ void __launch_bounds__(NTHREADS, 1) cluster_decode_kernel(const __grid_constant__ Params p) {
    if (threadIdx.x == 0) {
        for (int i = 0; i < NSLOT; i++) {
            mbar_init(&cl_sm.full[i], 1);
            mbar_init(&cl_sm.empty[i], NCW);   // every consumer warp releases every slot it read
        }
        mbar_init(&cl_sm.xbar, 1);
        mbar_init(&cl_sm.qbar, 1);
        mbar_init(&cl_sm.abar, 1);
        mbar_init(&cl_sm.hbar, 1);
        cl_sm.progress = 0;
        cl_sm.abort = 0;
        cl_sm.token = 0;
        cl_sm.prm = p;
        for (int w = 0; w <= NCW; w++) cl_sm.ring_it[w] = 0;
        cl_sm.n_issued = 0;
        const int g = (int)cluster_id_x(), r = (int)cluster_ctarank();
        cl_sm.g = g;
        cl_sm.r = r;
        // rows [A_ROWS r, A_ROWS (r+1)) of the cluster's block q(2g) | q(2g+1) | k(g) | v(g)
        const int b0 = A_ROWS * r;
        cl_sm.a_row0 = b0 < G * HD ? (uint32_t)(G * HD * g + b0)
                     : b0 < (G + 1) * HD ? (uint32_t)(QD + HD * g + b0 - G * HD)
                                         : (uint32_t)(QD + KVD + HD * g + b0 - (G + 1) * HD);
        const long long c = blockIdx.x, n = gridDim.x;
        cl_sm.lm_r0 = (uint32_t)((long long)p.V * c / n);
        cl_sm.lm_r1 = (uint32_t)((long long)p.V * (c + 1) / n);
        fence_mbar_init();
    }
    __syncthreads();
    // every CTA of the cluster has initialised its mbarriers before any peer pushes into it
    cluster_arrive();
    cluster_wait();
    if (CDecoder::warp() == NCW) {
        if (CDecoder::lane() == 0) CDecoder::produce();
    } else {
        CDecoder::consume();
    }
    // no CTA leaves while a peer may still write into its shared memory
    __syncwarp();
    cluster_arrive();
    cluster_wait();
}

}  // namespace cl
}  // namespace qw
