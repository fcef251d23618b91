// tcgen05 tensor-core GEMM for the batched prefill (sm_100a):
//
//   Y[M x N] (f32) = (A_hi + A_lo)[M x K] . B[N x K]^T
//
// A holds f32 activations split into two bf16 halves (A_hi = bf16(a), A_lo = bf16(a - A_hi)), so
// that the product keeps ~16 bits of each activation's mantissa against bf16 weights: the two
// halves accumulate into the same f32 accumulator. B is a weight matrix as stored ([out][in],
// row-major, bf16). Both operands are K-major, which is the nn.Linear layout.
//
// One CTA computes one BM x BN tile (BM = 128 rows, BN = 128 columns) with 4 warps:
//   * warp 0, one lane: TMA producer. Per K block of 64 it loads the A_hi, A_lo and B tiles with
//     2-D tiled bulk tensor copies (cp.async.bulk.tensor, 128-byte swizzle, no multicast) into a
//     STAGES-deep shared-memory ring, signalling a full mbarrier with the byte count;
//   * warp 1, one lane: MMA issuer. Per K block it issues 4 K-steps x 2 halves of
//     tcgen05.mma.cta_group::1.kind::f16 (M=128, N=128, K=16, bf16 x bf16 -> f32) accumulating in
//     tensor memory, then tcgen05.commit to the stage's empty mbarrier so the producer may refill
//     it; after the last block a final commit signals the epilogue;
//   * all 4 warps: epilogue. Warp w reads TMEM lanes 32w..32w+31 (its 32 rows) with
//     tcgen05.ld.32x32b and stores the f32 rows.
// TMEM: 128 columns (the accumulator) allocated by warp 1 and freed by it at the end.
//
// Every wait is bounded: a wait that runs out sets `err` (the kernel's error word) and the CTA
// skips the remaining work, still waiting (bounded) for the copies and MMAs it issued and freeing
// its tensor memory before it exits.
//
// gemm_skinny_kernel is the same product for M <= 16 activation rows (a decode batch, a short
// verify pass). There the weights are the only real traffic, so the roles swap: the weight tile
// is the MMA's A operand (M = 128 weight rows) and the activations its B operand (N = 16), giving
// D[128][16] = W . X^T per CTA in 32 TMEM columns. Tensor work per weight byte drops 8x against a
// 128-row activation tile, and a 20 KB stage (16 KB weights) lets an 8-deep ring keep 128 KB of
// weights in flight per SM.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "ptx.cuh"

namespace qw {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 64;                       // bf16 elements per 128-byte swizzle row
constexpr int STAGES = 4;
constexpr int TILE_A = BM * BK * 2;          // bytes of one A half tile (16 KB)
constexpr int TILE_B = BN * BK * 2;          // bytes of one B tile (16 KB)
constexpr int STAGE_BYTES = 2 * TILE_A + TILE_B;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack for the 1024-byte swizzle atoms
// launches of more tiles than SMs use 2 stages, so two CTAs share an SM (TMEM 2 x 128 columns) and
// one's MMAs overlap the other's pipeline fill and epilogue
constexpr int STAGES_WIDE = 2;
constexpr int SMEM_BYTES_WIDE = STAGES_WIDE * STAGE_BYTES + 1024;
constexpr int THREADS = 128;
constexpr int TMEM_COLS = BN;                // f32 accumulator columns
constexpr long long WAIT_LIMIT_NS = 2000000000ll;

// UMMA shared-memory descriptor of a K-major operand tile written by TMA with 128-byte swizzle:
// rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset), version 1 (sm_100),
// layout type 2 (SWIZZLE_128B). Addresses and offsets are in 16-byte units.
__device__ __forceinline__ uint64_t smem_desc_k128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);         // start address
    d |= (uint64_t)1u << 16;                              // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;                    // stride byte offset: next 8-row group
    d |= (uint64_t)1u << 46;                              // descriptor version (sm_100)
    d |= (uint64_t)2u << 61;                              // SWIZZLE_128B
    return d;
}

// instruction descriptor of kind::f16 with bf16 A and B, f32 accumulate, both K-major, M x N
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
    return (1u << 4)                   // D format: f32
         | (1u << 7)                   // A format: bf16
         | (1u << 10)                  // B format: bf16
         | ((uint32_t)(n >> 3) << 17)  // N / 8
         | ((uint32_t)(m >> 4) << 24); // M / 16
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(smem_dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// bounded wait on an mbarrier phase; false when it ran out (or another thread gave up)
__device__ __forceinline__ bool bounded_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++spins & 63) == 0) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > (uint64_t)WAIT_LIMIT_NS) {
                *abort_flag = 1;
                return false;
            }
        }
    }
    return true;
}

struct GemmArgs {
    float* y;          // [M][ldy] f32 output; split z writes y + z * split_stride
    int M, N, K;
    int ldy;
    int* err;          // kernel error word (nonzero: a wait ran out)
    long long split_stride;  // elements between the outputs of K splits (blockIdx.z)
    // SiLU epilogue (gemm_bf16x2_kernel, one K split): instead of y, columns 2i, 2i+1 of the output
    // (interleaved gate/up rows of B) become h = silu(gate) * up, stored as its bf16 high and low
    // halves silu_hi/silu_lo[row][i] with row pitch N / 2 (the down GEMM's input); null: plain y
    uint16_t* silu_hi = nullptr;
    uint16_t* silu_lo = nullptr;
};

template <int STG>
__global__ void __launch_bounds__(THREADS, 1)
gemm_bf16x2_kernel(const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo,
                   const __grid_constant__ CUtensorMap map_b, const GemmArgs args) {
    extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
    __shared__ uint64_t full[STG], empty[STG], done;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    // 1024-byte aligned ring (the 128-byte swizzle atom spans 8 rows x 128 bytes)
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // tiles in launch order with the M tile fastest (gridDim.y M tiles, gridDim.x N tiles): the CTAs
    // that share a weight tile start together, so a weight matrix larger than L2 (the lm_head's
    // 311 MB) is read from HBM once instead of once per M tile
    const int lin = (int)(blockIdx.x + blockIdx.y * gridDim.x);
    const int m0 = (lin % (int)gridDim.y) * BM, n0 = (lin / (int)gridDim.y) * BN;
    // split-K: CTA z of gridDim.z covers K blocks [kb0, kb0 + nkb) and writes its own output slice
    const int nkb_all = args.K / BK;
    const int kb0 = (int)((long long)nkb_all * blockIdx.z / gridDim.z);
    const int nkb = (int)((long long)nkb_all * (blockIdx.z + 1) / gridDim.z) - kb0;
    float* const y = args.y + (long long)blockIdx.z * args.split_stride;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STG; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {  // one warp allocates the accumulator's tensor-memory columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&tmem_base)), "r"((uint32_t)TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;
    const uint32_t idesc = idesc_bf16_f32(BM, BN);
    int issued_kb = 0;   // producer: K blocks whose copies were issued

    if (warp == 0 && lane == 0) {
        // the first stages' weight tiles do not depend on the previous kernel: issue them before
        // waiting for it (programmatic dependent launch), the activation tiles after
        const int pre = nkb < STG ? nkb : STG;
        for (int kb = 0; kb < pre; kb++) {
            uint8_t* st = ring + (kb % STG) * STAGE_BYTES;
            mbar_arrive_expect_tx(&full[kb], STAGE_BYTES);
            tma_load_2d(st + 2 * TILE_A, &map_b, (kb0 + kb) * BK, n0, &full[kb]);
        }
        pdl_wait();
        pdl_trigger();
        for (int kb = 0; kb < pre; kb++) {
            uint8_t* st = ring + (kb % STG) * STAGE_BYTES;
            tma_load_2d(st, &map_ahi, (kb0 + kb) * BK, m0, &full[kb]);
            tma_load_2d(st + TILE_A, &map_alo, (kb0 + kb) * BK, m0, &full[kb]);
        }
        issued_kb = pre;
        for (int kb = pre; kb < nkb; kb++) {
            const int s = kb % STG;
            if (!bounded_wait(&empty[s], ((kb / STG) - 1) & 1, &abort_flag)) break;
            uint8_t* st = ring + s * STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
            tma_load_2d(st, &map_ahi, (kb0 + kb) * BK, m0, &full[s]);
            tma_load_2d(st + TILE_A, &map_alo, (kb0 + kb) * BK, m0, &full[s]);
            tma_load_2d(st + 2 * TILE_A, &map_b, (kb0 + kb) * BK, n0, &full[s]);
            issued_kb = kb + 1;
        }
    } else if (warp == 1 && lane == 0) {
        for (int kb = 0; kb < nkb; kb++) {
            const int s = kb % STG;
            if (!bounded_wait(&full[s], (kb / STG) & 1, &abort_flag)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t st = smem_u32(ring + s * STAGE_BYTES);
            const uint64_t dhi = smem_desc_k128(st), dlo = smem_desc_k128(st + TILE_A), db = smem_desc_k128(st + 2 * TILE_A);
#pragma unroll
            for (int kk = 0; kk < BK / 16; kk++) {
                // a K step of 16 bf16 is 32 bytes along the swizzled row: +2 in 16-byte units
                mma_bf16(tmem, dhi + 2 * kk, db + 2 * kk, idesc, (kb | kk) != 0);
                mma_bf16(tmem, dlo + 2 * kk, db + 2 * kk, idesc, 1u);
            }
            mma_commit(&empty[s]);  // the stage may be refilled once these MMAs have read it
        }
        mma_commit(&done);          // arrives when every MMA issued above has completed
    }
    __syncwarp();
    // epilogue: wait for the accumulator (bounded), then TMEM -> registers -> global
    const bool ok = bounded_wait(&done, 0, &abort_flag) && !abort_flag;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok && args.silu_hi) {
        // cpu_inference.rs:166-170, :187: h = silu(gate) * up, the same expression and split as the
        // separate silu pass, so the values are identical to it
        const int row = m0 + warp * 32 + lane;
        const int ldh = args.N / 2;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, r);
            if (row < args.M && n0 + c < args.N) {
                const int np = (args.N - (n0 + c) < 32 ? args.N - (n0 + c) : 32) / 2;
                const size_t h0 = (size_t)row * ldh + (size_t)((n0 + c) >> 1);
                uint32_t hp[8], lp[8];
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const float g = __uint_as_float(r[2 * j]), u = __uint_as_float(r[2 * j + 1]);
                    const float v = g / (1.0f + __expf(-g)) * u;
                    const __nv_bfloat16 h = __float2bfloat16_rn(v);
                    const uint32_t hb = __bfloat16_as_ushort(h);
                    const uint32_t lb = __bfloat16_as_ushort(__float2bfloat16_rn(v - __bfloat162float(h)));
                    if (j & 1) { hp[j >> 1] |= hb << 16; lp[j >> 1] |= lb << 16; }
                    else { hp[j >> 1] = hb; lp[j >> 1] = lb; }
                }
                uint16_t* dh = args.silu_hi + h0;
                uint16_t* dl = args.silu_lo + h0;
                if (np == 16 && ((reinterpret_cast<uintptr_t>(dh) | reinterpret_cast<uintptr_t>(dl)) & 15) == 0) {
                    reinterpret_cast<uint4*>(dh)[0] = make_uint4(hp[0], hp[1], hp[2], hp[3]);
                    reinterpret_cast<uint4*>(dh)[1] = make_uint4(hp[4], hp[5], hp[6], hp[7]);
                    reinterpret_cast<uint4*>(dl)[0] = make_uint4(lp[0], lp[1], lp[2], lp[3]);
                    reinterpret_cast<uint4*>(dl)[1] = make_uint4(lp[4], lp[5], lp[6], lp[7]);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (j < np) {
                            dh[j] = (uint16_t)(hp[j >> 1] >> (16 * (j & 1)));
                            dl[j] = (uint16_t)(lp[j >> 1] >> (16 * (j & 1)));
                        }
                }
            }
        }
    } else if (ok) {
        const int row = m0 + warp * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, r);
            if (row < args.M && n0 + c < args.N) {
                float* dst = y + (size_t)row * args.ldy + n0 + c;
                const int nv = args.N - (n0 + c) < 32 ? args.N - (n0 + c) : 32;
                // float4 stores only where the row is 16-byte aligned (ldy need not be a multiple of 4,
                // e.g. an odd vocabulary size)
                if (nv == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(dst + j) = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                                          __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                } else {
#pragma unroll
                    for (int j = 0; j < 32; j++)  // unrolled: r stays in registers
                        if (j < nv) dst[j] = __uint_as_float(r[j]);
                }
            }
        }
    }
    if (!ok && threadIdx.x == 0) atomicExch(args.err, 1);
    // after an abort, the TMA copies still in flight must land before the CTA exits
    if (!ok && warp == 0 && lane == 0) {
        for (int kb = issued_kb - STG > 0 ? issued_kb - STG : 0; kb < issued_kb; kb++) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&full[kb % STG], (kb / STG) & 1))
                if (globaltimer_ns() - t0 > (uint64_t)WAIT_LIMIT_NS) break;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        // the MMAs issued before an abort must finish before their accumulator columns are freed:
        // the final commit arrives on `done` once they have (bounded wait, whatever abort_flag says)
        if (!ok && lane == 0) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&done, 0))
                if (globaltimer_ns() - t0 > (uint64_t)WAIT_LIMIT_NS) break;
        }
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)TMEM_COLS) : "memory");
    }
}

constexpr int SK_NB = 16;                          // most activation rows of the skinny GEMM
constexpr int SK_STAGES = 8;
constexpr int SK_TILE_W = BN * BK * 2;             // 16 KB weight tile (128 rows x 64)
constexpr int SK_TILE_X = SK_NB * BK * 2;          // 2 KB activation half tile (16 rows x 64)
constexpr int SK_STAGE_BYTES = SK_TILE_W + 2 * SK_TILE_X;
constexpr int SK_SMEM_BYTES = SK_STAGES * SK_STAGE_BYTES + 1024;
constexpr int SK_STAGES_WIDE = 4;                  // stages of a many-wave launch (two CTAs per SM)
constexpr int SK_SMEM_BYTES_WIDE = SK_STAGES_WIDE * SK_STAGE_BYTES + 1024;
constexpr int SK_TMEM_COLS = 32;                   // smallest allocation; columns 0..15 used

// Y[M][ldy] (M <= 16) = (X_hi + X_lo)[M][K] . W[N][K]^T; CTA = 128 weight rows x one K range
// STG ring stages: 8 for a layer's one-wave launches (the most weights in flight per SM); 4 for
// many-wave launches (the lm_head), where two CTAs per SM let one stream while the other fills or
// drains its pipeline
template <int STG>
__global__ void __launch_bounds__(THREADS, 1)
gemm_skinny_kernel(const __grid_constant__ CUtensorMap map_xhi, const __grid_constant__ CUtensorMap map_xlo,
                   const __grid_constant__ CUtensorMap map_w, const GemmArgs args) {
    extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
    __shared__ uint64_t full[STG], empty[STG], done;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN;
    const int nkb_all = args.K / BK;
    const int kb0 = (int)((long long)nkb_all * blockIdx.z / gridDim.z);
    const int nkb = (int)((long long)nkb_all * (blockIdx.z + 1) / gridDim.z) - kb0;
    float* const y = args.y + (long long)blockIdx.z * args.split_stride;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STG; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&tmem_base)), "r"((uint32_t)SK_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;
    const uint32_t idesc = idesc_bf16_f32(BN, SK_NB);
    int issued_kb = 0;

    if (warp == 0 && lane == 0) {
        // weight tiles of the first stages before waiting for the previous kernel, activations after
        const int pre = nkb < STG ? nkb : STG;
        for (int kb = 0; kb < pre; kb++) {
            mbar_arrive_expect_tx(&full[kb], SK_STAGE_BYTES);
            tma_load_2d(ring + kb * SK_STAGE_BYTES, &map_w, (kb0 + kb) * BK, n0, &full[kb]);
        }
        pdl_wait();
        pdl_trigger();
        for (int kb = 0; kb < pre; kb++) {
            uint8_t* st = ring + kb * SK_STAGE_BYTES;
            tma_load_2d(st + SK_TILE_W, &map_xhi, (kb0 + kb) * BK, 0, &full[kb]);
            tma_load_2d(st + SK_TILE_W + SK_TILE_X, &map_xlo, (kb0 + kb) * BK, 0, &full[kb]);
        }
        issued_kb = pre;
        for (int kb = pre; kb < nkb; kb++) {
            const int s = kb % STG;
            if (!bounded_wait(&empty[s], ((kb / STG) - 1) & 1, &abort_flag)) break;
            uint8_t* st = ring + s * SK_STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s], SK_STAGE_BYTES);
            tma_load_2d(st, &map_w, (kb0 + kb) * BK, n0, &full[s]);
            tma_load_2d(st + SK_TILE_W, &map_xhi, (kb0 + kb) * BK, 0, &full[s]);
            tma_load_2d(st + SK_TILE_W + SK_TILE_X, &map_xlo, (kb0 + kb) * BK, 0, &full[s]);
            issued_kb = kb + 1;
        }
    } else if (warp == 1 && lane == 0) {
        for (int kb = 0; kb < nkb; kb++) {
            const int s = kb % STG;
            if (!bounded_wait(&full[s], (kb / STG) & 1, &abort_flag)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t st = smem_u32(ring + s * SK_STAGE_BYTES);
            const uint64_t dw = smem_desc_k128(st), dhi = smem_desc_k128(st + SK_TILE_W),
                           dlo = smem_desc_k128(st + SK_TILE_W + SK_TILE_X);
#pragma unroll
            for (int kk = 0; kk < BK / 16; kk++) {
                mma_bf16(tmem, dw + 2 * kk, dhi + 2 * kk, idesc, (kb | kk) != 0);
                mma_bf16(tmem, dw + 2 * kk, dlo + 2 * kk, idesc, 1u);
            }
            mma_commit(&empty[s]);
        }
        mma_commit(&done);
    }
    __syncwarp();
    const bool ok = bounded_wait(&done, 0, &abort_flag) && !abort_flag;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok) {
        // thread = weight row n0 + 32 warp + lane (TMEM lane), column j = activation row j
        uint32_t r[16];
        tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16), r);
        const int row = n0 + warp * 32 + lane;
        if (row < args.N) {
#pragma unroll
            for (int j = 0; j < SK_NB; j++)
                if (j < args.M) y[(size_t)j * args.ldy + row] = __uint_as_float(r[j]);
        }
    }
    if (!ok && threadIdx.x == 0) atomicExch(args.err, 1);
    if (!ok && warp == 0 && lane == 0) {
        for (int kb = issued_kb - STG > 0 ? issued_kb - STG : 0; kb < issued_kb; kb++) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&full[kb % STG], (kb / STG) & 1))
                if (globaltimer_ns() - t0 > (uint64_t)WAIT_LIMIT_NS) break;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        if (!ok && lane == 0) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&done, 0))
                if (globaltimer_ns() - t0 > (uint64_t)WAIT_LIMIT_NS) break;
        }
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)SK_TMEM_COLS) : "memory");
    }
}

}  // namespace tc
}  // namespace qw
