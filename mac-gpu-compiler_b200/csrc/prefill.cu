// Batched prefill (the 512-token prompt workload, configs[3]): the tcgen05 GEMM's host side (tensor maps, launch) and
// the standalone entry point qw_gemm_bf16x2 (see tc_gemm.cuh for the kernel).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/cuda_inference.h"
#include "prefill.h"
#include "tc_gemm.cuh"

namespace qw {
int* device_err_word_for(int device);
int set_error(int code, const char* msg);
}  // namespace qw

using namespace qw;

namespace qw {

// Every kernel of the prefill and the batch step is launched with programmatic stream
// serialization: it may start (and run its prologue, e.g. a GEMM's first weight copies) while the
// previous kernel finishes; each calls pdl_wait() before it touches memory an earlier kernel wrote
// or reads. Launch errors surface through cudaGetLastError.
template <typename... KArgs, typename... Args>
void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

namespace tc {

// cuTensorMapEncodeTiled, fetched from the driver through the runtime (the library links the
// runtime statically and does not link libcuda itself)
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn(std::string& err) {
    static std::mutex mu;
    static EncodeTiledFn fn = nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p) {
            err = "cuTensorMapEncodeTiled is not available from the driver";
            return nullptr;
        }
        fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D tensor map of a row-major bf16 matrix [rows][cols] (cols contiguous, row pitch `pitch`
// elements), tiles of box_rows x 64 columns (128 bytes) with 128-byte swizzle; reads outside the
// matrix return zeros.
int make_map_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch, uint32_t box_rows,
                  std::string& err) {
    EncodeTiledFn fn = encode_fn(err);
    if (!fn) return QW_ERR_CUDA;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (pitch * 2) % 16 || cols % BK) {
        err = "tensor map: base must be 16-byte aligned, the row pitch a multiple of 16 bytes and cols a multiple of 64";
        return QW_ERR_ARG;
    }
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {pitch * 2};
    const cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        err = "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
        return QW_ERR_CUDA;
    }
    return QW_OK;
}

// Y[M][ldy] = (A_hi + A_lo)[M][K] . B[N][K]^T ; A halves with row pitch lda, B with row pitch ldb
// With ksplit > 1 the K blocks are split over ksplit CTAs per tile, each writing its partial
// product to its own slice y + z * M * ldy (the caller sums the slices in a fixed order).
// With silu_hi/silu_lo (M > 16, ksplit 1, N even): the SiLU epilogue of GemmArgs instead of y.
int gemm(const uint16_t* a_hi, const uint16_t* a_lo, int lda, const uint16_t* b, int ldb, float* y, int ldy, int M, int N,
         int K, int* err_word, cudaStream_t s, std::string& err, int ksplit, uint16_t* silu_hi = nullptr,
         uint16_t* silu_lo = nullptr) {
    if (M <= 0 || N <= 0 || K <= 0 || K % BK != 0 || ksplit < 1 || ksplit > K / BK) {
        err = "gemm: M, N, K must be positive, K a multiple of 64 and 1 <= ksplit <= K / 64";
        return QW_ERR_ARG;
    }
    if (silu_hi && (M <= SK_NB || ksplit != 1 || N % 2 != 0 || !silu_lo)) {
        err = "gemm: the SiLU epilogue needs M > 16, one K split and an even N";
        return QW_ERR_ARG;
    }
    CUtensorMap mh, ml, mb;
    int rc;
    if (M <= SK_NB) {  // weights-bound: the swapped-operand kernel
        if ((rc = make_map_bf16(&mh, a_hi, (uint64_t)M, (uint64_t)K, (uint64_t)lda, SK_NB, err))) return rc;
        if ((rc = make_map_bf16(&ml, a_lo, (uint64_t)M, (uint64_t)K, (uint64_t)lda, SK_NB, err))) return rc;
        if ((rc = make_map_bf16(&mb, b, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, BN, err))) return rc;
        // a launch of many waves (the lm_head: 1187 tiles) runs two 4-stage CTAs per SM
        const bool wide = (long long)((N + BN - 1) / BN) * ksplit > 2 * 148;
        if (cudaFuncSetAttribute(gemm_skinny_kernel<SK_STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM_BYTES) !=
                cudaSuccess ||
            cudaFuncSetAttribute(gemm_skinny_kernel<SK_STAGES_WIDE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 SK_SMEM_BYTES_WIDE) != cudaSuccess) {
            err = "cannot raise the skinny GEMM kernel's shared-memory limit";
            return QW_ERR_CUDA;
        }
        GemmArgs args{y, M, N, K, ldy, err_word, (long long)M * ldy};
        if (wide)
            launch(gemm_skinny_kernel<SK_STAGES_WIDE>, dim3((N + BN - 1) / BN, 1, ksplit), dim3(THREADS), SK_SMEM_BYTES_WIDE, s, mh,
                   ml, mb, args);
        else
            launch(gemm_skinny_kernel<SK_STAGES>, dim3((N + BN - 1) / BN, 1, ksplit), dim3(THREADS), SK_SMEM_BYTES, s, mh, ml, mb,
                   args);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            err = std::string("GEMM launch failed: ") + cudaGetErrorString(e);
            return QW_ERR_CUDA;
        }
        return QW_OK;
    }
    if ((rc = make_map_bf16(&mh, a_hi, (uint64_t)M, (uint64_t)K, (uint64_t)lda, BM, err))) return rc;
    if ((rc = make_map_bf16(&ml, a_lo, (uint64_t)M, (uint64_t)K, (uint64_t)lda, BM, err))) return rc;
    if ((rc = make_map_bf16(&mb, b, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, BN, err))) return rc;
    if (cudaFuncSetAttribute(gemm_bf16x2_kernel<STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_bf16x2_kernel<STAGES_WIDE>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES_WIDE) !=
            cudaSuccess) {
        err = "cannot raise the GEMM kernel's shared-memory limit";
        return QW_ERR_CUDA;
    }
    GemmArgs args{y, M, N, K, ldy, err_word, (long long)M * ldy, silu_hi, silu_lo};
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, ksplit);
    if ((long long)grid.x * grid.y * grid.z > 148)
        launch(gemm_bf16x2_kernel<STAGES_WIDE>, dim3(grid), dim3(THREADS), SMEM_BYTES_WIDE, s, mh, ml, mb, args);
    else
        launch(gemm_bf16x2_kernel<STAGES>, dim3(grid), dim3(THREADS), SMEM_BYTES, s, mh, ml, mb, args);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        err = std::string("GEMM launch failed: ") + cudaGetErrorString(e);
        return QW_ERR_CUDA;
    }
    return QW_OK;
}

}  // namespace tc

// ---------------------------------------------------------------------------------------------
// The prefill pipeline: one forward pass over n prompt tokens at positions start .. start+n-1
// (the reference feeds them one at a time, cpu_inference.rs:100-179; here every projection is
// one tensor-core GEMM over all n tokens). Residual stream X [n][H] f32; GEMM inputs are the
// bf16 hi/lo halves of f32 activations (see tc_gemm.cuh).
namespace pf {

constexpr int ROW_THREADS = 512;   // norm_split: one row per CTA (two hidden elements per thread at H = 1024)

int ksplit_for(int M, int N, int K) {
    const int tiles = ((M + 127) / 128) * ((N + 127) / 128);
    return std::max(1, std::min({148 / tiles, KSPLIT_MAX, K / 64}));
}

size_t y_floats(int n, int H, int I, int NQ, int NKV) {
    const int QD = NQ * 128, QKVR = QD + 2 * NKV * 128;
    const size_t a = (size_t)ksplit_for(n, QKVR, H) * QKVR, b = (size_t)ksplit_for(n, H, QD) * H,
                 c = (size_t)ksplit_for(n, 2 * I, H) * 2 * I, d = (size_t)ksplit_for(n, H, I) * H;
    return (size_t)n * std::max({a, b, c, d});
}

__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

__device__ __forceinline__ void split_store(float v, uint16_t* hi, uint16_t* lo, size_t i) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[i] = __bfloat16_as_ushort(h);
    lo[i] = __bfloat16_as_ushort(__float2bfloat16_rn(v - __bfloat162float(h)));
}

// four consecutive values split into bf16 hi/lo at hi[i..i+3], lo[i..i+3] (i a multiple of 4)
__device__ __forceinline__ void store_split4(uint16_t* hi, uint16_t* lo, size_t i, float4 v) {
    const __nv_bfloat162 h01 = __floats2bfloat162_rn(v.x, v.y), h23 = __floats2bfloat162_rn(v.z, v.w);
    const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
    const __nv_bfloat162 l01 = __floats2bfloat162_rn(v.x - f01.x, v.y - f01.y), l23 = __floats2bfloat162_rn(v.z - f23.x, v.w - f23.y);
    *reinterpret_cast<uint2*>(hi + i) = make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
    *reinterpret_cast<uint2*>(lo + i) = make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
}

// v + p[0] + p[stride] + ... over n <= NS slices, added in slice order
template <int NS>
__device__ __forceinline__ float add_slices(float v, const float* p, int n, size_t stride) {
    float pv[NS];
#pragma unroll
    for (int z = 0; z < NS; z++) pv[z] = z < n ? p[z * stride] : 0.f;
#pragma unroll
    for (int z = 0; z < NS; z++)
        if (z < n) v += pv[z];
    return v;
}

// 1 / sqrt(mean(x^2) + eps) of a row whose norm_part blocks left nblk sums of squares at ssq (added
// in block order, so every consumer of the row gets the same scale)
__device__ __forceinline__ float row_scale(const float* ssq, int nblk, int H, float eps) {
    float t = 0.f;
    for (int k = 0; k < nblk; k++) t += ssq[k];
    return rsqrtf(t / (float)H + eps);
}

// X[t] = f32(embed[ids[t]]) (cpu_inference.rs:109-111)
// X[t] = embed[ids[t]] (cpu_inference.rs:109-111). An id >= V (device memory the host did not
// check: qw_prefill_device, or a device first token of a batch decode) is never read through: the
// row is taken from id 0 and err[1] is set, which the host reports as QW_ERR_ARG.
__global__ void embed_rows(const uint32_t* ids, int H, int V, const uint16_t* embed, float* X, int* err) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    uint32_t id = ids[t];
    if (id >= (uint32_t)V) {
        if (threadIdx.x == 0) atomicExch(err + 1, 1);
        id = 0;
    }
    const uint16_t* e = embed + (size_t)id * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) X[(size_t)t * H + i] = bf16f(e[i]);
}

__device__ float block_sum(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < ROW_THREADS / 32; w++) t += red[w];
    __syncthreads();
    return t;
}

// X[t] += the nparts split-K slices of the previous projection (residual add, cpu_inference.rs:
// 163-164, :171-172; slices summed in order), then A_hi/A_lo[t] = split(rmsnorm(X[t]) * gain)
// (cpu_inference.rs:189-194)
// MANY: up to KSPLIT_MAX slices with every load in flight (row mode); else up to 4 per round (a
// prefill's few slices). Separate kernels, so the prefill's keeps the smaller register footprint.
// 512 threads per row (two elements each at H = 1024): a 512-token prefill pass took 3.254 ms with
// 1024-thread rows, 3.181 ms with 512 and 3.271 ms with 256 (same box).
template <bool MANY>
__global__ void __launch_bounds__(ROW_THREADS) norm_split(float* X, int H, const uint16_t* gain, float eps, uint16_t* hi,
                                                          uint16_t* lo, const float* parts, int nparts, size_t part_stride) {
    // rows of at most ROW_THREADS elements: one per thread, its gain fetched before waiting for the
    // kernels that produce X and the slices (the gains do not depend on them), its value kept in a
    // register for the output pass
    const bool one = H <= ROW_THREADS;
    float g1 = 0.f, v1 = 0.f;
    if (one && (int)threadIdx.x < H) g1 = bf16f(gain[threadIdx.x]);
    pdl_wait();
    pdl_trigger();
    __shared__ float red[ROW_THREADS / 32];
    const int t = blockIdx.x;
    float* x = X + (size_t)t * H;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += ROW_THREADS) {
        float v = x[i];
        const float* p = parts + (size_t)t * H + i;
        // slices added in slice order
        if (MANY) {
            v = add_slices<KSPLIT_MAX>(v, p, nparts, part_stride);
        } else {
            int z = 0;
            for (; z + 4 <= nparts; z += 4) {
                const float a = p[z * part_stride], b = p[(z + 1) * part_stride], c = p[(z + 2) * part_stride],
                            d = p[(z + 3) * part_stride];
                v += a;
                v += b;
                v += c;
                v += d;
            }
            for (; z < nparts; z++) v += p[z * part_stride];
        }
        if (nparts) x[i] = v;
        ss = fmaf(v, v, ss);
        v1 = v;
    }
    const float sc = rsqrtf(block_sum(ss, red) / (float)H + eps);
    if (one) {
        if ((int)threadIdx.x < H) split_store(v1 * sc * g1, hi, lo, (size_t)t * H + threadIdx.x);
    } else {
        for (int i = threadIdx.x; i < H; i += ROW_THREADS) split_store(x[i] * sc * bf16f(gain[i]), hi, lo, (size_t)t * H + i);
    }
}

// Row mode's residual add + RMSNorm input over many CTAs: CTA (b, t) takes columns
// [128 b, 128 b + 128) of row t. X[t] += the nparts slices (in slice order); A_hi/A_lo = split(X[t]
// * gain) WITHOUT the RMSNorm scale; ssq[t][b] = the block's sum of squares (warps in order). The
// consumers of the next projection's outputs apply the scale (row_scale): the projection is linear,
// so W (x * gain * s) = s * W (x * gain). Rows no longer wait on one CTA's 16-slice loads and
// block-wide reduction; the scale costs each consumer a few loads.
constexpr int NP_THREADS = 128;
__global__ void __launch_bounds__(NP_THREADS) norm_part(float* X, int H, const uint16_t* gain, uint16_t* hi, uint16_t* lo,
                                                        const float* parts, int nparts, size_t part_stride, float* ssq) {
    __shared__ float red[NP_THREADS / 32];
    const int t = blockIdx.y, i = blockIdx.x * NP_THREADS + threadIdx.x;
    const float g = i < H ? bf16f(gain[i]) : 0.f;  // the gains do not depend on earlier kernels
    pdl_wait();
    pdl_trigger();
    float v = 0.f;
    if (i < H) {
        v = add_slices<KSPLIT_MAX>(X[(size_t)t * H + i], parts + (size_t)t * H + i, nparts, part_stride);
        if (nparts) X[(size_t)t * H + i] = v;
        split_store(v * g, hi, lo, (size_t)t * H + i);
    }
    float ss = v * v;
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float c = 0.f;
        for (int w = 0; w < NP_THREADS / 32; w++) c += red[w];
        ssq[t * NORM_BLOCKS_MAX + blockIdx.x] = c;
    }
}

// A_hi/A_lo = split(src) over n rows of K
__global__ void split_rows(const float* src, size_t total, uint16_t* hi, uint16_t* lo) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x)
        split_store(src[i], hi, lo, i);
}

// X += the nparts slices of Y, in order (cpu_inference.rs:171-172)
__global__ void residual_add(float* X, const float* Y, size_t total, int nparts) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        float v = X[i];
        for (int z = 0; z < nparts; z++) v += Y[z * total + i];
        X[i] = v;
    }
}

// h[t][i] = silu(gate) * up from the interleaved gate/up outputs Y[t][2i], Y[t][2i+1] (the sum of
// nparts split-K slices, in order), split for the down GEMM (cpu_inference.rs:166-170, :187)
// (with ssq: the gate|up inputs were left unscaled by norm_part, and row i / I's RMSNorm scale is
// applied here, to the summed gate and up values, before the SiLU)
__global__ void silu_split(const float* Y, size_t n_inter, uint16_t* hi, uint16_t* lo, int nparts, const float* ssq,
                           int nblk, int I, int H, float eps) {
    pdl_wait();
    pdl_trigger();
    const size_t ps = 2 * n_inter;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_inter; i += (size_t)gridDim.x * blockDim.x) {
        float g = Y[2 * i], u = Y[2 * i + 1];
        for (int z = 1; z < nparts; z++) {
            g += Y[z * ps + 2 * i];
            u += Y[z * ps + 2 * i + 1];
        }
        if (ssq) {
            const float sc = row_scale(ssq + (i / I) * NORM_BLOCKS_MAX, nblk, H, eps);
            g *= sc;
            u *= sc;
        }
        split_store(g / (1.0f + __expf(-g)) * u, hi, lo, i);
    }
}

// One head's RMSNorm (gains gv) and rotate-half RoPE (cos/sin cs) across a warp: lane l holds
// dimensions 4 l .. 4 l + 3 (cpu_inference.rs:134-138, :196-215)
__device__ __forceinline__ float4 head_norm_rope(float4 v, const float (&gv)[4], const float2 (&cs)[4], float eps, int lane) {
    float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    const float s = rsqrtf(ss / 128.0f + eps);
    float e[4] = {v.x, v.y, v.z, v.w}, o4[4];
    for (int j = 0; j < 4; j++) e[j] = e[j] * s * gv[j];
    for (int j = 0; j < 4; j++) {
        const float other = __shfl_xor_sync(0xFFFFFFFFu, e[j], 16);  // element d +- 64
        o4[j] = lane < 16 ? e[j] * cs[j].x - other * cs[j].y : e[j] * cs[j].x + other * cs[j].y;
    }
    return make_float4(o4[0], o4[1], o4[2], o4[3]);
}

// the split-K slices of one head's 128 q|k|v outputs for token t, added in slice order (lane: 4 dims)
__device__ __forceinline__ float4 head_sum(const float* Y, int nparts, size_t ps, size_t off, int lane) {
    float4 v = reinterpret_cast<const float4*>(Y + off)[lane];
    for (int z = 1; z < nparts; z++) {
        const float4 w = reinterpret_cast<const float4*>(Y + z * ps + off)[lane];
        v.x += w.x;
        v.y += w.y;
        v.z += w.z;
        v.w += w.w;
    }
    return v;
}

// Per token and head of the q|k|v outputs Y[t][QKVR] (the sum of nparts split-K slices, in order):
// q heads get q_norm + RoPE into Q[t][NQ*128]; k heads k_norm + RoPE and v heads as they are go
// into the cache (cpu_inference.rs:134-141, :196-215; the RoPE table is the decode path's). One
// warp per head. Prefill: token t is at position start + t of cache `c`. Row mode (rows != null):
// token t is row t, at rows[t].pos of its own cache.
__global__ void qkv_post(const float* Y, int nparts, int n, int start, int NQ, int NKV, const uint16_t* qn,
                         const uint16_t* kn, float eps, CacheView c, const RowView* rows, int layer, float* Q) {
    const int warps = blockDim.x >> 5;
    const int item = blockIdx.x * warps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int per_tok = NQ + 2 * NKV;
    const bool live = item < n * per_tok;
    const int t = live ? item / per_tok : 0, hh = live ? item - t * per_tok : 0;
    int pos = start + t, max_seq = c.max_seq;
    float *Kc = c.k, *Vc = c.v;
    const float2* rope = c.rope;
    if (rows) {
        const RowView& rv = rows[t];
        pos = rv.pos;
        max_seq = rv.max_seq;
        Kc = rv.k;
        Vc = rv.v;
        rope = rv.rope;
    }
    // the head-norm gains and the RoPE row do not depend on earlier kernels (a row's position was
    // set by the previous step's argmax, which every later kernel of the chain waited for): fetch
    // them before waiting for the projection's output
    const int d0 = lane * 4;
    float gv[4] = {0.f, 0.f, 0.f, 0.f};
    float2 cs[4] = {};
    if (live && hh < NQ + NKV) {
        const uint16_t* gw = hh < NQ ? qn : kn;
        const float2* rr = rope + (size_t)pos * 64;
        for (int j = 0; j < 4; j++) {
            gv[j] = bf16f(gw[d0 + j]);
            cs[j] = rr[(d0 + j) & 63];
        }
    }
    pdl_wait();
    pdl_trigger();
    if (!live) return;
    const size_t head_stride_l = (size_t)layer * NKV * max_seq * 128;
    const int QKVR = per_tok * 128;
    const size_t ps = (size_t)n * QKVR;
    const float4 v = head_sum(Y, nparts, ps, (size_t)t * QKVR + (size_t)hh * 128, lane);
    if (hh >= NQ + NKV) {  // v head: straight into the cache
        const int g = hh - NQ - NKV;
        reinterpret_cast<float4*>(Vc + head_stride_l + ((size_t)g * max_seq + pos) * 128)[lane] = v;
        return;
    }
    const float4 out = head_norm_rope(v, gv, cs, eps, lane);
    if (hh < NQ) reinterpret_cast<float4*>(Q + (size_t)t * NQ * 128 + (size_t)hh * 128)[lane] = out;
    else reinterpret_cast<float4*>(Kc + head_stride_l + ((size_t)(hh - NQ) * max_seq + pos) * 128)[lane] = out;
}

// Causal GQA attention for the prefill as a small f32 flash attention on the CUDA cores (the
// same math as cpu_inference.rs:143-161, a running softmax over position chunks). CTA = (tile of
// QT query tokens, kv head g): its QT x G query rows meet chunks of PC cached positions staged in
// shared memory; per chunk every thread computes a 4 x 4 block of scores (rows x positions), the
// row groups update their running max / sum, and every thread adds P . V into a 4-row x 8-dim
// block of outputs. Positions after a row's own position are masked (causal).
//
// Causal tiles carry unequal work (the last tile reads every position, the first one chunk), so a
// tile that needs more than CMAX chunks is split over several CTAs by position range; each split
// writes its unnormalised output and running max / sum to a partial slot, and attention_merge
// combines the splits of a tile in split order. Work items are numbered longest tiles first.
constexpr int PC = 64;                 // positions per chunk
constexpr int CMAX = 3;                // most chunks one CTA processes
constexpr int AT_THREADS = 256;
constexpr int KPAD = 132;              // K row pitch in floats (bank spread for the score loads)
constexpr int PPITCH = 132;            // partial row: 128 output dims, running max, running sum, pad

// chunks tile `tile` (QT query tokens) reads: positions 0 .. its last token's position
__host__ __device__ inline int tile_chunks(int tile, int QT, int n, int start) {
    const int last = start + min(QT * (tile + 1), n) - 1;
    return last / PC + 1;
}
__host__ __device__ inline int tile_splits(int tile, int QT, int n, int start) {
    return (tile_chunks(tile, QT, n, start) + CMAX - 1) / CMAX;
}

// work items and partial slots of one KV head: tiles from the last down, each as its splits
struct AttPlan {
    int items = 0, slots = 0;  // CTAs per KV head; partial slots per KV head (split tiles only)
};
inline AttPlan att_plan(int QT, int n, int start) {
    AttPlan pl;
    for (int t = (n + QT - 1) / QT - 1; t >= 0; t--) {
        const int sp = tile_splits(t, QT, n, start);
        pl.items += sp;
        if (sp > 1) pl.slots += sp;
    }
    return pl;
}

// query tokens per CTA: 64 query rows for 1 or 2 query heads per KV head, 48 for 3
template <int G>
struct AttTile {
    static constexpr int QT = G == 1 ? 64 : G == 2 ? 32 : 16;
};

template <int G>
struct AttSmem {
    static constexpr int QT = AttTile<G>::QT;
    float q[QT * G][KPAD];
    float k[PC][KPAD];
    float v[PC][128];
    float p[QT * G][PC + 1];
    float corr[QT * G];
    float linv[QT * G];
};

template <int G>
__global__ void __launch_bounds__(AT_THREADS) attention(const float* Q, float* att, const float* Kc, const float* Vc, int n,
                                                        int start, int NQ, size_t head_stride_l, int max_seq, float scale,
                                                        float* part, int slots) {
    pdl_wait();
    pdl_trigger();
    constexpr int QT = AttTile<G>::QT;
    constexpr int R = QT * G;           // query rows of the tile
    constexpr int RB = R / 4;           // row blocks of 4
    static_assert(R % 4 == 0 && RB * 16 <= AT_THREADS, "row blocks x 16 must fit the CTA");
    extern __shared__ __align__(16) uint8_t att_raw[];
    AttSmem<G>& sm = *reinterpret_cast<AttSmem<G>*>(att_raw);
    const int g = blockIdx.y;
    // work item blockIdx.x -> (tile, split); slot = partial slot of a split tile (-1: write att)
    int tile = (n + QT - 1) / QT - 1, item = blockIdx.x, slot = 0, nsp = 1;
    for (; tile >= 0; tile--) {
        nsp = tile_splits(tile, QT, n, start);
        if (item < nsp) break;
        item -= nsp;
        if (nsp > 1) slot += nsp;
    }
    if (tile < 0) return;  // (the grid holds exactly the plan's items)
    slot = nsp > 1 ? slot + item : -1;
    const int nch = tile_chunks(tile, QT, n, start);
    const int c_begin = nch * item / nsp, c_end = nch * (item + 1) / nsp;
    const int t0 = tile * QT;
    const int tid = threadIdx.x;
    const int ntok = min(QT, n - t0);
    // query rows: row r = token (r / G) of the tile, head g*G + r % G
    for (int i = tid; i < R * 32; i += AT_THREADS) {
        const int r = i >> 5, c = i & 31, tl = r / G, h = r % G;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tl < ntok) v = reinterpret_cast<const float4*>(Q + (size_t)(t0 + tl) * NQ * 128 + (size_t)(g * G + h) * 128)[c];
        reinterpret_cast<float4*>(sm.q[r])[c] = v;
    }
    // score block: rows 4*rb.., positions pb + 16 j; output block: rows 4*rb.., dims 8*db..
    const int rb = tid >> 4, pb = tid & 15;
    const bool active = rb < RB;
    float m_run[4], l_run[4];
    float o[4][8];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m_run[i] = -INFINITY;
        l_run[i] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++) o[i][j] = 0.f;
    }
    const float* kb = Kc + head_stride_l + (size_t)g * max_seq * 128;
    const float* vb = Vc + head_stride_l + (size_t)g * max_seq * 128;
    const int last = min(start + t0 + ntok - 1, c_end * PC - 1);  // this item's last position
    for (int p0 = c_begin * PC; p0 <= last; p0 += PC) {
        const int np = min(PC, last + 1 - p0);
        __syncthreads();
        for (int i = tid; i < PC * 32; i += AT_THREADS) {
            const int r = i >> 5, c = i & 31;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (r < np) {
                kv = reinterpret_cast<const float4*>(kb + (size_t)(p0 + r) * 128)[c];
                vv = reinterpret_cast<const float4*>(vb + (size_t)(p0 + r) * 128)[c];
            }
            reinterpret_cast<float4*>(sm.k[r])[c] = kv;
            reinterpret_cast<float4*>(sm.v[r])[c] = vv;
        }
        __syncthreads();
        if (active) {
            // S = q . k for rows 4rb..4rb+3 and positions pb, pb+16, pb+32, pb+48
            float s[4][4];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) s[i][j] = 0.f;
#pragma unroll 4
            for (int d = 0; d < 128; d += 4) {
                float4 qv[4], kv[4];
#pragma unroll
                for (int i = 0; i < 4; i++) qv[i] = *reinterpret_cast<const float4*>(&sm.q[4 * rb + i][d]);
#pragma unroll
                for (int j = 0; j < 4; j++) kv[j] = *reinterpret_cast<const float4*>(&sm.k[pb + 16 * j][d]);
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        s[i][j] = fmaf(qv[i].x, kv[j].x, fmaf(qv[i].y, kv[j].y, fmaf(qv[i].z, kv[j].z, fmaf(qv[i].w, kv[j].w, s[i][j]))));
            }
            // running softmax per row over this chunk (the 16 threads of a row block share its rows)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int r = 4 * rb + i;
                const int pos = start + t0 + r / G;
                float mx = -INFINITY;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int pp = pb + 16 * j;
                    s[i][j] = (pp < np && p0 + pp <= pos) ? s[i][j] * scale : -INFINITY;
                    mx = fmaxf(mx, s[i][j]);
                }
#pragma unroll
                for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
                const float mn = fmaxf(m_run[i], mx);
                float sum = 0.f;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float e = mn == -INFINITY ? 0.f : __expf(s[i][j] - mn);
                    sm.p[r][pb + 16 * j] = e;
                    sum += e;
                }
#pragma unroll
                for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, off);
                const float corr = m_run[i] == -INFINITY ? 0.f : __expf(m_run[i] - mn);
                l_run[i] = l_run[i] * corr + sum;
                m_run[i] = mn;
                if (pb == 0) sm.corr[r] = corr;
            }
        }
        __syncthreads();
        if (active) {
            // O = O * corr + P . V for rows 4rb.. and dims 8pb..8pb+7
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float c = sm.corr[4 * rb + i];
#pragma unroll
                for (int j = 0; j < 8; j++) o[i][j] *= c;
            }
            for (int pp = 0; pp < np; pp++) {
                const float4 va = *reinterpret_cast<const float4*>(&sm.v[pp][8 * pb]);
                const float4 vb4 = *reinterpret_cast<const float4*>(&sm.v[pp][8 * pb + 4]);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float pw = sm.p[4 * rb + i][pp];
                    o[i][0] = fmaf(pw, va.x, o[i][0]);
                    o[i][1] = fmaf(pw, va.y, o[i][1]);
                    o[i][2] = fmaf(pw, va.z, o[i][2]);
                    o[i][3] = fmaf(pw, va.w, o[i][3]);
                    o[i][4] = fmaf(pw, vb4.x, o[i][4]);
                    o[i][5] = fmaf(pw, vb4.y, o[i][5]);
                    o[i][6] = fmaf(pw, vb4.z, o[i][6]);
                    o[i][7] = fmaf(pw, vb4.w, o[i][7]);
                }
            }
        }
    }
    if (!active) return;
    if (slot >= 0) {
        // partial: unnormalised output rows plus (running max, sum) for attention_merge
        float* po = part + ((size_t)g * slots + slot) * R * PPITCH;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float* dst = po + (size_t)(4 * rb + i) * PPITCH;
            reinterpret_cast<float4*>(dst + 8 * pb)[0] = make_float4(o[i][0], o[i][1], o[i][2], o[i][3]);
            reinterpret_cast<float4*>(dst + 8 * pb)[1] = make_float4(o[i][4], o[i][5], o[i][6], o[i][7]);
            if (pb == 0) {
                dst[128] = m_run[i];
                dst[129] = l_run[i];
            }
        }
        return;
    }
    // the row sums live with the score threads of the same row block (identical in all 16)
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = 4 * rb + i, tl = r / G, h = r % G;
        if (tl >= ntok) continue;
        const float inv = 1.0f / l_run[i];
        float* dst = att + (size_t)(t0 + tl) * NQ * 128 + (size_t)(g * G + h) * 128 + 8 * pb;
        reinterpret_cast<float4*>(dst)[0] = make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
        reinterpret_cast<float4*>(dst)[1] = make_float4(o[i][4] * inv, o[i][5] * inv, o[i][6] * inv, o[i][7] * inv);
    }
}

// Combines the splits of each split tile: per row, M = max of the splits' running maxima, then
// out = sum_j o_j e^(m_j - M) / sum_j l_j e^(m_j - M), splits in order. Grid (split tiles, KV heads,
// row groups of 4); warp w takes row 4 * blockIdx.z + w, lane the dims 4 lane .. 4 lane + 3.
template <int G, int QT>
__global__ void __launch_bounds__(128) attention_merge(float* att, const float* part, int n, int start, int NQ, int slots) {
    pdl_wait();
    pdl_trigger();
    constexpr int R = QT * G;
    const int g = blockIdx.y, lane = threadIdx.x & 31, r = blockIdx.z * 4 + (threadIdx.x >> 5);
    int tile = (n + QT - 1) / QT - 1, slot = 0, k = blockIdx.x, nsp = 1;
    for (; tile >= 0; tile--) {
        nsp = tile_splits(tile, QT, n, start);
        if (nsp > 1) {
            if (k == 0) break;
            k--;
            slot += nsp;
        }
    }
    if (tile < 0) return;
    const int t0 = tile * QT, ntok = min(QT, n - t0);
    const int tl = r / G, h = r % G;
    if (tl >= ntok) return;
    const float* po = part + ((size_t)g * slots + slot) * R * PPITCH;
    float M = -INFINITY;
    for (int j = 0; j < nsp; j++) M = fmaxf(M, po[((size_t)j * R + r) * PPITCH + 128]);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float l = 0.f;
    for (int j = 0; j < nsp; j++) {
        const float* pr = po + ((size_t)j * R + r) * PPITCH;
        const float mj = pr[128];
        const float w = mj == -INFINITY ? 0.f : __expf(mj - M);
        const float4 v = reinterpret_cast<const float4*>(pr)[lane];
        acc.x = fmaf(v.x, w, acc.x);
        acc.y = fmaf(v.y, w, acc.y);
        acc.z = fmaf(v.z, w, acc.z);
        acc.w = fmaf(v.w, w, acc.w);
        l = fmaf(pr[129], w, l);
    }
    const float inv = 1.0f / l;
    reinterpret_cast<float4*>(att + (size_t)(t0 + tl) * NQ * 128 + (size_t)(g * G + h) * 128)[lane] =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
}

template <int G>
int launch_attention(const float* Q, float* att, const float* Kc, const float* Vc, int n, int start, int NQ, int NKV,
                     size_t hsl, int max_seq, float scale, float* part, size_t part_cap, cudaStream_t s) {
    const int smem = (int)sizeof(AttSmem<G>);
    if (cudaFuncSetAttribute(attention<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return QW_ERR_CUDA;
    const AttPlan pl = att_plan(AttTile<G>::QT, n, start);
    if ((size_t)NKV * pl.slots * AttTile<G>::QT * G * PPITCH > part_cap) return QW_ERR_ARG;
    launch(attention<G>, dim3(pl.items, NKV), dim3(AT_THREADS), smem, s, Q, att, Kc, Vc, n, start, NQ, hsl, max_seq, scale,
           part, pl.slots);
    int split_tiles = 0;
    for (int t = (n + AttTile<G>::QT - 1) / AttTile<G>::QT - 1; t >= 0; t--)
        split_tiles += tile_splits(t, AttTile<G>::QT, n, start) > 1;
    if (split_tiles)
        launch(attention_merge<G, AttTile<G>::QT>, dim3(split_tiles, NKV, AttTile<G>::QT * G / 4), dim3(128), 0, s, att, part,
               n, start, NQ, pl.slots);
    return QW_OK;
}

// ---------------------------------------------------------------------------------------------
// Causal GQA attention for the prefill on the tensor cores (tcgen05), for G = 1, 2 or 4 query heads
// per KV head. A CTA takes 128 query rows (128 / G tokens x G heads of one KV head) and walks the
// same 64-position chunks and position-range splits as the CUDA-core kernel above:
//   S = Q . K^T   (M = 128 rows, N = 64 positions, K = 128 dims) into TMEM columns 0..63
//   online softmax: thread = row reads its 64 scores from TMEM, masks positions after its own,
//                   updates its running max / sum, writes P to shared memory and rescales its
//                   row of O in TMEM (tcgen05.ld / tcgen05.st)
//   O += P . V    (M = 128, N = 128 dims, K = 64 positions) into TMEM columns 64..191
// Q, K, V (f32 in memory) and P are split into bf16 hi/lo halves as they are written to shared
// memory in the 128-byte-swizzle K-major layout (V transposed: dims x positions); each product is
// hi.hi + hi.lo + lo.hi, so scores and outputs keep about 16 bits of every f32 operand. One
// thread issues the MMAs and commits them to an mbarrier per product; every wait is bounded.
constexpr int TA_THREADS = 256;  // 8 warps: warps w and w + 4 share TMEM lanes 32 (w % 4) .., split by columns
constexpr uint32_t TA_TMEM_COLS = 256, TA_S_COL = 0, TA_O_COL = 64;
constexpr int TA_Q = 0, TA_QLO = 32768;                  // Q: 2 K blocks x [128 rows x 128 B] per half
constexpr int TA_K = 65536, TA_KLO = TA_K + 16384;        // K chunk: 2 K blocks x [64 rows x 128 B] per half
constexpr int TA_V = TA_K + 32768, TA_VLO = TA_V + 16384; // V^T chunk: [128 dims x 64 positions] per half
constexpr int TA_P = TA_V + 32768, TA_PLO = TA_P + 16384; // P: [128 rows x 64 positions] per half
constexpr int TA_SMEM = TA_P + 32768 + 1024;

__device__ __forceinline__ uint32_t ta_sw128(int r, int c) {  // (row, column) of a [rows][64] bf16 swizzled tile
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((((c >> 3) ^ r) & 7) << 4) + (c & 7) * 2);
}
__device__ __forceinline__ void ta_split(uint8_t* hi, uint8_t* lo, uint32_t off, float v) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    *reinterpret_cast<__nv_bfloat16*>(hi + off) = h;
    *reinterpret_cast<__nv_bfloat16*>(lo + off) = __float2bfloat16_rn(v - __bfloat162float(h));
}
// 4 consecutive columns (8 bytes per half) of a swizzled tile row, c0 a multiple of 4
__device__ __forceinline__ void ta_split4(uint8_t* hi, uint8_t* lo, uint32_t off, float4 v) {
    const __nv_bfloat162 h01 = __floats2bfloat162_rn(v.x, v.y), h23 = __floats2bfloat162_rn(v.z, v.w);
    const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
    const __nv_bfloat162 l01 = __floats2bfloat162_rn(v.x - f01.x, v.y - f01.y), l23 = __floats2bfloat162_rn(v.z - f23.x, v.w - f23.y);
    *reinterpret_cast<uint2*>(hi + off) = make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
    *reinterpret_cast<uint2*>(lo + off) = make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
}
// 8 consecutive columns (one 16-byte swizzle chunk per half) of a swizzled tile row
__device__ __forceinline__ void ta_split8(uint8_t* hi, uint8_t* lo, uint32_t off, const float* v) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const __nv_bfloat162 hh = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        const float2 f = __bfloat1622float2(hh);
        const __nv_bfloat162 ll = __floats2bfloat162_rn(v[2 * j] - f.x, v[2 * j + 1] - f.y);
        h[j] = *reinterpret_cast<const uint32_t*>(&hh);
        l[j] = *reinterpret_cast<const uint32_t*>(&ll);
    }
    *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
          "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
          "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
          "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int G>
__global__ void __launch_bounds__(TA_THREADS, 1)
attention_tc(const float* Q, float* att, const float* Kc, const float* Vc, int n, int start, int NQ, size_t head_stride_l,
             int max_seq, float scale, float* part, int slots, int* err) {
    constexpr int QT = 128 / G;
    extern __shared__ __align__(1024) uint8_t ta_raw[];
    __shared__ uint64_t bar_s, bar_o;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    __shared__ float xmax[2][128], xsum[2][128];  // per row: the two score-column halves' max and sum
    pdl_wait();
    pdl_trigger();
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ta_raw) + 1023) & ~uintptr_t(1023));
    const int g = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // work item -> (tile, split), as attention<G>
    int tile = (n + QT - 1) / QT - 1, item = blockIdx.x, slot = 0, nsp = 1;
    for (; tile >= 0; tile--) {
        nsp = tile_splits(tile, QT, n, start);
        if (item < nsp) break;
        item -= nsp;
        if (nsp > 1) slot += nsp;
    }
    if (tile < 0) return;  // (the grid holds exactly the plan's items)
    slot = nsp > 1 ? slot + item : -1;
    const int nch = tile_chunks(tile, QT, n, start);
    const int c_begin = nch * item / nsp, c_end = nch * (item + 1) / nsp;
    const int t0 = tile * QT, ntok = min(QT, n - t0);
    const int last = min(start + t0 + ntok - 1, c_end * PC - 1);

    const float* kb = Kc + head_stride_l + (size_t)g * max_seq * 128;
    const float* vb = Vc + head_stride_l + (size_t)g * max_seq * 128;
    // K and V rows of a chunk, 8 rows x 64 contiguous bytes per warp load. K: warp w takes position
    // 8 w + (lane & 7), lane group lane >> 3 dims 4 (lane >> 3) + 16 u, u < 8. V: thread t takes
    // positions 8 (t & 7) .. + 7 of dims 4 (t >> 3) .. + 3, so that each dim's 8 positions leave as
    // one 16-byte chunk of the transposed tile. The next chunk's rows are loaded into registers
    // while this chunk's S MMA and softmax run, so their global-load latency is off the chunk's
    // critical path. The first chunk's loads go out before the Q tile's.
    const int kv_p = 8 * warp + (lane & 7), dg = lane >> 3;
    const int v_p = 8 * (tid & 7), v_d = 4 * (tid >> 3);
    float4 kv[8], vv[8];
    auto load_kv = [&](int p0n) {
        const int npn = min(PC, last + 1 - p0n);
#pragma unroll
        for (int u = 0; u < 8; u++) {
            kv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            vv[u] = kv[u];
            if (kv_p < npn) kv[u] = __ldcg(reinterpret_cast<const float4*>(kb + (size_t)(p0n + kv_p) * 128) + dg + 4 * u);
            if (v_p + u < npn) vv[u] = __ldcg(reinterpret_cast<const float4*>(vb + (size_t)(p0n + v_p + u) * 128 + v_d));
        }
    };
    if (c_begin * PC <= last) load_kv(c_begin * PC);

    if (tid == 0) {
        mbar_init(&bar_s, 1);
        mbar_init(&bar_o, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&tmem_base)), "r"(TA_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // Q tile: row r = token t0 + r / G, head g * G + r % G; 8 rows' loads in flight per batch
    // (the shared-memory stores in between would otherwise serialise every global load)
#pragma unroll 1
    for (int i0 = tid; i0 < 128 * 32; i0 += 8 * TA_THREADS) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = i0 + u * TA_THREADS, r = i >> 5;
            v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r / G < ntok)
                v[u] = __ldg(reinterpret_cast<const float4*>(Q + (size_t)(t0 + r / G) * NQ * 128 + (size_t)(g * G + r % G) * 128) +
                             (i & 31));
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = i0 + u * TA_THREADS, r = i >> 5, d0 = (i & 31) * 4;
            ta_split4(sm + TA_Q + (d0 >> 6) * 16384, sm + TA_QLO + (d0 >> 6) * 16384, ta_sw128(r, d0 & 63), v[u]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base, tS = tmem + TA_S_COL, tO = tmem + TA_O_COL;
    // warp w reads TMEM lanes 32 (w % 4) .. (its query rows) and column half w / 4 of S and O
    const int row = 32 * (warp & 3) + lane, half = warp >> 2;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const uint32_t idesc_s = tc::idesc_bf16_f32(128, 64), idesc_o = tc::idesc_bf16_f32(128, 128);
    const int pos_r = start + t0 + row / G;
    float m_run = -INFINITY, l_run = 0.f;
    int chunk = 0;
    bool ok = true;
    for (int p0 = c_begin * PC; p0 <= last; p0 += PC, chunk++) {
        const int np = min(PC, last + 1 - p0);
        // the previous chunk's P.V must be done before K, V and P are rewritten and O is rescaled
        if (chunk > 0 && tid == 0) ok = tc::bounded_wait(&bar_o, (chunk - 1) & 1, &abort_flag);
        if (!__syncthreads_and(ok && !abort_flag)) {
            ok = false;
            break;
        }
        {
            // K goes out as 8-byte row pieces; V^T (dims x positions) as one 16-byte chunk per dim
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int d0 = 4 * (dg + 4 * u);
                ta_split4(sm + TA_K + (d0 >> 6) * 8192, sm + TA_KLO + (d0 >> 6) * 8192, ta_sw128(kv_p, d0 & 63), kv[u]);
            }
            {
                float e[8];
#pragma unroll
                for (int u = 0; u < 8; u++) e[u] = vv[u].x;
                ta_split8(sm + TA_V, sm + TA_VLO, ta_sw128(v_d, v_p), e);
#pragma unroll
                for (int u = 0; u < 8; u++) e[u] = vv[u].y;
                ta_split8(sm + TA_V, sm + TA_VLO, ta_sw128(v_d + 1, v_p), e);
#pragma unroll
                for (int u = 0; u < 8; u++) e[u] = vv[u].z;
                ta_split8(sm + TA_V, sm + TA_VLO, ta_sw128(v_d + 2, v_p), e);
#pragma unroll
                for (int u = 0; u < 8; u++) e[u] = vv[u].w;
                ta_split8(sm + TA_V, sm + TA_VLO, ta_sw128(v_d + 3, v_p), e);
            }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 8; kk++) {
                const int blk = kk >> 2, w = kk & 3;
                const uint64_t qh = tc::smem_desc_k128(smem_u32(sm + TA_Q + blk * 16384)) + 2 * w;
                const uint64_t ql = tc::smem_desc_k128(smem_u32(sm + TA_QLO + blk * 16384)) + 2 * w;
                const uint64_t kh = tc::smem_desc_k128(smem_u32(sm + TA_K + blk * 8192)) + 2 * w;
                const uint64_t kl = tc::smem_desc_k128(smem_u32(sm + TA_KLO + blk * 8192)) + 2 * w;
                tc::mma_bf16(tS, qh, kh, idesc_s, kk > 0);
                tc::mma_bf16(tS, qh, kl, idesc_s, 1u);
                tc::mma_bf16(tS, ql, kh, idesc_s, 1u);
            }
            tc::mma_commit(&bar_s);
        }
        if (p0 + PC <= last) load_kv(p0 + PC);
        if (tid == 0) ok = tc::bounded_wait(&bar_s, chunk & 1, &abort_flag);
        if (!__syncthreads_and(ok && !abort_flag)) {
            ok = false;
            break;
        }
        tc_fence_after();
        // softmax for row `row` over this chunk; this warp holds score columns 32 half .. + 31
        uint32_t sr[32];
        tc::tmem_ld32(tS + lane_base + 32 * half, sr);
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const int c = 32 * half + j;
            const bool live = c < np && p0 + c <= pos_r;
            const float v = live ? __uint_as_float(sr[j]) * scale : -INFINITY;
            sr[j] = __float_as_uint(v);
            mx = fmaxf(mx, v);
        }
        xmax[half][row] = mx;
        __syncthreads();
        const float mn = fmaxf(m_run, fmaxf(xmax[0][row], xmax[1][row]));
        const float corr = m_run == -INFINITY ? 0.f : __expf(m_run - mn);
        float sum = 0.f;
#pragma unroll
        for (int c8 = 0; c8 < 32; c8 += 8) {  // one 16-byte swizzle chunk of P per half
            float e[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float v = __uint_as_float(sr[c8 + j]);
                e[j] = v == -INFINITY ? 0.f : __expf(v - mn);
                sum += e[j];
            }
            ta_split8(sm + TA_P, sm + TA_PLO, ta_sw128(row, 32 * half + c8), e);
        }
        xsum[half][row] = sum;
        if (chunk > 0) {  // this warp's half of the O row *= corr
#pragma unroll 1
            for (int cb = 64 * half; cb < 64 * half + 64; cb += 32) {
                uint32_t o[32];
                tc::tmem_ld32(tO + lane_base + cb, o);
#pragma unroll
                for (int j = 0; j < 32; j++) o[j] = __float_as_uint(__uint_as_float(o[j]) * corr);
                tmem_st32(tO + lane_base + cb, o);
            }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        l_run = l_run * corr + (xsum[0][row] + xsum[1][row]);
        m_run = mn;
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                const uint64_t ph = tc::smem_desc_k128(smem_u32(sm + TA_P)) + 2 * kk;
                const uint64_t pl = tc::smem_desc_k128(smem_u32(sm + TA_PLO)) + 2 * kk;
                const uint64_t vh = tc::smem_desc_k128(smem_u32(sm + TA_V)) + 2 * kk;
                const uint64_t vl = tc::smem_desc_k128(smem_u32(sm + TA_VLO)) + 2 * kk;
                tc::mma_bf16(tO, ph, vh, idesc_o, (chunk > 0 || kk > 0) ? 1u : 0u);
                tc::mma_bf16(tO, ph, vl, idesc_o, 1u);
                tc::mma_bf16(tO, pl, vh, idesc_o, 1u);
            }
            tc::mma_commit(&bar_o);
        }
    }
    // the last chunk's P.V, then this warp's half of the O row -> output
    if (ok && chunk > 0 && tid == 0) ok = tc::bounded_wait(&bar_o, (chunk - 1) & 1, &abort_flag);
    ok = __syncthreads_and(ok && !abort_flag);
    tc_fence_after();
    if (ok && chunk > 0) {
        const int tl = row / G, h = row % G;
        if (slot >= 0) {
            float* dst = part + (((size_t)g * slots + slot) * 128 + row) * PPITCH;
#pragma unroll 1
            for (int cb = 64 * half; cb < 64 * half + 64; cb += 32) {
                uint32_t o[32];
                tc::tmem_ld32(tO + lane_base + cb, o);
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(dst + cb + j) = make_float4(__uint_as_float(o[j]), __uint_as_float(o[j + 1]),
                                                                        __uint_as_float(o[j + 2]), __uint_as_float(o[j + 3]));
            }
            if (half == 0) {
                dst[128] = m_run;
                dst[129] = l_run;
            }
        } else {
            const float inv = 1.0f / l_run;
            float* dst = att + (size_t)(t0 + tl) * NQ * 128 + (size_t)(g * G + h) * 128;
#pragma unroll 1
            for (int cb = 64 * half; cb < 64 * half + 64; cb += 32) {
                uint32_t o[32];
                tc::tmem_ld32(tO + lane_base + cb, o);
                if (tl < ntok)
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(dst + cb + j) =
                            make_float4(__uint_as_float(o[j]) * inv, __uint_as_float(o[j + 1]) * inv,
                                        __uint_as_float(o[j + 2]) * inv, __uint_as_float(o[j + 3]) * inv);
            }
        }
    }
    if (!ok && tid == 0) {
        atomicExch(err, 1);
        // MMAs issued before the abort must finish before their TMEM is freed (bounded waits)
        const uint64_t w0 = globaltimer_ns();
        while (!mbar_try_wait(&bar_s, chunk & 1) && globaltimer_ns() - w0 < (uint64_t)tc::WAIT_LIMIT_NS) {
        }
        const uint64_t w1 = globaltimer_ns();
        while (chunk > 0 && !mbar_try_wait(&bar_o, (chunk - 1) & 1) && globaltimer_ns() - w1 < (uint64_t)tc::WAIT_LIMIT_NS) {
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TA_TMEM_COLS) : "memory");
    }
}

template <int G>
int launch_attention_tc(const float* Q, float* att, const float* Kc, const float* Vc, int n, int start, int NQ, int NKV,
                        size_t hsl, int max_seq, float scale, float* part, size_t part_cap, int* err, cudaStream_t s) {
    constexpr int QT = 128 / G;
    if (cudaFuncSetAttribute(attention_tc<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, TA_SMEM) != cudaSuccess)
        return QW_ERR_CUDA;
    const AttPlan pl = att_plan(QT, n, start);
    if ((size_t)NKV * pl.slots * 128 * PPITCH > part_cap) return QW_ERR_ARG;
    launch(attention_tc<G>, dim3(pl.items, NKV), dim3(TA_THREADS), TA_SMEM, s, Q, att, Kc, Vc, n, start, NQ, hsl, max_seq,
           scale, part, pl.slots, err);
    int split_tiles = 0;
    for (int t = (n + QT - 1) / QT - 1; t >= 0; t--) split_tiles += tile_splits(t, QT, n, start) > 1;
    if (split_tiles)
        launch(attention_merge<G, QT>, dim3(split_tiles, NKV, 128 / 4), dim3(128), 0, s, att, part, n, start, NQ, pl.slots);
    return QW_OK;
}


// floats of attention partials a pass over n tokens from `start` needs (G = query heads per KV head)
size_t attention_partial_floats(int n, int start, int NQ, int NKV) {
    const int G = NQ / NKV;
    const int QT = (G == 1 || G == 2 || G == 4) ? 128 / G : AttTile<3>::QT;  // tensor-core tiles, else CUDA-core
    return (size_t)NKV * att_plan(QT, n, start).slots * QT * G * PPITCH;
}

int grid_for(size_t total) { return (int)std::min<size_t>((total + 255) / 256, 148 * 8); }

// ---------------------------------------------------------------------------------------------
// Row mode (a decode batch): row b is one sequence's single token at its own position in its own
// cache. Attention is per (row, KV head, split of ROW_SPLIT positions) — flash-decoding — and the
// last split CTA of each (row, KV head) combines the splits into the o_proj input halves.

constexpr int RA_WARPS = 16;           // warp w takes positions p0 + w + 16 j, j < ROW_SPLIT / 16
constexpr int RA_THREADS = RA_WARPS * 32;
constexpr int RA_PER_WARP = ROW_SPLIT / RA_WARPS;

// One (row b, KV head g, split z): the G query heads of g against positions
// [z * ROW_SPLIT, min((z + 1) * ROW_SPLIT, pos + 1)) of the row's cache; writes (unnormalised
// output, running max, running sum) per head to part[((b * NQ + head) * splits + z) * PPITCH].
// The last of the row's live splits to finish (a ticket per (row, KV head), reset by that CTA)
// combines them in split order and writes the o_proj GEMM's input halves for the G heads. Same
// math as cpu_inference.rs:143-161 (scores scaled by 1/sqrt(128), softmax, sum of p . v), with the
// softmax done online.
//
// FUSED (rows in distinct caches, so no row reads another row's K/V of this step): the CTA also
// does qkv_post's work for itself. Warps 0 .. G-1 sum the split-K slices of Y for the G query heads
// and apply q_norm + RoPE into shared memory (every split of the row recomputes them); in the
// split holding the row's position, warps G and G+1 form that position's k (k_norm + RoPE) and v
// and write them into the cache before the CTA's K/V loads. Same helpers as the qkv_post pass.
// With ssq, the q|k|v outputs come from unscaled norm_part inputs and the row's RMSNorm scale is
// applied to the summed head values first.
template <int G, bool FUSED>
__global__ void __launch_bounds__(RA_THREADS) row_attention(const float* Q, const RowView* rows, int NQ, int NKV, int layer,
                                                            float scale, float* part, int splits, unsigned* tickets,
                                                            uint16_t* ahi, uint16_t* alo, const float* Y, int nparts,
                                                            const uint16_t* qn, const uint16_t* kn, float eps,
                                                            const float* ssq, int nblk, int H) {
    static_assert(!FUSED || G + 2 <= RA_WARPS, "fused q|k|v epilogue needs G + 2 warps");
    __shared__ float sm_o[RA_WARPS][G][128];
    __shared__ float sm_m[RA_WARPS][G], sm_l[RA_WARPS][G];
    __shared__ __align__(16) float sm_q[FUSED ? G : 1][128];
    const int b = blockIdx.x, g = blockIdx.y, z = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the row views were last written by the previous step's argmax, which every kernel since
    // waited for, so they (and this split's K/V range) are known before waiting for qkv_post
    const RowView rv = rows[b];
    const int p_begin = z * ROW_SPLIT;
    if (p_begin > rv.pos) return;  // past this row's positions (the merge reads only live splits)
    const int p_end = min(p_begin + ROW_SPLIT, rv.pos + 1);
    const size_t head_off = ((size_t)layer * NKV + g) * rv.max_seq * 128;
    float* kb = rv.k + head_off;
    float* vb = rv.v + head_off;
    // warm L2 with the split's K/V rows while the previous kernel finishes; the loads themselves
    // come after the wait (qkv_post writes this step's rows, and in a multi-position pass other
    // rows' positions too)
    if (threadIdx.x == 0) {
        bulk_prefetch_l2(kb + (size_t)p_begin * 128, (uint32_t)(p_end - p_begin) * 512u);
        bulk_prefetch_l2(vb + (size_t)p_begin * 128, (uint32_t)(p_end - p_begin) * 512u);
    }
    // fused: this warp's head (q heads g G .. g G + G - 1, then k and v of head g in the split that
    // holds the row's position), its gains and RoPE row, fetched before the wait
    const bool cur = p_end == rv.pos + 1;
    const int hw = FUSED ? (warp < G ? g * G + warp : warp == G && cur ? NQ + g : warp == G + 1 && cur ? NQ + NKV + g : -1) : -1;
    float gv[4] = {0.f, 0.f, 0.f, 0.f};
    float2 cs[4] = {};
    if (FUSED && hw >= 0 && hw < NQ + NKV) {
        const uint16_t* gw = hw < NQ ? qn : kn;
        const float2* rr = rv.rope + (size_t)rv.pos * 64;
        for (int j = 0; j < 4; j++) {
            gv[j] = bf16f(gw[lane * 4 + j]);
            cs[j] = rr[(lane * 4 + j) & 63];
        }
    }
    pdl_wait();
    pdl_trigger();
    if constexpr (FUSED) {
        if (hw >= 0) {
            const int QKVR = (NQ + 2 * NKV) * 128;
            float4 v = head_sum(Y, nparts, (size_t)gridDim.x * QKVR, (size_t)b * QKVR + (size_t)hw * 128, lane);
            if (ssq) {  // the input RMSNorm's scale, left out by norm_part
                const float sc = row_scale(ssq + b * NORM_BLOCKS_MAX, nblk, H, eps);
                v = make_float4(v.x * sc, v.y * sc, v.z * sc, v.w * sc);
            }
            if (hw >= NQ + NKV) {
                reinterpret_cast<float4*>(vb + (size_t)rv.pos * 128)[lane] = v;
            } else {
                const float4 e = head_norm_rope(v, gv, cs, eps, lane);
                if (hw < NQ) reinterpret_cast<float4*>(sm_q[warp])[lane] = e;
                else reinterpret_cast<float4*>(kb + (size_t)rv.pos * 128)[lane] = e;
            }
        }
        __syncthreads();  // q in shared memory; this position's k and v in the cache (CTA-visible)
    }
    float4 q[G], o[G];
    float m[G], l[G];
#pragma unroll
    for (int h = 0; h < G; h++) {
        if constexpr (FUSED) q[h] = reinterpret_cast<const float4*>(sm_q[h])[lane];
        else q[h] = reinterpret_cast<const float4*>(Q + (size_t)b * NQ * 128 + (size_t)(g * G + h) * 128)[lane];
        o[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        m[h] = -INFINITY;
        l[h] = 0.f;
    }
    // all of this warp's K and V rows in flight at once, then the online softmax over them
    float4 kr[RA_PER_WARP], vr[RA_PER_WARP];
#pragma unroll
    for (int j = 0; j < RA_PER_WARP; j++) {
        const int p = p_begin + warp + RA_WARPS * j;
        if (p < p_end) {
            kr[j] = reinterpret_cast<const float4*>(kb + (size_t)p * 128)[lane];
            vr[j] = reinterpret_cast<const float4*>(vb + (size_t)p * 128)[lane];
        }
    }
#pragma unroll
    for (int j = 0; j < RA_PER_WARP; j++) {
        if (p_begin + warp + RA_WARPS * j >= p_end) break;
        const float4 k4 = kr[j], v4 = vr[j];
#pragma unroll
        for (int h = 0; h < G; h++) {
            float d = q[h].x * k4.x + q[h].y * k4.y + q[h].z * k4.z + q[h].w * k4.w;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xFFFFFFFFu, d, off);
            const float sc = d * scale;
            const float mn = fmaxf(m[h], sc);
            const float corr = m[h] == -INFINITY ? 0.f : __expf(m[h] - mn);
            const float e = __expf(sc - mn);
            l[h] = l[h] * corr + e;
            o[h].x = fmaf(e, v4.x, o[h].x * corr);
            o[h].y = fmaf(e, v4.y, o[h].y * corr);
            o[h].z = fmaf(e, v4.z, o[h].z * corr);
            o[h].w = fmaf(e, v4.w, o[h].w * corr);
            m[h] = mn;
        }
    }
#pragma unroll
    for (int h = 0; h < G; h++) {
        reinterpret_cast<float4*>(sm_o[warp][h])[lane] = o[h];
        if (lane == 0) {
            sm_m[warp][h] = m[h];
            sm_l[warp][h] = l[h];
        }
    }
    __syncthreads();
    // combine the warps in warp order, one head per warp (dims 4 lane .. 4 lane + 3)
    for (int h = warp; h < G; h += RA_WARPS) {
        float M = -INFINITY;
        for (int w = 0; w < RA_WARPS; w++) M = fmaxf(M, sm_m[w][h]);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        float L = 0.f;
        for (int w = 0; w < RA_WARPS; w++) {
            const float mw = sm_m[w][h];
            const float f = mw == -INFINITY ? 0.f : __expf(mw - M);
            const float4 ow = reinterpret_cast<const float4*>(sm_o[w][h])[lane];
            acc.x = fmaf(ow.x, f, acc.x);
            acc.y = fmaf(ow.y, f, acc.y);
            acc.z = fmaf(ow.z, f, acc.z);
            acc.w = fmaf(ow.w, f, acc.w);
            L = fmaf(sm_l[w][h], f, L);
        }
        float* dst = part + (((size_t)b * NQ + g * G + h) * splits + z) * PPITCH;
        reinterpret_cast<float4*>(dst)[lane] = acc;
        if (lane == 0) {
            dst[128] = M;
            dst[129] = L;
        }
    }
    __shared__ int is_last;
    const int live = rv.pos / ROW_SPLIT + 1;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(&tickets[b * NKV + g], 1u) == (unsigned)(live - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int h = warp; h < G; h += RA_WARPS) {
        const float* base = part + ((size_t)b * NQ + g * G + h) * splits * PPITCH;
        float M = -INFINITY;
        for (int j = 0; j < live; j++) M = fmaxf(M, __ldcg(base + (size_t)j * PPITCH + 128));
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        float L = 0.f;
        for (int j = 0; j < live; j++) {
            const float* pj = base + (size_t)j * PPITCH;
            const float mj = __ldcg(pj + 128);
            const float f = mj == -INFINITY ? 0.f : __expf(mj - M);
            const float4 v = __ldcg(reinterpret_cast<const float4*>(pj) + lane);
            acc.x = fmaf(v.x, f, acc.x);
            acc.y = fmaf(v.y, f, acc.y);
            acc.z = fmaf(v.z, f, acc.z);
            acc.w = fmaf(v.w, f, acc.w);
            L = fmaf(__ldcg(pj + 129), f, L);
        }
        const float inv = 1.0f / L;
        store_split4(ahi, alo, (size_t)b * NQ * 128 + (size_t)(g * G + h) * 128 + 4 * lane,
                     make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
    }
    if (threadIdx.x == 0) tickets[b * NKV + g] = 0u;  // ready for the next layer
}

// argmax order: larger value wins, ties to the lower index, NaN never wins (the reference CPU rule,
// common/mod.rs:17-22)
constexpr unsigned AM_NONE = 0xFFFFFFFFu;
__device__ __forceinline__ bool am_wins(float av, unsigned ai, float bv, unsigned bi) {
    if (ai == AM_NONE) return false;
    if (bi == AM_NONE) return true;
    return av > bv || (av == bv && ai < bi);
}

constexpr int AR_THREADS = 256;

// Argmax of `rows` rows of V logits, AR_PARTS blocks per row (grid (rows, AR_PARTS)): block p
// takes elements p, p + AR_PARTS*..., in its share and writes its best (value, index); the last
// block of a row to finish (a ticket per row, reset by that block) picks the best of the parts,
// applies the CPU rule's NaN-at-index-0 case and stores the token. Row mode (rv != null): the
// token feeds the row's next step (tok[b]), is recorded at out[(pos - start) * rows + b], and the
// row advances to pos + 1. Otherwise out[b] = token.
__global__ void __launch_bounds__(AR_THREADS) argmax_rows_kernel(const float* logits, int V, int nrows, RowView* rv,
                                                                 uint32_t* tok, uint32_t* out, ArgmaxScratch* sc) {
    pdl_wait();
    pdl_trigger();
    __shared__ float sv[AR_THREADS / 32];
    __shared__ unsigned si[AR_THREADS / 32];
    __shared__ int is_last;
    const int b = blockIdx.x, part = blockIdx.y;
    const float* x = logits + (size_t)b * V;
    const int per = (V + AR_PARTS - 1) / AR_PARTS, i0 = part * per, i1 = min(V, i0 + per);
    float bv = -INFINITY;
    unsigned bi = AM_NONE;
    for (int i = i0 + threadIdx.x; i < i1; i += AR_THREADS) {
        const float v = x[i];
        if (!isnan(v) && am_wins(v, (unsigned)i, bv, bi)) {
            bv = v;
            bi = (unsigned)i;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
        const unsigned oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (am_wins(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < AR_THREADS / 32; w++)
            if (am_wins(sv[w], si[w], bv, bi)) {
                bv = sv[w];
                bi = si[w];
            }
        sc->val[b][part] = bv;
        sc->idx[b][part] = bi;
        __threadfence();
        is_last = atomicAdd(&sc->ticket[b], 1u) == AR_PARTS - 1;
    }
    __syncthreads();
    if (!is_last || threadIdx.x != 0) return;
    __threadfence();
    bv = -INFINITY;
    bi = AM_NONE;
    for (int q = 0; q < AR_PARTS; q++) {
        const float v = __ldcg(&sc->val[b][q]);
        const unsigned i = __ldcg(&sc->idx[b][q]);
        if (am_wins(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
    sc->ticket[b] = 0u;
    // a NaN at index 0 sticks, and with nothing comparable the CPU argmax stays at 0
    const unsigned t = (isnan(x[0]) || bi == AM_NONE) ? 0u : bi;
    if (rv) {
        tok[b] = t;
        RowView& r = rv[b];
        if (out) out[(size_t)(r.pos - r.start) * nrows + b] = t;
        r.pos += 1;
    } else {
        out[b] = t;
    }
}

int argmax_each(const float* d_logits, int V, int n, uint32_t* d_out, ArgmaxScratch* sc, cudaStream_t s, std::string& err) {
    launch(argmax_rows_kernel, dim3(n, AR_PARTS), dim3(AR_THREADS), 0, s, d_logits, V, n, (RowView*)nullptr,
           (uint32_t*)nullptr, d_out, sc);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        err = std::string("argmax launch failed: ") + cudaGetErrorString(e);
        return QW_ERR_CUDA;
    }
    return QW_OK;
}

size_t row_partial_floats(int B, int NQ, int splits) { return (size_t)B * NQ * splits * PPITCH; }

int argmax_rows(const float* d_logits, int V, int B, RowView* d_rows, uint32_t* d_tok, uint32_t* d_out, ArgmaxScratch* sc,
                cudaStream_t s, std::string& err) {
    launch(argmax_rows_kernel, dim3(B, AR_PARTS), dim3(AR_THREADS), 0, s, d_logits, V, B, d_rows, d_tok, d_out, sc);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        err = std::string("argmax launch failed: ") + cudaGetErrorString(e);
        return QW_ERR_CUDA;
    }
    return QW_OK;
}

// One forward pass over n rows: prefill (rows == null; token t at position start + t of cache c)
// or row mode (rows != null; token t at rows[t].pos of its own cache, `splits` attention splits).
typedef void (*NormSplitFn)(float*, int, const uint16_t*, float, uint16_t*, uint16_t*, const float*, int, size_t);
inline NormSplitFn norm_kernel(int nparts) { return nparts > 4 ? norm_split<true> : norm_split<false>; }

static int forward_pass(const Weights& w, const CacheView& c, const RowView* rows, int splits, bool fused,
                        const uint32_t* d_ids, int n, int start, float* d_logits, Scratch& sc, int* err_word,
                        cudaStream_t s, std::string& err) {
    const int H = w.H, I = w.I, NQ = w.NQ, NKV = w.NKV, QD = NQ * 128, KVD = NKV * 128, QKVR = QD + 2 * KVD;
    const size_t nH = (size_t)n * H;
    if (sc.ycap < y_floats(n, H, I, NQ, NKV)) {
        err = "GEMM output scratch too small";
        return QW_ERR_ARG;
    }
    launch(embed_rows, dim3(n), dim3(256), 0, s, d_ids, H, w.V, w.embed, sc.X, err_word);
    const int G = NQ / NKV;
    const float scale = 1.0f / sqrtf(128.0f);
    const int ks_qkv = ksplit_for(n, QKVR, H), ks_o = ksplit_for(n, H, QD), ks_gu = ksplit_for(n, 2 * I, H),
              ks_d = ksplit_for(n, H, I);
    // residual add of the previous projection's nparts slices + RMSNorm + bf16 split, one CTA per row;
    // in a fused row step (distinct caches) the layers' two norms run as norm_part over 128-column
    // blocks and leave the scale to the consumers (row attention for q|k|v, silu_split for gate|up)
    const int nblk = (H + NP_THREADS - 1) / NP_THREADS;
    const bool deferred = rows && fused && nblk <= NORM_BLOCKS_MAX && sc.row_ssq;
    float* const ssq_a = sc.row_ssq;
    float* const ssq_d = sc.row_ssq ? sc.row_ssq + ROWS_MAX * NORM_BLOCKS_MAX : nullptr;
    auto norm = [&](int nparts, const uint16_t* gain) {
        launch(norm_kernel(nparts), dim3(n), dim3(ROW_THREADS), 0, s, sc.X, H, gain, w.eps, sc.ahi, sc.alo, sc.Y, nparts, nH);
    };
    auto norm_deferred = [&](int nparts, const uint16_t* gain, float* ssq) {
        launch(norm_part, dim3(nblk, n), dim3(NP_THREADS), 0, s, sc.X, H, gain, sc.ahi, sc.alo, (const float*)sc.Y, nparts,
               nH, ssq);
    };
    for (int l = 0; l < w.L; l++) {
        const uint16_t* W = w.layer_w + (size_t)l * w.layer_stride;
        const uint16_t* nrm = w.layer_n + (size_t)l * w.norm_stride;
        int rc;
        // A: (the previous layer's down_proj slices into X) rmsnorm -> q|k|v
        if (deferred) norm_deferred(l == 0 ? 0 : ks_d, nrm, ssq_a);
        else norm(l == 0 ? 0 : ks_d, nrm);
        if ((rc = tc::gemm(sc.ahi, sc.alo, H, W, H, sc.Y, QKVR, n, QKVR, H, err_word, s, err, ks_qkv))) return rc;
        // B: q/k norm + RoPE, K/V into the cache, attention -> o_proj input halves
        const int items = n * (NQ + 2 * NKV);
        if (!(rows && fused))
            launch(qkv_post, dim3((items + 7) / 8), dim3(256), 0, s, sc.Y, ks_qkv, n, start, NQ, NKV, nrm + 2 * H,
                   nrm + 2 * H + 128, w.eps, c, rows, l, sc.Q);
        if (rows) {
            if (row_partial_floats(n, NQ, splits) > sc.attp_cap) {
                err = "row attention partial buffer too small";
                return QW_ERR_ARG;
            }
            const dim3 ag(n, NKV, splits);
            const uint16_t *qn = nrm + 2 * H, *kn = nrm + 2 * H + 128;
#define QW_ROW_ATT(GQ, F)                                                                                             \
    launch(row_attention<GQ, F>, dim3(ag), dim3(RA_THREADS), 0, s, sc.Q, rows, NQ, NKV, l, scale, sc.attp, splits,    \
           sc.att_tickets, sc.ahi, sc.alo, (const float*)sc.Y, ks_qkv, qn, kn, w.eps,                       \
           deferred ? (const float*)ssq_a : (const float*)nullptr, nblk, H)
            if (G == 1) fused ? QW_ROW_ATT(1, true) : QW_ROW_ATT(1, false);
            else if (G == 2) fused ? QW_ROW_ATT(2, true) : QW_ROW_ATT(2, false);
            else fused ? QW_ROW_ATT(3, true) : QW_ROW_ATT(3, false);
#undef QW_ROW_ATT
        } else {
            const size_t hsl = (size_t)l * NKV * c.max_seq * 128;
            rc = G == 1 ? launch_attention_tc<1>(sc.Q, sc.att, c.k, c.v, n, start, NQ, NKV, hsl, c.max_seq, scale, sc.attp,
                                                 sc.attp_cap, err_word, s)
               : G == 2 ? launch_attention_tc<2>(sc.Q, sc.att, c.k, c.v, n, start, NQ, NKV, hsl, c.max_seq, scale, sc.attp,
                                                 sc.attp_cap, err_word, s)
               : G == 4 ? launch_attention_tc<4>(sc.Q, sc.att, c.k, c.v, n, start, NQ, NKV, hsl, c.max_seq, scale, sc.attp,
                                                 sc.attp_cap, err_word, s)
                        : launch_attention<3>(sc.Q, sc.att, c.k, c.v, n, start, NQ, NKV, hsl, c.max_seq, scale, sc.attp,
                                              sc.attp_cap, s);
            if (rc) {
                err = rc == QW_ERR_ARG ? "prefill attention partial buffer too small"
                                       : "cannot raise the prefill attention kernel's shared-memory limit";
                return rc;
            }
            launch(split_rows, dim3(grid_for((size_t)n * QD)), dim3(256), 0, s, sc.att, (size_t)n * QD, sc.ahi, sc.alo);
        }
        // C: o_proj (its slices go into X in the next norm)
        if ((rc = tc::gemm(sc.ahi, sc.alo, QD, W + (size_t)QKVR * H, QD, sc.Y, H, n, H, QD, err_word, s, err, ks_o))) return rc;
        // D: residual + rmsnorm -> gate|up -> silu(gate) * up
        if (deferred) norm_deferred(ks_o, nrm + H, ssq_d);
        else norm(ks_o, nrm + H);
        const uint16_t* Wgu = W + (size_t)QKVR * H + (size_t)H * QD;
        const uint16_t* Wd = Wgu + (size_t)2 * I * H;
        if (ks_gu == 1 && n > tc::SK_NB && (size_t)I * 2 <= (size_t)QD * 4) {
            // SiLU * up in the gate|up GEMM's epilogue, its bf16 halves into the dead Q and att
            // buffers (their next writers are the next layer's qkv_post and attention); the GEMM's own
            // input halves stay in ahi/alo, which its CTAs are still reading
            uint16_t* hh = reinterpret_cast<uint16_t*>(sc.Q);
            uint16_t* hl = reinterpret_cast<uint16_t*>(sc.att);
            if ((rc = tc::gemm(sc.ahi, sc.alo, H, Wgu, H, sc.Y, 2 * I, n, 2 * I, H, err_word, s, err, 1, hh, hl))) return rc;
            // E: down (its slices go into X in the next layer's norm)
            if ((rc = tc::gemm(hh, hl, I, Wd, I, sc.Y, H, n, H, I, err_word, s, err, ks_d))) return rc;
        } else {
            if ((rc = tc::gemm(sc.ahi, sc.alo, H, Wgu, H, sc.Y, 2 * I, n, 2 * I, H, err_word, s, err, ks_gu))) return rc;
            launch(silu_split, dim3(grid_for((size_t)n * I)), dim3(256), 0, s, sc.Y, (size_t)n * I, sc.ahi, sc.alo, ks_gu,
                   deferred ? (const float*)ssq_d : (const float*)nullptr, nblk, I, H, w.eps);
            // E: down (its slices go into X in the next layer's norm)
            if ((rc = tc::gemm(sc.ahi, sc.alo, I, Wd, I, sc.Y, H, n, H, I, err_word, s, err, ks_d))) return rc;
        }
    }
    // the last down_proj's slices go into X with the final norm; without logits, add them alone
    if (d_logits) {
        norm(ks_d, w.final_norm);
        int rc;
        if ((rc = tc::gemm(sc.ahi, sc.alo, H, w.lm_head, H, d_logits, w.V, n, w.V, H, err_word, s, err, 1))) return rc;
    } else {
        launch(residual_add, dim3(grid_for(nH)), dim3(256), 0, s, sc.X, sc.Y, nH, ks_d);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        err = std::string("forward pass launch failed: ") + cudaGetErrorString(e);
        return QW_ERR_CUDA;
    }
    return QW_OK;
}

int run(const Weights& w, const CacheView& c, const uint32_t* d_ids, int n, int start, float* d_logits, Scratch& sc,
        int* err_word, cudaStream_t s, std::string& err) {
    return forward_pass(w, c, nullptr, 0, false, d_ids, n, start, d_logits, sc, err_word, s, err);
}

int run_rows(const Weights& w, const RowView* d_rows, int B, int splits, bool distinct_caches, const uint32_t* d_tok,
             float* d_logits, Scratch& sc, int* err_word, cudaStream_t s, std::string& err) {
    if (B < 1 || B > ROWS_MAX || splits < 1) {
        err = "row step: 1 <= rows <= 16 and splits >= 1";
        return QW_ERR_ARG;
    }
    return forward_pass(w, CacheView{}, d_rows, splits, distinct_caches, d_tok, B, 0, d_logits, sc, err_word, s, err);
}

}  // namespace pf
}  // namespace qw

extern "C" {

int qw_gemm_bf16x2(int device, const uint16_t* d_a_hi, const uint16_t* d_a_lo, const uint16_t* d_b, float* d_y, size_t M,
                   size_t N, size_t K, void* stream) {
    if (!d_a_hi || !d_a_lo || !d_b || !d_y || M == 0 || N == 0 || K == 0 || M > (1u << 30) || N > (1u << 30) ||
        K > (1u << 30))
        return set_error(QW_ERR_ARG, "bad GEMM arguments");
    if (cudaSetDevice(device) != cudaSuccess) return set_error(QW_ERR_CUDA, "cudaSetDevice failed");
    int* ew = device_err_word_for(device);
    if (!ew) return set_error(QW_ERR_NOMEM, "error word allocation failed");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(ew, 0, sizeof(int), s) != cudaSuccess) return set_error(QW_ERR_CUDA, "error word reset failed");
    std::string err;
    int rc = tc::gemm(d_a_hi, d_a_lo, (int)K, d_b, (int)K, d_y, (int)N, (int)M, (int)N, (int)K, ew, s, err, 1);
    if (rc) return set_error(rc, err.c_str());
    int h = 0;
    if (cudaMemcpyAsync(&h, ew, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
        return set_error(QW_ERR_CUDA, "GEMM failed on the device");
    if (h) return set_error(QW_ERR_DEVICE_TIMEOUT, "GEMM: a pipeline wait expired on the device");
    return QW_OK;
}

}  // extern "C"
