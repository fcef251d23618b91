// Standalone kernels behind qw_gemv_bf16 / qw_argmax_f32 / qw_read_probe.
//
// qw_gemv_bf16 runs the decode kernel's own GEMV machinery (Decoder::gemv_produce /
// gemv_consume: TMA bulk ring + register-resident activation segments) on one matrix, so the
// GEMV microbenchmark measures exactly the code the decode kernel streams its weights with.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/cuda_inference.h"
#include "decode_kernel.cuh"

using namespace qw;

namespace qw {
// shared error state lives in engine.cu
int* device_err_word_for(int device);
int set_error(int code, const char* msg);
}  // namespace qw

namespace {

// y[m] = W[m] x for m < count (matrices [count][rows][cols] back to back); count = 1 is the plain GEMV
__global__ void __launch_bounds__(NTHREADS, 1)
gemv_kernel(const __grid_constant__ DecodeParams p, const uint16_t* w, const float* x, float* y, int rows, int cols,
            int count) {
    if (threadIdx.x == 0) {
        for (int i = 0; i < NSLOT; i++) {
            mbar_init(&qw_sm.full[i], 1);
            mbar_init(&qw_sm.empty[i], NCW);
        }
        qw_sm.progress = 0;
        qw_sm.abort = 0;
        qw_sm.prm = p;
        for (int k = 0; k <= NCW; k++) qw_sm.ring_it[k] = 0;
        qw_sm.n_issued = 0;
        qw_sm.geo[0] = make_geo(rows, cols, blockIdx.x, gridDim.x, 0, 0);
        for (int w = 0; w < NCW; w++) qw_sm.wgeo[0][w] = make_warp_geo(qw_sm.geo[0], w);
        fence_mbar_init();
    }
    __syncthreads();
    const GemvGeo& g = qw_sm.geo[0];
    const size_t mat = (size_t)rows * cols;
    if (Decoder::warp() == NCW) {
        if (Decoder::lane() == 0) {
            for (int m = 0; m < count; m++) Decoder::gemv_produce(g, w + m * mat);
            Decoder::drain();
        }
        return;
    }
    for (int i = Decoder::tid(); i < cols; i += NCT) Decoder::xs()[xperm(i)] = x[i];
    named_bar_sync(1, NCT);
    for (int m = 0; m < count; m++) {
        Decoder::gemv_consume<EPI_PART>(g);
        float* ym = y + (size_t)m * rows;
        for (int i = Decoder::tid(); i < g.r1 - g.r0; i += NCT) ym[g.r0 + i] = Decoder::row_value(g, i);
        named_bar_sync(1, NCT);  // the next matrix's sums overwrite part()
    }
}

// argmax with the reference CPU rule, in two levels inside one launch (last-block reduction)
constexpr int AM_THREADS = 512;

__global__ void __launch_bounds__(AM_THREADS)
argmax_kernel(const float* __restrict__ x, size_t n, uint32_t* out, float* ws_val, unsigned* ws_idx, unsigned* ticket) {
    __shared__ float sv[AM_THREADS / 32];
    __shared__ unsigned si[AM_THREADS / 32];
    __shared__ int last;
    float bv = -INFINITY;
    unsigned bi = NONE_IDX;
    const size_t stride = (size_t)gridDim.x * AM_THREADS;
    for (size_t i = (size_t)blockIdx.x * AM_THREADS + threadIdx.x; i < n; i += stride) {
        const float v = x[i];
        if (!isnan(v) && am_better(v, (unsigned)i, bv, bi)) { bv = v; bi = (unsigned)i; }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
        const unsigned oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < AM_THREADS / 32; w++)
            if (am_better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
        ws_val[blockIdx.x] = bv;
        ws_idx[blockIdx.x] = bi;
        __threadfence();
        last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    bv = -INFINITY;
    bi = NONE_IDX;
    for (unsigned b = threadIdx.x; b < gridDim.x; b += AM_THREADS) {
        const float v = __ldcg(ws_val + b);
        const unsigned i = __ldcg(ws_idx + b);
        if (am_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
        const unsigned oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    __syncthreads();
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < AM_THREADS / 32; w++)
            if (am_better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
        // a NaN at index 0 sticks, and with nothing comparable the CPU argmax stays at 0
        *out = (n == 0 || isnan(x[0]) || bi == NONE_IDX) ? 0u : bi;
        *ticket = 0u;
    }
}

constexpr int RP_THREADS = 512;

__global__ void __launch_bounds__(RP_THREADS) read_probe_kernel(const float4* __restrict__ src, size_t n4, float* partials) {
    float4 a0 = make_float4(0, 0, 0, 0), a1 = a0, a2 = a0, a3 = a0;
    const size_t grid = (size_t)gridDim.x * RP_THREADS;
    size_t i = (size_t)blockIdx.x * RP_THREADS + threadIdx.x;
    for (; i + 3 * grid < n4; i += 4 * grid) {
        const float4 v0 = __ldcs(src + i), v1 = __ldcs(src + i + grid), v2 = __ldcs(src + i + 2 * grid),
                     v3 = __ldcs(src + i + 3 * grid);
        a0.x += v0.x; a0.y += v0.y; a0.z += v0.z; a0.w += v0.w;
        a1.x += v1.x; a1.y += v1.y; a1.z += v1.z; a1.w += v1.w;
        a2.x += v2.x; a2.y += v2.y; a2.z += v2.z; a2.w += v2.w;
        a3.x += v3.x; a3.y += v3.y; a3.z += v3.z; a3.w += v3.w;
    }
    for (; i < n4; i += grid) {
        const float4 v = __ldcs(src + i);
        a0.x += v.x; a0.y += v.y; a0.z += v.z; a0.w += v.w;
    }
    float s = (a0.x + a0.y + a0.z + a0.w) + (a1.x + a1.y + a1.z + a1.w) + (a2.x + a2.y + a2.z + a2.w) +
              (a3.x + a3.y + a3.z + a3.w);
    s = warp_sum(s);
    __shared__ float part[RP_THREADS / 32];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < RP_THREADS / 32 ? part[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) partials[blockIdx.x] = t;
    }
}

// Scratch of qw_argmax_f32_noalloc: the same layout as the caller workspace of qw_argmax_f32
// (a 4-byte ticket in the first 256 bytes, then up to 1024 block maxima and 1024 block indices).
// It is one file-scope device array: every GPU that loads this library holds these 8,448 bytes
// until the process exits, and all calls on a device share them.
constexpr size_t NOALLOC_ARGMAX_SCRATCH = 256 + 2 * 4 * 1024;
static __device__ __align__(256) uint8_t g_argmax_scratch[NOALLOC_ARGMAX_SCRATCH];

// Device address of g_argmax_scratch on `device`, looked up once per device with that device
// current (in host code the array's name is only a host-side stand-in, not a device address).
void* argmax_scratch_address(int device, std::string& err) {
    static std::mutex mu;
    static std::vector<void*> addr;
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0) { err = "bad device index"; return nullptr; }
    if ((int)addr.size() <= device) addr.resize(device + 1, nullptr);
    if (!addr[device]) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_argmax_scratch);
        if (e != cudaSuccess || !ptr) {
            err = std::string("cudaGetSymbolAddress(g_argmax_scratch) failed: ") + cudaGetErrorString(e);
            return nullptr;
        }
        addr[device] = ptr;
    }
    return addr[device];
}

int sm_count(int device) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    return n;
}

}  // namespace

extern "C" {

int qw_gemv_bf16(int device, const uint16_t* d_w, const float* d_x, float* d_y, size_t rows, size_t cols, void* stream) {
    return qw_gemv_bf16_seq(device, d_w, d_x, d_y, rows, cols, 1, stream);
}

int qw_gemv_bf16_seq(int device, const uint16_t* d_w, const float* d_x, float* d_y, size_t rows, size_t cols,
                     size_t count, void* stream) {
    if (!d_w || !d_x || !d_y || rows == 0 || count == 0 || count >= (1u << 20)) return set_error(QW_ERR_ARG, "bad gemv arguments");
    if (cols == 0 || cols > 12288 || seg_count((int)cols) == 0)
        return set_error(QW_ERR_UNSUPPORTED, "cols must split into 1, 2, 3, 4, 6 or 12 segments of 256-1024 columns");
    if (rows >= (1u << 30)) return set_error(QW_ERR_ARG, "rows too large");
    if (cudaSetDevice(device) != cudaSuccess) return set_error(QW_ERR_CUDA, "cudaSetDevice failed");
    int* err = device_err_word_for(device);
    if (!err) return set_error(QW_ERR_NOMEM, "error word allocation failed");
    const int n = sm_count(device);
    const size_t rows_per = (rows + n - 1) / n;
    DecodeParams p{};
    p.err = err;
    p.stall_cta = -1;
    p.H = (int)cols;
    p.I = 256;
    p.L = 1;
    p.NQ = 1;
    p.NKV = 1;
    p.V = (int)rows;
    p.S = 1;
    p.xs_cap = (int)((cols + 3) / 4 * 4);
    p.part_cap = (int)(((rows_per + 2) * seg_count((int)cols) + 3) / 4 * 4);
    p.xloc_cap = 4;
    p.timeout_ns = 4000000000LL;
    const size_t smem = (size_t)NSLOT * SLOT_BYTES + ((size_t)p.xs_cap + p.part_cap + p.xloc_cap) * 4;
    if (smem + sizeof(Smem) > 227 * 1024) return set_error(QW_ERR_UNSUPPORTED, "rows too large for one launch");
    if (cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return set_error(QW_ERR_CUDA, "cannot raise the gemv kernel's shared-memory limit");
    gemv_kernel<<<n, NTHREADS, smem, static_cast<cudaStream_t>(stream)>>>(p, d_w, d_x, d_y, (int)rows, (int)cols,
                                                                          (int)count);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(QW_ERR_CUDA, cudaGetErrorString(e));
    return QW_OK;
}

size_t qw_argmax_workspace_size(size_t n) {
    (void)n;
    return 256 + 2 * 4 * 1024;  // ticket + up to 1024 block partials
}

int qw_argmax_f32(int device, const float* d_x, size_t n, uint32_t* d_out, void* d_workspace, void* stream) {
    if (!d_x || !d_out || !d_workspace || n == 0 || n >= (1ull << 32)) return set_error(QW_ERR_ARG, "bad argmax arguments");
    if (cudaSetDevice(device) != cudaSuccess) return set_error(QW_ERR_CUDA, "cudaSetDevice failed");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int blocks = (int)std::min<size_t>(std::min<size_t>(1024, (size_t)sm_count(device) * 4), (n + AM_THREADS - 1) / AM_THREADS);
    uint8_t* ws = static_cast<uint8_t*>(d_workspace);
    unsigned* ticket = reinterpret_cast<unsigned*>(ws);
    float* vals = reinterpret_cast<float*>(ws + 256);
    unsigned* idxs = reinterpret_cast<unsigned*>(ws + 256 + 4 * 1024);
    if (cudaMemsetAsync(ticket, 0, 4, s) != cudaSuccess) return set_error(QW_ERR_CUDA, "workspace reset failed");
    argmax_kernel<<<blocks, AM_THREADS, 0, s>>>(d_x, n, d_out, vals, idxs, ticket);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(QW_ERR_CUDA, cudaGetErrorString(e));
    return QW_OK;
}

int qw_argmax_f32_noalloc(int device, const float* d_x, size_t n, uint32_t* d_out, void* stream) {
    if (!d_x || !d_out) return set_error(QW_ERR_ARG, "qw_argmax_f32_noalloc: null pointer");
    if (n == 0 || n > QW_ARGMAX_NOALLOC_MAX_N)
        return set_error(QW_ERR_ARG, "qw_argmax_f32_noalloc: n must be in [1, QW_ARGMAX_NOALLOC_MAX_N]");
    if (cudaSetDevice(device) != cudaSuccess) return set_error(QW_ERR_CUDA, "cudaSetDevice failed");
    std::string err;
    uint8_t* ws = static_cast<uint8_t*>(argmax_scratch_address(device, err));
    if (!ws) return set_error(QW_ERR_CUDA, err.c_str());
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int blocks = (int)std::min<size_t>(std::min<size_t>(1024, (size_t)sm_count(device) * 4), (n + AM_THREADS - 1) / AM_THREADS);
    unsigned* ticket = reinterpret_cast<unsigned*>(ws);
    // the ticket must start at zero; the partials are always written before they are read
    if (cudaMemsetAsync(ticket, 0, 4, s) != cudaSuccess) return set_error(QW_ERR_CUDA, "scratch reset failed");
    argmax_kernel<<<blocks, AM_THREADS, 0, s>>>(d_x, n, d_out, reinterpret_cast<float*>(ws + 256),
                                                reinterpret_cast<unsigned*>(ws + 256 + 4 * 1024), ticket);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(QW_ERR_CUDA, cudaGetErrorString(e));
    return QW_OK;
}

int qw_read_probe(int device, const float* d_src, size_t n_floats, float* d_partials, size_t n_partials, size_t* n_written,
                  void* stream) {
    if (!d_src || !d_partials || n_partials == 0 || n_floats % 4 != 0 || ((uintptr_t)d_src % 16) != 0)
        return set_error(QW_ERR_ARG, "bad read-probe arguments");
    if (cudaSetDevice(device) != cudaSuccess) return set_error(QW_ERR_CUDA, "cudaSetDevice failed");
    const int blocks = (int)std::min<size_t>(n_partials, (size_t)sm_count(device) * 4);
    read_probe_kernel<<<blocks, RP_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const float4*>(d_src), n_floats / 4, d_partials);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(QW_ERR_CUDA, cudaGetErrorString(e));
    if (n_written) *n_written = (size_t)blocks;
    return QW_OK;
}

}  // extern "C"
