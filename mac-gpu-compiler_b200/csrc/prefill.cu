// Batched prefill: the tcgen05 GEMM's host side (tensor maps, launch) and
// the standalone entry point qw_gemm_bf16x2 (see tc_gemm.cuh for the kernel).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "../../include/cuda_inference.h"
#include "tc_gemm.cuh"

namespace qw {
int* device_err_word_for(int device);
int set_error(int code, const char* msg);
}  // namespace qw

using namespace qw;

namespace qw {
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
int gemm(const uint16_t* a_hi, const uint16_t* a_lo, int lda, const uint16_t* b, int ldb, float* y, int ldy, int M, int N,
         int K, int* err_word, cudaStream_t s, std::string& err) {
    if (M <= 0 || N <= 0 || K <= 0 || K % BK != 0) {
        err = "gemm: M, N, K must be positive and K a multiple of 64";
        return QW_ERR_ARG;
    }
    CUtensorMap mh, ml, mb;
    int rc;
    if ((rc = make_map_bf16(&mh, a_hi, (uint64_t)M, (uint64_t)K, (uint64_t)lda, BM, err))) return rc;
    if ((rc = make_map_bf16(&ml, a_lo, (uint64_t)M, (uint64_t)K, (uint64_t)lda, BM, err))) return rc;
    if ((rc = make_map_bf16(&mb, b, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, BN, err))) return rc;
    if (cudaFuncSetAttribute(gemm_bf16x2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess) {
        err = "cannot raise the GEMM kernel's shared-memory limit";
        return QW_ERR_CUDA;
    }
    GemmArgs args{y, M, N, K, ldy, err_word};
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    gemm_bf16x2_kernel<<<grid, THREADS, SMEM_BYTES, s>>>(mh, ml, mb, args);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        err = std::string("GEMM launch failed: ") + cudaGetErrorString(e);
        return QW_ERR_CUDA;
    }
    return QW_OK;
}

}  // namespace tc
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
    int rc = tc::gemm(d_a_hi, d_a_lo, (int)K, d_b, (int)K, d_y, (int)N, (int)M, (int)N, (int)K, ew, s, err);
    if (rc) return set_error(rc, err.c_str());
    int h = 0;
    if (cudaMemcpyAsync(&h, ew, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
        return set_error(QW_ERR_CUDA, "GEMM failed on the device");
    if (h) return set_error(QW_ERR_DEVICE_TIMEOUT, "GEMM: a pipeline wait expired on the device");
    return QW_OK;
}

}  // extern "C"
