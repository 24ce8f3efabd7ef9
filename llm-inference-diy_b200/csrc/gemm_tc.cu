// gemm_tc.cu — host side of the tcgen05 GEMM: TMA tensor maps, launch, and
// the plain entry point C = A * W^T (fp16 out).  The prefill's fused
// epilogues live with the prefill (prefill_tc.cu) and reuse launch_gemm_tc.
#include <mutex>

#include "gemm_tc.cuh"
#include "gemm_tc_host.h"

namespace llmdiy {

namespace {
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

struct PlainStore {
    half* C;
    int ldc, N;
    __device__ void operator()(int row, int n, const float* v) const {
        half* dst = C + (size_t)row * ldc + n;
        if (n + 16 <= N && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
            *reinterpret_cast<uint4*>(dst) = pack8(v);
            *reinterpret_cast<uint4*>(dst + 8) = pack8(v + 8);
        } else {
            for (int j = 0; j < 16 && n + j < N; ++j) dst[j] = f2h(v[j]);
        }
    }
};
}  // namespace

// K-major fp16 operand [rows][K] (row pitch ld elements), box 64 x box_rows, 128-byte swizzle.
bool make_kmajor_map(CUtensorMap* m, const void* base, int rows, int K, int ld, int box_rows) {
    EncodeTiled enc = encode_fn();
    if (!enc || (reinterpret_cast<uintptr_t>(base) & 15) || (ld % 8) || K <= 0 || rows <= 0) return false;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)kGemmBK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_mnmajor_map(CUtensorMap* m, const void* base, int K, int N, int ld) {
    EncodeTiled enc = encode_fn();
    if (!enc || (reinterpret_cast<uintptr_t>(base) & 15) || (ld % 8) || K <= 0 || N <= 0) return false;
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)K};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)kGemmBK};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int* gemm_err_word() {
    static std::mutex mu;
    static int* words[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!words[dev] && cudaMalloc(&words[dev], sizeof(int)) == cudaSuccess) cudaMemset(words[dev], 0, sizeof(int));
    return words[dev];
}

int gemm_tc_status() {
    int* err = gemm_err_word();
    if (!err) return (int)cudaErrorMemoryAllocation;
    int h = 0;
    cudaError_t e = cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return (int)e;
    if (h) cudaMemset(err, 0, sizeof(int));
    return h;
}

}  // namespace llmdiy

using namespace llmdiy;

extern "C" int llmdiy_gemm_tc(const uint16_t* A, const uint16_t* W, uint16_t* C, int M, int N, int K, void* stream) {
    PlainStore epi{reinterpret_cast<half*>(C), N, N};
    return launch_gemm_tc(reinterpret_cast<const half*>(A), K, reinterpret_cast<const half*>(W), K, M, N, K, epi,
                          reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int llmdiy_gemm_tc_status(void) { return gemm_tc_status(); }

// C[M,N] = A[M,K] * B[K,N] with B in the reference's transposed-weight layout (test entry for
// the MN-major operand path; llmdiy_hgemm_swizzle_nn uses it).
extern "C" int llmdiy_gemm_tc_kn(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K,
                                 void* stream) {
    PlainStore epi{reinterpret_cast<half*>(C), N, N};
    return launch_gemm_tc_kn(reinterpret_cast<const half*>(A), K, reinterpret_cast<const half*>(B), N, M, N, K, epi,
                             reinterpret_cast<cudaStream_t>(stream));
}
