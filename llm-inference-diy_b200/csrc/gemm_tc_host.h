// gemm_tc_host.h — host-side launcher of the tcgen05 GEMM (C = A * W^T with a
// fused epilogue op) for every translation unit that instantiates one.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "gemm_tc.cuh"
#include "gemm_tc2.cuh"

namespace llmdiy {
constexpr int kGemmBN = 256;  // output columns per CTA tile (UMMA N = 256)
// K-major fp16 operand [rows][K] (row pitch ld elements), box 64 x box_rows, 128-byte swizzle.
bool make_kmajor_map(CUtensorMap* m, const void* base, int rows, int K, int ld, int box_rows);
// MN-major fp16 operand [K][N] (row pitch ld elements): box 64 N x 64 K rows, 128-byte swizzle.
bool make_mnmajor_map(CUtensorMap* m, const void* base, int K, int N, int ld);
int* gemm_err_word();  // per-device error word of the GEMM kernels (set when a wait expires)
int gemm_tc_status();  // 0, or 1 once any GEMM of this device recorded an expired wait

// C tile op `epi` is called per thread with (row, first column, 16 fp32 values).
// ksplit > 1: grid.z slices of the K blocks, each running `epi` on its partial sums.
inline int gemm_num_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    return sms;
}

// M > 128 without split-K: persistent 2-CTA clusters, 256 x 256 tiles per pair (gemm_tc2.cuh).
template <class Epi>
int launch_gemm_tc2(const half* A, int lda, const half* W, int ldw, int M, int N, int K, const Epi& epi,
                    cudaStream_t st) {
    CUtensorMap ta, tb;
    if (!make_kmajor_map(&ta, A, M, K, lda, 128) || !make_kmajor_map(&tb, W, N, K, ldw, 128))
        return (int)cudaErrorInvalidValue;
    int* err = gemm_err_word();
    if (!err) return (int)cudaErrorMemoryAllocation;
    auto kern = gemm_tc2_k<Epi>;
    static std::once_flag attr;
    std::call_once(attr, [&] {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Gemm2Smem));
    });
    const int sms = gemm_num_sms();
    const int tiles = ((M + 255) / 256) * ((N + 255) / 256);
    const int pairs = std::max(1, std::min(tiles, sms / 2));
    kern<<<2 * pairs, kGemm2Threads, sizeof(Gemm2Smem), st>>>(ta, tb, M, N, K, epi, err);
    return (int)cudaGetLastError();
}

// pdl: launch with programmatic stream serialization (the kernel prefetches its first weight
// blocks into L2, then waits for the previous kernel before reading A or running the epilogue).
template <class Epi>
int launch_gemm_tc(const half* A, int lda, const half* W, int ldw, int M, int N, int K, const Epi& epi,
                   cudaStream_t st, int ksplit = 1, bool pdl = false) {
    if (M <= 0 || N <= 0 || K <= 0) return (int)cudaErrorInvalidValue;
    // SM pairs when there are at least as many 256 x 256 tiles as pairs (below that, 128 x 256
    // tiles on single SMs cover more of the GPU)
    if (ksplit == 1 && M > kGemmBM && ((M + 255) / 256) * ((N + 255) / 256) >= gemm_num_sms() / 2)
        return launch_gemm_tc2(A, lda, W, ldw, M, N, K, epi, st);
    constexpr int BN = kGemmBN;
    CUtensorMap ta, tb;
    if (!make_kmajor_map(&ta, A, M, K, lda, kGemmBM) || !make_kmajor_map(&tb, W, N, K, ldw, BN))
        return (int)cudaErrorInvalidValue;
    int* err = gemm_err_word();
    if (!err) return (int)cudaErrorMemoryAllocation;
    auto kern = gemm_tc_k<BN, Epi>;
    static std::once_flag attr;
    std::call_once(attr, [&] {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(GemmSmem<BN>));
    });
    const int KB = (K + kGemmBK - 1) / kGemmBK;
    if (ksplit < 1 || ksplit > KB) return (int)cudaErrorInvalidValue;
    const int per = (KB + ksplit - 1) / ksplit;
    if ((ksplit - 1) * per >= KB) return (int)cudaErrorInvalidValue;  // an empty slice
    dim3 grid((N + BN - 1) / BN, (M + kGemmBM - 1) / kGemmBM, ksplit);
    if (!pdl) {
        kern<<<grid, kGemmThreads, sizeof(GemmSmem<BN>), st>>>(ta, tb, M, N, K, epi, err);
        return (int)cudaGetLastError();
    }
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = dim3(kGemmThreads);
    lc.dynamicSmemBytes = sizeof(GemmSmem<BN>);
    lc.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    return (int)cudaLaunchKernelEx(&lc, kern, ta, tb, M, N, K, epi, err);
}

// C = A[M,K] * B[K,N] with B in the reference's [K,N] layout (MN-major operand).
template <class Epi>
int launch_gemm_tc_kn(const half* A, int lda, const half* B, int ldb, int M, int N, int K, const Epi& epi,
                      cudaStream_t st) {
    if (M <= 0 || N <= 0 || K <= 0 || (N % 8) || (K % 8)) return (int)cudaErrorInvalidValue;
    constexpr int BN = kGemmBN;
    CUtensorMap ta, tb;
    if (!make_kmajor_map(&ta, A, M, K, lda, kGemmBM) || !make_mnmajor_map(&tb, B, K, N, ldb))
        return (int)cudaErrorInvalidValue;
    int* err = gemm_err_word();
    if (!err) return (int)cudaErrorMemoryAllocation;
    auto kern = gemm_tc_k<BN, Epi, true>;
    static std::once_flag attr;
    std::call_once(attr, [&] {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(GemmSmem<BN>));
    });
    dim3 grid((N + BN - 1) / BN, (M + kGemmBM - 1) / kGemmBM, 1);
    kern<<<grid, kGemmThreads, sizeof(GemmSmem<BN>), st>>>(ta, tb, M, N, K, epi, err);
    return (int)cudaGetLastError();
}

}  // namespace llmdiy
