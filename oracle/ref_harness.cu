// ref_harness.cu — TEST INFRASTRUCTURE ONLY.
//
// Exposes the reference's own kernels (LLM-inference-DIY, kernels/*.cuh) as
// extern "C" launchers with the engine's launch shapes, so that tests and the
// golden-fixture script can run them on a B200 from compute_89 PTX.  The
// reference headers are #included from the read-only reference tree at build
// time (oracle/Makefile passes -I to it); no reference source is copied here.
// The launch shapes below are the ones framework_src/qwen_infer.cu uses.
#include <cstdint>
#include <cstdlib>
#include <cmath>
#include <iostream>
#include <vector>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

// Same include order as framework_src/qwen_infer.cu:12-64.
#include "hgemm_mma_swizzle.cuh"
#include "flash_decode_q1_opt.cuh"
#include "rmsnorm.cuh"
#include "rope.cuh"
#include "swiglu.cuh"
#include "bias.cuh"
#include "argmax.cuh"
#include "hgemm_final.cuh"
#include "transpose.cuh"
#include "fused_qkv_rope_cache.cuh"
#define FLASH_ATTN_CAUSAL
#include "flash_attn.cu"
#include "gather_qkv.cuh"

extern "C" {

// qwen_infer.cu:626
int ref_rmsnorm(half* out, const half* in, const half* w, int d, float eps) {
    rmsnorm_kernel<<<1, 512>>>(out, in, w, d, eps);
    return (int)cudaDeviceSynchronize();
}

// qwen_infer.cu:631 / :704 (grid sized to n)
int ref_add_bias(half* out, const half* b, int n) {
    add_bias_kernel<<<(n + 255) / 256, 256>>>(out, b, n);
    return (int)cudaDeviceSynchronize();
}

// qwen_infer.cu:715
int ref_swiglu(half* out, const half* a, const half* b, int n) {
    swiglu_kernel<<<(n + 255) / 256, 256>>>(out, a, b, n);
    return (int)cudaDeviceSynchronize();
}

// qwen_infer.cu:634-642
int ref_fused_qkv_rope_cache(half* qkv, half* kc, half* vc, int pos, int max_seqlen, int nh, int hd) {
    fused_qkv_rope_cache_kernel<<<nh, hd / 2>>>(qkv, kc, vc, pos, max_seqlen, nh, hd);
    return (int)cudaDeviceSynchronize();
}

// qwen_infer.cu:360-363
int ref_hgemv(const half* A, const half* B, half* C, int N, int K) {
    hgemv_kernel<<<(N + 255) / 256, 256>>>(A, B, C, N, K);
    return (int)cudaDeviceSynchronize();
}

// qwen_infer.cu:666-668
int ref_fd_v5_fused(const half* Q, const half* K, const half* V, half* O, int L, int stride) {
    fd_v5_fused_kernel<128, 8, 32><<<1, 256>>>(Q, K, V, O, L, stride);
    return (int)cudaDeviceSynchronize();
}

// qwen_infer.cu:671-673
int ref_fd_v5_split_stage1(const half* Q, const half* K, const half* V, half* Opart, float* LSE,
                           int L, int num_chunks, int stride) {
    fd_v5_split_stage1_kernel<128, 256, 8><<<num_chunks, 256>>>(Q, K, V, Opart, LSE, L, num_chunks, stride);
    return (int)cudaDeviceSynchronize();
}

// qwen_infer.cu:674-676
int ref_fd_opt_stage2(const half* Opart, const float* LSE, half* O, int num_chunks) {
    fd_opt_stage2_kernel<128><<<1, 128>>>(Opart, LSE, O, num_chunks);
    return (int)cudaDeviceSynchronize();
}

// The decode step's whole attention launch sequence for one layer (qwen_infer.cu:646-677): per
// head, the fused kernel when L <= 256, else split stage 1 over ceil(L/256) chunks and stage 2,
// with the partials buffer reused head after head.  Launched on `stream` without synchronising
// (for timing, also inside a CUDA graph); q/out are [nh*128], K/V the cache rows at `stride`.
int ref_fd_layer(const half* q, const half* Kc, const half* Vc, half* out, half* Opart, float* LSE, int L, int nh,
                 int stride, cudaStream_t stream) {
    const int num_chunks = (L + 255) / 256;
    for (int h = 0; h < nh; h++) {
        if (num_chunks == 1) {
            fd_v5_fused_kernel<128, 8, 32><<<1, 256, 0, stream>>>(q + h * 128, Kc + h * 128, Vc + h * 128,
                                                                  out + h * 128, L, stride);
        } else {
            fd_v5_split_stage1_kernel<128, 256, 8><<<num_chunks, 256, 0, stream>>>(
                q + h * 128, Kc + h * 128, Vc + h * 128, Opart, LSE, L, num_chunks, stride);
            fd_opt_stage2_kernel<128><<<1, 128, 0, stream>>>(Opart, LSE, out + h * 128, num_chunks);
        }
    }
    return (int)cudaGetLastError();
}

// qwen_infer.cu:731
int ref_argmax(int* out, const half* logits, int V) {
    argmax_kernel<<<1, 512>>>(out, logits, V);
    return (int)cudaDeviceSynchronize();
}

// qwen_infer.cu:364-366
int ref_hgemm_swizzle_nn(half* A, half* B, half* C, int M, int N, int K) {
    hgemm_swizzle_nn(A, B, C, M, N, K);
    return (int)cudaDeviceSynchronize();
}

// qwen_infer.cu:501-516: one head, per-head contiguous Q/K/V/O [N,128]
int ref_flash_attn_causal_head(half* Q, half* K, half* V, half* O, int N) {
    constexpr int Br = 128, Bc = 128;
    int Tr = (N + Br - 1) / Br;
    dim3 g(1, Tr), b(256);
    constexpr int Q_sz = Br * (16 + 8), K_sz = Bc * (16 + 8);
    int smem = 2 * (Q_sz + K_sz) * sizeof(half);
    auto fa = flash_attn_tuned_A_kernel<128, 16, 8, 16, 8, 1, 1, 16, 1, 0, 8, 8, 8, 2, 1>;
    cudaFuncSetAttribute(fa, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    fa<<<g, b, smem>>>(Q, K, V, O, N, 1, 128, 128, 0, 0, 0, 0);
    return (int)cudaDeviceSynchronize();
}

// qwen_infer.cu:486-490 and :527-528
int ref_gather_q_from_qkv(const half* qkv, half* dst, int N, int nh) {
    gather_q_from_qkv(qkv, dst, N, nh, 128);
    return (int)cudaDeviceSynchronize();
}
int ref_gather_kv_from_cache(const half* cache, half* dst, int N, int nh) {
    gather_kv_from_cache(cache, dst, N, nh, 128);
    return (int)cudaDeviceSynchronize();
}
int ref_scatter_interleaved(const half* src, half* dst, int N, int nh, int H) {
    scatter_interleaved_kernel<128, 256><<<(N * nh * 128 + 255) / 256, 256>>>(src, dst, N, nh, H);
    return (int)cudaDeviceSynchronize();
}

// qwen_infer.cu:233-242 (kernel only: out[c*rows+r] = in[r*cols+c])
int ref_transpose(half* out, const half* in, int rows, int cols) {
    dim3 block(16, 16), grid((cols + 15) / 16, (rows + 15) / 16);
    transpose_weight_kernel<<<grid, block>>>(out, in, rows, cols);
    return (int)cudaDeviceSynchronize();
}

}  // extern "C"
