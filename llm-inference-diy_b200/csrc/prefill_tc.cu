// prefill_tc.cu — the prompt forward (QwenEngine::prefill, qwen_infer.cu:372-611)
// on the tensor cores: per layer
//   RMSNorm(ln_1) rows -> QKV GEMM [epilogue: bias, RoPE, K/V appended to the
//   cache, Q kept] -> causal flash attention over the cache (flash_tc.cuh)
//   -> o_proj GEMM [epilogue:
//   residual add] -> RMSNorm(ln_2) rows -> w1|w2 GEMM [epilogue: SwiGLU] ->
//   c_proj GEMM [epilogue: residual add].
// The GEMMs are the tcgen05 kernel (gemm_tc.cuh) over the engine's device
// weights (QKV rows permuted into RoPE pairs, w1/w2 interleaved — the pairs an
// epilogue needs sit in adjacent output columns of one thread).  The fp16
// rounding points and fast-math intrinsics are those of the decode kernel's
// epilogues, so a prompt row gets the same arithmetic as a decode step except
// for the GEMM summation order.  Prompts are processed in chunks of at most
// kPrefillChunk rows; a chunk attends over every cached row before it.
#include <mutex>

#include "decode.h"
#include "flash_tc.cuh"
#include "gemm_tc_host.h"
#include "ops.cuh"
#include "prefill_tc.h"
#include "rows.cuh"

namespace llmdiy {
namespace {

// QKV epilogue: columns (2u, 2u+1) are RoPE partners (t, t+64) of unit u =
// sec*1024 + h*64 + t.  bias -> RoPE (q, k) -> q kept in [row][H], k and v
// appended to the cache at position p0 + row (fused_qkv_rope_cache.cuh:6-55).
struct EpiQKV {
    const half* bias;
    half* q;
    half* kc;
    half* vc;
    int p0;
    // The 16 columns [n, n+16) are units u0..u0+7 = dims t0..t0+7 (and +64) of one
    // head of one section (n is a multiple of 16), so the 8 first values and the 8
    // second values of the pairs are each one 16-byte row segment.
    __device__ void operator()(int row, int n, const float* v) const {
        const int pos = p0 + row;
        const int u0 = n >> 1, sec = u0 / (kHidden / 2), vv = u0 % (kHidden / 2), h = vv / 64, t0 = vv % 64;
        const int i1 = sec * kHidden + h * kHeadDim + t0;
        float b1[8], b2[8], y1[8], y2[8];
        unpack8(*reinterpret_cast<const uint4*>(bias + i1), b1);
        unpack8(*reinterpret_cast<const uint4*>(bias + i1 + 64), b2);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            y1[j] = h2f(f2h(h2f(f2h(v[2 * j])) + b1[j]));
            y2[j] = h2f(f2h(h2f(f2h(v[2 * j + 1])) + b2[j]));
        }
        const int o1 = h * kHeadDim + t0;
        if (sec == 2) {
            *reinterpret_cast<uint4*>(vc + (size_t)pos * kHidden + o1) = pack8(y1);
            *reinterpret_cast<uint4*>(vc + (size_t)pos * kHidden + o1 + 64) = pack8(y2);
            return;
        }
        float r1[8], r2[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float theta =
                (float)pos * __powf(10000.0f, __fdividef(-2.0f * (float)(t0 + j), (float)kHeadDim));
            const float cs = __cosf(theta), sn = __sinf(theta);
            r1[j] = y1[j] * cs - y2[j] * sn;
            r2[j] = y2[j] * cs + y1[j] * sn;
        }
        half* dst = sec == 1 ? kc + (size_t)pos * kHidden : q + (size_t)row * kHidden;
        *reinterpret_cast<uint4*>(dst + o1) = pack8(r1);
        *reinterpret_cast<uint4*>(dst + o1 + 64) = pack8(r2);
    }
};

}  // namespace

int flash_tc_causal(const half* q, int ldq, const half* k, const half* v, int ldkv, int kv_rows, half* o, int ldo,
                    int n, int p0, int heads, cudaStream_t st) {
    static std::once_flag attr;
    std::call_once(attr, [] {
        cudaFuncSetAttribute(flash_tc_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(FlashTcSmem));
    });
    CUtensorMap tq, tk, tv;
    const int width = heads * kHeadDim;
    if (!make_kmajor_map(&tq, q, n, width, ldq, kFtRows) || !make_kmajor_map(&tk, k, kv_rows, width, ldkv, kFtKeys) ||
        !make_kmajor_map(&tv, v, kv_rows, width, ldkv, kFtKeys))
        return (int)cudaErrorInvalidValue;
    int* err = gemm_err_word();
    if (!err) return (int)cudaErrorMemoryAllocation;
    flash_tc_k<<<dim3((n + kFtRows - 1) / kFtRows, heads), kFtThreads, sizeof(FlashTcSmem), st>>>(tq, tk, tv, o, ldo,
                                                                                                  n, p0, err);
    return (int)cudaGetLastError();
}

int prefill_tc(const PrefillArgs& p, const int* tokens_dev, int n, int p0, cudaStream_t st) {
    int rc = 0;
    cudaError_t e;
    for (int c0 = 0; c0 < n; c0 += kPrefillChunk) {
        const int m = n - c0 < kPrefillChunk ? n - c0 : kPrefillChunk;
        const int pos0 = p0 + c0;
        embed_rows_k<<<m, 256, 0, st>>>(p.wte, tokens_dev + c0, p.x);
        for (int l = 0; l < p.NL; ++l) {
            const LayerPtrs& L = p.layers[l];
            half* kcl = p.kc + (size_t)l * p.layer_stride;
            half* vcl = p.vc + (size_t)l * p.layer_stride;
            rmsnorm_rows_k<<<m, 256, 0, st>>>(p.xn, p.x, L.ln1);
            rc = launch_gemm_tc(p.xn, kHidden, L.qkv_w, kHidden, m, 3 * kHidden, kHidden,
                                EpiQKV{L.qkv_b, p.q, kcl, vcl, pos0}, st);
            if (rc) return rc;
            rc = flash_tc_causal(p.q, kHidden, kcl, vcl, kHidden, p.max_seqlen, p.att, kHidden, m, pos0, kHeads, st);
            if (rc) return rc;
            rc = launch_gemm_tc(p.att, kHidden, L.proj_w, kHidden, m, kHidden, kHidden, EpiResidual{p.x}, st);
            if (rc) return rc;
            rmsnorm_rows_k<<<m, 256, 0, st>>>(p.xn, p.x, L.ln2);
            rc = launch_gemm_tc(p.xn, kHidden, L.w12, kHidden, m, 2 * p.IM, kHidden, EpiSwiGLU{p.act, p.IM}, st);
            if (rc) return rc;
            rc = launch_gemm_tc(p.act, p.IM, L.cproj, p.IM, m, kHidden, p.IM, EpiResidual{p.x}, st);
            if (rc) return rc;
        }
        // the last row's residual stream is the engine's hidden state after this prompt
        e = cudaMemcpyAsync(p.hidden, p.x + (size_t)(m - 1) * kHidden, kHidden * sizeof(half),
                            cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return (int)e;
    }
    e = cudaGetLastError();
    return (int)e;
}

}  // namespace llmdiy
