// prefill_tc.cu — the prompt forward (QwenEngine::prefill, qwen_infer.cu:372-611)
// on the tensor cores: per layer
//   RMSNorm(ln_1) rows -> QKV GEMM [epilogue: bias, RoPE, K/V appended to the
//   cache, Q kept] -> causal flash attention over the cache (flash_prefill.cuh)
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
#include "flash_prefill.cuh"
#include "gemm_tc_host.h"
#include "ops.cuh"
#include "prefill_tc.h"

namespace llmdiy {
namespace {

__global__ void __launch_bounds__(256) embed_rows_k(const half* __restrict__ wte, const int* __restrict__ tokens,
                                                    half* __restrict__ x) {
    const int r = blockIdx.x, t = threadIdx.x;
    const half* src = wte + (size_t)tokens[r] * kHidden;
    *reinterpret_cast<uint4*>(x + (size_t)r * kHidden + 8 * t) = *reinterpret_cast<const uint4*>(src + 8 * t);
}

// out = half((x * r) * w) per row with the reference's reduction tree (rmsnorm.cuh:6-57)
__global__ void __launch_bounds__(256) rmsnorm_rows_k(half* __restrict__ out, const half* __restrict__ x,
                                                      const half* __restrict__ w) {
    __shared__ float red[17];
    const int r = blockIdx.x, t = threadIdx.x;
    const half* xr = x + (size_t)r * kHidden;
    const float s = rms_scale_tree256(xr, kHidden, 1e-6f, red, t, 1);
    float xf[8], wf[8], of[8];
    unpack8(*reinterpret_cast<const uint4*>(xr + 8 * t), xf);
    unpack8(*reinterpret_cast<const uint4*>(w + 8 * t), wf);
#pragma unroll
    for (int e = 0; e < 8; ++e) of[e] = (xf[e] * s) * wf[e];
    *reinterpret_cast<uint4*>(out + (size_t)r * kHidden + 8 * t) = pack8(of);
}

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

// x[row][n..n+15] = half(x + half(acc))  (the residual adds, bias.cuh:6-11)
struct EpiResidual {
    half* x;
    __device__ void operator()(int row, int n, const float* v) const {
        half* p = x + (size_t)row * kHidden + n;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            float xf[8], of[8];
            unpack8(*reinterpret_cast<const uint4*>(p + 8 * k), xf);
#pragma unroll
            for (int e = 0; e < 8; ++e) of[e] = xf[e] + h2f(f2h(v[8 * k + e]));
            *reinterpret_cast<uint4*>(p + 8 * k) = pack8(of);
        }
    }
};

// SwiGLU epilogue: columns (2u, 2u+1) = (w1 row u, w2 row u); act = half(g * up / (1 + e^-up))
// with g, up the fp16-rounded GEMM outputs (swiglu.cuh:6-15).
struct EpiSwiGLU {
    half* act;
    int IM;
    __device__ void operator()(int row, int n, const float* v) const {
        const int u0 = n >> 1;
        float of[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float g = h2f(f2h(v[2 * j])), up = h2f(f2h(v[2 * j + 1]));
            of[j] = g * __fdividef(up, 1.0f + __expf(-up));
        }
        half* dst = act + (size_t)row * IM + u0;
        if (u0 + 8 <= IM && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
            *reinterpret_cast<uint4*>(dst) = pack8(of);
        } else {
            for (int j = 0; j < 8 && u0 + j < IM; ++j) dst[j] = f2h(of[j]);
        }
    }
};

}  // namespace

int prefill_tc(const PrefillArgs& p, const int* tokens_dev, int n, int p0, cudaStream_t st) {
    int rc = 0;
    cudaError_t e;
    static std::once_flag attr;
    std::call_once(attr, [] {
        cudaFuncSetAttribute(flash_prefill_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(FlashPrefillSmem));
    });
    for (int c0 = 0; c0 < n; c0 += kPrefillChunk) {
        const int m = n - c0 < kPrefillChunk ? n - c0 : kPrefillChunk;
        const int pos0 = p0 + c0;
        embed_rows_k<<<m, 256, 0, st>>>(p.wte, tokens_dev + c0, p.x);
        for (int l = 0; l < p.NL; ++l) {
            const LayerPtrs& L = p.layers[l];
            half* kcl = p.kc + (size_t)l * p.max_seqlen * kHidden;
            half* vcl = p.vc + (size_t)l * p.max_seqlen * kHidden;
            rmsnorm_rows_k<<<m, 256, 0, st>>>(p.xn, p.x, L.ln1);
            rc = launch_gemm_tc(p.xn, kHidden, L.qkv_w, kHidden, m, 3 * kHidden, kHidden,
                                EpiQKV{L.qkv_b, p.q, kcl, vcl, pos0}, st);
            if (rc) return rc;
            flash_prefill_k<<<dim3((m + kFpRows - 1) / kFpRows, kHeads), kFpThreads, sizeof(FlashPrefillSmem), st>>>(
                p.q, kcl, vcl, p.att, m, pos0, kHidden, kHidden);
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
