// rows.cuh — row-wise kernels and GEMM epilogue ops shared by the prompt
// forward (prefill_tc.cu) and the batched decode (batch.cu): embedding rows,
// RMSNorm rows with the reference's reduction tree, and the residual / SwiGLU
// epilogues of the tcgen05 GEMM (fp16 rounding points of the decode kernel).
#pragma once
#include "decode.h"
#include "ops.cuh"

namespace llmdiy {

static __global__ void __launch_bounds__(256) embed_rows_k(const half* __restrict__ wte, const int* __restrict__ tokens,
                                                    half* __restrict__ x) {
    const int r = blockIdx.x, t = threadIdx.x;
    pdl_wait();
    pdl_launch_dependents();
    const half* src = wte + (size_t)tokens[r] * kHidden;
    *reinterpret_cast<uint4*>(x + (size_t)r * kHidden + 8 * t) = *reinterpret_cast<const uint4*>(src + 8 * t);
}

// out = half((x * r) * w) per row with the reference's reduction tree (rmsnorm.cuh:6-57)
static __global__ void __launch_bounds__(256) rmsnorm_rows_k(half* __restrict__ out, const half* __restrict__ x,
                                                      const half* __restrict__ w) {
    __shared__ float red[17];
    const int r = blockIdx.x, t = threadIdx.x;
    const uint4 wv = *reinterpret_cast<const uint4*>(w + 8 * t);  // weights: no dependence on earlier kernels
    pdl_wait();
    pdl_launch_dependents();
    const uint4 v = *reinterpret_cast<const uint4*>(x + (size_t)r * kHidden + 8 * t);  // this thread's 8 values
    const float s = rms_scale_regs2048(v, 1e-6f, red, t, 1);
    float xf[8], wf[8], of[8];
    unpack8(v, xf);
    unpack8(wv, wf);
#pragma unroll
    for (int e = 0; e < 8; ++e) of[e] = (xf[e] * s) * wf[e];
    *reinterpret_cast<uint4*>(out + (size_t)r * kHidden + 8 * t) = pack8(of);
}

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

}  // namespace llmdiy
