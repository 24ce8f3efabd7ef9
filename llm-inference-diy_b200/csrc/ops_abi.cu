// ops_abi.cu — sm_100a kernels behind the reference's launch signatures.
//
// Each extern "C" launcher keeps the parameter list of the reference kernel
// it replaces (declared in include/llmdiy_kernels.h with the reference
// file:line), adds a trailing stream (NULL = legacy default stream, as the
// reference uses) and returns the cudaError_t of the launch.  Buffers are
// fp16 bit patterns (uint16_t) so the header needs no CUDA types.
#include "ops.cuh"

using namespace llmdiy;

namespace {

inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline int last_err() { return (int)cudaGetLastError(); }
__host__ __device__ inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- RMSNorm
// kernels/rmsnorm.cuh:6-57.  One CTA of 256 threads; bit-identical
// reduction tree (rms_scale_tree256), output half((x * r) * w).
__global__ void __launch_bounds__(256) rmsnorm_k(half* __restrict__ out, const half* __restrict__ in,
                                                  const half* __restrict__ w, int d, float eps) {
    __shared__ float red[17];
    const int tid = threadIdx.x;
    float r = rms_scale_tree256(in, d, eps, red, tid, 1);
    const int n = (d / 512) * 512;  // the reference writes only ipt*512 items
    if ((n & 7) == 0 && aligned16(in) && aligned16(w) && aligned16(out)) {
        for (int i = tid * 8; i < n; i += 256 * 8) {
            float xf[8], wf[8], of[8];
            unpack8(*reinterpret_cast<const uint4*>(in + i), xf);
            unpack8(*reinterpret_cast<const uint4*>(w + i), wf);
#pragma unroll
            for (int e = 0; e < 8; ++e) of[e] = (xf[e] * r) * wf[e];
            *reinterpret_cast<uint4*>(out + i) = pack8(of);
        }
    } else {
        for (int i = tid; i < n; i += 256) out[i] = f2h((h2f(in[i]) * r) * h2f(w[i]));
    }
}

// ---------------------------------------------------------------- bias / residual
// kernels/bias.cuh:6-11: out = half(out + b)
__global__ void add_bias_k(half* __restrict__ out, const half* __restrict__ b, int n, int vec) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        int j = i * 8;
        if (j + 8 <= n) {
            float of[8], bf[8];
            unpack8(*reinterpret_cast<const uint4*>(out + j), of);
            unpack8(*reinterpret_cast<const uint4*>(b + j), bf);
#pragma unroll
            for (int e = 0; e < 8; ++e) of[e] = of[e] + bf[e];
            *reinterpret_cast<uint4*>(out + j) = pack8(of);
        } else {
            for (; j < n; ++j) out[j] = f2h(h2f(out[j]) + h2f(b[j]));
        }
    } else if (i < n) {
        out[i] = f2h(h2f(out[i]) + h2f(b[i]));
    }
}

// ---------------------------------------------------------------- SwiGLU
// kernels/swiglu.cuh:6-15 (built with --use_fast_math): out = w1 * (w2 / (1 + exp(-w2)))
LLMDIY_DEV float swiglu1(float a, float b) { return a * __fdividef(b, 1.0f + __expf(-b)); }

__global__ void swiglu_k(half* __restrict__ out, const half* __restrict__ w1o, const half* __restrict__ w2o,
                         int n, int vec) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        int j = i * 8;
        if (j + 8 <= n) {
            float a[8], b[8];
            unpack8(*reinterpret_cast<const uint4*>(w1o + j), a);
            unpack8(*reinterpret_cast<const uint4*>(w2o + j), b);
#pragma unroll
            for (int e = 0; e < 8; ++e) a[e] = swiglu1(a[e], b[e]);
            *reinterpret_cast<uint4*>(out + j) = pack8(a);
        } else {
            for (; j < n; ++j) out[j] = f2h(swiglu1(h2f(w1o[j]), h2f(w2o[j])));
        }
    } else if (i < n) {
        out[i] = f2h(swiglu1(h2f(w1o[i]), h2f(w2o[i])));
    }
}

// ---------------------------------------------------------------- RoPE + KV append
// kernels/fused_qkv_rope_cache.cuh:6-55 with the Makefile's fast-math
// intrinsics (__powf/__cosf/__sinf).  One thread per (head, t) pair.
__global__ void rope_cache_k(half* __restrict__ qkv, half* __restrict__ kc, half* __restrict__ vc, int pos,
                             int num_heads, int head_dim) {
    const int half_dim = head_dim / 2;
    const int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= num_heads * half_dim) return;
    const int h = g / half_dim, t = g % half_dim;
    const int H = num_heads * head_dim;
    const int i1 = h * head_dim + t, i2 = i1 + half_dim;
    float q1 = h2f(qkv[i1]), q2 = h2f(qkv[i2]);
    float k1 = h2f(qkv[H + i1]), k2 = h2f(qkv[H + i2]);
    half v1 = qkv[2 * H + i1], v2 = qkv[2 * H + i2];
    float theta = (float)pos * __powf(10000.0f, __fdividef(-2.0f * (float)t, (float)head_dim));
    float c = __cosf(theta), s = __sinf(theta);
    qkv[i1] = f2h(q1 * c - q2 * s);
    qkv[i2] = f2h(q2 * c + q1 * s);
    const size_t off = (size_t)pos * H;
    kc[off + i1] = f2h(k1 * c - k2 * s);
    kc[off + i2] = f2h(k2 * c + k1 * s);
    vc[off + i1] = v1;
    vc[off + i2] = v2;
}

// ---------------------------------------------------------------- ArgMax
// kernels/argmax.cuh:7-72.  One CTA of 1024 threads computes the
// reference's winner directly from order keys (argmax_key), so the result is
// the reference's for every input, ties included.
__global__ void __launch_bounds__(1024) argmax_k(int* __restrict__ out, const half* __restrict__ logits, int V) {
    __shared__ unsigned long long wk[32];
    const int ipt = (V + 511) / 512;
    unsigned long long best = 0;
    const uint16_t* lg = reinterpret_cast<const uint16_t*>(logits);
    if ((V & 7) == 0 && aligned16(logits)) {
        for (int j = threadIdx.x * 8; j < V; j += 1024 * 8) {
            uint4 u = *reinterpret_cast<const uint4*>(lg + j);
            const uint16_t* h = reinterpret_cast<const uint16_t*>(&u);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                unsigned long long k = argmax_key(h[e], j + e, ipt);
                best = k > best ? k : best;
            }
        }
    } else {
        for (int j = threadIdx.x; j < V; j += 1024) {
            unsigned long long k = argmax_key(lg[j], j, ipt);
            best = k > best ? k : best;
        }
    }
    best = warp_max_u64(best);
    if ((threadIdx.x & 31) == 0) wk[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        best = warp_max_u64(wk[threadIdx.x]);
        if (threadIdx.x == 0) *out = argmax_key_index(best);
    }
}

// ---------------------------------------------------------------- GEMV, weight [K,N]
// kernels/hgemm_final.cuh:274-295: C[n] = half(sum_k A[k] * B[k*N+n]).
// One CTA per 32 output columns; 256 threads = 4 column groups of 8 x 64
// k-slices, 16-byte loads of B, fp32 partials reduced through shared memory.
__global__ void __launch_bounds__(256) hgemv_kn_k(const half* __restrict__ A, const half* __restrict__ B,
                                                   half* __restrict__ C, int N, int K) {
    __shared__ float part[64][33];
    const int cg = threadIdx.x & 3, ks = threadIdx.x >> 2;
    const int n0 = blockIdx.x * 32 + cg * 8;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    if (n0 < N) {
        for (int k = ks; k < K; k += 64) {
            float a = h2f(A[k]);
            float bf[8];
            unpack8(ld_stream_u4(B + (size_t)k * N + n0), bf);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(a, bf[e], acc[e]);
        }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) part[ks][cg * 8 + e] = acc[e];
    __syncthreads();
    if (threadIdx.x < 32) {
        const int n = blockIdx.x * 32 + threadIdx.x;
        float s = 0.f;
        for (int j = 0; j < 64; ++j) s += part[j][threadIdx.x];
        if (n < N) C[n] = f2h(s);
    }
}
// any N / alignment: one thread per column, sequential k (the reference's shape)
__global__ void hgemv_kn_scalar_k(const half* __restrict__ A, const half* __restrict__ B, half* __restrict__ C,
                                  int N, int K) {
    int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    float s = 0.f;
    for (int k = 0; k < K; ++k) s = __fmaf_rn(h2f(A[k]), h2f(B[(size_t)k * N + n]), s);
    C[n] = f2h(s);
}

// ---------------------------------------------------------------- flash decoding (one head)
// kernels/flash_decode_q1_opt.cuh:434-537 (fused, rows [0, min(L,256)))
// and :548-656 (split stage 1, 256 rows per CTA).  8 warps; each warp owns
// 32 consecutive rows like the reference, read with 16-byte loads by
// half-warps; the 8 warp states merge through shared memory.
template <bool kSplit>
__global__ void __launch_bounds__(256) fd_head_k(const half* __restrict__ Q, const half* __restrict__ K,
                                                  const half* __restrict__ V, half* __restrict__ O,
                                                  float* __restrict__ LSE, int L, int stride) {
    __shared__ float sm[8], sl[8];
    __shared__ float so[8][128];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, dl = (lane & 15) * 8;
    const int base = kSplit ? blockIdx.x * 256 : 0;
    const int lim = kSplit ? L : (L < 256 ? L : 256);
    float q8[8];
    unpack8(*reinterpret_cast<const uint4*>(Q + dl), q8);
    const float scale = __frcp_rn(sqrtf(128.0f));
    float m = -INFINITY, l = 0.f, o8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o8[e] = 0.f;
    int r0 = base + warp * 32, r1 = r0 + 32;
    if (r1 > lim) r1 = lim;
    if (r0 < r1) attend_rows<false>(K, V, stride, r0, r1, q8, scale, m, l, o8);
    combine_halfwarps(m, l, o8);
    if (lane < 16) {
#pragma unroll
        for (int e = 0; e < 8; ++e) so[warp][dl + e] = o8[e];
    }
    if (lane == 0) { sm[warp] = m; sl[warp] = l; }
    __syncthreads();
    if (threadIdx.x < 128) {
        const int d = threadIdx.x;
        float M = -INFINITY;
        for (int w = 0; w < 8; ++w) M = fmaxf(M, sm[w]);
        float Ls = 0.f, acc = 0.f;
        for (int w = 0; w < 8; ++w) {
            float c = (sm[w] == -INFINITY) ? 0.f : __expf(sm[w] - M);
            Ls += sl[w] * c;
            acc = __fmaf_rn(c, so[w][d], acc);
        }
        half* dst = kSplit ? O + (size_t)blockIdx.x * 128 : O;
        dst[d] = f2h(acc * __frcp_rn(Ls));
        if (kSplit && d == 0) LSE[blockIdx.x] = __logf(Ls) + M;
    }
}

// kernels/flash_decode_q1_opt.cuh:666-724: O = sum_c e^{LSE_c - M} Opart_c / sum_c e^{LSE_c - M}
__global__ void __launch_bounds__(128) fd_stage2_k(const half* __restrict__ Opart, const float* __restrict__ LSE,
                                                    half* __restrict__ O, int nc) {
    __shared__ float red[4];
    float mx = -INFINITY;
    for (int c = threadIdx.x; c < nc; c += 128) mx = fmaxf(mx, LSE[c]);
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const int d = threadIdx.x;
    float sw = 0.f, acc = 0.f;
    for (int c = 0; c < nc; ++c) {
        float w = __expf(LSE[c] - mx);
        sw += w;
        acc = __fmaf_rn(w, h2f(Opart[(size_t)c * 128 + d]), acc);
    }
    O[d] = f2h(acc * __frcp_rn(sw));
}

// ---------------------------------------------------------------- layout kernels
// kernels/transpose.cuh:6-30: out[c*rows + r] = in[r*cols + c]
__global__ void transpose_k(half* __restrict__ out, const half* __restrict__ in, int rows, int cols) {
    __shared__ half tile[32][34];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += 8) {
        int r = r0 + j, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[j][threadIdx.x] = in[(size_t)r * cols + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += 8) {
        int c = c0 + j, r = r0 + threadIdx.x;
        if (r < rows && c < cols) out[(size_t)c * rows + r] = tile[threadIdx.x][j];
    }
}

// kernels/gather_qkv.cuh:14-60: [N, cols] (heads interleaved) <-> [nh*N, 128]
// moved in 16-byte units (16 per 128-wide head row).
__global__ void gather_k(const half* __restrict__ src, half* __restrict__ dst, int N, int nh, int src_cols) {
    long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long total = (long long)N * nh * 16;
    if (u >= total) return;
    int seg = (int)(u % 16), h = (int)((u / 16) % nh), row = (int)(u / (16LL * nh));
    const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)row * src_cols + h * 128 + seg * 8);
    *reinterpret_cast<uint4*>(dst + ((size_t)h * N + row) * 128 + seg * 8) = *s;
}
__global__ void scatter_k(const half* __restrict__ src, half* __restrict__ dst, int N, int nh, int dst_cols) {
    long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long total = (long long)N * nh * 16;
    if (u >= total) return;
    int seg = (int)(u % 16), h = (int)((u / 16) % nh), row = (int)(u / (16LL * nh));
    *reinterpret_cast<uint4*>(dst + (size_t)row * dst_cols + h * 128 + seg * 8) =
        *reinterpret_cast<const uint4*>(src + ((size_t)h * N + row) * 128 + seg * 8);
}

}  // namespace

#define H(p) reinterpret_cast<half*>(p)
#define CH(p) reinterpret_cast<const half*>(p)

extern "C" {

int llmdiy_rmsnorm(uint16_t* out, const uint16_t* in, const uint16_t* weight, int d, float eps, void* stream) {
    if (d < 512) return (int)cudaErrorInvalidValue;
    rmsnorm_k<<<1, 256, 0, S(stream)>>>(H(out), CH(in), CH(weight), d, eps);
    return last_err();
}

int llmdiy_add_bias(uint16_t* out, const uint16_t* bias, int size, void* stream) {
    if (size <= 0) return 0;
    int vec = aligned16(out) && aligned16(bias);
    int threads = 256, items = vec ? (size + 7) / 8 : size;
    add_bias_k<<<(items + threads - 1) / threads, threads, 0, S(stream)>>>(H(out), CH(bias), size, vec);
    return last_err();
}

int llmdiy_swiglu(uint16_t* out, const uint16_t* w1o, const uint16_t* w2o, int size, void* stream) {
    if (size <= 0) return 0;
    int vec = aligned16(out) && aligned16(w1o) && aligned16(w2o);
    int threads = 256, items = vec ? (size + 7) / 8 : size;
    swiglu_k<<<(items + threads - 1) / threads, threads, 0, S(stream)>>>(H(out), CH(w1o), CH(w2o), size, vec);
    return last_err();
}

int llmdiy_fused_qkv_rope_cache(uint16_t* qkv, uint16_t* kc, uint16_t* vc, int pos, int max_seqlen, int num_heads,
                                int head_dim, void* stream) {
    if (pos < 0 || pos >= max_seqlen || (head_dim & 1)) return (int)cudaErrorInvalidValue;
    int n = num_heads * head_dim / 2;
    rope_cache_k<<<(n + 255) / 256, 256, 0, S(stream)>>>(H(qkv), H(kc), H(vc), pos, num_heads, head_dim);
    return last_err();
}

int llmdiy_argmax(int* out, const uint16_t* logits, int V, void* stream) {
    if (V <= 0) return (int)cudaErrorInvalidValue;
    argmax_k<<<1, 1024, 0, S(stream)>>>(out, CH(logits), V);
    return last_err();
}

int llmdiy_hgemv(const uint16_t* A, const uint16_t* B, uint16_t* C, int N, int K, void* stream) {
    if (N <= 0 || K <= 0) return 0;
    if ((N & 7) == 0 && aligned16(B))
        hgemv_kn_k<<<(N + 31) / 32, 256, 0, S(stream)>>>(CH(A), CH(B), H(C), N, K);
    else
        hgemv_kn_scalar_k<<<(N + 255) / 256, 256, 0, S(stream)>>>(CH(A), CH(B), H(C), N, K);
    return last_err();
}

int llmdiy_fd_v5_fused(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O, int L, int stride,
                       void* stream) {
    if (L <= 0 || (stride & 7) || !aligned16(Q) || !aligned16(K) || !aligned16(V)) return (int)cudaErrorInvalidValue;
    fd_head_k<false><<<1, 256, 0, S(stream)>>>(CH(Q), CH(K), CH(V), H(O), nullptr, L, stride);
    return last_err();
}

int llmdiy_fd_v5_split_stage1(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* Opart, float* LSE,
                              int L, int num_chunks, int stride, void* stream) {
    if (L <= 0 || num_chunks <= 0 || (stride & 7) || !aligned16(Q) || !aligned16(K) || !aligned16(V))
        return (int)cudaErrorInvalidValue;
    fd_head_k<true><<<num_chunks, 256, 0, S(stream)>>>(CH(Q), CH(K), CH(V), H(Opart), LSE, L, stride);
    return last_err();
}

int llmdiy_fd_opt_stage2(const uint16_t* Opart, const float* LSE, uint16_t* O, int num_chunks, void* stream) {
    if (num_chunks <= 0) return (int)cudaErrorInvalidValue;
    fd_stage2_k<<<1, 128, 0, S(stream)>>>(CH(Opart), LSE, H(O), num_chunks);
    return last_err();
}

int llmdiy_transpose_weight(uint16_t* out, const uint16_t* in, int rows, int cols, void* stream) {
    dim3 block(32, 8), grid((cols + 31) / 32, (rows + 31) / 32);
    transpose_k<<<grid, block, 0, S(stream)>>>(H(out), CH(in), rows, cols);
    return last_err();
}

// kernels/transpose.cuh:17-30: allocate, transpose, free the old buffer, swap.
int llmdiy_transpose_weight_gpu(uint16_t** w, int rows, int cols) {
    uint16_t* t = nullptr;
    cudaError_t e = cudaMalloc(&t, (size_t)rows * cols * sizeof(uint16_t));
    if (e != cudaSuccess) return (int)e;
    int r = llmdiy_transpose_weight(t, *w, rows, cols, nullptr);
    if (r) { cudaFree(t); return r; }
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { cudaFree(t); return (int)e; }
    cudaFree(*w);
    *w = t;
    return 0;
}

int llmdiy_gather_q_from_qkv(const uint16_t* qkv, uint16_t* buf, int N, int num_heads, int head_dim, void* stream) {
    if (head_dim != 128 || !aligned16(qkv) || !aligned16(buf)) return (int)cudaErrorInvalidValue;
    long long total = (long long)N * num_heads * 16;
    gather_k<<<(unsigned)((total + 255) / 256), 256, 0, S(stream)>>>(CH(qkv), H(buf), N, num_heads, num_heads * 128 * 3);
    return last_err();
}

int llmdiy_gather_kv_from_cache(const uint16_t* cache, uint16_t* buf, int N, int num_heads, int head_dim, void* stream) {
    if (head_dim != 128 || !aligned16(cache) || !aligned16(buf)) return (int)cudaErrorInvalidValue;
    long long total = (long long)N * num_heads * 16;
    gather_k<<<(unsigned)((total + 255) / 256), 256, 0, S(stream)>>>(CH(cache), H(buf), N, num_heads, num_heads * 128);
    return last_err();
}

int llmdiy_scatter_interleaved(const uint16_t* src, uint16_t* dst, int N, int num_heads, int dst_cols, void* stream) {
    if (!aligned16(src) || !aligned16(dst) || (dst_cols & 7)) return (int)cudaErrorInvalidValue;
    long long total = (long long)N * num_heads * 16;
    scatter_k<<<(unsigned)((total + 255) / 256), 256, 0, S(stream)>>>(CH(src), H(dst), N, num_heads, dst_cols);
    return last_err();
}

}  // extern "C"
