// fd_noalloc.cu — single-launch split-KV flash decoding whose scratch lives
// in a file-scope device array, so a call allocates nothing.
//
// It computes what llmdiy_fd_v5_split_stage1 followed by llmdiy_fd_opt_stage2
// compute (kernels/flash_decode_q1_opt.cuh:548-656 and :666-724): one query
// head of 128 dims against L cache rows, in chunks of 256 rows.  The chunk
// partials (fp16 output, LSE) go to g_fd_scratch instead of caller buffers,
// and the last CTA to finish merges them with the stage-2 arithmetic, in the
// same order, so the result is bit-identical to the two-launch pair.
//
// Scratch: one array shared by every call on a device.  The arrival counter
// must start at zero and is cleared on the call's stream before each launch;
// the partials need no clearing (each chunk writes its own before the merge
// reads it).  Two calls whose work overlaps on the GPU (different streams,
// no ordering between them) race on the array and give undefined results.
#include <cuda.h>

#include <mutex>

#include "ops.cuh"

using namespace llmdiy;

namespace {

constexpr int kNoAllocMaxChunks = 128;                        // 256 rows each
constexpr int kNoAllocMaxRows = kNoAllocMaxChunks * 256;      // 32768
constexpr size_t kOpartOff = 0;                               // half [chunks][128]
constexpr size_t kLseOff = kOpartOff + (size_t)kNoAllocMaxChunks * 128 * 2;  // float [chunks]
constexpr size_t kCounterOff = kLseOff + (size_t)kNoAllocMaxChunks * 4;      // unsigned int
constexpr size_t kScratchBytes = (kCounterOff + 4 + 255) / 256 * 256;        // 33,536 bytes

static __device__ __align__(256) unsigned char g_fd_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_ptr_mu;
void* g_ptr[kMaxDevices];                // cudaGetSymbolAddress(g_fd_scratch) per device
unsigned long long g_ctx_id[kMaxDevices];  // the context that address belongs to (0 = none yet)

__global__ void __launch_bounds__(256) fd_split_noalloc_k(const half* __restrict__ Q, const half* __restrict__ K,
                                                         const half* __restrict__ V, half* __restrict__ O, int L,
                                                         int stride, unsigned char* __restrict__ scratch) {
    __shared__ float sm[8], sl[8];
    __shared__ float so[8][128];
    __shared__ float red[4];
    __shared__ int is_last;
    half* opart = reinterpret_cast<half*>(scratch + kOpartOff);
    float* lse = reinterpret_cast<float*>(scratch + kLseOff);
    unsigned int* arrivals = reinterpret_cast<unsigned int*>(scratch + kCounterOff);
    const int nc = gridDim.x;

    // ---- stage 1: this CTA's 256-row chunk, 8 warps x 32 rows
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, dl = (lane & 15) * 8;
    float q8[8];
    unpack8(*reinterpret_cast<const uint4*>(Q + dl), q8);
    const float scale = __frcp_rn(sqrtf(128.0f));
    float m = -INFINITY, l = 0.f, o8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o8[e] = 0.f;
    int r0 = blockIdx.x * 256 + warp * 32, r1 = r0 + 32;
    if (r1 > L) r1 = L;
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
        opart[(size_t)blockIdx.x * 128 + d] = f2h(acc * __frcp_rn(Ls));
        if (d == 0) lse[blockIdx.x] = __logf(Ls) + M;
    }
    // publish the partial, then count arrivals; the last CTA merges
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = (atomicAdd(arrivals, 1u) == (unsigned)(nc - 1));
    __syncthreads();
    if (!is_last) return;
    __threadfence();

    // ---- stage 2 (last CTA, 128 threads): O = sum_c e^{LSE_c - M} Opart_c / sum_c e^{LSE_c - M}
    float mx = -INFINITY;
    if (threadIdx.x < 128)
        for (int c = threadIdx.x; c < nc; c += 128) mx = fmaxf(mx, __ldcg(lse + c));
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
    if (threadIdx.x < 128 && lane == 0) red[warp] = mx;
    __syncthreads();
    if (threadIdx.x < 128) {
        mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
        const int d = threadIdx.x;
        const unsigned short* op = reinterpret_cast<const unsigned short*>(opart);
        float sw = 0.f, acc = 0.f;
        for (int c = 0; c < nc; ++c) {
            float w = __expf(__ldcg(lse + c) - mx);
            sw += w;
            acc = __fmaf_rn(w, h2f(__ushort_as_half(__ldcg(op + (size_t)c * 128 + d))), acc);
        }
        O[d] = f2h(acc * __frcp_rn(sw));
    }
}

// The unique id of the calling thread's current CUDA context (cuCtxGetCurrent + cuCtxGetId,
// through the runtime's driver entry points), or 0 when there is none or the driver lacks them.
unsigned long long current_ctx_id() {
    using GetCurrent = CUresult (*)(CUcontext*);
    using GetId = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(p);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

// Device address of g_fd_scratch for the current device, looked up once per device and context:
// the first call on a device (and the first after cudaDeviceReset, whose new context gets a new id)
// does the lookup and must not be inside a stream capture; later calls reuse the address.
int scratch_ptr(unsigned char** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_ptr_mu);
    const unsigned long long id = current_ctx_id();
    if (!g_ptr[dev] || id == 0 || id != g_ctx_id[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_fd_scratch);
        if (e != cudaSuccess) return (int)e;
        g_ptr[dev] = p;
        g_ctx_id[dev] = current_ctx_id();  // the lookup made the device's context current if it was not
    }
    *out = static_cast<unsigned char*>(g_ptr[dev]);
    return 0;
}

}  // namespace

extern "C" int llmdiy_fd_split_noalloc(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O, int L,
                                       int stride, void* stream) {
    if (L > kNoAllocMaxRows) return -1;
    if (L <= 0 || (stride & 7) || (reinterpret_cast<uintptr_t>(Q) & 15) || (reinterpret_cast<uintptr_t>(K) & 15) ||
        (reinterpret_cast<uintptr_t>(V) & 15))
        return (int)cudaErrorInvalidValue;
    unsigned char* scratch = nullptr;
    int rc = scratch_ptr(&scratch);
    if (rc) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(scratch + kCounterOff, 0, sizeof(unsigned int), s);
    if (e != cudaSuccess) return (int)e;
    const int nc = (L + 255) / 256;
    fd_split_noalloc_k<<<nc, 256, 0, s>>>(reinterpret_cast<const half*>(Q), reinterpret_cast<const half*>(K),
                                          reinterpret_cast<const half*>(V), reinterpret_cast<half*>(O), L, stride,
                                          scratch);
    return (int)cudaGetLastError();
}
