// flash_prefill.cuh — causal flash attention for the prefill (kernels/flash_attn.cu:1854-2179
// computes the same quantity per head with its own tiling): query rows at
// positions p0 .. p0+n-1 of one head attend cache rows [0, pos].
//
// CTA = 4 warps x 16 query rows (64 rows) of one head; K/V tiles of 64 keys
// stream through a double-buffered shared-memory ring (cp.async, 16-byte
// chunks XOR-swizzled by row so ldmatrix is conflict-free).  Per warp and key
// tile: S = Q K^T (m16n8k16, fp16 in, fp32 accumulate), online softmax on the
// accumulator fragments (scale 1/sqrt(128), __expf), P reused in registers as
// the A operand of O += P V (V fragments by ldmatrix.trans).
#pragma once
#include "decode.h"
#include "ops.cuh"

namespace llmdiy {

constexpr int kFpRows = 64;  // query rows per CTA
constexpr int kFpKeys = 64;  // keys per tile
constexpr int kFpThreads = 128;

struct FlashPrefillSmem {
    half k[2][kFpKeys * kHeadDim];
    half v[2][kFpKeys * kHeadDim];
};

LLMDIY_DEV uint32_t fp_swz(int row, int chunk) {  // byte offset of 16-byte chunk `chunk` of row `row`
    return (uint32_t)(row * 256 + ((chunk ^ (row & 7)) << 4));
}
LLMDIY_DEV void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
LLMDIY_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
LLMDIY_DEV void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
LLMDIY_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
LLMDIY_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
LLMDIY_DEV void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
LLMDIY_DEV uint32_t pack_h2(float lo, float hi) {
    const half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// q: [n][ldq] rows of the prompt (head h at h*128); kc, vc: cache [rows][ldkv];
// att: [n][ldq].  Grid (ceil(n/64), heads); the x index runs longest tiles first.
static __global__ void __launch_bounds__(kFpThreads) flash_prefill_k(const half* __restrict__ q, const half* __restrict__ kc,
                                                             const half* __restrict__ vc, half* __restrict__ att,
                                                             int n, int p0, int ldq, int ldkv) {
    extern __shared__ __align__(128) uint8_t fp_smem_raw[];
    FlashPrefillSmem& s = *reinterpret_cast<FlashPrefillSmem*>(fp_smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    const int h = blockIdx.y;
    const int qt = (int)gridDim.x - 1 - (int)blockIdx.x;
    const int i0 = qt * kFpRows;
    const int last_pos = p0 + min(n, i0 + kFpRows) - 1;  // largest key any row of the tile needs
    const int ntiles = last_pos / kFpKeys + 1;
    const half* kh = kc + h * kHeadDim;
    const half* vh = vc + h * kHeadDim;

    auto load_tile = [&](int kt, int buf) {
        // 64 keys x 16 chunks of K and of V: 8 + 8 copies per thread
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = tid + i * kFpThreads, r = idx >> 4, c = idx & 15;
            int key = kt * kFpKeys + r;
            key = key <= last_pos ? key : last_pos;  // rows past the last needed key are masked anyway
            cp_async16(reinterpret_cast<uint8_t*>(s.k[buf]) + fp_swz(r, c), kh + (size_t)key * ldkv + 8 * c);
            cp_async16(reinterpret_cast<uint8_t*>(s.v[buf]) + fp_swz(r, c), vh + (size_t)key * ldkv + 8 * c);
        }
        cp_async_commit();
    };
    load_tile(0, 0);

    // Q fragments of this warp's 16 rows (A operand, 8 k-steps of 16 dims)
    const int rA = min(i0 + warp * 16 + g, n - 1), rB = min(i0 + warp * 16 + g + 8, n - 1);
    uint32_t qa[8][4];
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
        const half* pa = q + (size_t)rA * ldq + h * kHeadDim + ks * 16 + 2 * t4;
        const half* pb = q + (size_t)rB * ldq + h * kHeadDim + ks * 16 + 2 * t4;
        qa[ks][0] = *reinterpret_cast<const uint32_t*>(pa);
        qa[ks][1] = *reinterpret_cast<const uint32_t*>(pb);
        qa[ks][2] = *reinterpret_cast<const uint32_t*>(pa + 8);
        qa[ks][3] = *reinterpret_cast<const uint32_t*>(pb + 8);
    }
    const int posA = p0 + i0 + warp * 16 + g, posB = posA + 8;
    const float scale = __frcp_rn(sqrtf((float)kHeadDim));
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;

    for (int kt = 0; kt < ntiles; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < ntiles) {
            load_tile(kt + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const uint32_t kbase = smem_u32(s.k[buf]), vbase = smem_u32(s.v[buf]);
        // ---- S = Q K^T: 8 key blocks of 8
        float sc[8][4];
#pragma unroll
        for (int nb = 0; nb < 8; ++nb) {
            sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.f;
#pragma unroll
            for (int kp = 0; kp < 4; ++kp) {  // pairs of k-steps (32 dims) per ldmatrix.x4
                uint32_t b0, b1, b2, b3;
                const int r = nb * 8 + (lane & 7), c = kp * 4 + (lane >> 3);
                ldsm_x4(kbase + fp_swz(r, c), b0, b1, b2, b3);
                mma16816(sc[nb], qa[2 * kp][0], qa[2 * kp][1], qa[2 * kp][2], qa[2 * kp][3], b0, b1);
                mma16816(sc[nb], qa[2 * kp + 1][0], qa[2 * kp + 1][1], qa[2 * kp + 1][2], qa[2 * kp + 1][3], b2, b3);
            }
        }
        // ---- online softmax (rows A = g, B = g + 8 of the warp's 16)
        float mxA = mA, mxB = mB;
#pragma unroll
        for (int nb = 0; nb < 8; ++nb) {
            const int key = kt * kFpKeys + nb * 8 + 2 * t4;
            sc[nb][0] = key <= posA ? sc[nb][0] * scale : -INFINITY;
            sc[nb][1] = key + 1 <= posA ? sc[nb][1] * scale : -INFINITY;
            sc[nb][2] = key <= posB ? sc[nb][2] * scale : -INFINITY;
            sc[nb][3] = key + 1 <= posB ? sc[nb][3] * scale : -INFINITY;
            mxA = fmaxf(mxA, fmaxf(sc[nb][0], sc[nb][1]));
            mxB = fmaxf(mxB, fmaxf(sc[nb][2], sc[nb][3]));
        }
        mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
        mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
        mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
        mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
        const float cA = mA == -INFINITY ? 0.f : __expf(mA - mxA);
        const float cB = mB == -INFINITY ? 0.f : __expf(mB - mxB);
        mA = mxA;
        mB = mxB;
        float sA = 0.f, sB = 0.f;
        uint32_t pa[4][4];  // P as A fragments: 4 k-steps of 16 keys
#pragma unroll
        for (int nb = 0; nb < 8; ++nb) {
            const float p0v = mxA == -INFINITY ? 0.f : __expf(sc[nb][0] - mxA);
            const float p1v = mxA == -INFINITY ? 0.f : __expf(sc[nb][1] - mxA);
            const float p2v = mxB == -INFINITY ? 0.f : __expf(sc[nb][2] - mxB);
            const float p3v = mxB == -INFINITY ? 0.f : __expf(sc[nb][3] - mxB);
            sA += p0v + p1v;
            sB += p2v + p3v;
            const int kk = nb >> 1, hi = nb & 1;
            pa[kk][hi ? 2 : 0] = pack_h2(p0v, p1v);
            pa[kk][hi ? 3 : 1] = pack_h2(p2v, p3v);
        }
        sA += __shfl_xor_sync(0xffffffffu, sA, 1);
        sA += __shfl_xor_sync(0xffffffffu, sA, 2);
        sB += __shfl_xor_sync(0xffffffffu, sB, 1);
        sB += __shfl_xor_sync(0xffffffffu, sB, 2);
        lA = lA * cA + sA;
        lB = lB * cB + sB;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            o[j][0] *= cA;
            o[j][1] *= cA;
            o[j][2] *= cB;
            o[j][3] *= cB;
        }
        // ---- O += P V: 16 dim blocks of 8, 4 key steps of 16
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int dp = 0; dp < 8; ++dp) {  // pairs of dim blocks per ldmatrix.x4.trans
                uint32_t b0, b1, b2, b3;
                const int r = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), c = dp * 2 + (lane >> 4);
                ldsm_x4_t(vbase + fp_swz(r, c), b0, b1, b2, b3);
                mma16816(o[2 * dp], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
                mma16816(o[2 * dp + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
            }
        }
        __syncthreads();  // the buffer is refilled by the next iteration's load
    }
    // ---- normalise and store rows A and B
    const int iA = i0 + warp * 16 + g, iB = iA + 8;
    const float invA = __frcp_rn(lA), invB = __frcp_rn(lB);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int d = h * kHeadDim + j * 8 + 2 * t4;
        if (iA < n) *reinterpret_cast<uint32_t*>(att + (size_t)iA * ldq + d) = pack_h2(o[j][0] * invA, o[j][1] * invA);
        if (iB < n) *reinterpret_cast<uint32_t*>(att + (size_t)iB * ldq + d) = pack_h2(o[j][2] * invB, o[j][3] * invB);
    }
}

}  // namespace llmdiy
