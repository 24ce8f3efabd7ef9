// ops.cuh — device routines shared by the op-level launchers and the fused
// decode kernel.
#pragma once
#include "common.cuh"

namespace llmdiy {

// Reference RMSNorm scale (kernels/rmsnorm.cuh:6-57, blockDim 512), computed
// by 256 threads with the reference's exact summation tree:
//   * reference thread v (0..511) sums its ipt = d/512 contiguous squares with
//     an FMA chain; here thread u plays v = 2u and v = 2u+1;
//   * the reference's per-warp xor butterfly (masks 16..1 over the virtual
//     lane 2*(u%16)+b) becomes xor 8,4,2,1 over u plus the in-thread b add;
//   * warp 0's butterfly over the 16 warp sums (lanes 16..31 zero) is
//     replayed by one thread in the same pairing order.
// `x` may be shared or global memory; `red` is >= 17 floats of shared memory.
// Must be called by all 256 threads of the group identified by bar_id.
LLMDIY_DEV float rms_scale_tree256(const half* x, int d, float eps, float* red, int tid, int bar_id) {
    const int ipt = d / 512;
    float p0 = 0.f, p1 = 0.f;
    const half* a = x + (2 * tid) * ipt;
    const half* b = a + ipt;
    for (int i = 0; i < ipt; ++i) {
        float v = __half2float(a[i]);
        p0 = __fmaf_rn(v, v, p0);
    }
    for (int i = 0; i < ipt; ++i) {
        float v = __half2float(b[i]);
        p1 = __fmaf_rn(v, v, p1);
    }
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1) {
        p0 += __shfl_xor_sync(0xffffffffu, p0, m);
        p1 += __shfl_xor_sync(0xffffffffu, p1, m);
    }
    float s = p0 + p1;
    const int lane = tid & 31, warp = tid >> 5;
    if (lane == 0) red[2 * warp] = s;
    if (lane == 16) red[2 * warp + 1] = s;
    named_bar_sync(bar_id, 256);
    if (tid == 0) {
        float t[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) t[j] = red[j] + 0.0f;
#pragma unroll
        for (int m = 8; m >= 1; m >>= 1) {
            float u[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) u[j] = t[j] + t[j ^ m];
#pragma unroll
            for (int j = 0; j < 16; ++j) t[j] = u[j];
        }
        float var = __fdividef(t[0], (float)d);
        red[16] = rsqrtf(var + eps);
    }
    named_bar_sync(bar_id, 256);
    return red[16];
}

// rms_scale_tree256 for d = 2048 (same summation tree, same bits) with each
// thread's own eight elements (x[8*tid .. 8*tid+7], fp16 pairs in v) already
// in registers, and one barrier: after the per-warp stage every warp replays
// the final 16-value tree itself (lane j holds warp-sum j; the xor butterfly
// computes t[j] + t[j^m] exactly as the serial replay does) and takes lane
// 0's total.  `red` (>= 16 floats of shared memory) must not be rewritten
// before every warp has read it (the caller's next barrier orders that).
LLMDIY_DEV float rms_scale_regs2048(const uint4& v, float eps, float* red, int tid, int bar_id) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float p0 = 0.f, p1 = 0.f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        p0 = __fmaf_rn(f.x, f.x, p0);
        p0 = __fmaf_rn(f.y, f.y, p0);
    }
#pragma unroll
    for (int i = 2; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        p1 = __fmaf_rn(f.x, f.x, p1);
        p1 = __fmaf_rn(f.y, f.y, p1);
    }
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1) {
        p0 += __shfl_xor_sync(0xffffffffu, p0, m);
        p1 += __shfl_xor_sync(0xffffffffu, p1, m);
    }
    const float s = p0 + p1;
    const int lane = tid & 31, warp = tid >> 5;
    if (lane == 0) red[2 * warp] = s;
    if (lane == 16) red[2 * warp + 1] = s;
    named_bar_sync(bar_id, 256);
    float t = lane < 16 ? red[lane] + 0.0f : 0.f;
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1) t = t + __shfl_xor_sync(0xffffffffu, t, m);
    const float total = __shfl_sync(0xffffffffu, t, 0);
    return rsqrtf(__fdividef(total, 2048.0f) + eps);
}

// Online-softmax state of one attention partial: running max m (over scaled
// scores), running sum l, unnormalised output o.
struct SoftmaxState {
    float m, l;
};

// Merge (m2,l2,o2) into (m1,l1,o1); empty states carry m = -inf and l = 0.
LLMDIY_DEV void merge_state(float& m1, float& l1, float* o1, float m2, float l2, const float* o2, int n) {
    if (m2 == -INFINITY) return;
    if (m1 == -INFINITY) {
        m1 = m2; l1 = l2;
        for (int i = 0; i < n; ++i) o1[i] = o2[i];
        return;
    }
    float mn = fmaxf(m1, m2);
    float a = __expf(m1 - mn), b = __expf(m2 - mn);
    l1 = l1 * a + l2 * b;
    for (int i = 0; i < n; ++i) o1[i] = o1[i] * a + o2[i] * b;
    m1 = mn;
}

// Accumulate rows [r0, r1) of one head into a half-warp's online-softmax
// state.  Each of the 16 lanes of a half-warp owns 8 of the 128 dims (one
// 16-byte load per row); the two half-warps of a warp take alternate rows.
// K and V rows are `stride` halves apart.  q8 holds the lane's 8 q values.
// Rows are processed four per half-warp at a time so that eight 16-byte
// loads are in flight per lane.
template <bool kCacheGlobal>
LLMDIY_DEV void attend_rows(const half* __restrict__ K, const half* __restrict__ V, int stride, int r0, int r1,
                            const float* q8, float scale, float& m, float& l, float* o8) {
    const int lane = threadIdx.x & 31, hw = lane >> 4, dl = (lane & 15) * 8;
    // Batches of 8 rows per warp; the batch base b is warp-uniform so the
    // shuffles below always run with all 32 lanes.
    int b = r0;
    for (; b + 8 <= r1; b += 8) {
        uint4 kr[4], vr[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int r = b + 2 * j + hw;
            const half* kp = K + (size_t)r * stride + dl;
            const half* vp = V + (size_t)r * stride + dl;
            kr[j] = kCacheGlobal ? ld_cg_u4(kp) : ld_stream_u4(kp);
            vr[j] = kCacheGlobal ? ld_cg_u4(vp) : ld_stream_u4(vp);
        }
        float sc[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float kf[8];
            unpack8(kr[j], kf);
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) d = __fmaf_rn(q8[e], kf[e], d);
            sc[j] = d;
        }
#pragma unroll
        for (int mk = 8; mk >= 1; mk >>= 1)
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[j] += __shfl_xor_sync(0xffffffffu, sc[j], mk);
        float mx = m;
#pragma unroll
        for (int j = 0; j < 4; ++j) { sc[j] *= scale; mx = fmaxf(mx, sc[j]); }
        float corr = __expf(m - mx);
        l *= corr;
#pragma unroll
        for (int e = 0; e < 8; ++e) o8[e] *= corr;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float p = __expf(sc[j] - mx);
            l += p;
            float vf[8];
            unpack8(vr[j], vf);
#pragma unroll
            for (int e = 0; e < 8; ++e) o8[e] = __fmaf_rn(p, vf[e], o8[e]);
        }
        m = mx;
    }
    // Tail (< 8 rows): the loop bound depends only on warp-uniform values.
    for (int j = 0; b + 2 * j < r1; ++j) {
        const int rj = b + 2 * j + hw;
        const bool valid = rj < r1;
        float d = 0.f;
        uint4 vr = make_uint4(0, 0, 0, 0);
        if (valid) {
            const half* kp = K + (size_t)rj * stride + dl;
            const half* vp = V + (size_t)rj * stride + dl;
            uint4 kr = kCacheGlobal ? ld_cg_u4(kp) : ld_stream_u4(kp);
            vr = kCacheGlobal ? ld_cg_u4(vp) : ld_stream_u4(vp);
            float kf[8];
            unpack8(kr, kf);
#pragma unroll
            for (int e = 0; e < 8; ++e) d = __fmaf_rn(q8[e], kf[e], d);
        }
#pragma unroll
        for (int mk = 8; mk >= 1; mk >>= 1) d += __shfl_xor_sync(0xffffffffu, d, mk);
        if (valid) {
            float s = d * scale;
            float mx = fmaxf(m, s);
            float corr = __expf(m - mx);
            float p = __expf(s - mx);
            l = l * corr + p;
            float vf[8];
            unpack8(vr, vf);
#pragma unroll
            for (int e = 0; e < 8; ++e) o8[e] = __fmaf_rn(p, vf[e], o8[e] * corr);
            m = mx;
        }
    }
}

// Combine the two half-warp states of a warp (lanes l and l^16 own the same dims).
LLMDIY_DEV void combine_halfwarps(float& m, float& l, float* o8) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, 16);
    float l2 = __shfl_xor_sync(0xffffffffu, l, 16);
    float o2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o2[e] = __shfl_xor_sync(0xffffffffu, o8[e], 16);
    merge_state(m, l, o8, m2, l2, o2, 8);
}

}  // namespace llmdiy
