// fd_multihead.cu — multi-head split-KV flash decoding (one query token).
//
// The reference attends one head per launch (fd_v5_split_stage1_kernel +
// fd_opt_stage2_kernel, kernels/flash_decode_q1_opt.cuh:548-724, launched per
// head at qwen_infer.cu:650-677).  Here all heads and all KV positions go in
// one launch: CTA (split, head) streams its rows of K and V for that head
// through a 4-stage shared-memory pipeline of 64-row TMA tiles (2-D tensor
// maps over the [L][stride] cache, box 128 x 64), keeps an online softmax
// state per half-warp, and writes its unnormalised partial (o[128], m, l) in
// fp32.  A second kernel merges each head's partials (log-sum-exp) into the
// fp16 output or into one fp32 partial per head — the form the multi-GPU path
// exchanges (over peer memory with fd_p2p_merge_k, or by an NCCL all-gather)
// before the final merge of the shards' partials.
//
// Short caches (L <= 2048 rows) take a single launch instead: one thread-block
// cluster of 8 CTAs per head (fd_cluster_k), each CTA reading its share of the
// head's rows with 16-byte loads straight into registers (sixteen in flight per
// lane) and reducing them to a partial, then CTA 0 of the cluster merging the 8
// partials through distributed shared memory.  No global scratch, no memset, no
// second kernel.
#include <cooperative_groups.h>
#include <cuda.h>
#include <algorithm>
#include <cstring>
#include <mutex>

#include "llmdiy_kernels.h"
#include "ops.cuh"

using namespace llmdiy;

namespace {

constexpr int kFdHeadDim = 128;
constexpr int kFdRows = 64;  // rows per TMA tile
constexpr int kFdStages = 3;    // K/V tiles in flight per CTA; two CTAs share an SM (6 per SM)
constexpr int kFdCtasPerSm = 2;
constexpr int kFdThreads = 128;  // 4 warps x 16 rows of a tile
constexpr int kFdPart = kFdHeadDim + 2;
constexpr int kFdTileBytes = kFdRows * kFdHeadDim * 2;

constexpr int kFdMergeMax = 1024;  // most partials one merge combines

struct FdSmem {
    half k[kFdStages][kFdRows * kFdHeadDim];
    half v[kFdStages][kFdRows * kFdHeadDim];
    uint64_t full[kFdStages];
    float so[4][kFdHeadDim];
    float sm[4], sl[4];
};

// Log-sum-exp merge of n partials of one head by the 128 threads of a CTA, in
// order j = 0..n-1: O = sum_j e^{m_j - M} o_j / sum_j e^{m_j - M} l_j.  Partial
// j is at p + j * jstride (floats).  Partials are staged through shared memory
// (`scratch`, cap floats) in batches with coalesced, independent loads, so a
// batch costs one L2 round trip.  Writes the fp16 output and/or the merged
// fp32 partial (o unnormalised, M, L).
__device__ __forceinline__ void fd_merge_head(const float* p, int n, int jstride, float* scratch, int cap,
                                              float* red, half* O, float* out_part) {
    const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
    float mx = -INFINITY;
    for (int j = d; j < n; j += kFdHeadDim) mx = fmaxf(mx, __ldcg(p + (size_t)j * jstride + kFdHeadDim));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    const float M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const int per = cap / kFdPart;
    float Ls = 0.f, acc = 0.f;
    for (int j0 = 0; j0 < n; j0 += per) {
        const int nb = min(per, n - j0);
#pragma unroll 4
        for (int i = d; i < nb * kFdPart; i += kFdHeadDim) {
            const int j = i / kFdPart, e = i - j * kFdPart;
            scratch[i] = __ldcg(p + (size_t)(j0 + j) * jstride + e);
        }
        __syncthreads();
        for (int j = 0; j < nb; ++j) {
            const float mj = scratch[j * kFdPart + kFdHeadDim];
            const float f = mj == -INFINITY ? 0.f : __expf(mj - M);
            Ls = __fmaf_rn(scratch[j * kFdPart + kFdHeadDim + 1], f, Ls);
            acc = __fmaf_rn(f, scratch[j * kFdPart + d], acc);
        }
        __syncthreads();
    }
    if (O) O[d] = f2h(acc * __frcp_rn(Ls));
    if (out_part) {
        out_part[d] = acc;
        if (d == 0) { out_part[kFdHeadDim] = M; out_part[kFdHeadDim + 1] = Ls; }
    }
}

// Exchange + merge over peer memory (one CTA per head): push this rank's partial of head h into
// slot `rank` of every rank's buffer as flag-carrying 8-byte words (the fp32 value in the low half,
// the call's tag in the high half, one single-copy-atomic store each: no fence and no separate
// flag), poll the world's words of head h in the own buffer until every one carries the tag, then
// merge the world's partials in rank order.
//
// Each buffer holds two regions of [world][H][130] words, and call `tag` uses region (tag & 1).  A
// rank that has finished call t saw every rank's call-t words, and a rank writes those only after
// its own call t-1 kernel (same stream) has finished merging; so the earliest next write into a
// region, call t+1's, lands after every reader of call t-1 in that region is done, while call t's
// region may still be read.  One region would let a fast rank's call t+1 overwrite a slot that a
// slower rank's call t merge is still reading.
constexpr uint32_t kP2pPollLimit = 1u << 20;  // about a second of polling
constexpr int kP2pMaxWorld = 16;              // ranks one exchange merges (shared-memory staging)
constexpr int kP2pStage = 40;                 // partials staged per pass (the split merge: one pass up to 40 splits)

__host__ __device__ inline size_t p2p_region_words(int world, int H) { return (size_t)world * H * kFdPart; }

// One head's exchange by the 128 threads of a CTA (a CTA-uniform call): merge the head's S split
// partials (part_h = [S][130]; S = 1: already merged, the merge is then exact), push the result as
// tagged words into slot `rank` of every rank's buffer, wait (bounded) until every rank's words of
// head h in the own buffer carry the tag, and merge them in rank order into O[h].  scratch holds
// `cap` >= kP2pMaxWorld * 130 floats.  Returns false (and sets *err) when the wait expired.
__device__ bool exchange_head(const float* part_h, int S, const unsigned long long* __restrict__ peers, int world,
                              int rank, int H, int h, uint32_t tag, half* __restrict__ O, int* err, float* scratch,
                              int cap, float* red, float* mine) {
    const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
    const size_t region = (tag & 1u) * p2p_region_words(world, H);  // words before this call's region
    fd_merge_head(part_h, S, kFdPart, scratch, cap, red, nullptr, mine);
    __syncthreads();
    const unsigned long long hi = (unsigned long long)tag << 32;
    for (int p = 0; p < world; ++p) {
        unsigned long long* dst = reinterpret_cast<unsigned long long*>(peers[p]) + region + ((size_t)rank * H + h) * kFdPart;
        for (int i = d; i < kFdPart; i += kFdHeadDim) {
            const unsigned long long w = hi | __float_as_uint(mine[i]);
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst + i), "l"(w) : "memory");
        }
    }
    // every word of head h from every rank, polled in the own buffer: thread d takes element d of
    // each rank (and threads 0, 1 elements 128, 129)
    const unsigned long long* own = reinterpret_cast<const unsigned long long*>(peers[rank]) + region;
    const int per = d < kFdPart - kFdHeadDim ? 2 : 1;
    uint32_t pending = world * per >= 32 ? 0xffffffffu : (1u << (world * per)) - 1u;  // bit j * per + k: rank j, element d + 128 k
    for (uint32_t it = 0; pending && it < kP2pPollLimit; ++it) {
        for (int j = 0; j < world; ++j) {
            for (int k = 0; k < per; ++k) {
                const uint32_t bit = 1u << (j * per + k);
                if (!(pending & bit)) continue;
                const int e = d + k * kFdHeadDim;
                unsigned long long w;
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];"
                             : "=l"(w)
                             : "l"(own + ((size_t)j * H + h) * kFdPart + e)
                             : "memory");
                if ((uint32_t)(w >> 32) == tag) {
                    scratch[j * kFdPart + e] = __uint_as_float((uint32_t)w);
                    pending &= ~bit;
                }
            }
        }
        if (pending && it > 64) __nanosleep(64);
    }
    if (!__syncthreads_and(pending == 0)) {
        if (d == 0) atomicExch(err, 1);
        return false;
    }
    // merge in rank order (fd_merge_head's arithmetic, from shared memory)
    float mx = -INFINITY;
    for (int j = d; j < world; j += kFdHeadDim) mx = fmaxf(mx, scratch[j * kFdPart + kFdHeadDim]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    const float M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    float Ls = 0.f, acc = 0.f;
    for (int j = 0; j < world; ++j) {
        const float mj = scratch[j * kFdPart + kFdHeadDim];
        const float f = mj == -INFINITY ? 0.f : __expf(mj - M);
        Ls = __fmaf_rn(scratch[j * kFdPart + kFdHeadDim + 1], f, Ls);
        acc = __fmaf_rn(f, scratch[j * kFdPart + d], acc);
    }
    O[(size_t)h * kFdHeadDim + d] = f2h(acc * __frcp_rn(Ls));
    return true;
}

// The exchange alone, one CTA per head, on partials already in memory ([H][S][130]).
__global__ void __launch_bounds__(kFdHeadDim) fd_p2p_merge_k(const float* __restrict__ part, int S,
                                                             const unsigned long long* __restrict__ peers, int world,
                                                             int rank, int H, uint32_t tag, half* __restrict__ O,
                                                             int* err) {
    static_assert(kP2pStage >= kP2pMaxWorld, "the rank merge stages every rank at once");
    __shared__ float scratch[kP2pStage * kFdPart];
    __shared__ float red[4];
    __shared__ float mine[kFdPart];
    const int h = blockIdx.x;
    (void)exchange_head(part + (size_t)h * S * kFdPart, S, peers, world, rank, H, h, tag, O, err, scratch,
                        kP2pStage * kFdPart, red, mine);
}

// Persistent: CTA b takes work items (head, split) b, b + grid, ... and its
// TMA pipeline runs across item boundaries, so the next item's tiles are
// already in flight when one item ends.  Item i: head i / S, split i % S,
// rows [split * rows_per_split, min(L, (split + 1) * rows_per_split)).
struct FdCursor {
    int item, tile, ntiles, r0;  // current item, tile within it, its tile count and first row
};

__device__ __forceinline__ void fd_item(int item, int S, int L, int rows_per_split, FdCursor& c) {
    c.item = item;
    c.tile = 0;
    const int sp = item % S;
    c.r0 = sp * rows_per_split;
    const int r1 = min(L, c.r0 + rows_per_split);
    c.ntiles = r1 > c.r0 ? (r1 - c.r0 + kFdRows - 1) / kFdRows : 0;
}

__global__ void __launch_bounds__(kFdThreads, kFdCtasPerSm)
    fd_partials_k(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                  const half* __restrict__ Q, int L, int S, int H, int rows_per_split, float* __restrict__ part,
                  int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    FdSmem& s = *reinterpret_cast<FdSmem*>(smem_raw);
    const int tid = threadIdx.x, G = gridDim.x, nitems = S * H;
    const int warp = tid >> 5, lane = tid & 31, hw = lane >> 4, dl = (lane & 15) * 8;
    const uint64_t pol = l2_policy_evict_first();
    if (tid == 0) {
        for (int i = 0; i < kFdStages; ++i) mbar_init(&s.full[i], 1);
        mbar_fence_init();
    }
    __syncthreads();
    // producer cursor (thread 0) and the count of tiles issued / consumed in this CTA's sequence
    FdCursor pc;
    fd_item(blockIdx.x, S, L, rows_per_split, pc);
    uint32_t issued = 0, consumed = 0;
    auto produce = [&]() {  // issue the next tile of the sequence, if any
        while (pc.item < nitems && pc.tile >= pc.ntiles) fd_item(pc.item + G, S, L, rows_per_split, pc);
        if (pc.item >= nitems) return;
        const int st = issued % kFdStages, h = pc.item / S, y = pc.r0 + pc.tile * kFdRows;
        mbar_arrive_expect_tx(&s.full[st], 2 * kFdTileBytes);
        tma_load_2d_hint(s.k[st], &tk, h * kFdHeadDim, y, &s.full[st], pol);
        tma_load_2d_hint(s.v[st], &tv, h * kFdHeadDim, y, &s.full[st], pol);
        ++pc.tile;
        ++issued;
    };
    if (tid == 0)
        for (int i = 0; i < kFdStages; ++i) produce();
    const float scale = __frcp_rn(sqrtf((float)kFdHeadDim));
    bool failed = false;
    for (int item = blockIdx.x; item < nitems && !failed; item += G) {
        FdCursor cc;
        fd_item(item, S, L, rows_per_split, cc);
        const int h = item / S;
        const int r1 = min(L, cc.r0 + rows_per_split);
        float q8[8];
        unpack8(*reinterpret_cast<const uint4*>(Q + (size_t)h * kFdHeadDim + dl), q8);
        float m = -INFINITY, l = 0.f, o8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o8[e] = 0.f;
        for (int t = 0; t < cc.ntiles; ++t, ++consumed) {
            const int st = consumed % kFdStages;
            const bool ok = mbar_wait(&s.full[st], (consumed / kFdStages) & 1);
            if (__syncthreads_or(!ok)) {
                failed = true;
                break;
            }
            const int nvalid = min(kFdRows, r1 - (cc.r0 + t * kFdRows));
            const half* kt = s.k[st];
            const half* vt = s.v[st];
            float sc[8];
            uint4 vr[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int r = warp * 16 + 2 * j + hw;
                float kf[8];
                unpack8(*reinterpret_cast<const uint4*>(kt + r * kFdHeadDim + dl), kf);
                vr[j] = *reinterpret_cast<const uint4*>(vt + r * kFdHeadDim + dl);
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < 8; ++e) d = __fmaf_rn(q8[e], kf[e], d);
                sc[j] = d;
            }
#pragma unroll
            for (int mk = 8; mk >= 1; mk >>= 1)
#pragma unroll
                for (int j = 0; j < 8; ++j) sc[j] += __shfl_xor_sync(0xffffffffu, sc[j], mk);
            float mx = m;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const bool valid = warp * 16 + 2 * j + hw < nvalid;
                sc[j] = valid ? sc[j] * scale : -INFINITY;
                mx = fmaxf(mx, sc[j]);
            }
            if (mx != -INFINITY) {
                const float corr = __expf(m - mx);
                l *= corr;
#pragma unroll
                for (int e = 0; e < 8; ++e) o8[e] *= corr;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float p = __expf(sc[j] - mx);
                    l += p;
                    float vf[8];
                    unpack8(vr[j], vf);
#pragma unroll
                    for (int e = 0; e < 8; ++e) o8[e] = __fmaf_rn(p, vf[e], o8[e]);
                }
                m = mx;
            }
            __syncthreads();  // every warp is done with stage st: refill it
            if (tid == 0) produce();
        }
        if (failed) break;
        combine_halfwarps(m, l, o8);
        if (lane < 16) {
#pragma unroll
            for (int e = 0; e < 8; ++e) s.so[warp][dl + e] = o8[e];
        }
        if (lane == 0) { s.sm[warp] = m; s.sl[warp] = l; }
        __syncthreads();
        const int d = tid;
        float M = -INFINITY;
        for (int w = 0; w < 4; ++w) M = fmaxf(M, s.sm[w]);
        float Ls = 0.f, acc = 0.f;
        for (int w = 0; w < 4; ++w) {
            if (s.sm[w] == -INFINITY) continue;
            const float f = __expf(s.sm[w] - M);
            Ls += s.sl[w] * f;
            acc = __fmaf_rn(f, s.so[w][d], acc);
        }
        float* p = part + (size_t)item * kFdPart;  // item = h * S + split
        p[d] = acc;
        if (d == 0) { p[kFdHeadDim] = M; p[kFdHeadDim + 1] = Ls; }
        __syncthreads();  // s.so / s.sm / s.sl are reused by the next item
    }
    if (failed && tid == 0) {
        atomicExch(err, 1);
        // copies still in flight land in this CTA's shared memory: wait for them (bounded)
        for (uint32_t i = consumed; i < issued; ++i) (void)mbar_wait(&s.full[i % kFdStages], (i / kFdStages) & 1);
    }
}

// ------------------------------------------------------------------ short caches: one cluster per head
constexpr int kFcCluster = 8;        // CTAs per head (portable cluster size)
constexpr int kFcMaxRows = 2048;     // rows per head at most (256 per CTA)
constexpr int kFcThreads = 256;

struct FcSmem {
    float so[kFcThreads / 32][kFdHeadDim];
    float sm[kFcThreads / 32], sl[kFcThreads / 32];
    float po[kFdHeadDim];  // this CTA's partial: o (unnormalised), then m and l
    float pm, pl;
};

// Cluster h (CTAs 8h .. 8h+7) attends head h; CTA rank r takes rows [r R, min(L, (r+1) R)).  Each
// half-warp folds every 16th row into its online softmax (16-byte loads, a lane holds 8 of the 128
// dims), then the CTA merges its 8 warps into a partial in shared memory.  After a cluster barrier,
// CTA 0 reads the 8 partials over distributed shared memory and writes the head's fp16 output; a
// second barrier keeps every CTA's shared memory alive until then.  The kernel has no waits of its
// own besides the two cluster barriers, which every CTA reaches.
__global__ void __cluster_dims__(kFcCluster, 1, 1) __launch_bounds__(kFcThreads, 1)
    fd_cluster_k(const half* __restrict__ Kp, const half* __restrict__ Vp, int stride,
                 const half* __restrict__ Q, int L, int R, half* __restrict__ O) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    FcSmem& s = *reinterpret_cast<FcSmem*>(smem_raw);
    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, hw = lane >> 4, dl = (lane & 15) * 8;
    const int rank = (int)cluster.block_rank(), h = blockIdx.x / kFcCluster;
    const int r0 = rank * R, r1 = min(L, r0 + R);
    // direct 16-byte loads, no staging: half-warp q (of 16) takes rows r0 + q, r0 + q + 16, ...,
    // eight at a time with all sixteen loads of a batch in flight
    const int hq = warp * 2 + hw;
    float q8[8];
    unpack8(*reinterpret_cast<const uint4*>(Q + (size_t)h * kFdHeadDim + dl), q8);
    const float scale = __frcp_rn(sqrtf((float)kFdHeadDim));
    float m = -INFINITY, l = 0.f, o8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o8[e] = 0.f;
    const half* Kh = reinterpret_cast<const half*>(Kp) + (size_t)h * kFdHeadDim + dl;
    const half* Vh = reinterpret_cast<const half*>(Vp) + (size_t)h * kFdHeadDim + dl;
    // the loop bound is CTA-uniform (every lane iterates together: the q.k sums shuffle across the
    // half-warp); rows past r1 are masked
    for (int base = r0; base < r1; base += 8 * 16) {
        const int b0 = base + hq;
        uint4 kr[8], vr[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int r = b0 + 16 * j;
            kr[j] = vr[j] = make_uint4(0u, 0u, 0u, 0u);
            if (r < r1) {
                kr[j] = __ldcs(reinterpret_cast<const uint4*>(Kh + (size_t)r * stride));
                vr[j] = __ldcs(reinterpret_cast<const uint4*>(Vh + (size_t)r * stride));
            }
        }
        float sc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
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
            for (int j = 0; j < 8; ++j) sc[j] += __shfl_xor_sync(0xffffffffu, sc[j], mk);
        float mx = m;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            sc[j] = b0 + 16 * j < r1 ? sc[j] * scale : -INFINITY;
            mx = fmaxf(mx, sc[j]);
        }
        if (mx != -INFINITY) {
            const float corr = __expf(m - mx);
            l *= corr;
#pragma unroll
            for (int e = 0; e < 8; ++e) o8[e] *= corr;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float p = __expf(sc[j] - mx);
                l += p;
                float vf[8];
                unpack8(vr[j], vf);
#pragma unroll
                for (int e = 0; e < 8; ++e) o8[e] = __fmaf_rn(p, vf[e], o8[e]);
            }
            m = mx;
        }
    }
    combine_halfwarps(m, l, o8);
    if (lane < 16) {
#pragma unroll
        for (int e = 0; e < 8; ++e) s.so[warp][dl + e] = o8[e];
    }
    if (lane == 0) { s.sm[warp] = m; s.sl[warp] = l; }
    __syncthreads();
    if (tid < kFdHeadDim) {
        float M = -INFINITY;
        for (int w = 0; w < kFcThreads / 32; ++w) M = fmaxf(M, s.sm[w]);
        float Ls = 0.f, acc = 0.f;
        for (int w = 0; w < kFcThreads / 32; ++w) {
            if (s.sm[w] == -INFINITY) continue;
            const float f = __expf(s.sm[w] - M);
            Ls += s.sl[w] * f;
            acc = __fmaf_rn(f, s.so[w][tid], acc);
        }
        s.po[tid] = acc;
        if (tid == 0) { s.pm = M; s.pl = Ls; }
    }
    cluster.sync();  // every CTA's partial is in its shared memory
    if (rank == 0 && tid < kFdHeadDim) {
        float pm[kFcCluster], pl[kFcCluster], po[kFcCluster];
        float M = -INFINITY;
#pragma unroll
        for (int c = 0; c < kFcCluster; ++c) {
            const FcSmem* peer = cluster.map_shared_rank(&s, c);
            pm[c] = peer->pm;
            pl[c] = peer->pl;
            po[c] = peer->po[tid];
            M = fmaxf(M, pm[c]);
        }
        float Ls = 0.f, acc = 0.f;
#pragma unroll
        for (int c = 0; c < kFcCluster; ++c) {
            if (pm[c] == -INFINITY) continue;
            const float f = __expf(pm[c] - M);
            Ls = __fmaf_rn(pl[c], f, Ls);
            acc = __fmaf_rn(f, po[c], acc);
        }
        O[(size_t)h * kFdHeadDim + tid] = f2h(acc * __frcp_rn(Ls));
    }
    cluster.sync();  // CTA 0 has read every peer's partial
}

// Merge of a head's S split partials (part = [H][S][130]) with 256 threads:
// the weights e^{m_j - M} are computed once per partial, then thread group g
// (threads g*128 .. g*128+127, one per dimension) sums partials j = g, g+2, ...
// sixteen loads in flight at a time, and the two group sums are added.
constexpr int kFdMergeThreads = 256;

__global__ void __launch_bounds__(kFdMergeThreads)
    fd_merge_splits_k(const float* __restrict__ part, int S, half* __restrict__ O, float* __restrict__ out_part) {
    __shared__ float wgt[kFdMergeMax];
    __shared__ float red[8], red2[8], acc2[kFdHeadDim];
    const int h = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const float* p = part + (size_t)h * S * kFdPart;
    float mx = -INFINITY;
    for (int j = t; j < S; j += kFdMergeThreads) mx = fmaxf(mx, p[(size_t)j * kFdPart + kFdHeadDim]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    float M = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) M = fmaxf(M, red[w]);
    float lsum = 0.f;
    for (int j = t; j < S; j += kFdMergeThreads) {
        const float mj = p[(size_t)j * kFdPart + kFdHeadDim];
        const float f = mj == -INFINITY ? 0.f : __expf(mj - M);
        wgt[j] = f;
        lsum = __fmaf_rn(p[(size_t)j * kFdPart + kFdHeadDim + 1], f, lsum);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (lane == 0) red2[warp] = lsum;
    __syncthreads();
    float Ls = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) Ls += red2[w];
    const int g = t >> 7, d = t & (kFdHeadDim - 1);
    float acc = 0.f;
    for (int j0 = g; j0 < S; j0 += 32) {
        float v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const int j = j0 + 2 * k;
            v[k] = j < S ? p[(size_t)j * kFdPart + d] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const int j = j0 + 2 * k;
            if (j < S) acc = __fmaf_rn(wgt[j], v[k], acc);
        }
    }
    if (g == 1) acc2[d] = acc;
    __syncthreads();
    if (g == 0) {
        acc += acc2[d];
        if (O) O[(size_t)h * kFdHeadDim + d] = f2h(acc * __frcp_rn(Ls));
        if (out_part) {
            float* q = out_part + (size_t)h * kFdPart;
            q[d] = acc;
            if (d == 0) { q[kFdHeadDim] = M; q[kFdHeadDim + 1] = Ls; }
        }
    }
}

// Merge of G shards' partials (parts = [G][H][130]): one CTA per head.
__global__ void __launch_bounds__(kFdHeadDim) fd_merge_ranks_k(const float* __restrict__ parts, int G, int H,
                                                               half* __restrict__ O) {
    __shared__ float scratch[8 * kFdPart];
    __shared__ float red[4];
    const int h = blockIdx.x;
    fd_merge_head(parts + (size_t)h * kFdPart, G, H * kFdPart, scratch, 8 * kFdPart, red, O + (size_t)h * kFdHeadDim,
                  nullptr);
}

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

// Tensor map over one [L][stride] fp16 cache: box = 128 columns x 64 rows.
bool make_map(CUtensorMap* m, const void* base, int L, int stride) {
    EncodeTiled enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)stride, (cuuint64_t)L};
    cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
    cuuint32_t box[2] = {(cuuint32_t)kFdHeadDim, (cuuint32_t)kFdRows};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// CTAs of the persistent partials grid: two per SM (two independent TMA pipelines of three
// stages each per SM stream 11% faster than one of six: 187 -> 166 µs at 16 x 131072 rows).
int partials_ctas() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return kFdCtasPerSm * (n > 0 ? n : 148);
}

// Split plan: rows per split (a multiple of the 64-row tile).  Items (head, split) are dealt to the
// persistent grid of partials_ctas() CTAs round-robin (item i to CTA i % ctas), so a call lasts as
// long as its busiest CTA: ceil(items / ctas) items of `tps` tiles each (the last split of a head
// may be shorter).  The plan minimises that CTA's tiles plus half a tile per item (its query load
// and partial write), and among equal plans takes the smaller split count (fewer partials to
// merge).  E.g. 16 heads x 16384 rows on 296 CTAs: 37 splits of 7 tiles, two items per CTA
// (2 x 15 half tiles), where 18 splits of 15 tiles would give one item per CTA (31 half tiles).
void plan(int L, int H, int* S, int* rows) {
    const int tiles = (L + kFdRows - 1) / kFdRows;
    const long long sms = partials_ctas();
    const int smax = std::min(tiles, kFdMergeMax);
    long long best = -1;
    int best_tps = tiles;
    for (int s = 1; s <= smax; ++s) {
        const int tps = (tiles + s - 1) / s;
        const int sa = (tiles + tps - 1) / tps;  // splits actually needed with tps tiles each
        if (sa != s) continue;                   // the same plan as a smaller s
        const long long load = ((long long)sa * H + sms - 1) / sms * (2LL * tps + 1);  // in half tiles
        if (best < 0 || load < best) {
            best = load;
            best_tps = tps;
        }
    }
    *rows = best_tps * kFdRows;
    *S = (L + *rows - 1) / *rows;
}

int check_args(const void* Q, const void* K, const void* V, int L, int stride, int H) {
    if (L <= 0 || H <= 0 || stride < H * kFdHeadDim || (stride & 7)) return (int)cudaErrorInvalidValue;
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!a16(Q) || !a16(K) || !a16(V)) return (int)cudaErrorInvalidValue;
    return 0;
}

// Workspace: a 16-byte control block at the same place for every L (word 0: the error word, which
// a kernel only ever sets and llmdiy_fd_mh_status reads and clears), then the split partials
// [H][S][130] fp32.  Zero-filled by the caller before first use; a workspace sized for one L serves
// every shorter L (the error word does not move with the split count).
constexpr size_t kFdCtl = 4;  // floats
size_t work_floats(int H, int S) { return kFdCtl + (size_t)H * S * kFdPart; }

// The persistent split kernel alone: per-split partials [H][S][130] in `work`.
int launch_split_partials(const uint16_t* Q, const uint16_t* K, const uint16_t* V, int L, int stride, int H,
                          float* work, int S, int rows, cudaStream_t st) {
    CUtensorMap tk, tv;
    if (!make_map(&tk, K, L, stride) || !make_map(&tv, V, L, stride)) return (int)cudaErrorInvalidValue;
    int* err = reinterpret_cast<int*>(work);  // set by the kernel, cleared by the status query
    cudaError_t e;
    static std::once_flag attr;
    std::call_once(attr, [] {
        cudaFuncSetAttribute(fd_partials_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(FdSmem));
    });
    const int grid = std::min(S * H, partials_ctas());
    fd_partials_k<<<grid, kFdThreads, sizeof(FdSmem), st>>>(tk, tv, reinterpret_cast<const half*>(Q), L, S, H, rows,
                                                             work + kFdCtl, err);
    e = cudaGetLastError();
    return (int)e;
}

int launch_partials(const uint16_t* Q, const uint16_t* K, const uint16_t* V, int L, int stride, int H, float* work,
                    int S, int rows, uint16_t* O, float* out_part, cudaStream_t st) {
    const int rc = launch_split_partials(Q, K, V, L, stride, H, work, S, rows, st);
    if (rc) return rc;
    fd_merge_splits_k<<<H, kFdMergeThreads, 0, st>>>(work + kFdCtl, S, reinterpret_cast<half*>(O), out_part);
    return (int)cudaGetLastError();
}

// Short caches: one launch of fd_cluster_k, H clusters of 8 CTAs (no bounded waits, so the
// workspace's error word is left as it is).
int launch_cluster(const uint16_t* Q, const uint16_t* K, const uint16_t* V, int L, int stride, int H,
                   uint16_t* O, cudaStream_t st) {
    const int per = (L + kFcCluster - 1) / kFcCluster;  // rows per CTA
    fd_cluster_k<<<H * kFcCluster, kFcThreads, sizeof(FcSmem), st>>>(
        reinterpret_cast<const half*>(K), reinterpret_cast<const half*>(V), stride, reinterpret_cast<const half*>(Q),
        L, per, reinterpret_cast<half*>(O));
    return (int)cudaGetLastError();
}

}  // namespace

extern "C" size_t llmdiy_fd_mh_work_bytes(int L, int num_heads) {
    if (L <= 0 || num_heads <= 0) return 0;
    int S, rows;
    plan(L, num_heads, &S, &rows);
    return work_floats(num_heads, S) * sizeof(float);
}

extern "C" int llmdiy_fd_multihead(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O, int L,
                                   int stride, int num_heads, float* work, size_t work_bytes, void* stream) {
    int rc = check_args(Q, K, V, L, stride, num_heads);
    if (rc) return rc;
    int S, rows;
    plan(L, num_heads, &S, &rows);
    if (!O || !work || work_bytes < work_floats(num_heads, S) * sizeof(float)) return (int)cudaErrorInvalidValue;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (L <= kFcMaxRows) return launch_cluster(Q, K, V, L, stride, num_heads, O, st);
    return launch_partials(Q, K, V, L, stride, num_heads, work, S, rows, O, nullptr, st);
}

extern "C" int llmdiy_fd_mh_partials(const uint16_t* Q, const uint16_t* K, const uint16_t* V, int L, int stride,
                                     int num_heads, float* part, float* work, size_t work_bytes, void* stream) {
    int rc = check_args(Q, K, V, L, stride, num_heads);
    if (rc) return rc;
    int S, rows;
    plan(L, num_heads, &S, &rows);
    if (!part || !work || work_bytes < work_floats(num_heads, S) * sizeof(float)) return (int)cudaErrorInvalidValue;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    return launch_partials(Q, K, V, L, stride, num_heads, work, S, rows, nullptr, part, st);
}

extern "C" int llmdiy_fd_mh_merge(const float* parts, int G, int num_heads, uint16_t* O, void* stream) {
    if (!parts || !O || G <= 0 || G > kFdMergeMax || num_heads <= 0) return (int)cudaErrorInvalidValue;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    fd_merge_ranks_k<<<num_heads, kFdHeadDim, 0, st>>>(parts, G, num_heads, reinterpret_cast<half*>(O));
    return (int)cudaGetLastError();
}

extern "C" int llmdiy_fd_mh_status(const float* work, int L, int num_heads) {
    if (!work || L <= 0 || num_heads <= 0) return (int)cudaErrorInvalidValue;
    int h = 0;
    int* word = reinterpret_cast<int*>(const_cast<float*>(work));  // word 0 for every L
    cudaError_t e = cudaMemcpy(&h, word, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return (int)e;
    if (h) cudaMemset(word, 0, sizeof(int));  // the kernels only ever set it
    return h ? -5 : 0;
}

extern "C" size_t llmdiy_p2p_buffer_bytes(int world, int num_heads) {
    if (world <= 0 || num_heads <= 0) return 0;
    const size_t b = 2 * p2p_region_words(world, num_heads) * sizeof(unsigned long long);  // two regions (tag parity)
    return (b + 255) / 256 * 256;
}

extern "C" int llmdiy_p2p_alloc(size_t bytes, void** ptr, uint8_t* ipc_handle) {
    if (!ptr || !ipc_handle || bytes == 0) return (int)cudaErrorInvalidValue;
    *ptr = nullptr;
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);  // flags start below every tag
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, *ptr);
    if (e != cudaSuccess) {
        if (*ptr) cudaFree(*ptr);
        *ptr = nullptr;
        return (int)e;
    }
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    std::memcpy(ipc_handle, &h, sizeof(h));
    return 0;
}

extern "C" int llmdiy_p2p_open(const uint8_t* ipc_handle, void** ptr) {
    if (!ipc_handle || !ptr) return (int)cudaErrorInvalidValue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    return (int)cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

extern "C" int llmdiy_p2p_close(void* peer_ptr) { return (int)cudaIpcCloseMemHandle(peer_ptr); }

extern "C" int llmdiy_p2p_free(void* ptr) { return (int)cudaFree(ptr); }

extern "C" int llmdiy_fd_p2p_merge(const float* part, const uint64_t* peers, int world, int rank, int num_heads,
                                   uint32_t tag, uint16_t* O, int* err, void* stream) {
    if (!part || !peers || !O || !err || world <= 0 || world > kP2pMaxWorld || rank < 0 || rank >= world ||
        num_heads <= 0 || tag == 0)
        return (int)cudaErrorInvalidValue;
    fd_p2p_merge_k<<<num_heads, kFdHeadDim, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        part, 1, reinterpret_cast<const unsigned long long*>(peers), world, rank, num_heads, tag,
        reinterpret_cast<half*>(O), err);
    return (int)cudaGetLastError();
}

extern "C" int llmdiy_fd_mh_p2p(const uint16_t* Q, const uint16_t* K, const uint16_t* V, int L, int stride,
                                int num_heads, float* work, size_t work_bytes, const uint64_t* peers, int world,
                                int rank, uint32_t tag, uint16_t* O, int* err, void* stream) {
    int rc = check_args(Q, K, V, L, stride, num_heads);
    if (rc) return rc;
    if (!peers || !O || !err || world <= 0 || world > kP2pMaxWorld || rank < 0 || rank >= world || tag == 0)
        return (int)cudaErrorInvalidValue;
    int S, rows;
    plan(L, num_heads, &S, &rows);
    if (!work || work_bytes < work_floats(num_heads, S) * sizeof(float)) return (int)cudaErrorInvalidValue;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    rc = launch_split_partials(Q, K, V, L, stride, num_heads, work, S, rows, st);
    if (rc) return rc;
    fd_p2p_merge_k<<<num_heads, kFdHeadDim, 0, st>>>(work + kFdCtl, S, reinterpret_cast<const unsigned long long*>(peers),
                                                     world, rank, num_heads, tag, reinterpret_cast<half*>(O), err);
    return (int)cudaGetLastError();
}
