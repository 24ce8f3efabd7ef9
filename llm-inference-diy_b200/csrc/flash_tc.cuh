// flash_tc.cuh — causal flash attention of the prefill on the tcgen05 tensor cores.
// Computes what kernels/flash_attn.cu:1854-2179 computes per head (softmax(Q K^T /
// sqrt(128)) V with the causal mask, fp16 P, fp32 accumulation), with query rows at
// positions p0 .. p0+n-1 attending cache rows [0, pos] in place (no gather pass).
//
// CTA = 128 query rows of one head.  Warp 4 (one lane) loads Q once and streams
// 64-key K and V tiles through 2-stage TMA rings, and issues the MMAs:
//   S(j)  = Q K(j)^T          128 x 64,  K = 128 dims  -> TMEM (two S buffers)
//   O    += P(j) V(j)         128 x 128, K = 64 keys   -> TMEM (one O accumulator; P from TMEM)
// with S(j+1) issued before PV(j), so the rows find it ready when they finish softmax(j).  Warps 0-3 own the query rows
// (thread = row = TMEM lane): each reads its S row, applies the causal mask and the
// online softmax in base 2, writes its P row (fp16 pairs) back into TMEM over its S row,
// where PV takes it as the A operand, and signals the issuer.  O is rescaled (TMEM load, scale,
// store) only when a row's running maximum grows by more than 2^8; otherwise the stale
// maximum is kept, which leaves O / l unchanged (P stays <= 256, exact in fp16 range).
// At the end each thread reads its O row, divides by l and stores fp16.
//
// Every wait is bounded; on expiry the CTA records an error in *err, waits (bounded)
// for its in-flight copies and MMAs, frees its TMEM and returns.
#pragma once
#include <cuda.h>

#include "decode.h"
#include "tc.cuh"

namespace llmdiy {

constexpr int kFtRows = 128;     // query rows per CTA (MMA M)
constexpr int kFtKeys = 64;      // keys per tile
constexpr int kFtStages = 2;     // K/V tiles in flight (two CTAs share an SM: 112 KB of smem each)
constexpr int kFtThreads = 160;  // warps 0-3: rows (TMEM lanes 32w..32w+31); warp 4: TMA + MMA issue

LLMDIY_DEV uint32_t pack_h2f(float lo, float hi) {  // two fp16 (round to nearest) in one 32-bit word
    const half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

LLMDIY_DEV float ex2_approx(float x) {  // 2^x (the MUFU approximation; 2^-inf = 0)
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct FlashTcSmem {
    half q[2][kFtRows * 64];             // dims 0-63 | 64-127: K-major, 128-byte swizzle (16 KB each)
    half k[kFtStages][2][kFtKeys * 64];  // per stage, dims 0-63 | 64-127, K-major (8 KB each)
    half v[kFtStages][2][kFtKeys * 64];  // per stage, dims 0-63 | 64-127, MN-major (8 KB each)
    uint64_t q_full, k_full[kFtStages], k_empty[kFtStages], v_full[kFtStages], v_empty[kFtStages];
    uint64_t s_full[2], p_full[2], o_done[2], drain;
    uint32_t tmem_base;
    int fail;
};

// tq: the query rows [n][heads*128] (box 64 x 128); tk, tv: the K / V rows [rows][heads*128]
// (box 64 x 64), head h in columns h*128 .. h*128+127 of each.  att: [n] rows of ldo elements,
// head h at column h*128.  Grid (ceil(n/128), heads).
__global__ void __launch_bounds__(kFtThreads, 2)
    flash_tc_k(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
               const __grid_constant__ CUtensorMap tv, half* __restrict__ att, int ldo, int n, int p0, int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    FlashTcSmem& s = *reinterpret_cast<FlashTcSmem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y;
    const int q0 = ((int)gridDim.x - 1 - (int)blockIdx.x) * kFtRows;  // longest tiles first
    const int last_row = min(q0 + kFtRows, n) - 1;
    const int T = (p0 + last_row) / kFtKeys + 1;  // key tiles up to the last row's position
    constexpr uint32_t kCols = 256;                // S0 | S1 | O (128 columns)
    if (tid == 0) {
        mbar_init(&s.q_full, 1);
        for (int i = 0; i < kFtStages; ++i) {
            mbar_init(&s.k_full[i], 1);
            mbar_init(&s.k_empty[i], 1);
            mbar_init(&s.v_full[i], 1);
            mbar_init(&s.v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s.s_full[i], 1);
            mbar_init(&s.p_full[i], 128);
            mbar_init(&s.o_done[i], 1);
        }
        mbar_init(&s.drain, 1);
        s.fail = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        tmem_alloc(&s.tmem_base, kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;
    const uint32_t tO = tmem + 128;  // S(j) lives at tmem + 64 * (j & 1)

    if (warp == 4) {
        if (lane == 0) {
            // ---------------- producer + MMA issuer
            // K and V tiles have their own rings: K(t) can stream in as soon as S(t-2) is done,
            // well before PV(t-2) releases V's stage
            int kloaded = 0, vloaded = 0;
            auto load_k = [&](int t) {
                const int st = t % kFtStages, y = t * kFtKeys;
                mbar_arrive_expect_tx(&s.k_full[st], 2 * kFtKeys * 64 * 2);
                tma_load_2d(s.k[st][0], &tk, h * kHeadDim, y, &s.k_full[st]);
                tma_load_2d(s.k[st][1], &tk, h * kHeadDim + 64, y, &s.k_full[st]);
                ++kloaded;
            };
            auto load_v = [&](int t) {
                const int st = t % kFtStages, y = t * kFtKeys;
                mbar_arrive_expect_tx(&s.v_full[st], 2 * kFtKeys * 64 * 2);
                tma_load_2d(s.v[st][0], &tv, h * kHeadDim, y, &s.v_full[st]);
                tma_load_2d(s.v[st][1], &tv, h * kHeadDim + 64, y, &s.v_full[st]);
                ++vloaded;
            };
            mbar_arrive_expect_tx(&s.q_full, 2 * kFtRows * 64 * 2);
            tma_load_2d(s.q[0], &tq, h * kHeadDim, q0, &s.q_full);
            tma_load_2d(s.q[1], &tq, h * kHeadDim + 64, q0, &s.q_full);
            for (int t = 0; t < T && t < kFtStages; ++t) load_k(t);
            for (int t = 0; t < T && t < kFtStages; ++t) load_v(t);
            constexpr uint32_t idS = umma_idesc_f16_f32(kFtRows, kFtKeys, false);
            constexpr uint32_t idO = umma_idesc_f16_f32(kFtRows, kHeadDim, true);
            const uint32_t qa = smem_u32(s.q[0]);
            bool ok = mbar_wait(&s.q_full, 0, &s.fail);
            auto pv = [&](int i) -> bool {  // O += P(i) V(i), then release the P tile and V(i)'s stage
                if (!mbar_wait(&s.p_full[i & 1], (i >> 1) & 1, &s.fail)) return false;
                if (!mbar_wait(&s.v_full[i % kFtStages], (i / kFtStages) & 1, &s.fail)) return false;
                tc_fence_after();
                // A = P(i) in TMEM (packed over S(i)'s first 32 columns), B = V(i) in shared memory
                const uint32_t pa = tmem + 64u * (i & 1), vb = smem_u32(s.v[i % kFtStages][0]);
#pragma unroll
                for (int kk = 0; kk < kFtKeys / 16; ++kk)
                    umma_f16_tmem_a(tO, pa + 8 * kk, umma_desc_sw128_mn(vb + 2048 * kk, 8192, 1024), idO,
                                    (i | kk) != 0 ? 1u : 0u);
                umma_commit(&s.o_done[i & 1]);
                umma_commit(&s.v_empty[i % kFtStages]);
                return true;
            };
            // S(j) = Q K(j)^T into TMEM buffer j & 1, then release K(j)'s stage
            auto qk = [&](int j) -> bool {
                const int st = j % kFtStages;
                if (!mbar_wait(&s.k_full[st], (j / kFtStages) & 1, &s.fail)) return false;
                tc_fence_after();
                const uint32_t kb = smem_u32(s.k[st][0]);
#pragma unroll
                for (int kk = 0; kk < kHeadDim / 16; ++kk)
                    umma_f16(tmem + 64u * (j & 1), umma_desc_sw128(qa + (kk >> 2) * 16384 + 32 * (kk & 3)),
                             umma_desc_sw128(kb + (kk >> 2) * 8192 + 32 * (kk & 3)), idS, kk != 0 ? 1u : 0u);
                umma_commit(&s.s_full[j & 1]);
                umma_commit(&s.k_empty[st]);
                return true;
            };
            if (ok && !qk(0)) ok = false;
            for (int j = 0; ok && j < T; ++j) {
                // K(j+2) into the stage S(j) released (S(j) was issued an iteration ago)
                if (j + kFtStages < T) {
                    if (!mbar_wait(&s.k_empty[j % kFtStages], (j / kFtStages) & 1, &s.fail)) { ok = false; break; }
                    load_k(j + kFtStages);
                }
                // S(j+1) before PV(j), so it is ready when the rows finish softmax(j); its TMEM
                // buffer held P(j-1): PV(j-1) must be complete
                if (j + 1 < T) {
                    const bool freed = j < 1 || mbar_wait(&s.o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, &s.fail);
                    if (!freed || !qk(j + 1)) { ok = false; break; }
                }
                // V(j+1) into the stage PV(j-1) released
                const int i = j - 1;
                if (i >= 0 && i + kFtStages < T) {
                    if (!mbar_wait(&s.v_empty[i % kFtStages], (i / kFtStages) & 1, &s.fail)) { ok = false; break; }
                    load_v(i + kFtStages);
                }
                if (!pv(j)) { ok = false; break; }
            }
            if (!ok) {
                s.fail = 1;
                // every MMA issued so far, and the copies that no MMA consumed, complete before the CTA exits
                umma_commit(&s.drain);
                (void)mbar_wait(&s.drain, 0);
                for (int t = kloaded > kFtStages ? kloaded - kFtStages : 0; t < kloaded; ++t)
                    (void)mbar_wait(&s.k_full[t % kFtStages], (t / kFtStages) & 1);
                for (int t = vloaded > kFtStages ? vloaded - kFtStages : 0; t < vloaded; ++t)
                    (void)mbar_wait(&s.v_full[t % kFtStages], (t / kFtStages) & 1);
                (void)mbar_wait(&s.q_full, 0);
            }
        }
        __syncwarp();
    } else {
        // ---------------- rows: softmax and epilogue (thread = query row = TMEM lane)
        const int r = tid;  // 0..127
        const int qp = p0 + q0 + r;  // this row's position
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        constexpr float kScaleLog2 = 1.4426950408889634f * 0.08838834764831845f;  // log2(e) / sqrt(128)
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < T; ++j) {
            if (!mbar_wait(&s.s_full[j & 1], (j >> 1) & 1, &s.fail)) { ok = false; break; }
            tc_fence_after();
            float x[kFtKeys];
#pragma unroll
            for (int c = 0; c < kFtKeys; c += 16)
                tmem_ld16(tmem + 64u * (j & 1) + lane_off + c, reinterpret_cast<uint32_t*>(x + c));
            tmem_ld_wait();
            const int k0 = j * kFtKeys;
            if (k0 + kFtKeys - 1 > p0 + q0) {  // a tile on the diagonal (CTA-uniform): mask keys after the row
#pragma unroll
                for (int c = 0; c < kFtKeys; ++c) x[c] = (k0 + c <= qp) ? x[c] : -INFINITY;
            }
            // row maximum of the raw scores (8 independent chains), then scaled (the scale is positive)
            float mx[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) mx[e] = x[e];
#pragma unroll
            for (int c = 8; c < kFtKeys; ++c) mx[c & 7] = fmaxf(mx[c & 7], x[c]);
            const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                   fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * kScaleLog2;
            if (j == 0) {
                m = mt;  // key 0 is visible to every row: m is finite from here on
            } else if (mt > m + 8.f) {
                // the running maximum grew by more than 2^8: rescale O (complete through PV(j-1))
                if (!mbar_wait(&s.o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, &s.fail)) { ok = false; break; }
                tc_fence_after();
                const float f = exp2f(m - mt);
#pragma unroll 1
                for (int c = 0; c < kHeadDim; c += 16) {
                    uint32_t o[16];
                    tmem_ld16(tO + lane_off + c, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
                    tmem_st16(tO + lane_off + c, o);
                }
                tmem_st_wait();
                l *= f;
                m = mt;
            }
            // P(j) in fp16 pairs over the first 32 columns of S(j)'s buffer (S(j) is in registers)
            const float nm = -m;
            float ls[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) ls[e] = 0.f;
            uint32_t pk[kFtKeys / 2];
#pragma unroll
            for (int c = 0; c < kFtKeys; c += 2) {
                const float p0 = ex2_approx(__fmaf_rn(x[c], kScaleLog2, nm));  // masked keys: 2^-inf = 0
                const float p1 = ex2_approx(__fmaf_rn(x[c + 1], kScaleLog2, nm));
                ls[c & 7] += p0;
                ls[(c + 1) & 7] += p1;
                pk[c / 2] = pack_h2f(p0, p1);
            }
            l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
#pragma unroll
            for (int c = 0; c < kFtKeys / 2; c += 16) tmem_st16(tmem + 64u * (j & 1) + lane_off + c, pk + c);
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&s.p_full[j & 1]);
        }
        // epilogue: O / l once the last PV is complete
        if (ok && mbar_wait(&s.o_done[(T - 1) & 1], ((T - 1) >> 1) & 1, &s.fail)) {
            tc_fence_after();
            const bool live = q0 + r < n;
            const float inv = 1.f / l;
            half* dst = att + (size_t)(q0 + r) * ldo + h * kHeadDim;
#pragma unroll 1
            for (int c = 0; c < kHeadDim; c += 16) {
                uint32_t o[16];
                tmem_ld16(tO + lane_off + c, o);
                tmem_ld_wait();
                float v[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] = __uint_as_float(o[e]) * inv;
                if (live) {
                    *reinterpret_cast<uint4*>(dst + c) = pack8(v);
                    *reinterpret_cast<uint4*>(dst + c + 8) = pack8(v + 8);
                }
            }
        } else {
            s.fail = 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && s.fail) atomicExch(err, 1);
    if (warp == 0) tmem_dealloc(tmem, kCols);
}

}  // namespace llmdiy
