// gemm_tc.cuh — C[M, N] = A[M, K] * B[N, K]^T on the tcgen05 tensor cores
// (fp16 operands, fp32 accumulation in TMEM), with the output op fused into
// the epilogue.  Both operands are K-major (row-major A; B = weights in the
// file's [out, in] layout), staged by 2-D TMA loads with 128-byte swizzling
// through a STAGES-deep shared-memory ring.
//
// One 128 x BN output tile per CTA (BN = 256: one 128x256x16 MMA per K step of 16), 4 warps:
//   warp 0 lane 0  TMA producer (waits for a stage to be released, loads A, B)
//   warp 1 lane 0  MMA issuer (4 x 128xBNx16 per 64-wide K block, commit
//                  releases the stage; a final commit signals the accumulator)
//   warps 0-3      epilogue: warp w owns accumulator rows 32w..32w+31 (its
//                  TMEM lanes), reads 16 columns at a time, applies the op.
// Every wait is bounded; on expiry the CTA records an error, waits (bounded)
// for its in-flight work, frees its TMEM and returns.
#pragma once
#include <cuda.h>

#include "tc.cuh"

namespace llmdiy {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // 128 bytes of fp16: one swizzle row
constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 128;
constexpr int kGemmPrefetchBlocks = 8;  // weight K blocks per CTA prefetched into L2 before pdl_wait

template <int BN>
struct GemmSmem {
    half a[kGemmStages][kGemmBM * kGemmBK];  // each stage 16 KB, 1024-byte aligned
    half b[kGemmStages][BN * kGemmBK];
    uint64_t full[kGemmStages];
    uint64_t empty[kGemmStages];
    uint64_t accum;
    uint32_t tmem_base;
    int fail;
};

// The epilogue op receives, per thread, one output row and 16 consecutive
// columns [n, n+16) of fp32 accumulators (already masked to n < N by the caller
// only at whole-16 granularity: the op checks its own column bound).
// kBMN: B is stored [K][N] (N contiguous, the reference's transposed-weight layout) and staged
// MN-major: per stage BN/64 TMA boxes of 64 N x 64 K rows, 8 KB apart.
template <int BN, class Epi, bool kBMN = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_k(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb, int M, int N, int K,
              Epi epi, int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    GemmSmem<BN>& s = *reinterpret_cast<GemmSmem<BN>*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.y * kGemmBM, n0 = blockIdx.x * BN;
    // split-K: z-slice blockIdx.z of gridDim.z takes K blocks [kb0, kb0 + KB) (the host makes
    // every slice non-empty); the epilogue then writes a partial sum
    const int KBall = (K + kGemmBK - 1) / kGemmBK;
    const int per = (KBall + (int)gridDim.z - 1) / (int)gridDim.z;
    const int kb0 = (int)blockIdx.z * per;
    const int KB = min(per, KBall - kb0);
    constexpr uint32_t kStageBytes = (kGemmBM + BN) * kGemmBK * 2;
    constexpr uint32_t kCols = BN < 32 ? 32 : BN;  // TMEM columns: a power of two >= 32
    if (tid == 0) {
        for (int i = 0; i < kGemmStages; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        mbar_init(&s.accum, 1);
        s.fail = 0;
        mbar_fence_init();
        // the first weight blocks into L2 while an earlier kernel may still run (weights are
        // constant, so this needs no ordering); the loads below then find them there.  Only with
        // one M tile: with more, every M tile's CTA would prefetch the same weight blocks
        for (int kb = 0; gridDim.y == 1 && kb < KB && kb < kGemmPrefetchBlocks; ++kb) {
            if constexpr (kBMN) {
#pragma unroll
                for (int j = 0; j < BN / 64; ++j) tma_prefetch_2d(&tmb, n0 + 64 * j, (kb0 + kb) * kGemmBK);
            } else {
                tma_prefetch_2d(&tmb, (kb0 + kb) * kGemmBK, n0);
            }
        }
    }
    if (warp == 0) {
        tmem_alloc(&s.tmem_base, kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;
    pdl_wait();  // A and the epilogue's outputs depend on earlier kernels
    pdl_launch_dependents();

    int issued = 0;  // producer: K blocks whose loads were issued
    if (warp == 0 && lane == 0) {
        for (int kb = 0; kb < KB; ++kb) {
            const int st = kb % kGemmStages;
            if (kb >= kGemmStages && !mbar_wait(&s.empty[st], ((kb / kGemmStages) - 1) & 1, &s.fail)) {
                s.fail = 1;
                break;
            }
            mbar_arrive_expect_tx(&s.full[st], kStageBytes);
            tma_load_2d(s.a[st], &tma, (kb0 + kb) * kGemmBK, m0, &s.full[st]);
            if constexpr (kBMN) {
#pragma unroll
                for (int j = 0; j < BN / 64; ++j)
                    tma_load_2d(s.b[st] + j * 64 * kGemmBK, &tmb, n0 + 64 * j, (kb0 + kb) * kGemmBK, &s.full[st]);
            } else {
                tma_load_2d(s.b[st], &tmb, (kb0 + kb) * kGemmBK, n0, &s.full[st]);
            }
            ++issued;
        }
    } else if (warp == 1 && lane == 0) {
        constexpr uint32_t idesc = umma_idesc_f16_f32(kGemmBM, BN, kBMN);
        int kb = 0;
        for (; kb < KB; ++kb) {
            const int st = kb % kGemmStages;
            if (!mbar_wait(&s.full[st], (kb / kGemmStages) & 1, &s.fail)) {
                s.fail = 1;
                break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(s.a[st]), b0 = smem_u32(s.b[st]);
#pragma unroll
            for (int k = 0; k < kGemmBK / 16; ++k) {
                // K-major: 16 K-elements = 32 bytes within each 128-byte row; MN-major: 16 K-rows = 2 KB
                const uint64_t bdesc = kBMN ? umma_desc_sw128_mn(b0 + 2048 * k, 64 * kGemmBK * 2, 1024)
                                            : umma_desc_sw128(b0 + 32 * k);
                umma_f16(tmem, umma_desc_sw128(a0 + 32 * k), bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
            }
            umma_commit(&s.empty[st]);  // frees the stage once these MMAs have read it
        }
        umma_commit(&s.accum);  // all MMAs issued so far (a failed loop commits what it has)
    }
    __syncwarp();
    // epilogue
    const bool ok = __syncthreads_and(mbar_wait(&s.accum, 0, &s.fail) && !s.fail);  // CTA-uniform
    tc_fence_after();
    if (ok) {
        const int row = m0 + warp * 32 + lane;
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
            if (n0 + c >= N) break;  // warp-uniform
            uint32_t r[16];
            tmem_ld16(lane_addr + (uint32_t)c, r);
            tmem_ld_wait();
            if (row < M) epi(row, n0 + c, reinterpret_cast<const float*>(r));
        }
    } else if (tid == 0) {
        atomicExch(err, 1);
    }
    // the producer's loads that no MMA consumed must land before the CTA exits
    if (warp == 0 && lane == 0 && !ok) {
        for (int kb = issued > kGemmStages ? issued - kGemmStages : 0; kb < issued; ++kb)
            (void)mbar_wait(&s.full[kb % kGemmStages], (kb / kGemmStages) & 1);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kCols);
}

}  // namespace llmdiy
