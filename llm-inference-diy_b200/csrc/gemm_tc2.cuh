// gemm_tc2.cuh — C[M, N] = A[M, K] * B[N, K]^T on a pair of SMs: a 2-CTA cluster issues
// 256 x 256 x 16 tcgen05 MMAs (cta_group::2).  CTA r of the pair stages rows
// [128r, 128r+128) of the pair's A tile and columns [128r, 128r+128) of its B tile, so each
// SM streams 32 KB per 64-wide K block for a 128 x 256 output tile — two thirds of what a
// single-SM 128 x 256 tile needs — and the MMA reads the other half from the peer's shared
// memory.  Output rows [128r, 128r+128) of the pair tile accumulate in CTA r's TMEM.
//
// Roles, per CTA: warp 0 lane 0 loads its halves (TMA, completing on the LEADER's full
// barrier, which expects both CTAs' bytes); in the leader (rank 0) warp 1 lane 0 issues the
// MMAs and commits to both CTAs' empty / accumulator barriers; warps 2-5 run the epilogue on
// their TMEM lanes and release the accumulator buffer on the leader's barrier.  Every wait is
// bounded; a CTA whose wait expires records an error, and both CTAs still meet at the final
// cluster barrier.
#pragma once
#include <cuda.h>

#include "gemm_tc.cuh"

namespace llmdiy {

constexpr int kGemm2Stages = 6;

struct Gemm2Smem {
    half a[kGemm2Stages][128 * kGemmBK];  // 16 KB per stage
    half b[kGemm2Stages][128 * kGemmBK];  // 16 KB per stage (this CTA's half of the B tile)
    uint64_t full[kGemm2Stages];          // used in the leader: both CTAs' loads complete here
    uint64_t empty[kGemm2Stages];         // each CTA: the pair's MMAs are done with the stage
    uint64_t acc_full[2];                 // each CTA: accumulator buffer b holds a finished tile
    uint64_t acc_empty[2];                // leader: both CTAs' epilogues have drained buffer b
    uint32_t tmem_base;
    int fail;
};

LLMDIY_DEV uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Shared-memory address (cluster window) of the same variable in CTA `rank` of the cluster.
LLMDIY_DEV uint32_t map_to_rank(const void* p, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_u32(p)), "r"(rank));
    return d;
}
LLMDIY_DEV void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 2-D tile load into this CTA's shared memory, completing bytes on a barrier that may live
// in the peer CTA (cluster-window address `bar_cluster`).
LLMDIY_DEV void tma_load_2d_pair(void* smem_dst, const void* tmap, int32_t x, int32_t y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}
LLMDIY_DEV void umma2_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
// Arrive on `bar` (same offset) in both CTAs of the pair once the MMAs issued so far complete.
LLMDIY_DEV void umma2_commit_both(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}"
        ::"r"(smem_u32(bar))
        : "memory");
}

constexpr int kGemm2Threads = 192;  // warp 0: TMA, warp 1: MMA (leader), warps 2-5: epilogue

// Persistent: pair p of the grid's pairs takes pair tiles t = p, p + pairs, ... (256 x 256 output
// each; t runs down the M tiles of one N column first).  The accumulator is double-buffered in
// TMEM (2 x 256 columns), so the epilogue of tile i overlaps the MMAs of tile i+1.
template <class Epi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemm2Threads, 1)
    gemm_tc2_k(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb, int M, int N, int K,
               Epi epi, int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Gemm2Smem& s = *reinterpret_cast<Gemm2Smem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int pair = (int)blockIdx.x >> 1, pairs = (int)gridDim.x >> 1;
    const int nTM = (M + 255) / 256, nTN = (N + 255) / 256, T = nTM * nTN;
    const int KB = (K + kGemmBK - 1) / kGemmBK;
    constexpr uint32_t kCols = 512;
    if (tid == 0) {
        for (int i = 0; i < kGemm2Stages; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s.acc_full[i], 1);
            mbar_init(&s.acc_empty[i], 2 * 128);  // both CTAs' epilogue threads (used in the leader)
        }
        s.fail = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&s.tmem_base)), "r"(kCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
    }
    tc_fence_before();
    cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- producer (both CTAs): this CTA's halves of every k-block of every tile
            int g = 0;
            for (int t = pair; t < T && !s.fail; t += pairs) {
                const int m0 = (t % nTM) * 256 + (int)rank * 128, nb = (t / nTM) * 256 + (int)rank * 128;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int st = g % kGemm2Stages;
                    if (g >= kGemm2Stages && !mbar_wait(&s.empty[st], ((g / kGemm2Stages) - 1) & 1, &s.fail)) {
                        s.fail = 1;
                        break;
                    }
                    // the leader's full barrier expects both CTAs' bytes; its own arrive carries the count
                    if (leader) mbar_arrive_expect_tx(&s.full[st], 2 * 2 * 128 * kGemmBK * 2);
                    const uint32_t bar = map_to_rank(&s.full[st], 0);
                    tma_load_2d_pair(s.a[st], &tma, kb * kGemmBK, m0, bar);
                    tma_load_2d_pair(s.b[st], &tmb, kb * kGemmBK, nb, bar);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------- MMA issuer (leader only): 256 x 256 x 16 per instruction
            constexpr uint32_t idesc = umma_idesc_f16_f32(256, 256, false);
            int g = 0, it = 0;
            bool ok = true;
            for (int t = pair; ok && t < T; t += pairs, ++it) {
                const int buf = it & 1;
                // both CTAs' epilogues are done with this accumulator (used two tiles ago)
                if (it >= 2 && !mbar_wait(&s.acc_empty[buf], ((it >> 1) - 1) & 1, &s.fail)) { ok = false; break; }
                tc_fence_after();
                const uint32_t acc = tmem + 256u * buf;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int st = g % kGemm2Stages;
                    if (!mbar_wait(&s.full[st], (g / kGemm2Stages) & 1, &s.fail)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(s.a[st]), b0 = smem_u32(s.b[st]);
#pragma unroll
                    for (int k = 0; k < kGemmBK / 16; ++k)
                        umma2_f16(acc, umma_desc_sw128(a0 + 32 * k), umma_desc_sw128(b0 + 32 * k), idesc,
                                  (kb | k) != 0);
                    umma2_commit_both(&s.empty[st]);  // both CTAs may refill the stage once these MMAs read it
                }
                umma2_commit_both(&s.acc_full[buf]);  // the tile's accumulator, in both CTAs
            }
            if (!ok) s.fail = 1;
        }
    } else {
        // ---------------- epilogue (warps 2-5 of both CTAs): TMEM lanes 32q .. 32q+31
        const int q = warp & 3;
        const uint32_t empty_leader = map_to_rank(&s.acc_empty[0], 0);
        int it = 0;
        for (int t = pair; t < T; t += pairs, ++it) {
            const int buf = it & 1;
            if (!mbar_wait(&s.acc_full[buf], (it >> 1) & 1, &s.fail)) {
                s.fail = 1;
                break;
            }
            tc_fence_after();
            const int row = (t % nTM) * 256 + (int)rank * 128 + q * 32 + lane, n0 = (t / nTM) * 256;
            const uint32_t lane_addr = tmem + 256u * buf + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
            for (int c = 0; c < 256; c += 16) {
                if (n0 + c >= N) break;  // warp-uniform
                uint32_t r[16];
                tmem_ld16(lane_addr + (uint32_t)c, r);
                tmem_ld_wait();
                if (row < M) epi(row, n0 + c, reinterpret_cast<const float*>(r));
            }
            tc_fence_before();
            // release the buffer in the leader (cluster-scope arrive on its barrier)
            asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];"
                         ::"r"(empty_leader + 8u * buf)
                         : "memory");
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && s.fail) atomicExch(err, 1);
    // the peer's MMAs and loads no longer touch this CTA's shared memory or TMEM after this point
    // (every MMA was waited for through acc_full; a failed run waits out its bounded waits first)
    cluster_sync_all();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

}  // namespace llmdiy
