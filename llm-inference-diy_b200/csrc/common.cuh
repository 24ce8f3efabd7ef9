// common.cuh — device helpers shared by the sm_100a kernels of llmdiy_b200.
//
// Thin inline-PTX wrappers for the Blackwell features the kernels use:
// mbarriers, 1-D bulk async copies (TMA without a tensor map), 2-D tiled
// tensor copies, L2 cache policies, cross-CTA acquire/release, and fp16
// helpers.  No multicast form of any bulk or tensor copy is used anywhere
// in this library.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define LLMDIY_DEV __device__ __forceinline__

namespace llmdiy {

// Upper bound on polls of any spin-wait (mbarrier or a global flag).  A wait
// that runs out sets an error flag and the kernel returns instead of hanging.
// With the nanosleep back-off below this is on the order of a few seconds.
constexpr uint32_t kSpinLimit = 1u << 24;

// Error codes a kernel may record in its error word.
enum : int {
    kErrNone = 0,
    kErrGridBarrierTimeout = 1,
    kErrRingTimeout = 2,
    kErrHeadMergeTimeout = 3,
    kErrBadToken = 4,
};

LLMDIY_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------- mbarrier ----------------
LLMDIY_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
LLMDIY_DEV void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
LLMDIY_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
LLMDIY_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// `count` arrivals at once (release semantics at CTA scope, like a plain arrive).
LLMDIY_DEV void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
LLMDIY_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: returns false if the phase did not complete within the limit.
LLMDIY_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, const volatile int* abort_flag = nullptr) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (abort_flag && *abort_flag) return false;
        if (i > 64) __nanosleep(64);
    }
    return false;
}

// ---------------- bulk copies (TMA engine) ----------------
LLMDIY_DEV uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
LLMDIY_DEV uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// 1-D global -> shared bulk copy completing on `bar` (bytes: multiple of 16,
// both addresses 16-byte aligned).
LLMDIY_DEV void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// 2-D tiled tensor copy global -> shared (no multicast).  x is the inner
// coordinate in elements and must be a multiple of 16 bytes' worth.
LLMDIY_DEV void tma_load_2d(void* smem_dst, const void* tmap, int32_t x, int32_t y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(smem_dst)), "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
LLMDIY_DEV void tma_load_2d_hint(void* smem_dst, const void* tmap, int32_t x, int32_t y, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;"
        ::"r"(smem_u32(smem_dst)), "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// L2 prefetch of one box of a 2-D tensor map (no shared memory, no completion); x follows the
// same 16-byte rule as the tiled loads.
LLMDIY_DEV void tma_prefetch_2d(const void* tmap, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(tmap), "r"(x), "r"(y)
                 : "memory");
}

// ---------------- programmatic dependent launch ----------------
// A kernel launched with programmatic stream serialization may start while its predecessor in the
// stream still runs.  pdl_wait() returns once the predecessor has completed and its memory is
// visible: a kernel calls it before its first access to memory that earlier kernels write (or
// read, for its own writes), so the chain keeps stream order as long as every kernel in it does.
// pdl_launch_dependents() lets the successor start its own independent prologue.  Both are
// no-ops in a kernel launched without the attribute.
LLMDIY_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LLMDIY_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Bulk prefetch of a global range into L2 (no shared memory, no completion).
LLMDIY_DEV void bulk_prefetch_l2(const void* gmem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem_src), "r"(bytes) : "memory");
}
LLMDIY_DEV void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------- global memory ordering ----------------
LLMDIY_DEV uint32_t ld_acquire_gpu(const unsigned int* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
LLMDIY_DEV void red_release_gpu_add(unsigned int* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
LLMDIY_DEV uint32_t atom_add_acq_rel_gpu(unsigned int* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
// L2-only (L1-bypassing) 16-byte load, for data another CTA wrote this launch.
LLMDIY_DEV uint4 ld_cg_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
LLMDIY_DEV uint16_t ld_cg_u16(const void* p) {
    uint16_t r;
    asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}
// Streaming 16-byte load that does not allocate in L1.
LLMDIY_DEV uint4 ld_stream_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Named barrier over `nthreads` threads (a multiple of 32) with id 1..15.
LLMDIY_DEV void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Named barrier that also ORs a predicate over the participating threads:
// every thread receives the same value.
LLMDIY_DEV bool named_bar_or(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n"
        " setp.ne.u32 p, %1, 0;\n"
        " barrier.cta.red.or.pred q, %2, %3, p;\n"
        " selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

LLMDIY_DEV unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------- fp16 helpers ----------------
LLMDIY_DEV float h2f(half h) { return __half2float(h); }
LLMDIY_DEV half f2h(float f) { return __float2half_rn(f); }
LLMDIY_DEV void unpack8(const uint4& u, float* f) {
    const half2* h = reinterpret_cast<const half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}
LLMDIY_DEV uint4 pack8(const float* f) {
    uint4 u;
    half2* h = reinterpret_cast<half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    return u;
}

// Order-preserving 16-bit key of an fp16 value (NaN and -inf excluded by the
// caller; -0 is folded onto +0 so that equal float values get equal keys).
LLMDIY_DEV uint32_t half_order_key(uint16_t h) {
    if (h == 0x8000u) h = 0;
    return (h & 0x8000u) ? (uint32_t)(~h & 0xFFFFu) : (uint32_t)(h | 0x8000u);
}
LLMDIY_DEV uint32_t brev5(uint32_t v) { return __brev(v) >> 27; }

// Greedy-argmax candidate key reproducing kernels/argmax.cuh:7-72 with
// blockDim 512: among equal maxima the winner minimises
// (bitrev5(warp), bitrev5(lane), index) of the scanning thread t = idx / ipt.
// Larger key = preferred.  Returns 0 for values the reference never selects.
LLMDIY_DEV unsigned long long argmax_key(uint16_t h, int idx, int ipt) {
    bool is_nan = ((h & 0x7C00u) == 0x7C00u) && (h & 0x03FFu);
    if (is_nan || h == 0xFC00u) return 0ull;
    uint32_t t = (uint32_t)(idx / ipt);
    uint32_t w = (t >> 5) & 31u, l = t & 31u;
    unsigned long long k = (unsigned long long)half_order_key(h) << 48;
    k |= (unsigned long long)(31u - brev5(w)) << 43;
    k |= (unsigned long long)(31u - brev5(l)) << 38;
    k |= (unsigned long long)((1u << 30) - 1u - (uint32_t)idx) & ((1ull << 38) - 1);
    return k;
}
LLMDIY_DEV int argmax_key_index(unsigned long long k) {
    if (k == 0ull) return -1;
    return (int)((1u << 30) - 1u - (uint32_t)(k & ((1ull << 30) - 1)));
}

LLMDIY_DEV unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        unsigned long long o = __shfl_xor_sync(0xffffffffu, v, m);
        v = o > v ? o : v;
    }
    return v;
}

}  // namespace llmdiy
