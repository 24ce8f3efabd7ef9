// decode_kernel.cu — the persistent bs1 decode kernel (QwenEngine::step,
// framework_src/qwen_infer.cu:614-737, for many steps per launch).
//
// One CTA of 8 consumer warps and 1 producer warp per SM.  Each CTA streams
// its share of every weight matrix through an 8-slot ring of 24 KB
// shared-memory slots with 1-D bulk copies (TMA): chunk g of the CTA's chunk
// sequence goes to slot g % 8.  The producer (one lane) issues chunk g as soon
// as the consumers have released chunk g - 8 (an "empty" mbarrier per slot),
// and prefetches a later chunk into L2.  Weights never depend on activations,
// so those copies run ahead across phase, layer and token boundaries and HBM
// keeps streaming while the consumers wait for activations.  A phase's units
// (two weight rows each) are dealt round-robin to the 8 consumer warps, unit i
// to warp i % 8, so the warps work through the ring in sequence order and the
// oldest slots free up first; a warp consumes its unit's two rows (fp32 FMA dot
// products against the activation held in registers or shared memory), with the
// reference's small ops fused into the epilogues:
//   QKV  : RMSNorm(ln_1) prologue; bias; RoPE; K/V append at row pos
//   ATT  : 16 heads x 9 position splits; split 0 of a head merges the (m,l,o) partials
//   O    : residual add
//   W12  : RMSNorm(ln_2) prologue; SwiGLU (silu on the w2 output)
//   C    : residual add
//   LM   : RMSNorm(ln_f) prologue; logits; greedy argmax key (reference tie rule)
// Between phases the small activation vectors travel as flag-carrying words
// (decode.h): a consumer waits for exactly the words it needs, so there is no
// grid barrier inside a step.  One grid barrier per step publishes the argmax
// and orders the KV-cache rows for the next step.  Every spin-wait is bounded;
// on expiry the kernel records an error code in DecodeControl and returns.
#include "decode.h"
#include "ops.cuh"

namespace llmdiy {
namespace {

enum PhaseId { PH_QKV = 0, PH_ATT = 1, PH_O = 2, PH_W12 = 3, PH_C = 4, PH_LM = 5 };

constexpr int kMaxIM = 6144;
constexpr int kQkvBiasUnits = 64;  // QKV units per CTA whose bias pairs are staged in shared memory
constexpr uint32_t kPollLimit = 1u << 21;  // polls of one flag-carrying word or of the step barrier
constexpr int kDecodeBlock = kDecodeThreads + 32;  // 8 consumer warps + the producer warp
constexpr uint32_t kEmptyArrivals = 3;  // per chunk: one per unit, the last unit of a chunk tops up to 3

struct __align__(128) Smem {
    uint8_t ring[kRingStages][kStageBytes];
    half xs[kHidden];    // normalised activation of the current phase
    half xraw[kHidden];  // residual stream entering the current phase
    half act[kMaxIM];
    float so[kConsumerWarps][kHeadDim];
    half qkv_new[3][kHeadDim];  // attention: q, k and v of the new row for this CTA's head
    float sm[kConsumerWarps], sl[kConsumerWarps];
    float red[32];
    unsigned long long wkey[kConsumerWarps];
    uint64_t full[kRingStages];   // chunk landed (the producer's expect_tx + the copy's bytes)
    uint64_t empty[kRingStages];  // chunk consumed (kEmptyArrivals per chunk from the consumer warps)
    LayerPtrs layers[kMaxLayers];  // copy of a.layers (read at every phase change)
    int range[5][4];               // per phase (qkv, o, w12, c, lm): this CTA's units [u0, u1), units per chunk, K
    float qbias[kQkvBiasUnits][2];  // this layer's QKV bias pairs of the CTA's QKV units (loaded ahead)
    volatile int fail;  // a consumer wait expired
    volatile int stop;  // the consumers have left the step loop: the producer stops issuing
    int token;
    int last;
};


// acc0 += lo(w) * lo(x), acc1 += hi(w) * hi(x): fp16 operands, exact product,
// fp32 accumulate (the same arithmetic as fmaf(float(w), float(x), acc)).
__device__ __forceinline__ void fma2_f16(float& acc0, float& acc1, uint32_t w, uint32_t x) {
    asm("{\n\t.reg .f16 wl, wh, xl, xh;\n\t"
        "mov.b32 {wl, wh}, %2;\n\t"
        "mov.b32 {xl, xh}, %3;\n\t"
        "fma.rn.f32.f16 %0, wl, xl, %0;\n\t"
        "fma.rn.f32.f16 %1, wh, xh, %1;\n\t}"
        : "+f"(acc0), "+f"(acc1)
        : "r"(w), "r"(x));
}


// The two rows (a unit) of K = 2048 starting at `r0` against the lane's
// activation slice in registers (lane holds elements 256 j + 8 lane .. +7),
// then a transposing butterfly: every lane ends with both sums.
__device__ __forceinline__ void dot2_regs(const half* r0, const uint32_t* xh, int lane, float& s0, float& s1) {
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint4 w0 = *reinterpret_cast<const uint4*>(r0 + 256 * j + 8 * lane);
        const uint4 w1 = *reinterpret_cast<const uint4*>(r0 + kHidden + 256 * j + 8 * lane);
        fma2_f16(a0, a1, w0.x, xh[4 * j + 0]);
        fma2_f16(b0, b1, w1.x, xh[4 * j + 0]);
        fma2_f16(a0, a1, w0.y, xh[4 * j + 1]);
        fma2_f16(b0, b1, w1.y, xh[4 * j + 1]);
        fma2_f16(a0, a1, w0.z, xh[4 * j + 2]);
        fma2_f16(b0, b1, w1.z, xh[4 * j + 2]);
        fma2_f16(a0, a1, w0.w, xh[4 * j + 3]);
        fma2_f16(b0, b1, w1.w, xh[4 * j + 3]);
    }
    const float v0 = a0 + a1, v1 = b0 + b1;
    // lanes < 16 keep row 0 and send row 1, lanes >= 16 the other way round: one shuffle halves both
    const bool hi = lane & 16;
    float t = (hi ? v1 : v0) + __shfl_xor_sync(0xffffffffu, hi ? v0 : v1, 16);
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1) t += __shfl_xor_sync(0xffffffffu, t, m);
    const float o = __shfl_xor_sync(0xffffffffu, t, 16);
    s0 = hi ? o : t;
    s1 = hi ? t : o;
}

// fp32-accumulated dot products of two weight rows (a unit) of any K against
// the activation in shared memory; after the butterfly every lane holds both.
__device__ __forceinline__ void dot2_smem(const half* r0, const half* r1, const half* xs, int K, int lane, float& s0,
                                          float& s1) {
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll 2
    for (int k = 8 * lane; k < K; k += 256) {
        const uint4 w0 = *reinterpret_cast<const uint4*>(r0 + k);
        const uint4 w1 = *reinterpret_cast<const uint4*>(r1 + k);
        const uint4 xv = *reinterpret_cast<const uint4*>(xs + k);
        fma2_f16(a0, a1, w0.x, xv.x);
        fma2_f16(b0, b1, w1.x, xv.x);
        fma2_f16(a0, a1, w0.y, xv.y);
        fma2_f16(b0, b1, w1.y, xv.y);
        fma2_f16(a0, a1, w0.z, xv.z);
        fma2_f16(b0, b1, w1.z, xv.z);
        fma2_f16(a0, a1, w0.w, xv.w);
        fma2_f16(b0, b1, w1.w, xv.w);
    }
    s0 = a0 + a1;
    s1 = b0 + b1;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        s0 += __shfl_xor_sync(0xffffffffu, s0, m);
        s1 += __shfl_xor_sync(0xffffffffu, s1, m);
    }
}

__device__ void record_error(DecodeControl* ctl, int code, int where) {
    if (atomicCAS(&ctl->err, 0, code) == 0) ctl->err_where = where;
}

// ------------------------------------------------------------------ flag-carrying words
__device__ __forceinline__ void ll_store(unsigned long long* p, uint32_t data, uint32_t tag) {
    const unsigned long long v = ((unsigned long long)tag << 32) | data;
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ll_load(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Read N words p[i*stride] that must carry `tag`; data to out[i].  Every
// poll issues all N loads back to back (a word already received is loaded
// again and ignored), so one round costs one L2 round trip, not N.  Returns
// false when the words did not arrive within the poll bound.
template <int N>
__device__ __forceinline__ bool ll_read(const unsigned long long* p, int stride, uint32_t tag, uint32_t* out) {
    uint32_t pending = (N == 32) ? 0xffffffffu : ((1u << N) - 1u);
    for (uint32_t it = 0; it < kPollLimit; ++it) {
        unsigned long long v[N];
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = ll_load(p + (size_t)i * stride);
#pragma unroll
        for (int i = 0; i < N; ++i) {
            if ((pending & (1u << i)) && (uint32_t)(v[i] >> 32) == tag) {
                out[i] = (uint32_t)v[i];
                pending &= ~(1u << i);
            }
        }
        if (!pending) return true;
        __nanosleep(16);
    }
    return false;
}

// As ll_read for the first n <= N of the N words (the rest are not touched).
template <int N>
__device__ __forceinline__ bool ll_read_n(const unsigned long long* p, int stride, int n, uint32_t tag, uint32_t* out) {
    uint32_t pending = (n >= 32) ? 0xffffffffu : ((1u << n) - 1u);
    for (uint32_t it = 0; it < kPollLimit; ++it) {
        unsigned long long v[N];
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = (i < n) ? ll_load(p + (size_t)i * stride) : 0ull;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            if ((pending & (1u << i)) && (uint32_t)(v[i] >> 32) == tag) {
                out[i] = (uint32_t)v[i];
                pending &= ~(1u << i);
            }
        }
        if (!pending) return true;
        __nanosleep(16);
    }
    return false;
}

// The SwiGLU output (one fp16 per word, IM <= kMaxIM words): thread tid
// gathers words tid, tid+256, ... into out[] (shared memory), 12 loads in
// flight per round.
__device__ __forceinline__ bool ll_gather_act(const unsigned long long* p, int n, uint32_t tag, half* out) {
    static_assert(kMaxIM <= 24 * kDecodeThreads, "two rounds of 12 words per thread");
    uint32_t pending = (1u << n) - 1u;  // n <= 24
    for (uint32_t it = 0; it < kPollLimit; ++it) {
#pragma unroll
        for (int j0 = 0; j0 < 24; j0 += 12) {
            if (!(pending >> j0)) continue;
            unsigned long long v[12];
#pragma unroll
            for (int j = 0; j < 12; ++j) v[j] = (j0 + j < n) ? ll_load(p + (size_t)(j0 + j) * kDecodeThreads) : 0ull;
#pragma unroll
            for (int j = 0; j < 12; ++j) {
                const int k = j0 + j;
                if ((pending & (1u << k)) && (uint32_t)(v[j] >> 32) == tag) {
                    out[(size_t)k * kDecodeThreads] = __ushort_as_half((uint16_t)v[j]);
                    pending &= ~(1u << k);
                }
            }
        }
        if (!pending) return true;
        __nanosleep(16);
    }
    return false;
}

// Timing probe (development aid, off when a.prof is null): at consecutive
// boundaries of its row of a.prof, each CTA records %globaltimer when warp 0
// arrives (slot 0) and when the last of its warps arrives (slot 1).
__device__ __forceinline__ void probe(const DecodeArgs& a, int tid, int& np) {
    if (a.prof) {
        if ((tid & 31) == 0 && np < a.prof_cap) {
            const unsigned long long t = globaltimer();
            unsigned long long* p = a.prof + ((size_t)blockIdx.x * a.prof_cap + np) * 2;
            if (tid == 0) p[0] = t;
            atomicMax(p + 1, t);
        }
        ++np;
    }
}

struct Tags {
    uint32_t base;
    int NL;
    __device__ __forceinline__ uint32_t operator()(int step, int layer, int slot) const {
        return base + (uint32_t)((step * NL + layer) * LL_PER_LAYER + slot) + 1u;
    }
};

// ------------------------------------------------------------------ producer
// One lane of the producer warp walks this CTA's chunk sequence (DecodeArgs::feed_tbl: per step,
// per layer the chunks of qkv_w, proj_w, w12, cproj, then unless skip_lm lm_head's) and copies
// chunk g into ring slot g % 8 once the consumers have released chunk g - 8 there.  With each
// copy it prefetches chunk g + 8 * l2_ahead into L2, so HBM keeps streaming while the ring is
// full.  Every wait is bounded and gives up when the consumers have stopped or failed; before
// returning, the producer waits (bounded) for its copies in flight, so none lands in the shared
// memory of an exited CTA.
__device__ void producer(const DecodeArgs& a, Smem& s) {
    if ((threadIdx.x & 31) != 0) return;
    const int b = blockIdx.x;
    const int E = a.feed_cnt[2 * b] + (a.skip_lm ? 0 : a.feed_cnt[2 * b + 1]);
    const uint2* tbl = a.feed_tbl + (size_t)b * a.feed_stride;
    const uint32_t total = (uint32_t)E * (uint32_t)a.n_steps;
    const uint32_t ahead = (uint32_t)(kRingStages * a.l2_ahead);
    const uint64_t pol = l2_policy_evict_first();
    int i = 0, ip = (int)(ahead % (uint32_t)(E > 0 ? E : 1));  // table index of chunk g and of chunk g + ahead
    uint32_t g = 0;
    for (; g < total; ++g) {
        const int slot = (int)(g & (kRingStages - 1));
        if (g >= (uint32_t)kRingStages) {
            // use k = g / 8 of the slot needs use k - 1 released
            const uint32_t par = ((g >> 3) - 1) & 1;
            bool ok = false;
            for (uint32_t it = 0; it < kSpinLimit; ++it) {
                if (mbar_try_wait(&s.empty[slot], par)) { ok = true; break; }
                if (s.stop || s.fail) break;
                if (it > 64) __nanosleep(32);
            }
            if (!ok) break;  // the consumers left (end of the launch, a stop id or a failure)
        }
        const uint2 ent = tbl[i];
        mbar_arrive_expect_tx(&s.full[slot], ent.y);
        bulk_g2s(s.ring[slot], a.wbase + (size_t)ent.x * 16u, ent.y, &s.full[slot], pol);
        if (ahead && g + ahead < total) {
            const uint2 pe = tbl[ip];
            bulk_prefetch_l2(a.wbase + (size_t)pe.x * 16u, pe.y);
        }
        if (++i == E) i = 0;
        if (++ip == E) ip = 0;
    }
    // drain: the last copy issued into each slot has landed
    for (uint32_t k = g > (uint32_t)kRingStages ? g - kRingStages : 0; k < g; ++k)
        (void)mbar_wait(&s.full[k & (kRingStages - 1)], (k >> 3) & 1);
}

// ------------------------------------------------------------------ consumers
struct StepCtx {
    int pos, step, layer;
    half* kcl;
    half* vcl;
    const half* bias;
    int ipt;
    uint32_t tag;             // tag of the words the current phase writes
    unsigned long long best;  // lane u of each warp: best argmax key of its units in the LM phase
};

// The one grid-wide barrier of a step (publishes the argmax, orders KV rows).
__device__ bool grid_sync(const DecodeArgs& a, Smem& s, uint32_t& nbar, int tid, bool bad, int& np) {
    const bool any_bad = named_bar_or(1, 256, bad);
    ++nbar;
    bool failed = any_bad;
    probe(a, tid, np);
    if (tid == 0) {
        red_release_gpu_add(&a.ctl->bar, 1u);
        if (!failed) {
            const uint32_t target = nbar * gridDim.x;
            bool ok = false;
            for (uint32_t i = 0; i < kPollLimit; ++i) {
                if (ld_acquire_gpu(&a.ctl->bar) >= target) { ok = true; break; }
                if ((i & 63) == 63 && *(volatile int*)&a.ctl->err != 0) break;
                if (i > 256) __nanosleep(32);
            }
            if (!ok) {
                record_error(a.ctl, kErrGridBarrierTimeout, PH_LM);
                failed = true;
            }
        }
    }
    probe(a, tid, np);
    // every consumer thread gets the same verdict, so later branches stay CTA-uniform
    return !named_bar_or(1, 256, failed);
}

__device__ __forceinline__ void prefetch_l2_line(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
// As prefetch_l2_line, with the line marked to be evicted last: the small per-layer vectors on
// the critical path (norm weights, QKV bias) stay in L2 while the weight stream (evict-first)
// passes through it.
__device__ __forceinline__ void prefetch_l2_keep(const void* p) {
    asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}
// 16-byte load that keeps its L2 line evict-last (see prefetch_l2_keep).
__device__ __forceinline__ uint4 ld_keep_u4(const void* p, uint64_t pol) {
    uint4 v;
    asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}

// Stage a residual-stream vector in shared memory (raw copy in xraw),
// RMSNorm it with the reference tree and leave each lane's 64-element slice
// of the normalised vector in xr.  The source is either a plain fp16 row (the
// embedding) or flag-carrying words with `tag`.  Returns the CTA-wide failure
// verdict (true = a wait expired somewhere in the CTA).
__device__ bool load_norm(const DecodeArgs& a, const half* plain, const unsigned long long* ll, uint32_t tag,
                          const half* w, Smem& s, int tid, uint32_t* xr, bool bad, int& np,
                          float* stage_dst = nullptr, float stage_val = 0.f) {
    const uint4 wv = ld_keep_u4(w + tid * 8, l2_policy_evict_last());  // in flight while polling
    uint4 v;
    uint32_t d[4];
    if (plain) {
        v = *reinterpret_cast<const uint4*>(plain + tid * 8);
    } else {
        // coalesced polls: thread t takes words t, t + 256, t + 512, t + 768
        bad |= !ll_read<4>(ll + tid, kDecodeThreads, tag, d);
    }
    // the previous phase may still read xraw / xs: wait before overwriting
    if (named_bar_or(1, 256, bad)) return true;
    probe(a, tid, np);
    if (plain) {
        *reinterpret_cast<uint4*>(s.xraw + tid * 8) = v;
    } else {
        uint32_t* xw = reinterpret_cast<uint32_t*>(s.xraw);
#pragma unroll
        for (int k = 0; k < 4; ++k) xw[tid + k * kDecodeThreads] = d[k];
        named_bar_sync(1, 256);
        v = *reinterpret_cast<const uint4*>(s.xraw + tid * 8);
    }
    const float r = rms_scale_regs2048(v, 1e-6f, s.red, tid, 1);  // v = this thread's eight elements
    float xf[8], wf[8], of[8];
    unpack8(v, xf);
    unpack8(wv, wf);
#pragma unroll
    for (int e = 0; e < 8; ++e) of[e] = (xf[e] * r) * wf[e];
    *reinterpret_cast<uint4*>(s.xs + tid * 8) = pack8(of);
    if (stage_dst) *stage_dst = stage_val;  // a value loaded before the poll, visible after the barrier
    named_bar_sync(1, 256);
    const int lane = tid & 31;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint4 q = *reinterpret_cast<const uint4*>(s.xs + 256 * j + 8 * lane);
        xr[4 * j] = q.x; xr[4 * j + 1] = q.y; xr[4 * j + 2] = q.z; xr[4 * j + 3] = q.w;
    }
    return false;
}

__device__ __forceinline__ void epilogue(int ph, const DecodeArgs& a, const Smem& s, StepCtx& c, int u, float s0,
                                         float s1, float bias0, float bias1) {
    if (ph == PH_QKV) {
        const int sec = u / (kHidden / 2), v = u % (kHidden / 2), h = v / 64, t = v % 64;
        const float y1 = h2f(f2h(h2f(f2h(s0)) + bias0));
        const float y2 = h2f(f2h(h2f(f2h(s1)) + bias1));
        const int o1 = h * kHeadDim + t, o2 = o1 + 64;
        const size_t row = (size_t)c.pos * kHidden;
        half r1, r2;
        if (sec == 2) {
            r1 = f2h(y1);
            r2 = f2h(y2);
            c.vcl[row + o1] = r1;
            c.vcl[row + o2] = r2;
        } else {
            // fused_qkv_rope_cache.cuh:36-43 with the fast-math intrinsics
            const float theta = (float)c.pos * __powf(10000.0f, __fdividef(-2.0f * (float)t, (float)kHeadDim));
            const float cs = __cosf(theta), sn = __sinf(theta);
            r1 = f2h(y1 * cs - y2 * sn);
            r2 = f2h(y2 * cs + y1 * sn);
            if (sec == 1) {
                c.kcl[row + o1] = r1;
                c.kcl[row + o2] = r2;
            }
        }
        ll_store(a.ll_qkv + u, (uint32_t)__half_as_ushort(r1) | ((uint32_t)__half_as_ushort(r2) << 16), c.tag);
    } else if (ph == PH_O || ph == PH_C) {
        const int n = 2 * u;
        const half2 xo = *reinterpret_cast<const half2*>(s.xraw + n);
        const half2 r = __floats2half2_rn(h2f(__low2half(xo)) + h2f(f2h(s0)), h2f(__high2half(xo)) + h2f(f2h(s1)));
        const uint32_t bits = *reinterpret_cast<const uint32_t*>(&r);
        if (ph == PH_O) {
            ll_store(a.ll_xo + u, bits, c.tag);
        } else {
            ll_store(a.ll_xc + u, bits, c.tag);
            if (c.layer == a.NL - 1) *reinterpret_cast<half2*>(a.x + n) = r;
        }
    } else if (ph == PH_W12) {
        const float g = h2f(f2h(s0)), up = h2f(f2h(s1));
        ll_store(a.ll_act + u, (uint32_t)__half_as_ushort(f2h(g * __fdividef(up, 1.0f + __expf(-up)))), c.tag);
    } else {  // PH_LM
        const int n = 2 * u;
        const half l0 = f2h(s0), l1 = f2h(s1);
        *reinterpret_cast<half2*>(a.logits + n) = __halves2half2(l0, l1);
        const unsigned long long k0 = argmax_key(__half_as_ushort(l0), n, c.ipt);
        const unsigned long long k1 = argmax_key(__half_as_ushort(l1), n + 1, c.ipt);
        const unsigned long long k = k0 > k1 ? k0 : k1;
        c.best = k > c.best ? k : c.best;
    }
}

// Consume this CTA's units of one weight matrix (two rows each): unit i of the phase goes to
// warp i % 8, so the warps take the ring's chunks in sequence order and release the oldest slot
// first.  Each unit's warp releases it on the chunk's "empty" barrier (kEmptyArrivals per chunk:
// the last unit of a chunk adds the arrivals of the units the chunk does not have).  A wait that
// expires marks `bad` and the remaining units are skipped.  Phases run through one call site so
// the kernel's code stays small enough for the instruction caches (the phase id selects range,
// dot and epilogue).
__device__ __forceinline__ void gemv_phase(int PH, const DecodeArgs& a, Smem& s, StepCtx& c, uint32_t& chunk,
                                           const uint32_t* xr, int warp, int lane, bool& bad) {
    const int R = PH == PH_LM ? 4 : PH == PH_C ? 3 : PH == PH_W12 ? 2 : PH == PH_O ? 1 : 0;
    const int u0 = s.range[R][0], u1 = s.range[R][1], CH = s.range[R][2], K = s.range[R][3];
    unsigned long long pw = 0, pc = 0;  // per-unit cycle sums (profiling only)
    unsigned long long pmaxw = 0;       // longest single wait (profiling only)
    const int nu = u1 - u0;
    const uint32_t c0 = chunk;
    chunk = c0 + (uint32_t)((nu + CH - 1) / CH);
    for (int i = warp; i < nu; i += kConsumerWarps) {
        const int j = CH == 1 ? i : i / CH, r = i - j * CH;  // chunk of the phase, unit within it
        const uint32_t g = c0 + (uint32_t)j;
        const int slot = (int)(g & (kRingStages - 1));
        if (bad || s.fail) continue;
        const unsigned long long t0 = a.prof_prod ? (unsigned long long)clock64() : 0ull;
        if (!mbar_wait(&s.full[slot], (g >> 3) & 1, &s.fail)) {
            if (lane == 0) record_error(a.ctl, kErrRingTimeout, PH);
            s.fail = 1;
            bad = true;
            continue;
        }
        const unsigned long long t1 = a.prof_prod ? (unsigned long long)clock64() : 0ull;
        const half* rows = reinterpret_cast<const half*>(s.ring[slot]) + (size_t)r * 2 * K;
        float s0, s1;
        if (PH == PH_C) dot2_smem(rows, rows + K, s.act, K, lane, s0, s1);
        else dot2_regs(rows, xr, lane, s0, s1);
        const int u = u0 + i;
        // QKV: the unit's bias pair, read after the dot products (read before them, it put about
        // 1.5 us per layer on the critical path)
        float b0 = 0.f, b1 = 0.f;
        if (PH == PH_QKV && lane == 0) {
            if (nu <= kQkvBiasUnits) {  // staged by the QKV prologue
                b0 = s.qbias[i][0];
                b1 = s.qbias[i][1];
            } else {
                const int sec = u / (kHidden / 2), v = u % (kHidden / 2);
                const int i1 = sec * kHidden + (v / 64) * kHeadDim + (v % 64);
                b0 = h2f(c.bias[i1]);
                b1 = h2f(c.bias[i1 + 64]);
            }
        }
        if (lane == 0) {
            epilogue(PH, a, s, c, u, s0, s1, b0, b1);
            // every lane's reads of the slot are done (the butterfly consumed them): release it
            const int nun = nu - j * CH < CH ? nu - j * CH : CH;
            mbar_arrive_cnt(&s.empty[slot], r == nun - 1 ? kEmptyArrivals - (uint32_t)nun + 1u : 1u);
        }
        if (a.prof_prod) {
            pw += t1 - t0;
            pmaxw = (t1 - t0) > pmaxw ? (t1 - t0) : pmaxw;
            pc += (unsigned long long)clock64() - t1;
        }
    }
    if (a.prof_prod && lane == 0) {
        // per CTA, phase and warp: SM cycles waiting for chunks, computing; the longest wait
        unsigned long long* q = a.prof_prod + (((size_t)blockIdx.x * 6 + PH) * kConsumerWarps + warp) * 4;
        atomicAdd(q, pw);  // reductions: no round trip on the phase's critical path
        atomicAdd(q + 1, pc);
        atomicMax(q + 3, pmaxw);
    }
}


// Every layer's norm weights and QKV bias (and ln_f), spread over the grid, into L2 as evict-last
// lines at the start of a launch: together a few hundred KB that every step reads on its critical
// path, and that a demand miss would fetch from an HBM saturated by the weight stream.
__device__ void prefetch_small_vectors(const DecodeArgs& a, const Smem& s, int tid) {
    constexpr int kLinesPerLayer = (kHidden * 2 + kHidden * 2 + 3 * kHidden * 2) / 128;  // ln_1, ln_2, qkv_b
    const int total = a.NL * kLinesPerLayer + kHidden * 2 / 128;
    for (int i = blockIdx.x * kDecodeThreads + tid; i < total; i += gridDim.x * kDecodeThreads) {
        const int l = i / kLinesPerLayer, j = i % kLinesPerLayer;
        if (l >= a.NL) {
            prefetch_l2_keep(a.lnf + (size_t)(i - a.NL * kLinesPerLayer) * 64);
        } else {
            const LayerPtrs& L = s.layers[l];
            const half* p = j < 32 ? L.ln1 + j * 64 : j < 64 ? L.ln2 + (j - 32) * 64 : L.qkv_b + (j - 64) * 64;
            prefetch_l2_keep(p);
        }
    }
}
// L2 prefetch, one line per thread, of what the critical path of the coming
// phases reads from global memory besides flag words: the next layer's ln_1,
// ln_2 and QKV bias (ln_f as well at the last layer), and this CTA's rows of
// the KV cache for the attention phase (rows before pos, written by earlier
// steps).  With HBM saturated by the weight stream, a demand miss on these
// would cost several microseconds on the critical path.
__device__ void prefetch_norms(const DecodeArgs& a, const Smem& s, int l, int tid) {
    const LayerPtrs& N = s.layers[l + 1 < a.NL ? l + 1 : 0];
    if (tid < 32) prefetch_l2_keep(N.ln1 + tid * 64);
    else if (tid < 64) prefetch_l2_keep(N.ln2 + (tid - 32) * 64);
    else if (tid < 160) prefetch_l2_keep(N.qkv_b + (tid - 64) * 64);
    else if (tid < 192 && l + 1 == a.NL) prefetch_l2_keep(a.lnf + (tid - 160) * 64);
}
__device__ void prefetch_kv_rows(const DecodeArgs& a, int l, int pos, int tid) {
    const int b = blockIdx.x;
    if (b < kHeads * kAttnSplits) {
        const half* kcl = a.kc + (size_t)l * a.max_seqlen * kHidden;
        const half* vcl = a.vc + (size_t)l * a.max_seqlen * kHidden;
        const int h = b / kAttnSplits, sp = b % kAttnSplits, L = pos + 1;
        const int r0 = (int)((long long)L * sp / kAttnSplits), r1 = (int)((long long)L * (sp + 1) / kAttnSplits);
        const int rend = (r1 == L) ? L - 1 : r1;
        for (int i = tid; i < (rend - r0) * 4; i += kDecodeThreads) {
            const half* base = ((i & 2) ? vcl : kcl) + (size_t)(r0 + (i >> 2)) * kHidden + h * kHeadDim;
            prefetch_l2_line(base + (i & 1) * 64);
        }
    }
}

// Cached rows of one warp's attention share: half-warp hw takes rows
// w0 + 2j + hw (j < 4) of [w0, w1); lane (l & 15) holds dims 8(l & 15) ..
// +7 of each.  Loads past w1 are skipped (zero registers).  The rows were
// written by earlier steps (ordered by the step barrier) and prefetched to L2
// at the start of the layer; .cg keeps them out of the non-coherent L1.
__device__ __forceinline__ void kv_rows_load(const half* K, const half* V, int w0, int w1, int lane, uint4* kr,
                                             uint4* vr) {
    const int hw = lane >> 4, dl = (lane & 15) * 8;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int r = w0 + 2 * j + hw;
        kr[j] = vr[j] = make_uint4(0u, 0u, 0u, 0u);
        if (r < w1) {
            kr[j] = ld_cg_u4(K + (size_t)r * kHidden + dl);
            vr[j] = ld_cg_u4(V + (size_t)r * kHidden + dl);
        }
    }
}

// Fold the (up to 8) rows loaded by kv_rows_load into the half-warp's
// online-softmax state (m over scaled scores, l, unnormalised o8).  w0 and
// w1 are warp-uniform, so every shuffle runs with all 32 lanes.
__device__ __forceinline__ void kv_rows_fold(const uint4* kr, const uint4* vr, int w0, int w1, int lane,
                                             const float* q8, float scale, float& m, float& l, float* o8) {
    const int hw = lane >> 4;
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
    for (int j = 0; j < 4; ++j) {
        sc[j] = (w0 + 2 * j + hw < w1) ? sc[j] * scale : -INFINITY;
        mx = fmaxf(mx, sc[j]);
    }
    if (mx == -INFINITY) return;  // no row for this half-warp yet
    const float corr = (m == -INFINITY) ? 0.f : __expf(m - mx);
    l *= corr;
#pragma unroll
    for (int e = 0; e < 8; ++e) o8[e] *= corr;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float p = sc[j] == -INFINITY ? 0.f : __expf(sc[j] - mx);
        l += p;
        float vf[8];
        unpack8(vr[j], vf);
#pragma unroll
        for (int e = 0; e < 8; ++e) o8[e] = __fmaf_rn(p, vf[e], o8[e]);
    }
    m = mx;
}

// Split-KV attention of one (head, split) per CTA (qwen_infer.cu:646-677 with
// the reference's split-KV flash decoding, kernels/flash_decode_q1_opt.cuh:548-724): the
// CTA's rows < pos come from the KV cache, the query and row pos from the
// QKV phase's words.  Each warp folds its cached rows eight at a time (one
// L2 round trip per eight rows).  Splits 1..8 publish (o, m, l) partials as
// flag words; split 0 merges them in split order and publishes att for the
// head.  Returns the CTA-wide failure verdict.
__device__ bool attention_phase(const DecodeArgs& a, Smem& s, const StepCtx& c, const Tags& tags, int tid,
                                bool bad) {
    const int b = blockIdx.x;
    constexpr int S = kAttnSplits;
    const bool active = b < kHeads * S;
    const int h = active ? b / S : 0, sp = active ? b % S : 0, L = c.pos + 1;
    const int warp = tid >> 5, lane = tid & 31, dl = (lane & 15) * 8;
    const int r0 = (int)((long long)L * sp / S), r1 = (int)((long long)L * (sp + 1) / S);
    const bool has_new = active && r0 < L && r1 == L;  // this split owns row pos
    const int rend = has_new ? L - 1 : r1;             // rows from the cache
    const int n = active ? rend - r0 : 0;
    const int w0 = r0 + n * warp / 8, w1 = r0 + n * (warp + 1) / 8;
    const half* K = c.kcl + h * kHeadDim;
    const half* V = c.vcl + h * kHeadDim;
    uint4 kr[4], vr[4];
    const uint32_t tq = tags(c.step, c.layer, LL_QKV);
    float q8[8], m = -INFINITY, l = 0.f, o8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o8[e] = 0.f;
    // Each word is polled by one thread: threads 0..63 the query, 64..191 the
    // new row's k and v (only the split that owns row pos needs them).
    if (active && (tid < 64 || (has_new && tid < 192))) {
        const int sec = tid >> 6, t = tid & 63;
        uint32_t w[1] = {0};
        bad |= !ll_read<1>(a.ll_qkv + sec * (kHidden / 2) + h * 64 + t, 1, tq, w);
        s.qkv_new[sec][t] = __ushort_as_half((uint16_t)(w[0] & 0xffffu));
        s.qkv_new[sec][t + 64] = __ushort_as_half((uint16_t)(w[0] >> 16));
    }
    if (named_bar_or(1, 256, bad)) return true;
    if (active) {
        unpack8(*reinterpret_cast<const uint4*>(&s.qkv_new[0][dl]), q8);
        const float scale = __frcp_rn(sqrtf((float)kHeadDim));
#pragma unroll 1
        for (int r = w0; r < w1; r += 8) {
            const int re = w1 < r + 8 ? w1 : r + 8;
            kv_rows_load(K, V, r, re, lane, kr, vr);
            kv_rows_fold(kr, vr, r, re, lane, q8, scale, m, l, o8);
        }
        combine_halfwarps(m, l, o8);
        if (has_new && warp == 0) {
            // row pos from the QKV phase's words
            float kf[8], vf[8];
            unpack8(*reinterpret_cast<const uint4*>(&s.qkv_new[1][dl]), kf);
            unpack8(*reinterpret_cast<const uint4*>(&s.qkv_new[2][dl]), vf);
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) d = __fmaf_rn(q8[e], kf[e], d);
#pragma unroll
            for (int mk = 8; mk >= 1; mk >>= 1) d += __shfl_xor_sync(0xffffffffu, d, mk);
            const float sc = d * scale;
            const float mx = fmaxf(m, sc);
            const float corr = (m == -INFINITY) ? 0.f : __expf(m - mx);
            const float p = __expf(sc - mx);
            l = l * corr + p;
#pragma unroll
            for (int e = 0; e < 8; ++e) o8[e] = __fmaf_rn(p, vf[e], o8[e] * corr);
            m = mx;
        }
        if (lane < 16) {
#pragma unroll
            for (int e = 0; e < 8; ++e) s.so[warp][dl + e] = o8[e];
        }
        if (lane == 0) { s.sm[warp] = m; s.sl[warp] = l; }
    }
    if (named_bar_or(1, 256, bad)) return true;
    if (!active) return false;
    // This CTA's partial (o[128] normalised by nothing, m, l) over its rows.
    const uint32_t tp = tags(c.step, c.layer, LL_APART);
    float acc = 0.f, Ls = 0.f, M = -INFINITY;
    if (tid < kHeadDim) {
        for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, s.sm[w]);
        for (int w = 0; w < kConsumerWarps; ++w) {
            if (s.sm[w] == -INFINITY) continue;
            const float f = __expf(s.sm[w] - M);
            Ls += s.sl[w] * f;
            acc += s.so[w][tid] * f;
        }
    }
    unsigned long long* part = a.ll_apart + (size_t)h * S * 130;
    if (sp != 0) {
        // publish as flag-carrying words; split 0 of the head merges
        if (tid < kHeadDim) ll_store(part + sp * 130 + tid, __float_as_uint(acc), tp);
        if (tid == 0) {
            ll_store(part + sp * 130 + 128, __float_as_uint(M), tp);
            ll_store(part + sp * 130 + 129, __float_as_uint(Ls), tp);
        }
        return false;
    }
    // split 0: gather the other splits' partials into shared memory (s.so rows
    // 0..S-2 hold o of splits 1..S-1, s.sm / s.sl their m and l), then merge
    named_bar_sync(1, 256);  // every warp is done reading s.so / s.sm / s.sl
    static_assert(kAttnSplits - 1 <= kConsumerWarps, "one shared row per other split");
    {
        constexpr int kWords = (S - 1) * 130, kPer = (kWords + kDecodeThreads - 1) / kDecodeThreads;
        const int nw = (kWords - tid + kDecodeThreads - 1) / kDecodeThreads;
        uint32_t d[kPer];
        bad |= !ll_read_n<kPer>(part + 130 + tid, kDecodeThreads, nw, tp, d);
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            if (k >= nw) break;
            const int i = tid + k * kDecodeThreads, j = i / 130, e = i % 130;
            const float v = __uint_as_float(d[k]);
            if (e < kHeadDim) s.so[j][e] = v;
            else if (e == kHeadDim) s.sm[j] = v;
            else s.sl[j] = v;
        }
    }
    if (named_bar_or(1, 256, bad)) return true;
    if (tid < kHeadDim) {
        // merge in split order: own partial first, then splits 1..S-1
        float Mx = M;
        for (int j = 0; j < S - 1; ++j) Mx = fmaxf(Mx, s.sm[j]);
        float L2 = 0.f, o = 0.f;
        if (M != -INFINITY) {
            const float f = __expf(M - Mx);
            L2 += Ls * f;
            o += acc * f;
        }
        for (int j = 0; j < S - 1; ++j) {
            if (s.sm[j] == -INFINITY) continue;
            const float f = __expf(s.sm[j] - Mx);
            L2 += s.sl[j] * f;
            o += s.so[j][tid] * f;
        }
        const float r = o * __frcp_rn(L2);
        // dims (2i, 2i+1) travel as one word: pair up through shared memory
        s.so[kConsumerWarps - 1][tid] = r;
    }
    named_bar_sync(1, 256);
    if (tid < kHeadDim / 2) {
        const half2 r = __floats2half2_rn(s.so[kConsumerWarps - 1][2 * tid], s.so[kConsumerWarps - 1][2 * tid + 1]);
        ll_store(a.ll_att + h * 64 + tid, *reinterpret_cast<const uint32_t*>(&r), tags(c.step, c.layer, LL_ATT));
    }
    return false;
}

__device__ void consumers(const DecodeArgs& a, Smem& s) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t chunk = 0, nbar = 0;
    int token = a.first_token;
    StepCtx c;
    uint32_t xr[32];  // this lane's 64 fp16 activation values of the current phase
    c.ipt = (a.V + 511) / 512;
    const Tags tags{a.flag_base, a.NL};
    bool bad = false;
    int np = 0;  // probe index
    prefetch_small_vectors(a, s, tid);
    for (int step = 0; step < a.n_steps; ++step) {
        c.pos = a.pos0 + step;
        c.step = step;
        bool failed = false;
        // Phases of the step: per layer QKV, O, W12, C (qwen_infer.cu:626-721), then LM
        // (qwen_infer.cu:725-731).  Each phase: probe A, prologue (its input vector
        // into xr or s.act; probe B once the input words have arrived), probe C, GEMV.
        const int nph = a.NL * 4 + (a.skip_lm ? 0 : 1);
#pragma unroll 1
        for (int k = 0; k < nph; ++k) {
            const int ph = k == a.NL * 4 ? PH_LM : (k & 3) == 0 ? PH_QKV : (k & 3) == 1 ? PH_O : (k & 3) == 2 ? PH_W12 : PH_C;
            const int l = ph == PH_LM ? a.NL - 1 : k >> 2;
            const LayerPtrs& L = s.layers[l];
            if (ph == PH_QKV) {
                c.layer = l;
                c.kcl = a.kc + (size_t)l * a.max_seqlen * kHidden;
                c.vcl = a.vc + (size_t)l * a.max_seqlen * kHidden;
                c.bias = L.qkv_b;
                prefetch_norms(a, s, l, tid);
                if (l == 0) prefetch_kv_rows(a, 0, c.pos, tid);
            }
            probe(a, tid, np);
            if (ph == PH_O) {
                // attention (qwen_infer.cu:646-677), then each thread polls its own
                // four words of att into shared memory and every warp takes its slice
                failed = attention_phase(a, s, c, tags, tid, bad);
                if (failed) break;
                probe(a, tid, np);
                uint32_t d[4];
                bad |= !ll_read<4>(a.ll_att + tid, kDecodeThreads, tags(step, l, LL_ATT), d);
                failed = named_bar_or(1, 256, bad);  // the previous phase is done with s.xs
                if (failed) break;
#pragma unroll
                for (int k = 0; k < 4; ++k) reinterpret_cast<uint32_t*>(s.xs)[tid + k * kDecodeThreads] = d[k];
                named_bar_sync(1, 256);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint4 q = *reinterpret_cast<const uint4*>(s.xs + 256 * j + 8 * lane);
                    xr[4 * j] = q.x; xr[4 * j + 1] = q.y; xr[4 * j + 2] = q.z; xr[4 * j + 3] = q.w;
                }
            } else if (ph == PH_C) {
                // SwiGLU output into s.act.  s.act was last read by the previous
                // layer's C phase, which every warp has left (several named
                // barriers since), so the words go straight to shared memory.
                if (l + 1 < a.NL) prefetch_kv_rows(a, l + 1, c.pos, tid);
                const int n = (a.IM - tid + kDecodeThreads - 1) / kDecodeThreads;
                bad |= !ll_gather_act(a.ll_act + tid, n, tags(step, l, LL_ACT), s.act + tid);
                failed = named_bar_or(1, 256, bad);
                if (failed) break;
                probe(a, tid, np);
            } else {
                // RMSNorm of the residual stream: the embedding row (first layer),
                // the previous layer's output, or this layer's attention residual
                const half* plain = (ph == PH_QKV && l == 0) ? a.wte + (size_t)token * kHidden : nullptr;
                const unsigned long long* src = ph == PH_W12 ? a.ll_xo : a.ll_xc;
                const uint32_t tag = ph == PH_W12 ? tags(step, l, LL_XO)
                                     : ph == PH_LM ? tags(step, l, LL_XC)
                                                   : (l > 0 ? tags(step, l - 1, LL_XC) : 0u);
                const half* w = ph == PH_QKV ? L.ln1 : ph == PH_W12 ? L.ln2 : a.lnf;
                // QKV: thread i loads half (i & 1) of the bias pair of QKV unit u0 + i / 2 now;
                // load_norm stores it into s.qbias once its poll is over
                float* bdst = nullptr;
                float bval = 0.f;
                if (ph == PH_QKV) {
                    const int u0 = s.range[0][0], nu = s.range[0][1] - u0;
                    if (nu <= kQkvBiasUnits && tid < 2 * nu) {
                        const int u = u0 + (tid >> 1), sec = u / (kHidden / 2), v = u % (kHidden / 2);
                        const int i1 = sec * kHidden + (v / 64) * kHeadDim + (v % 64) + (tid & 1) * 64;
                        bval = h2f(L.qkv_b[i1]);
                        bdst = &s.qbias[tid >> 1][tid & 1];
                    }
                }
                failed = load_norm(a, plain, src, tag, w, s, tid, xr, bad, np, bdst, bval);
                if (failed) break;
            }
            c.tag = tags(step, l, ph == PH_QKV ? LL_QKV : ph == PH_O ? LL_XO : ph == PH_W12 ? LL_ACT : LL_XC);
            c.best = 0ull;
            probe(a, tid, np);
            gemv_phase(ph, a, s, c, chunk, xr, warp, lane, bad);
        }
        if (failed) break;
        if (a.skip_lm) {
            // prefill through the decode path: the step barrier orders this step's KV rows
            if (!grid_sync(a, s, nbar, tid, bad, np)) break;
            if (step + 1 < a.n_steps) token = a.forced[step + 1];
            if (blockIdx.x == 0 && tid == 0) a.ctl->n_done = step + 1;
            continue;
        }
        // argmax over the CTAs' best keys (argmax.cuh tie rule, see argmax_key)
        c.best = warp_max_u64(c.best);  // the epilogue lanes each tracked their own units
        if (lane == 0) s.wkey[warp] = c.best;
        named_bar_sync(1, 256);
        if (tid == 0) {
            unsigned long long k = 0ull;
            for (int w = 0; w < kConsumerWarps; ++w) k = s.wkey[w] > k ? s.wkey[w] : k;
            if (k) atomicMax(&a.ctl->best[step & 1], k);
        }
        if (!grid_sync(a, s, nbar, tid, bad, np)) break;
        if (tid == 0) {
            const unsigned long long k = atomicOr(&a.ctl->best[step & 1], 0ull);
            const int t = argmax_key_index(k);
            s.token = t;
            if (blockIdx.x == 0) {
                if (a.tokens_out) a.tokens_out[step] = t;
                if (a.host_tokens) {
                    *(volatile int*)(a.host_tokens + step) = t;
                    __threadfence_system();
                    *(volatile int*)a.host_count = step + 1;
                }
                a.ctl->best[(step + 1) & 1] = 0ull;
                a.ctl->n_done = step + 1;
            }
        }
        named_bar_sync(1, 256);
        token = s.token;
        if (token < 0 || token >= a.V) {
            if (tid == 0 && blockIdx.x == 0) record_error(a.ctl, kErrBadToken, PH_LM);
            break;
        }
        if (token == a.stop0 || token == a.stop1) break;
    }
    if (bad) record_error(a.ctl, kErrHeadMergeTimeout, -1);
    // the producer stops issuing once it sees this (and drains its copies in flight)
    if (tid == 0) s.stop = 1;
}

__global__ void __launch_bounds__(kDecodeBlock, 1) decode_kernel(const DecodeArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);
    if (threadIdx.x == 0) {
        for (int i = 0; i < kRingStages; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], kEmptyArrivals);
        }
        s.fail = 0;
        s.stop = 0;
        mbar_fence_init();
    }
    for (int i = threadIdx.x; i < a.NL * (int)(sizeof(LayerPtrs) / sizeof(uint64_t)); i += blockDim.x)
        reinterpret_cast<uint64_t*>(s.layers)[i] = reinterpret_cast<const uint64_t*>(a.layers)[i];
    if (threadIdx.x < 5) {
        // this CTA's unit range of each phase: the same for every layer and step
        const PhaseRange r = phase_range(threadIdx.x, a.IM, a.V, blockIdx.x, gridDim.x);
        s.range[threadIdx.x][0] = r.u0;
        s.range[threadIdx.x][1] = r.u1;
        s.range[threadIdx.x][2] = r.CH;
        s.range[threadIdx.x][3] = r.K;
    }
    __syncthreads();
    // from here on the consumer warps synchronise on named barrier 1 (256 threads) only
    if (threadIdx.x >= kDecodeThreads) producer(a, s);
    else consumers(a, s);
}

}  // namespace

static_assert(sizeof(Smem) <= 232448, "the decode kernel's shared memory exceeds the 227 KB opt-in limit");
size_t decode_smem_bytes() { return sizeof(Smem); }

// Number of flag tags one launch of n_steps consumes (the host advances its
// running tag base by this much after every launch).
uint32_t decode_tags_per_launch(int n_steps, int num_layers) {
    return (uint32_t)(n_steps * num_layers * LL_PER_LAYER + 1);
}

cudaError_t launch_decode(const DecodeArgs& a, int grid, cudaStream_t stream) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(Smem));
    if (e != cudaSuccess) return e;
    void* args[] = {const_cast<DecodeArgs*>(&a)};
    return cudaLaunchCooperativeKernel((const void*)decode_kernel, dim3(grid), dim3(kDecodeBlock), args,
                                       sizeof(Smem), stream);
}

}  // namespace llmdiy
