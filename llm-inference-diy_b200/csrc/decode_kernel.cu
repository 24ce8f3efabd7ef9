// decode_kernel.cu — the persistent bs1 decode kernel (QwenEngine::step,
// framework_src/qwen_infer.cu:614-737, for many steps per launch).
//
// One CTA per SM.  Warp 8 lane 0 is a producer that streams this CTA's share
// of every weight matrix, in the exact order the consumers use it, through an
// 8-stage ring of 24 KB shared-memory slots with 1-D bulk copies (TMA).
// Weights never depend on activations, so the producer runs ahead across
// phase, layer and token boundaries and HBM keeps streaming while the
// consumers wait at grid barriers.  Warps 0-7 are consumers: slot s is always
// drained by warp s, two rows at a time (fp32 FMA dot products against the
// activation held in registers or shared memory), with the reference's small
// ops fused into the epilogues:
//   QKV  : RMSNorm(ln_1) prologue; bias; RoPE; K/V append at row pos; q out
//   ATT  : 16 heads x 9 position splits; last CTA of a head merges (m,l,o)
//   O    : residual add into x
//   W12  : RMSNorm(ln_2) prologue; SwiGLU (silu on the w2 output)
//   C    : residual add into x
//   LM   : RMSNorm(ln_f) prologue; logits; greedy argmax key (reference tie rule)
// Phases are separated by grid barriers on one monotonically increasing
// counter.  Every spin-wait is bounded; on expiry the kernel records an error
// code in DecodeControl and returns.
#include "decode.h"
#include "ops.cuh"

namespace llmdiy {
namespace {

enum PhaseId { PH_QKV = 0, PH_ATT = 1, PH_O = 2, PH_W12 = 3, PH_C = 4, PH_LM = 5 };

constexpr int kMaxIM = 6144;

struct __align__(128) Smem {
    uint8_t ring[kRingStages][kStageBytes];
    half xs[kHidden];
    half act[kMaxIM];
    float so[kConsumerWarps][kHeadDim];
    float sm[kConsumerWarps], sl[kConsumerWarps];
    float red[32];
    unsigned long long wkey[kConsumerWarps];
    uint64_t full[kRingStages], empty[kRingStages];
    volatile int stop;  // consumers -> producer: stop streaming and drain
    volatile int fail;  // consumer-side failure broadcast
    int token;
    int last;
};

__device__ __forceinline__ int chunk_units(int K) {
    int u = kStageBytes / (4 * K);
    return u < 1 ? 1 : u;
}

__device__ void record_error(DecodeControl* ctl, int code, int where) {
    if (atomicCAS(&ctl->err, 0, code) == 0) ctl->err_where = where;
}

// ------------------------------------------------------------------ producer
__device__ bool stream_phase(const half* W, int U, int K, uint32_t& chunk, Smem& s, uint64_t pol) {
    const int b = blockIdx.x, G = gridDim.x;
    const int u0 = (int)((long long)U * b / G), u1 = (int)((long long)U * (b + 1) / G);
    const int CH = chunk_units(K);
    for (int cu = u0; cu < u1; cu += CH) {
        const int nun = (u1 - cu) < CH ? (u1 - cu) : CH;
        const int slot = chunk & (kRingStages - 1);
        if (chunk >= (uint32_t)kRingStages) {
            if (!mbar_wait(&s.empty[slot], ((chunk >> 3) - 1) & 1, &s.stop)) return false;
        }
        const uint32_t bytes = (uint32_t)nun * 4u * (uint32_t)K;
        mbar_arrive_expect_tx(&s.full[slot], bytes);
        bulk_g2s(s.ring[slot], W + (size_t)cu * 2 * K, bytes, &s.full[slot], pol);
        ++chunk;
    }
    return true;
}

__device__ void producer(const DecodeArgs& a, Smem& s) {
    const uint64_t pol = l2_policy_evict_first();
    uint32_t chunk = 0;
    bool ok = true;
    for (int step = 0; step < a.n_steps && ok; ++step) {
        for (int l = 0; l < a.NL && ok; ++l) {
            const LayerPtrs L = a.layers[l];
            ok = stream_phase(L.qkv_w, 3 * kHidden / 2, kHidden, chunk, s, pol) &&
                 stream_phase(L.proj_w, kHidden / 2, kHidden, chunk, s, pol) &&
                 stream_phase(L.w12, a.IM, kHidden, chunk, s, pol) &&
                 stream_phase(L.cproj, kHidden / 2, a.IM, chunk, s, pol);
        }
        if (ok && !a.skip_lm) ok = stream_phase(a.lm_head, a.V / 2, kHidden, chunk, s, pol);
    }
    // Drain: wait until every copy this CTA issued has landed before exiting.
    for (int slot = 0; slot < kRingStages; ++slot) {
        if (chunk > (uint32_t)slot) {
            const uint32_t c = slot + 8u * ((chunk - 1u - slot) / 8u);
            mbar_wait(&s.full[slot], (c >> 3) & 1);
        }
    }
}

// ------------------------------------------------------------------ consumers
__device__ __forceinline__ void dot2_regs(const half* r0, const half* r1, const float* xr, int lane, float& s0,
                                          float& s1) {
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint4 w0 = *reinterpret_cast<const uint4*>(r0 + 256 * j + 8 * lane);
        const uint4 w1 = *reinterpret_cast<const uint4*>(r1 + 256 * j + 8 * lane);
        float f0[8], f1[8];
        unpack8(w0, f0);
        unpack8(w1, f1);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            a0 = __fmaf_rn(f0[e], xr[8 * j + e], a0);
            a1 = __fmaf_rn(f0[e + 1], xr[8 * j + e + 1], a1);
            b0 = __fmaf_rn(f1[e], xr[8 * j + e], b0);
            b1 = __fmaf_rn(f1[e + 1], xr[8 * j + e + 1], b1);
        }
    }
    s0 = a0 + a1;
    s1 = b0 + b1;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        s0 += __shfl_xor_sync(0xffffffffu, s0, m);
        s1 += __shfl_xor_sync(0xffffffffu, s1, m);
    }
}

__device__ __forceinline__ void dot2_smem(const half* r0, const half* r1, const half* xs, int K, int lane, float& s0,
                                          float& s1) {
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll 2
    for (int k = 8 * lane; k < K; k += 256) {
        const uint4 w0 = *reinterpret_cast<const uint4*>(r0 + k);
        const uint4 w1 = *reinterpret_cast<const uint4*>(r1 + k);
        const uint4 xv = *reinterpret_cast<const uint4*>(xs + k);
        float f0[8], f1[8], xf[8];
        unpack8(w0, f0);
        unpack8(w1, f1);
        unpack8(xv, xf);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            a0 = __fmaf_rn(f0[e], xf[e], a0);
            a1 = __fmaf_rn(f0[e + 1], xf[e + 1], a1);
            b0 = __fmaf_rn(f1[e], xf[e], b0);
            b1 = __fmaf_rn(f1[e + 1], xf[e + 1], b1);
        }
    }
    s0 = a0 + a1;
    s1 = b0 + b1;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        s0 += __shfl_xor_sync(0xffffffffu, s0, m);
        s1 += __shfl_xor_sync(0xffffffffu, s1, m);
    }
}

struct StepCtx {
    int pos, step;
    half* kcl;
    half* vcl;
    const half* bias;
    int ipt;
    unsigned long long best;  // lane 0 of each warp: best argmax key seen in the LM phase
};

// Grid-wide barrier over all CTAs (called by the 256 consumer threads).  The
// named barriers always run, so a failure anywhere in the CTA never leaves a
// consumer warp waiting on bar.sync; the global spin gives up when the count
// does not arrive within the bound or when another CTA has recorded an error.
__device__ bool grid_sync(const DecodeArgs& a, Smem& s, uint32_t& nbar, int tid, int where) {
    named_bar_sync(1, 256);
    ++nbar;
    bool failed = false;
    if (tid == 0) {
        __threadfence();
        red_release_gpu_add(&a.ctl->bar, 1u);
        failed = s.fail != 0;
        if (!failed) {
            const uint32_t target = nbar * gridDim.x;
            bool ok = false;
            for (uint32_t i = 0; i < kSpinLimit; ++i) {
                if (ld_acquire_gpu(&a.ctl->bar) >= target) { ok = true; break; }
                if ((i & 63) == 63 && *(volatile int*)&a.ctl->err != 0) break;
                if (i > 512) __nanosleep(32);
            }
            if (!ok) {
                record_error(a.ctl, kErrGridBarrierTimeout, where);
                s.fail = 1;
                failed = true;
            }
        }
        __threadfence();
    }
    // every consumer thread gets the same verdict, so later branches stay CTA-uniform
    return !named_bar_or(1, 256, failed);
}

// Stage x (global) in shared memory, RMSNorm it with the reference tree, and
// leave each lane's 64-element slice of the normalised vector in xr.
__device__ void load_norm(const half* src, bool written_this_launch, const half* w, half* copy_out, Smem& s,
                          int tid, float* xr) {
    const uint4 v = written_this_launch ? ld_cg_u4(src + tid * 8) : *reinterpret_cast<const uint4*>(src + tid * 8);
    *reinterpret_cast<uint4*>(s.xs + tid * 8) = v;
    if (copy_out) *reinterpret_cast<uint4*>(copy_out + tid * 8) = v;
    const float r = rms_scale_tree256(s.xs, kHidden, 1e-6f, s.red, tid, 1);
    float xf[8], wf[8], of[8];
    unpack8(v, xf);
    unpack8(*reinterpret_cast<const uint4*>(w + tid * 8), wf);
#pragma unroll
    for (int e = 0; e < 8; ++e) of[e] = (xf[e] * r) * wf[e];
    *reinterpret_cast<uint4*>(s.xs + tid * 8) = pack8(of);
    named_bar_sync(1, 256);
    const int lane = tid & 31;
#pragma unroll
    for (int j = 0; j < 8; ++j) unpack8(*reinterpret_cast<const uint4*>(s.xs + 256 * j + 8 * lane), xr + 8 * j);
}

template <int PH>
__device__ __forceinline__ void epilogue(const DecodeArgs& a, StepCtx& c, int u, float s0, float s1) {
    if constexpr (PH == PH_QKV) {
        const int sec = u / (kHidden / 2), v = u % (kHidden / 2), h = v / 64, t = v % 64;
        const int i1 = sec * kHidden + h * kHeadDim + t, i2 = i1 + 64;
        const float y1 = h2f(f2h(h2f(f2h(s0)) + h2f(c.bias[i1])));
        const float y2 = h2f(f2h(h2f(f2h(s1)) + h2f(c.bias[i2])));
        const int o1 = h * kHeadDim + t, o2 = o1 + 64;
        const size_t row = (size_t)c.pos * kHidden;
        if (sec == 2) {
            c.vcl[row + o1] = f2h(y1);
            c.vcl[row + o2] = f2h(y2);
        } else {
            // fused_qkv_rope_cache.cuh:36-43 with the fast-math intrinsics
            const float theta = (float)c.pos * __powf(10000.0f, __fdividef(-2.0f * (float)t, (float)kHeadDim));
            const float cs = __cosf(theta), sn = __sinf(theta);
            const half r1 = f2h(y1 * cs - y2 * sn);
            const half r2 = f2h(y2 * cs + y1 * sn);
            if (sec == 0) {
                a.q[o1] = r1;
                a.q[o2] = r2;
            } else {
                c.kcl[row + o1] = r1;
                c.kcl[row + o2] = r2;
            }
        }
    } else if constexpr (PH == PH_O || PH == PH_C) {
        const int n = 2 * u;
        const half2 xo = __halves2half2(__ushort_as_half(ld_cg_u16(a.x + n)), __ushort_as_half(ld_cg_u16(a.x + n + 1)));
        const float r0 = h2f(__low2half(xo)) + h2f(f2h(s0));
        const float r1 = h2f(__high2half(xo)) + h2f(f2h(s1));
        *reinterpret_cast<half2*>(a.x + n) = __floats2half2_rn(r0, r1);
    } else if constexpr (PH == PH_W12) {
        const float g = h2f(f2h(s0)), up = h2f(f2h(s1));
        a.act[u] = f2h(g * __fdividef(up, 1.0f + __expf(-up)));
    } else if constexpr (PH == PH_LM) {
        const int n = 2 * u;
        const half l0 = f2h(s0), l1 = f2h(s1);
        *reinterpret_cast<half2*>(a.logits + n) = __halves2half2(l0, l1);
        const unsigned long long k0 = argmax_key(__half_as_ushort(l0), n, c.ipt);
        const unsigned long long k1 = argmax_key(__half_as_ushort(l1), n + 1, c.ipt);
        const unsigned long long k = k0 > k1 ? k0 : k1;
        c.best = k > c.best ? k : c.best;
    }
}

template <int PH, bool kRegs>
__device__ void gemv_phase(const DecodeArgs& a, Smem& s, StepCtx& c, int U, int K, uint32_t& chunk, const float* xr,
                           int warp, int lane) {
    const int b = blockIdx.x, G = gridDim.x;
    const int u0 = (int)((long long)U * b / G), u1 = (int)((long long)U * (b + 1) / G);
    const int CH = chunk_units(K);
    for (int cu = u0; cu < u1; cu += CH, ++chunk) {
        if ((int)(chunk & (kRingStages - 1)) != warp) continue;
        const int nun = (u1 - cu) < CH ? (u1 - cu) : CH;
        if (s.fail) continue;
        if (!mbar_wait(&s.full[warp], (chunk >> 3) & 1, &s.fail)) {
            if (lane == 0) record_error(a.ctl, kErrRingTimeout, PH);
            s.fail = 1;
            continue;
        }
        const half* buf = reinterpret_cast<const half*>(s.ring[warp]);
        for (int j = 0; j < nun; ++j) {
            const half* r0 = buf + (size_t)j * 2 * K;
            float s0, s1;
            if constexpr (kRegs) dot2_regs(r0, r0 + K, xr, lane, s0, s1);
            else dot2_smem(r0, r0 + K, s.act, K, lane, s0, s1);
            if (lane == 0) epilogue<PH>(a, c, cu + j, s0, s1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.empty[warp]);
    }
}

// Split-KV attention of one (head, split) per CTA; the last CTA to finish a
// head merges the 9 partials into att[h*128 .. +128] (fp16).
__device__ void attention_phase(const DecodeArgs& a, Smem& s, const StepCtx& c, int tid) {
    const int b = blockIdx.x;
    constexpr int S = kAttnSplits;
    if (b >= kHeads * S) return;
    const int h = b / S, sp = b % S, L = c.pos + 1;
    const int warp = tid >> 5, lane = tid & 31, dl = (lane & 15) * 8;
    const int r0 = (int)((long long)L * sp / S), r1 = (int)((long long)L * (sp + 1) / S);
    const int n = r1 - r0;
    const int w0 = r0 + n * warp / 8, w1 = r0 + n * (warp + 1) / 8;
    float q8[8];
    unpack8(ld_cg_u4(a.q + h * kHeadDim + dl), q8);
    const float scale = __frcp_rn(sqrtf((float)kHeadDim));
    float m = -INFINITY, l = 0.f, o8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o8[e] = 0.f;
    if (w0 < w1) attend_rows<true>(c.kcl + h * kHeadDim, c.vcl + h * kHeadDim, kHidden, w0, w1, q8, scale, m, l, o8);
    combine_halfwarps(m, l, o8);
    if (lane < 16) {
#pragma unroll
        for (int e = 0; e < 8; ++e) s.so[warp][dl + e] = o8[e];
    }
    if (lane == 0) { s.sm[warp] = m; s.sl[warp] = l; }
    named_bar_sync(1, 256);
    float* part = a.att_part + (size_t)(h * S + sp) * 130;
    if (tid < kHeadDim) {
        float M = -INFINITY;
        for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, s.sm[w]);
        float Ls = 0.f, acc = 0.f;
        for (int w = 0; w < kConsumerWarps; ++w) {
            if (s.sm[w] == -INFINITY) continue;
            const float f = __expf(s.sm[w] - M);
            Ls += s.sl[w] * f;
            acc += s.so[w][tid] * f;
        }
        part[tid] = acc;
        if (tid == 0) { part[128] = M; part[129] = Ls; }
    }
    named_bar_sync(1, 256);
    if (tid == 0) {
        __threadfence();
        const unsigned int old = atomicAdd(&a.ctl->head_ctr[h], 1u);
        s.last = ((old + 1u) % (unsigned)S) == 0u;
        __threadfence();
    }
    named_bar_sync(1, 256);
    if (s.last && tid < kHeadDim) {
        const float* base = a.att_part + (size_t)h * S * 130;
        float M = -INFINITY;
        for (int j = 0; j < S; ++j) M = fmaxf(M, __ldcg(base + j * 130 + 128));
        float Ls = 0.f, acc = 0.f;
        for (int j = 0; j < S; ++j) {
            const float mj = __ldcg(base + j * 130 + 128);
            if (mj == -INFINITY) continue;
            const float f = __expf(mj - M);
            Ls += __ldcg(base + j * 130 + 129) * f;
            acc += __ldcg(base + j * 130 + tid) * f;
        }
        a.att[h * kHeadDim + tid] = f2h(acc * __frcp_rn(Ls));
    }
}

__device__ void consumers(const DecodeArgs& a, Smem& s) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t chunk = 0, nbar = 0;
    int token = a.first_token;
    float xr[64];
    StepCtx c;
    c.ipt = (a.V + 511) / 512;
    for (int step = 0; step < a.n_steps; ++step) {
        c.pos = a.pos0 + step;
        c.step = step;
        const half* emb = a.wte + (size_t)token * kHidden;
        bool ok = true;
        for (int l = 0; l < a.NL && ok; ++l) {
            const LayerPtrs L = a.layers[l];
            c.kcl = a.kc + (size_t)l * a.max_seqlen * kHidden;
            c.vcl = a.vc + (size_t)l * a.max_seqlen * kHidden;
            c.bias = L.qkv_b;
            // QKV (qwen_infer.cu:626-642)
            if (l == 0) load_norm(emb, false, L.ln1, blockIdx.x == 0 ? a.x : nullptr, s, tid, xr);
            else load_norm(a.x, true, L.ln1, nullptr, s, tid, xr);
            gemv_phase<PH_QKV, true>(a, s, c, 3 * kHidden / 2, kHidden, chunk, xr, warp, lane);
            if (!grid_sync(a, s, nbar, tid, PH_QKV)) { ok = false; break; }
            // attention (qwen_infer.cu:646-677)
            attention_phase(a, s, c, tid);
            if (!grid_sync(a, s, nbar, tid, PH_ATT)) { ok = false; break; }
            // o_proj + residual (qwen_infer.cu:701-704)
#pragma unroll
            for (int j = 0; j < 8; ++j) unpack8(ld_cg_u4(a.att + 256 * j + 8 * lane), xr + 8 * j);
            gemv_phase<PH_O, true>(a, s, c, kHidden / 2, kHidden, chunk, xr, warp, lane);
            if (!grid_sync(a, s, nbar, tid, PH_O)) { ok = false; break; }
            // RMSNorm + w1/w2 + SwiGLU (qwen_infer.cu:708-715)
            load_norm(a.x, true, L.ln2, nullptr, s, tid, xr);
            gemv_phase<PH_W12, true>(a, s, c, a.IM, kHidden, chunk, xr, warp, lane);
            if (!grid_sync(a, s, nbar, tid, PH_W12)) { ok = false; break; }
            // c_proj + residual (qwen_infer.cu:718-721)
            for (int i = tid * 8; i < a.IM; i += 256 * 8)
                *reinterpret_cast<uint4*>(s.act + i) = ld_cg_u4(a.act + i);
            named_bar_sync(1, 256);
            gemv_phase<PH_C, false>(a, s, c, kHidden / 2, a.IM, chunk, xr, warp, lane);
            if (!grid_sync(a, s, nbar, tid, PH_C)) { ok = false; break; }
        }
        if (!ok) break;
        if (a.skip_lm) {
            if (step + 1 < a.n_steps) token = a.forced[step + 1];
            if (blockIdx.x == 0 && tid == 0) a.ctl->n_done = step + 1;
            continue;
        }
        // final RMSNorm + lm_head + argmax (qwen_infer.cu:725-731)
        load_norm(a.x, true, a.lnf, nullptr, s, tid, xr);
        c.best = 0ull;
        gemv_phase<PH_LM, true>(a, s, c, a.V / 2, kHidden, chunk, xr, warp, lane);
        if (lane == 0) s.wkey[warp] = c.best;
        named_bar_sync(1, 256);
        if (tid == 0) {
            unsigned long long k = 0ull;
            for (int w = 0; w < kConsumerWarps; ++w) k = s.wkey[w] > k ? s.wkey[w] : k;
            if (k) atomicMax(&a.ctl->best[step & 1], k);
        }
        if (!grid_sync(a, s, nbar, tid, PH_LM)) break;
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
    if (tid == 0) s.stop = 1;
}

__global__ void __launch_bounds__(kDecodeThreads, 1) decode_kernel(const DecodeArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);
    if (threadIdx.x == 0) {
        for (int i = 0; i < kRingStages; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        s.stop = 0;
        s.fail = 0;
        mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x >= kConsumerWarps * 32) {
        if (threadIdx.x == kConsumerWarps * 32) producer(a, s);
        return;
    }
    consumers(a, s);
}

}  // namespace

size_t decode_smem_bytes() { return sizeof(Smem); }

cudaError_t launch_decode(const DecodeArgs& a, int grid, cudaStream_t stream) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(Smem));
    if (e != cudaSuccess) return e;
    void* args[] = {const_cast<DecodeArgs*>(&a)};
    return cudaLaunchCooperativeKernel((const void*)decode_kernel, dim3(grid), dim3(kDecodeThreads), args,
                                       sizeof(Smem), stream);
}

}  // namespace llmdiy
