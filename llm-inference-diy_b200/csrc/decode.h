// decode.h — host/device contract of the persistent decode kernel.
//
// Device weight layout (chosen by this engine; the .bin file keeps the
// reference's [out,in] = [N,K] row-major layout, model_weights/convert_weights.py:107-185):
//   * every GEMV weight stays [N,K] (output rows contiguous along K), so a
//     group of consecutive rows is one contiguous byte range that a single
//     bulk copy moves into shared memory;
//   * qkv_w rows are permuted so that RoPE partners sit next to each other:
//     unit u of section s (0=q,1=k,2=v), head h, t<64 holds rows
//     (s*H + h*128 + t, s*H + h*128 + 64 + t);
//   * ffn_w1 / ffn_w2 are interleaved row by row (w12 row 2n = w1 row n,
//     row 2n+1 = w2 row n), so one unit carries both SwiGLU operands.
// Every phase therefore works on "units" of two rows.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace llmdiy {

constexpr int kHidden = 2048;       // hidden size the fused kernel is specialised for
constexpr int kHeadDim = 128;
constexpr int kHeads = kHidden / kHeadDim;
constexpr int kRingStages = 8;       // == consumer warps: slot s is always drained by warp s
constexpr int kStageBytes = 24576;   // 3 units of K=2048 (6 rows) or 1 unit of K<=6144
constexpr int kConsumerWarps = 8;
constexpr int kDecodeThreads = kConsumerWarps * 32;
constexpr int kAttnSplits = 9;       // 16 heads x 9 position splits = 144 attention CTAs
constexpr int kMaxLayers = 64;       // layer pointers are cached in shared memory

// Units (two weight rows of K elements) in one ring slot: 3 for K = 2048, 1 for K up to 6144.
__host__ __device__ constexpr int chunk_units(int K) {
    return kStageBytes / (4 * K) < 1 ? 1 : kStageBytes / (4 * K);
}

// This CTA's share of one phase's matrix: units [u0, u1), units per chunk, row length K.
// Phases: 0 qkv (3H/2 units), 1 o_proj (H/2), 2 w12 (IM), 3 c_proj (H/2, K = IM), 4 lm_head (V/2).
struct PhaseRange {
    int u0, u1, CH, K;
};
__host__ __device__ inline PhaseRange phase_range(int ph, int IM, int V, int b, int G) {
    const int U = ph == 0 ? 3 * kHidden / 2 : ph == 1 ? kHidden / 2 : ph == 2 ? IM : ph == 3 ? kHidden / 2 : V / 2;
    const int K = ph == 3 ? IM : kHidden;
    PhaseRange r;
    r.u0 = (int)((long long)U * b / G);
    r.u1 = (int)((long long)U * (b + 1) / G);
    r.CH = chunk_units(K);
    r.K = K;
    return r;
}

struct LayerPtrs {
    const half* ln1;     // [H]
    const half* qkv_w;   // [3H, H], RoPE-pair permuted rows
    const half* qkv_b;   // [3H], original order
    const half* proj_w;  // [H, H]
    const half* ln2;     // [H]
    const half* w12;     // [2*IM, H], w1/w2 interleaved rows
    const half* cproj;   // [H, IM]
};

// Flag-carrying words ("LL" words) pass the small per-phase vectors between
// CTAs without grid barriers: each 8-byte word holds 32 bits of data in its
// low half and a 32-bit phase tag in its high half, written with one 64-bit
// store; a reader polls exactly the words it needs until they carry the tag
// of the phase instance it expects.  Tags are unique per (launch, step,
// layer, phase), so no buffer ever needs clearing between phases.
enum LLSlot : uint32_t { LL_QKV = 0, LL_ATT = 1, LL_XO = 2, LL_ACT = 3, LL_XC = 4, LL_APART = 5, LL_PER_LAYER = 6 };

// Per-launch control words, zeroed by the host before every launch.
struct DecodeControl {
    unsigned int bar;                  // grid barrier arrivals
    int err;                           // first error code (0 = none)
    int err_where;                     // diagnostic: phase id of the failure
    int n_done;                        // steps completed
    unsigned long long best[2];        // argmax keys, double-buffered by step parity
};

struct DecodeArgs {
    const LayerPtrs* layers;  // device array [NL]
    const half* wte;          // [V, H]
    const half* lnf;          // [H]
    const half* lm_head;      // [V, H]
    half* kc;                 // [NL][max_seqlen][H]
    half* vc;
    half* x;                  // [H]   residual stream after the last layer (plain copy)
    half* logits;             // [V]
    unsigned long long* ll_qkv;  // [3H/2] unit u = (value of row 2u, row 2u+1) after bias/RoPE
    unsigned long long* ll_att;  // [H/2]  attention output pairs
    unsigned long long* ll_xo;   // [H/2]  residual stream after o_proj
    unsigned long long* ll_act;  // [IM]   SwiGLU output, one value per word
    unsigned long long* ll_xc;   // [H/2]  residual stream after c_proj
    unsigned long long* ll_apart;  // [kHeads][kAttnSplits][130] split partials (o[128], m, l) as fp32 words
    uint32_t flag_base;          // tag of this launch's first phase instance minus 1
    DecodeControl* ctl;
    int* tokens_out;          // [n_steps] device copy of generated tokens (may be null)
    int* host_tokens;         // mapped host buffer for streaming (may be null)
    int* host_count;          // mapped host word: number of tokens published
    const int* forced;        // [n_steps] input tokens when skip_lm (prefill through the decode path)
    int NL, IM, V, max_seqlen;
    int first_token, pos0, n_steps;
    int skip_lm;              // 1: no lm_head; the input of step t+1 is forced[t+1]
    int stop0, stop1;         // stop ids (-1 = none)
    // Weight-chunk schedule of one step, per CTA: entry i = (byte offset / 16 from wbase, bytes) of
    // the CTA's i-th chunk (all layers' qkv, o, w12, c chunks, then lm_head's); feed_cnt[2*cta] =
    // chunks of the layers, feed_cnt[2*cta+1] = chunks of lm_head.  Built once per engine.
    const uint2* feed_tbl;    // [grid][feed_stride]
    const int* feed_cnt;      // [grid][2]
    int feed_stride;
    const uint8_t* wbase;
    int l2_ahead;             // chunks prefetched into L2 ahead of the copy issued: 8 * l2_ahead (0 = off)
    // optional timing probes (null in production): per CTA and grid barrier,
    // %globaltimer at arrival and at release; per CTA the producer's time
    // blocked on a full ring and the consumers' time waiting for data.
    unsigned long long* prof;       // [grid][prof_cap][2]
    unsigned long long* prof_prod;  // [grid][6 phases][8 warps][4]: wait, compute, issue cycles, longest wait
    int prof_cap;
};

}  // namespace llmdiy
