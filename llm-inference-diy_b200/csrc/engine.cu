// engine.cu — host runtime of the B200 decode engine (the QwenEngine of
// framework_src/qwen_infer.cu:69-738, re-designed around one persistent
// decode kernel per request instead of ~700 launches and 24 host syncs per
// token).
//
// Device memory: one allocation for all weights (each tensor 256-byte
// aligned, GEMV matrices kept in the file's [N,K] layout, qkv_w rows
// permuted into RoPE pairs and ffn_w1/ffn_w2 interleaved, see decode.h), the
// KV cache [layers][max_seqlen][hidden] for K and V, a handful of
// activation vectors, and a small control block the kernel zeroes' state in.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "decode.h"
#include "engine_internal.h"
#include "gemm_tc_host.h"
#include "llmdiy_engine.h"
#include "prefill_tc.h"
#include "qwdf.h"

namespace llmdiy {
size_t decode_smem_bytes();
uint32_t decode_tags_per_launch(int n_steps, int num_layers);
cudaError_t launch_decode(const DecodeArgs& a, int grid, cudaStream_t stream);

namespace {

// qkv_w [3H,H] -> RoPE-pair order: dst unit u (rows 2u, 2u+1) = src rows
// (s*H + h*128 + t, s*H + h*128 + 64 + t), u = s*(H/2) + h*64 + t.
__global__ void permute_qkv_k(half* __restrict__ dst, const half* __restrict__ src, int H) {
    const int row = blockIdx.x;  // destination row
    const int u = row >> 1, j = row & 1;
    const int sec = u / (H / 2), v = u % (H / 2), h = v / 64, t = v % 64;
    const int srow = sec * H + h * 128 + t + 64 * j;
    const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)srow * H);
    uint4* d = reinterpret_cast<uint4*>(dst + (size_t)row * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) d[i] = s[i];
}

// w12 row 2n = w1 row n, row 2n+1 = w2 row n
__global__ void interleave_k(half* __restrict__ dst, const half* __restrict__ w1, const half* __restrict__ w2, int K) {
    const int row = blockIdx.x, n = row >> 1;
    const uint4* s = reinterpret_cast<const uint4*>(((row & 1) ? w2 : w1) + (size_t)n * K);
    uint4* d = reinterpret_cast<uint4*>(dst + (size_t)row * K);
    for (int i = threadIdx.x; i < K / 8; i += blockDim.x) d[i] = s[i];
}

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace
}  // namespace llmdiy

using namespace llmdiy;

struct llmdiy_engine {
    llmdiy_config cfg{};
    int device = 0;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    std::string err;

    // weights
    uint8_t* wbuf = nullptr;
    size_t wbytes = 0;
    half* wte = nullptr;
    half* lnf = nullptr;
    half* lm_head = nullptr;
    std::vector<LayerPtrs> layers;
    LayerPtrs* d_layers = nullptr;

    // state
    half* kc = nullptr;
    half* vc = nullptr;
    half *x = nullptr, *logits = nullptr;
    unsigned long long* ll = nullptr;  // flag-carrying words: qkv | att | xo | act | xc
    size_t ll_words = 0;
    uint32_t tag_base = 0;
    half* pf = nullptr;  // tensor-core prefill scratch: x, xn, q, att [rows][H], act [rows][IM]
    int pf_rows = 0;
    uint2* feed_tbl = nullptr;  // decode kernel's per-CTA weight-chunk schedule of one step
    int* feed_cnt = nullptr;
    int feed_stride = 0;
    int l2_ahead = 1;  // decode kernel: rings of chunks prefetched into L2 beyond the copy ring (env LLMDIY_L2_AHEAD)
    DecodeControl* ctl = nullptr;
    int* tokens_dev = nullptr;
    int* forced_dev = nullptr;
    int* host_tokens = nullptr;  // mapped pinned
    int* host_tokens_dev = nullptr;
    int* host_count = nullptr;   // mapped pinned
    int* host_count_dev = nullptr;
    int last_steps = 0;
};

namespace {

int fail(llmdiy_engine* e, int code, const std::string& msg) {
    if (e) e->err = msg;
    return code;
}

int cuda_fail(llmdiy_engine* e, cudaError_t c, const char* what) {
    if (e) e->err = std::string(what) + ": " + cudaGetErrorString(c);
    return (int)c;
}

#define CK(call, what)                                        \
    do {                                                      \
        cudaError_t _c = (call);                              \
        if (_c != cudaSuccess) return cuda_fail(e, _c, what); \
    } while (0)

int check_config(llmdiy_engine* e, const llmdiy_config& c) {
    static_assert(kHidden == 2048 && kHeads == 16 && kMaxLayers == 64, "qwdf_unsupported states these limits");
    if (const char* why = qwdf_unsupported(c)) return fail(e, LLMDIY_ERR_UNSUPPORTED, why);
    return LLMDIY_OK;
}

// Sizes and offsets of every tensor in the device weight buffer.
struct Layout {
    size_t wte, lnf, lm_head, total;
    std::vector<size_t> ln1, qkv_w, qkv_b, proj, ln2, w12, cproj;
};

Layout plan(const llmdiy_config& c) {
    const size_t H = c.hidden_size, IM = c.intermediate_size, V = c.vocab_size;
    Layout L;
    size_t off = 0;
    auto take = [&](size_t elems) { size_t o = off; off += align256(elems * 2); return o; };
    L.wte = take(V * H);
    for (uint32_t l = 0; l < c.num_layers; ++l) {
        L.ln1.push_back(take(H));
        L.qkv_w.push_back(take(3 * H * H));
        L.qkv_b.push_back(take(3 * H));
        L.proj.push_back(take(H * H));
        L.ln2.push_back(take(H));
        L.w12.push_back(take(2 * IM * H));
        L.cproj.push_back(take(H * IM));
    }
    L.lnf = take(H);
    L.lm_head = take(V * H);
    L.total = off;
    return L;
}

// Source of tensor data in file order: either a QWDF file or the seeded generator.
struct Source {
    FILE* f = nullptr;
    bool random = false;
    uint64_t seed = 0;
    float std_dev = 0.02f;
    int nthreads = 8;
};

// Stream tensor `id` (n fp16 elements) from the source into device memory at dst.
int upload_tensor(llmdiy_engine* e, Source& src, int id, size_t n, half* dst, std::vector<uint16_t*>& pinned) {
    const size_t chunk = (size_t)1 << 23;  // 16 MB per staging buffer, double-buffered
    for (size_t i = 0, k = 0; i < n; i += chunk, ++k) {
        const size_t m = std::min(chunk, n - i);
        uint16_t* buf = pinned[k & 1];
        // the copy that used this staging buffer two chunks ago must be done
        CK(cudaStreamSynchronize(e->stream), "upload sync");
        if (src.random) {
            qwdf_fill(e->cfg, id, src.seed, src.std_dev, i, m, buf, src.nthreads);
        } else if (std::fread(buf, 2, m, src.f) != m) {
            return fail(e, LLMDIY_ERR_FORMAT, "weight file truncated");
        }
        CK(cudaMemcpyAsync(dst + i, buf, m * 2, cudaMemcpyHostToDevice, e->stream), "weight upload");
    }
    return LLMDIY_OK;
}

int load_weights(llmdiy_engine* e, Source& src) {
    const llmdiy_config& c = e->cfg;
    const size_t H = c.hidden_size, IM = c.intermediate_size, V = c.vocab_size;
    Layout L = plan(c);
    e->wbytes = L.total;
    CK(cudaMalloc(&e->wbuf, L.total), "cudaMalloc weights");
    auto P = [&](size_t off) { return reinterpret_cast<half*>(e->wbuf + off); };
    std::vector<uint16_t*> pinned(2, nullptr);
    for (auto& p : pinned) CK(cudaMallocHost(&p, ((size_t)1 << 23) * 2), "cudaMallocHost staging");
    half* tmp = nullptr;
    const size_t tmp_elems = std::max(3 * H * H, 2 * IM * H);
    int rc = LLMDIY_OK;
    cudaError_t ce = cudaMalloc(&tmp, tmp_elems * 2);
    if (ce != cudaSuccess) rc = cuda_fail(e, ce, "cudaMalloc staging");
    int id = 0;
    if (!rc) rc = upload_tensor(e, src, id++, V * H, P(L.wte), pinned);
    e->layers.resize(c.num_layers);
    for (uint32_t l = 0; l < c.num_layers && !rc; ++l) {
        LayerPtrs& lp = e->layers[l];
        rc = upload_tensor(e, src, id++, H, P(L.ln1[l]), pinned);
        if (!rc) rc = upload_tensor(e, src, id++, 3 * H * H, tmp, pinned);
        if (!rc) {
            permute_qkv_k<<<(unsigned)(3 * H), 256, 0, e->stream>>>(P(L.qkv_w[l]), tmp, (int)H);
            ce = cudaStreamSynchronize(e->stream);
            if (ce != cudaSuccess) rc = cuda_fail(e, ce, "qkv permute");
        }
        if (!rc) rc = upload_tensor(e, src, id++, 3 * H, P(L.qkv_b[l]), pinned);
        if (!rc) rc = upload_tensor(e, src, id++, H * H, P(L.proj[l]), pinned);
        if (!rc) rc = upload_tensor(e, src, id++, H, P(L.ln2[l]), pinned);
        if (!rc) rc = upload_tensor(e, src, id++, IM * H, tmp, pinned);
        if (!rc) rc = upload_tensor(e, src, id++, IM * H, tmp + IM * H, pinned);
        if (!rc) {
            interleave_k<<<(unsigned)(2 * IM), 256, 0, e->stream>>>(P(L.w12[l]), tmp, tmp + IM * H, (int)H);
            ce = cudaStreamSynchronize(e->stream);
            if (ce != cudaSuccess) rc = cuda_fail(e, ce, "w1/w2 interleave");
        }
        if (!rc) rc = upload_tensor(e, src, id++, H * IM, P(L.cproj[l]), pinned);
        lp.ln1 = P(L.ln1[l]);
        lp.qkv_w = P(L.qkv_w[l]);
        lp.qkv_b = P(L.qkv_b[l]);
        lp.proj_w = P(L.proj[l]);
        lp.ln2 = P(L.ln2[l]);
        lp.w12 = P(L.w12[l]);
        lp.cproj = P(L.cproj[l]);
    }
    if (!rc) rc = upload_tensor(e, src, id++, H, P(L.lnf), pinned);
    if (!rc) rc = upload_tensor(e, src, id++, V * H, P(L.lm_head), pinned);
    cudaStreamSynchronize(e->stream);
    for (auto& p : pinned) cudaFreeHost(p);
    cudaFree(tmp);
    if (rc) return rc;
    e->wte = P(L.wte);
    e->lnf = P(L.lnf);
    e->lm_head = P(L.lm_head);
    CK(cudaMalloc(&e->d_layers, sizeof(LayerPtrs) * c.num_layers), "cudaMalloc layers");
    CK(cudaMemcpy(e->d_layers, e->layers.data(), sizeof(LayerPtrs) * c.num_layers, cudaMemcpyHostToDevice),
       "layers upload");
    return LLMDIY_OK;
}

int alloc_state(llmdiy_engine* e) {
    const llmdiy_config& c = e->cfg;
    const size_t H = c.hidden_size, kv = (size_t)c.num_layers * c.max_seqlen * H;
    CK(cudaMalloc(&e->kc, kv * 2), "cudaMalloc K cache");
    CK(cudaMalloc(&e->vc, kv * 2), "cudaMalloc V cache");
    CK(cudaMalloc(&e->x, H * 2), "alloc x");
    e->ll_words = 3 * H / 2 + H / 2 + H / 2 + c.intermediate_size + H / 2 + (size_t)kHeads * kAttnSplits * 130;
    CK(cudaMalloc(&e->ll, e->ll_words * 8), "alloc flag words");
    CK(cudaMemset(e->ll, 0, e->ll_words * 8), "clear flag words");
    CK(cudaMalloc(&e->logits, (size_t)c.vocab_size * 2), "alloc logits");
    CK(cudaMalloc(&e->ctl, sizeof(DecodeControl)), "alloc control");
    CK(cudaMalloc(&e->tokens_dev, sizeof(int) * (c.max_seqlen + 1)), "alloc tokens");
    CK(cudaMalloc(&e->forced_dev, sizeof(int) * (c.max_seqlen + 1)), "alloc forced");
    CK(cudaHostAlloc(&e->host_tokens, sizeof(int) * (c.max_seqlen + 1), cudaHostAllocMapped), "alloc mapped tokens");
    CK(cudaHostGetDevicePointer(&e->host_tokens_dev, e->host_tokens, 0), "map tokens");
    CK(cudaHostAlloc(&e->host_count, sizeof(int) * 4, cudaHostAllocMapped), "alloc mapped count");
    CK(cudaHostGetDevicePointer(&e->host_count_dev, e->host_count, 0), "map count");
    e->pf_rows = (int)std::min<uint32_t>(c.max_seqlen, (uint32_t)kPrefillChunk);
    CK(cudaMalloc(&e->pf, (size_t)e->pf_rows * (4 * H + c.intermediate_size) * 2), "alloc prefill scratch");
    return llmdiy_engine_reset(e);
}

// The decode kernel's weight-chunk schedule: for every CTA, the chunks it
// streams in one step, in consumption order (per layer qkv, o_proj, w12,
// c_proj; then lm_head), as (offset / 16 from the weight buffer, bytes).
int build_feed_table(llmdiy_engine* e) {
    const llmdiy_config& c = e->cfg;
    const int G = e->num_sms, NL = (int)c.num_layers, IM = (int)c.intermediate_size, V = (int)c.vocab_size;
    std::vector<std::vector<uint2>> per(G);
    std::vector<int> cnt(2 * G);
    auto add = [&](std::vector<uint2>& v, const half* W, const PhaseRange& r) {
        for (int cu = r.u0; cu < r.u1; cu += r.CH) {
            const int nun = std::min(r.CH, r.u1 - cu);
            const size_t off = (size_t)(reinterpret_cast<const uint8_t*>(W + (size_t)cu * 2 * r.K) - e->wbuf);
            v.push_back(make_uint2((uint32_t)(off / 16), (uint32_t)nun * 4u * (uint32_t)r.K));
        }
    };
    for (int b = 0; b < G; ++b) {
        PhaseRange r[5];
        for (int ph = 0; ph < 5; ++ph) r[ph] = phase_range(ph, IM, V, b, G);
        for (int l = 0; l < NL; ++l) {
            const LayerPtrs& L = e->layers[l];
            add(per[b], L.qkv_w, r[0]);
            add(per[b], L.proj_w, r[1]);
            add(per[b], L.w12, r[2]);
            add(per[b], L.cproj, r[3]);
        }
        cnt[2 * b] = (int)per[b].size();
        add(per[b], e->lm_head, r[4]);
        cnt[2 * b + 1] = (int)per[b].size() - cnt[2 * b];
        e->feed_stride = std::max(e->feed_stride, (int)per[b].size());
    }
    std::vector<uint2> flat((size_t)G * e->feed_stride, make_uint2(0, 0));
    for (int b = 0; b < G; ++b) std::copy(per[b].begin(), per[b].end(), flat.begin() + (size_t)b * e->feed_stride);
    CK(cudaMalloc(&e->feed_tbl, flat.size() * sizeof(uint2)), "alloc chunk schedule");
    CK(cudaMalloc(&e->feed_cnt, cnt.size() * sizeof(int)), "alloc chunk counts");
    CK(cudaMemcpy(e->feed_tbl, flat.data(), flat.size() * sizeof(uint2), cudaMemcpyHostToDevice), "upload schedule");
    CK(cudaMemcpy(e->feed_cnt, cnt.data(), cnt.size() * sizeof(int), cudaMemcpyHostToDevice), "upload counts");
    return LLMDIY_OK;
}

int create_common(llmdiy_engine* e, Source& src) {
    CK(cudaSetDevice(e->device), "cudaSetDevice");
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, e->device), "cudaGetDeviceProperties");
    if (prop.major != 10) return fail(e, LLMDIY_ERR_UNSUPPORTED, "this library is built for sm_100a (B200)");
    e->num_sms = prop.multiProcessorCount;
    if (!prop.cooperativeLaunch) return fail(e, LLMDIY_ERR_UNSUPPORTED, "device lacks cooperative launch");
    if (prop.sharedMemPerBlockOptin < decode_smem_bytes())
        return fail(e, LLMDIY_ERR_UNSUPPORTED, "not enough shared memory per block for the decode kernel");
    CK(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking), "cudaStreamCreate");
    if (const char* v = std::getenv("LLMDIY_L2_AHEAD")) e->l2_ahead = std::max(0, std::atoi(v));
    int rc = load_weights(e, src);
    if (!rc) rc = build_feed_table(e);
    if (!rc) rc = alloc_state(e);
    if (rc) return rc;
    // the uploads and clears above ran on the legacy stream, which does not order against the
    // engine's non-blocking stream or a caller's stream: finish them before any launch
    CK(cudaDeviceSynchronize(), "finish set-up");
    return LLMDIY_OK;
}

// Launch the decode kernel for n_steps steps (first input token, first position).
int launch(llmdiy_engine* e, int first_token, int pos0, int n_steps, bool skip_lm, bool stop_on_eos, bool stream_host,
           cudaStream_t st, unsigned long long* prof = nullptr, unsigned long long* prof_prod = nullptr,
           int prof_cap = 0) {
    const llmdiy_config& c = e->cfg;
    if (n_steps <= 0) return LLMDIY_OK;
    if (pos0 < 0 || (long long)pos0 + n_steps > (long long)c.max_seqlen)
        return fail(e, LLMDIY_ERR_ARG, "position beyond max_seqlen");
    if (first_token < 0 || first_token >= (int)c.vocab_size) return fail(e, LLMDIY_ERR_ARG, "token id out of range");
    CK(cudaMemsetAsync(e->ctl, 0, sizeof(DecodeControl), st), "reset control");
    if (stream_host) *(volatile int*)e->host_count = 0;
    DecodeArgs a{};
    a.layers = e->d_layers;
    a.wte = e->wte;
    a.lnf = e->lnf;
    a.lm_head = e->lm_head;
    a.kc = e->kc;
    a.vc = e->vc;
    a.x = e->x;
    a.logits = e->logits;
    const size_t H = c.hidden_size;
    a.ll_qkv = e->ll;
    a.ll_att = a.ll_qkv + 3 * H / 2;
    a.ll_xo = a.ll_att + H / 2;
    a.ll_act = a.ll_xo + H / 2;
    a.ll_xc = a.ll_act + c.intermediate_size;
    a.ll_apart = a.ll_xc + H / 2;
    // tags are unique per phase instance across launches; on wrap-around the
    // words are cleared so no stale word can carry a future tag
    const uint32_t need = decode_tags_per_launch(n_steps, (int)c.num_layers);
    if ((uint64_t)e->tag_base + need >= 0xFFFFFFF0ull) {
        CK(cudaMemsetAsync(e->ll, 0, e->ll_words * 8, st), "clear flag words");
        e->tag_base = 0;
    }
    a.flag_base = e->tag_base;
    e->tag_base += need;
    a.ctl = e->ctl;
    a.tokens_out = e->tokens_dev;
    a.host_tokens = stream_host ? e->host_tokens_dev : nullptr;
    a.host_count = stream_host ? e->host_count_dev : nullptr;
    a.forced = e->forced_dev;
    a.NL = (int)c.num_layers;
    a.IM = (int)c.intermediate_size;
    a.V = (int)c.vocab_size;
    a.max_seqlen = (int)c.max_seqlen;
    a.first_token = first_token;
    a.pos0 = pos0;
    a.n_steps = n_steps;
    a.skip_lm = skip_lm ? 1 : 0;
    a.stop0 = stop_on_eos ? 151645 : -1;  // qwen_infer.cu:808
    a.stop1 = stop_on_eos ? 151643 : -1;
    a.feed_tbl = e->feed_tbl;
    a.feed_cnt = e->feed_cnt;
    a.feed_stride = e->feed_stride;
    a.wbase = e->wbuf;
    a.l2_ahead = e->l2_ahead;
    a.prof = prof;
    a.prof_prod = prof_prod;
    a.prof_cap = prof_cap;
    CK(launch_decode(a, e->num_sms, st), "decode launch");
    e->last_steps = n_steps;
    return LLMDIY_OK;
}

int read_status(llmdiy_engine* e, int* n_done) {
    DecodeControl h;
    CK(cudaMemcpy(&h, e->ctl, sizeof(h), cudaMemcpyDeviceToHost), "read control");
    if (n_done) *n_done = h.n_done;
    if (h.err) {
        char buf[160];
        std::snprintf(buf, sizeof(buf), "decode kernel error %d in phase %d after %d steps", h.err, h.err_where,
                      h.n_done);
        return fail(e, LLMDIY_ERR_DEVICE, buf);
    }
    return LLMDIY_OK;
}

int prefill_impl(llmdiy_engine* e, const int* tokens, int n) {
    if (n <= 0) return LLMDIY_OK;
    if ((uint32_t)n > e->cfg.max_seqlen) return fail(e, LLMDIY_ERR_ARG, "prompt longer than max_seqlen");
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= (int)e->cfg.vocab_size) return fail(e, LLMDIY_ERR_ARG, "token id out of range");
    CK(cudaMemcpyAsync(e->forced_dev, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, e->stream), "upload prompt");
    const llmdiy_config& c = e->cfg;
    const size_t H = c.hidden_size, R = (size_t)e->pf_rows;
    PrefillArgs p{};
    p.layers = e->layers.data();
    p.wte = e->wte;
    p.kc = e->kc;
    p.vc = e->vc;
    p.NL = (int)c.num_layers;
    p.IM = (int)c.intermediate_size;
    p.max_seqlen = (int)c.max_seqlen;
    p.layer_stride = (size_t)c.max_seqlen * H;
    p.x = e->pf;
    p.xn = p.x + R * H;
    p.q = p.xn + R * H;
    p.att = p.q + R * H;
    p.act = p.att + R * H;
    p.hidden = e->x;
    int rc = prefill_tc(p, e->forced_dev, n, 0, e->stream);
    if (rc) return cuda_fail(e, (cudaError_t)rc, "prefill");
    CK(cudaStreamSynchronize(e->stream), "prefill");
    if (gemm_tc_status()) return fail(e, LLMDIY_ERR_DEVICE, "prefill GEMM pipeline wait expired");
    return LLMDIY_OK;
}

}  // namespace

namespace llmdiy {
EngineView engine_view(const llmdiy_engine* e) {
    EngineView v{};
    v.cfg = e->cfg;
    v.device = e->device;
    v.num_sms = e->num_sms;
    v.stream = e->stream;
    v.layers = e->layers.data();
    v.wte = e->wte;
    v.lnf = e->lnf;
    v.lm_head = e->lm_head;
    return v;
}
}  // namespace llmdiy

extern "C" {

int llmdiy_engine_create(const char* bin_path, int device, llmdiy_engine** out) {
    if (!out || !bin_path) return LLMDIY_ERR_ARG;
    *out = nullptr;
    llmdiy_config c;
    int rc = llmdiy_qwdf_read_config(bin_path, &c);
    if (rc) return rc;
    llmdiy_engine* e = new llmdiy_engine();
    e->cfg = c;
    e->device = device;
    rc = check_config(e, c);
    Source src;
    if (!rc) {
        src.f = std::fopen(bin_path, "rb");
        if (!src.f) rc = fail(e, LLMDIY_ERR_FILE, "cannot open weight file");
        else std::fseek(src.f, sizeof(QwdfHeader), SEEK_SET);
    }
    if (!rc) rc = create_common(e, src);
    if (src.f) std::fclose(src.f);
    if (rc) {
        std::fprintf(stderr, "[llmdiy] engine create failed: %s\n", e->err.c_str());
        llmdiy_engine_destroy(e);
        return rc;
    }
    *out = e;
    return LLMDIY_OK;
}

int llmdiy_engine_create_random(const llmdiy_config* cfg, uint64_t seed, float std_dev, int device,
                                llmdiy_engine** out) {
    if (!out || !cfg) return LLMDIY_ERR_ARG;
    *out = nullptr;
    llmdiy_engine* e = new llmdiy_engine();
    e->cfg = *cfg;
    e->device = device;
    int rc = check_config(e, *cfg);
    Source src;
    src.random = true;
    src.seed = seed;
    src.std_dev = std_dev;
    src.nthreads = (int)std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
    if (!rc) rc = create_common(e, src);
    if (rc) {
        std::fprintf(stderr, "[llmdiy] engine create failed: %s\n", e->err.c_str());
        llmdiy_engine_destroy(e);
        return rc;
    }
    *out = e;
    return LLMDIY_OK;
}

void llmdiy_engine_destroy(llmdiy_engine* e) {
    if (!e) return;
    cudaSetDevice(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    cudaFree(e->wbuf);
    cudaFree(e->pf);
    cudaFree(e->feed_tbl);
    cudaFree(e->feed_cnt);
    cudaFree(e->d_layers);
    cudaFree(e->kc);
    cudaFree(e->vc);
    cudaFree(e->x);
    cudaFree(e->ll);
    cudaFree(e->logits);
    cudaFree(e->ctl);
    cudaFree(e->tokens_dev);
    cudaFree(e->forced_dev);
    if (e->host_tokens) cudaFreeHost(e->host_tokens);
    if (e->host_count) cudaFreeHost(e->host_count);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
}

int llmdiy_engine_get_config(const llmdiy_engine* e, llmdiy_config* out) {
    if (!e || !out) return LLMDIY_ERR_ARG;
    *out = e->cfg;
    return LLMDIY_OK;
}

const char* llmdiy_engine_last_error(const llmdiy_engine* e) { return e ? e->err.c_str() : "null engine"; }

int llmdiy_engine_num_sms(const llmdiy_engine* e) { return e ? e->num_sms : 0; }

// qwen_infer.cu:318-356: zero the KV cache and the activations.
int llmdiy_engine_reset(llmdiy_engine* e) {
    if (!e) return LLMDIY_ERR_ARG;
    CK(cudaSetDevice(e->device), "cudaSetDevice");
    const llmdiy_config& c = e->cfg;
    const size_t H = c.hidden_size, kv = (size_t)c.num_layers * c.max_seqlen * H;
    CK(cudaMemsetAsync(e->kc, 0, kv * 2, e->stream), "reset K");
    CK(cudaMemsetAsync(e->vc, 0, kv * 2, e->stream), "reset V");
    CK(cudaMemsetAsync(e->x, 0, H * 2, e->stream), "reset x");
    CK(cudaMemsetAsync(e->logits, 0, (size_t)c.vocab_size * 2, e->stream), "reset logits");
    CK(cudaMemsetAsync(e->ctl, 0, sizeof(DecodeControl), e->stream), "reset control");
    CK(cudaStreamSynchronize(e->stream), "reset");
    return LLMDIY_OK;
}

int llmdiy_engine_prefill(llmdiy_engine* e, const int* tokens, int n) {
    if (!e || (n > 0 && !tokens)) return LLMDIY_ERR_ARG;
    CK(cudaSetDevice(e->device), "cudaSetDevice");
    return prefill_impl(e, tokens, n);
}

int llmdiy_engine_step(llmdiy_engine* e, int token, int pos, int* next) {
    if (!e || !next) return LLMDIY_ERR_ARG;
    CK(cudaSetDevice(e->device), "cudaSetDevice");
    int rc = launch(e, token, pos, 1, false, false, false, e->stream);
    if (rc) return rc;
    CK(cudaStreamSynchronize(e->stream), "step");
    rc = read_status(e, nullptr);
    if (rc) return rc;
    CK(cudaMemcpy(next, e->tokens_dev, sizeof(int), cudaMemcpyDeviceToHost), "read token");
    return LLMDIY_OK;
}

int llmdiy_engine_generate_stream(llmdiy_engine* e, const int* prompt, int n, int max_new, int stop_on_eos,
                                  llmdiy_token_cb cb, void* user, int* n_out) {
    if (!e || !prompt || n <= 0 || max_new < 0) return LLMDIY_ERR_ARG;
    if (n_out) *n_out = 0;
    CK(cudaSetDevice(e->device), "cudaSetDevice");
    int rc = prefill_impl(e, prompt, n - 1);
    if (rc) return rc;
    const int pos0 = n - 1;
    const int steps = std::min(max_new, (int)e->cfg.max_seqlen - pos0);
    if (steps <= 0) return LLMDIY_OK;
    rc = launch(e, prompt[n - 1], pos0, steps, false, stop_on_eos != 0, cb != nullptr, e->stream);
    if (rc) return rc;
    int emitted = 0;
    if (cb) {
        // Publish tokens as the kernel writes them into mapped host memory.
        for (;;) {
            const int avail = *(volatile int*)e->host_count;
            while (emitted < avail) {
                const int t = ((volatile int*)e->host_tokens)[emitted];
                if (stop_on_eos && (t == 151645 || t == 151643)) { emitted = steps; break; }
                cb(t, user);
                ++emitted;
                if (n_out) *n_out = emitted;
            }
            if (emitted >= steps) break;
            cudaError_t q = cudaStreamQuery(e->stream);
            if (q == cudaSuccess) {
                // kernel finished: flush whatever it published last
                const int fin = *(volatile int*)e->host_count;
                while (emitted < fin) {
                    const int t = ((volatile int*)e->host_tokens)[emitted];
                    if (stop_on_eos && (t == 151645 || t == 151643)) break;
                    cb(t, user);
                    ++emitted;
                    if (n_out) *n_out = emitted;
                }
                break;
            }
            if (q != cudaErrorNotReady) return cuda_fail(e, q, "decode");
            std::this_thread::sleep_for(std::chrono::microseconds(20));
        }
    }
    CK(cudaStreamSynchronize(e->stream), "decode");
    int done = 0;
    rc = read_status(e, &done);
    if (rc) return rc;
    if (!cb && n_out) *n_out = done;
    return LLMDIY_OK;
}

int llmdiy_engine_generate(llmdiy_engine* e, const int* prompt, int n, int max_new, int stop_on_eos, int* out,
                           int* n_out) {
    if (!e || !out || !n_out) return LLMDIY_ERR_ARG;
    int done = 0;
    int rc = llmdiy_engine_generate_stream(e, prompt, n, max_new, stop_on_eos, nullptr, nullptr, &done);
    if (rc) return rc;
    std::vector<int> t(done > 0 ? done : 1);
    if (done > 0) CK(cudaMemcpy(t.data(), e->tokens_dev, sizeof(int) * done, cudaMemcpyDeviceToHost), "read tokens");
    int k = 0;
    for (int i = 0; i < done; ++i) {
        if (stop_on_eos && (t[i] == 151645 || t[i] == 151643)) break;
        out[k++] = t[i];
    }
    *n_out = k;
    return LLMDIY_OK;
}

int llmdiy_engine_decode_async(llmdiy_engine* e, int first_token, int pos, int n_steps, int stop_on_eos,
                               void* stream) {
    if (!e) return LLMDIY_ERR_ARG;
    cudaStream_t st = stream ? reinterpret_cast<cudaStream_t>(stream) : e->stream;
    return launch(e, first_token, pos, n_steps, false, stop_on_eos != 0, false, st);
}

// Timing probes of one decode launch: out[(cta*cap + i)*2] = %globaltimer (ns)
// at the i-th phase boundary of CTA `cta`; prod[((cta*6 + phase)*8 + warp)*4 +
// {0,1,2,3}] = SM cycles waiting for ring chunks, computing, issuing copies; chunks.
int llmdiy_engine_profile(llmdiy_engine* e, int first_token, int pos, int n_steps, int cap, uint64_t* out,
                          uint64_t* prod) {
    if (!e || !out || !prod || cap <= 0) return LLMDIY_ERR_ARG;
    CK(cudaSetDevice(e->device), "cudaSetDevice");
    unsigned long long *d = nullptr, *dp = nullptr;
    const size_t n = (size_t)e->num_sms * cap * 2;
    CK(cudaMalloc(&d, n * 8), "alloc probes");
    const size_t np = (size_t)e->num_sms * 6 * kConsumerWarps * 4;
    CK(cudaMalloc(&dp, np * 8), "alloc probes");
    cudaMemsetAsync(d, 0, n * 8, e->stream);
    cudaMemsetAsync(dp, 0, np * 8, e->stream);
    int rc = launch(e, first_token, pos, n_steps, false, false, false, e->stream, d, dp, cap);
    if (!rc) {
        cudaError_t c = cudaStreamSynchronize(e->stream);
        if (c != cudaSuccess) rc = cuda_fail(e, c, "profile");
    }
    if (!rc) rc = read_status(e, nullptr);
    if (!rc) {
        cudaMemcpy(out, d, n * 8, cudaMemcpyDeviceToHost);
        cudaMemcpy(prod, dp, np * 8, cudaMemcpyDeviceToHost);
    }
    cudaFree(d);
    cudaFree(dp);
    return rc;
}

int llmdiy_engine_status(llmdiy_engine* e, int* n_done) {
    if (!e) return LLMDIY_ERR_ARG;
    return read_status(e, n_done);
}

int llmdiy_engine_copy_tokens(llmdiy_engine* e, int* out, int n) {
    if (!e || !out || n < 0 || n > (int)e->cfg.max_seqlen) return LLMDIY_ERR_ARG;
    CK(cudaMemcpy(out, e->tokens_dev, sizeof(int) * n, cudaMemcpyDeviceToHost), "copy tokens");
    return LLMDIY_OK;
}

int llmdiy_engine_copy_logits(llmdiy_engine* e, uint16_t* out) {
    if (!e || !out) return LLMDIY_ERR_ARG;
    CK(cudaMemcpy(out, e->logits, (size_t)e->cfg.vocab_size * 2, cudaMemcpyDeviceToHost), "copy logits");
    return LLMDIY_OK;
}

int llmdiy_engine_copy_hidden(llmdiy_engine* e, uint16_t* out) {
    if (!e || !out) return LLMDIY_ERR_ARG;
    CK(cudaMemcpy(out, e->x, (size_t)e->cfg.hidden_size * 2, cudaMemcpyDeviceToHost), "copy hidden");
    return LLMDIY_OK;
}

int llmdiy_engine_copy_kv(llmdiy_engine* e, int layer, int pos0, int n, uint16_t* k, uint16_t* v) {
    if (!e || layer < 0 || layer >= (int)e->cfg.num_layers || pos0 < 0 || n < 0 ||
        (long long)pos0 + n > (long long)e->cfg.max_seqlen)
        return LLMDIY_ERR_ARG;
    const size_t H = e->cfg.hidden_size;
    const size_t off = ((size_t)layer * e->cfg.max_seqlen + pos0) * H;
    if (k) CK(cudaMemcpy(k, e->kc + off, (size_t)n * H * 2, cudaMemcpyDeviceToHost), "copy K");
    if (v) CK(cudaMemcpy(v, e->vc + off, (size_t)n * H * 2, cudaMemcpyDeviceToHost), "copy V");
    return LLMDIY_OK;
}

}  // extern "C"
