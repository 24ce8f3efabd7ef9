/*
 * qwen_oracle.c — TEST INFRASTRUCTURE ONLY (see qwen_oracle.h).
 *
 * CPU restatement of the reference decode path.  Every function names the
 * reference lines it follows.  Built with -ffp-contract=off so that the only
 * fused multiply-adds are the explicit fmaf()/_mm256_fmadd_ps calls that
 * stand for the FFMA instructions nvcc emits for the reference's
 * `sum += a * b` loops.
 */
#include "qwen_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef orc_f16 f16;

float   orc_h2f(f16 h) { return _cvtsh_ss(h); }
f16     orc_f2h(float f) { return (f16)_cvtss_sh(f, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC); }
#define h2f orc_h2f
#define f2h orc_f2h

void orc_f32_to_f16(const float* in, f16* out, int64_t n) { for (int64_t i = 0; i < n; i++) out[i] = f2h(in[i]); }
void orc_f16_to_f32(const f16* in, float* out, int64_t n) { for (int64_t i = 0; i < n; i++) out[i] = h2f(in[i]); }

/* ------------------------------------------------------------------------ */
/* A small persistent thread pool: par_for(n) splits [0,n) into contiguous   */
/* ranges, one per worker.                                                    */
/* ------------------------------------------------------------------------ */
typedef void (*range_fn)(void* ctx, int64_t b, int64_t e);

typedef struct {
    pthread_t* th;
    int n;
    pthread_mutex_t mu;
    pthread_cond_t cv_go, cv_done;
    long gen;
    int pending;
    int quit;
    range_fn fn;
    void* ctx;
    int64_t total, grain;
} pool_t;

typedef struct { pool_t* p; int id; } worker_arg;

static void pool_run_part(pool_t* p, int id) {
    int64_t units = (p->total + p->grain - 1) / p->grain;
    int64_t ub = units * id / p->n, ue = units * (id + 1) / p->n;
    int64_t b = ub * p->grain, e = ue * p->grain;
    if (e > p->total) e = p->total;
    if (b < e) p->fn(p->ctx, b, e);
}

static void* pool_main(void* a) {
    worker_arg* w = (worker_arg*)a;
    pool_t* p = w->p;
    long seen = 0;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        while (p->gen == seen && !p->quit) pthread_cond_wait(&p->cv_go, &p->mu);
        if (p->quit) { pthread_mutex_unlock(&p->mu); break; }
        seen = p->gen;
        pthread_mutex_unlock(&p->mu);
        pool_run_part(p, w->id);
        pthread_mutex_lock(&p->mu);
        if (--p->pending == 0) pthread_cond_signal(&p->cv_done);
        pthread_mutex_unlock(&p->mu);
    }
    free(w);
    return NULL;
}

static pool_t* pool_new(int n) {
    pool_t* p = (pool_t*)calloc(1, sizeof(pool_t));
    p->n = n < 1 ? 1 : n;
    pthread_mutex_init(&p->mu, NULL);
    pthread_cond_init(&p->cv_go, NULL);
    pthread_cond_init(&p->cv_done, NULL);
    p->th = (pthread_t*)calloc((size_t)p->n, sizeof(pthread_t));
    for (int i = 1; i < p->n; i++) {
        worker_arg* w = (worker_arg*)malloc(sizeof(worker_arg));
        w->p = p; w->id = i;
        pthread_create(&p->th[i], NULL, pool_main, w);
    }
    return p;
}

static void pool_free(pool_t* p) {
    if (!p) return;
    pthread_mutex_lock(&p->mu);
    p->quit = 1;
    pthread_cond_broadcast(&p->cv_go);
    pthread_mutex_unlock(&p->mu);
    for (int i = 1; i < p->n; i++) pthread_join(p->th[i], NULL);
    free(p->th);
    free(p);
}

static void par_for(pool_t* p, int64_t total, int64_t grain, range_fn fn, void* ctx) {
    if (!p || p->n == 1 || total <= grain) { fn(ctx, 0, total); return; }
    pthread_mutex_lock(&p->mu);
    p->fn = fn; p->ctx = ctx; p->total = total; p->grain = grain;
    p->pending = p->n - 1;
    p->gen++;
    pthread_cond_broadcast(&p->cv_go);
    pthread_mutex_unlock(&p->mu);
    pool_run_part(p, 0);
    pthread_mutex_lock(&p->mu);
    while (p->pending > 0) pthread_cond_wait(&p->cv_done, &p->mu);
    pthread_mutex_unlock(&p->mu);
}

/* one-shot pool for the stateless per-op entry points */
static void par_for_once(int nthreads, int64_t total, int64_t grain, range_fn fn, void* ctx) {
    if (nthreads <= 1 || total <= grain) { fn(ctx, 0, total); return; }
    pool_t* p = pool_new(nthreads);
    par_for(p, total, grain, fn, ctx);
    pool_free(p);
}

/* ------------------------------------------------------------------------ */
/* RMSNorm — kernels/rmsnorm.cuh:6-57 with blockDim 512.                     */
/* Thread t sums items [t*ipt, t*ipt+ipt) with an FMA chain (:17-20), then a */
/* xor butterfly per warp (:24-26), then warp 0 butterflies the 16 warp sums */
/* with lanes 16..31 contributing 0 (:36-41); variance = sum / d (:43).      */
/* ------------------------------------------------------------------------ */
static void butterfly_sum32(float* v) {
    float t[32];
    for (int mask = 16; mask >= 1; mask >>= 1) {
        for (int l = 0; l < 32; l++) t[l] = v[l] + v[l ^ mask];
        memcpy(v, t, sizeof(t));
    }
}

static float rms_scale(const f16* in, int d, float eps) {
    enum { T = 512 };
    int ipt = d / T;
    float part[T];
    for (int t = 0; t < T; t++) {
        float s = 0.0f;
        for (int i = 0; i < ipt; i++) {
            float v = h2f(in[t * ipt + i]);
            s = fmaf(v, v, s);
        }
        part[t] = s;
    }
    float ws[32];
    for (int w = 0; w < T / 32; w++) {
        butterfly_sum32(part + w * 32);
        ws[w] = part[w * 32];
    }
    for (int l = T / 32; l < 32; l++) ws[l] = 0.0f;
    butterfly_sum32(ws);
    float var = ws[0] / (float)d;
    return 1.0f / sqrtf(var + eps);
}

void orc_rmsnorm(f16* out, const f16* in, const f16* w, int d, float eps) {
    float r = rms_scale(in, d, eps);
    int n = (d / 512) * 512;
    for (int i = 0; i < n; i++) out[i] = f2h(h2f(in[i]) * r * h2f(w[i]));
}

/* kernels/bias.cuh:6-11 */
void orc_add_bias(f16* out, const f16* bias, int n) {
    for (int i = 0; i < n; i++) out[i] = f2h(h2f(out[i]) + h2f(bias[i]));
}

/* kernels/swiglu.cuh:6-15: out = w1 * (w2 / (1 + exp(-w2))) */
void orc_swiglu(f16* out, const f16* w1o, const f16* w2o, int n) {
    for (int i = 0; i < n; i++) {
        float a = h2f(w1o[i]), b = h2f(w2o[i]);
        float s = b / (1.0f + expf(-b));
        out[i] = f2h(a * s);
    }
}

/* kernels/fused_qkv_rope_cache.cuh:6-55 */
void orc_fused_qkv_rope_cache(f16* qkv, f16* kc, f16* vc, int pos, int max_seqlen,
                              int num_heads, int head_dim) {
    (void)max_seqlen;
    int H = num_heads * head_dim, half_dim = head_dim / 2;
    for (int h = 0; h < num_heads; h++) {
        for (int t = 0; t < half_dim; t++) {
            int i1 = h * head_dim + t, i2 = h * head_dim + half_dim + t;
            float q1 = h2f(qkv[i1]), q2 = h2f(qkv[i2]);
            float k1 = h2f(qkv[H + i1]), k2 = h2f(qkv[H + i2]);
            float v1 = h2f(qkv[2 * H + i1]), v2 = h2f(qkv[2 * H + i2]);
            float theta = (float)pos * powf(10000.0f, -2.0f * (float)t / (float)head_dim);
            float c = cosf(theta), s = sinf(theta);
            qkv[i1] = f2h(q1 * c - q2 * s);
            qkv[i2] = f2h(q2 * c + q1 * s);
            size_t off = (size_t)pos * H;
            kc[off + i1] = f2h(k1 * c - k2 * s);
            kc[off + i2] = f2h(k2 * c + k1 * s);
            vc[off + i1] = f2h(v1);
            vc[off + i2] = f2h(v2);
        }
    }
}

/* ------------------------------------------------------------------------ */
/* GEMV, weight [K,N] — kernels/hgemm_final.cuh:274-295.                     */
/* C[n] = half(sum_k A[k]*B[k*N+n]) summed in k order by FMA.  Vectorised    */
/* across columns only, so every column keeps the reference's exact chain.   */
/* ------------------------------------------------------------------------ */
typedef struct { const f16* A; const f16* B; f16* C; int N, K, M; } gemv_ctx;

static void gemv_kn_cols(const f16* A, const f16* B, f16* C, int N, int K, int64_t n0, int64_t n1) {
    int64_t n = n0;
    for (; n + 64 <= n1; n += 64) {
        __m256 acc[8];
        for (int j = 0; j < 8; j++) acc[j] = _mm256_setzero_ps();
        for (int k = 0; k < K; k++) {
            __m256 a = _mm256_set1_ps(h2f(A[k]));
            const f16* row = B + (size_t)k * N + n;
            for (int j = 0; j < 8; j++) {
                __m256 b = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(row + 8 * j)));
                acc[j] = _mm256_fmadd_ps(a, b, acc[j]);
            }
        }
        for (int j = 0; j < 8; j++)
            _mm_storeu_si128((__m128i*)(C + n + 8 * j), _mm256_cvtps_ph(acc[j], _MM_FROUND_TO_NEAREST_INT));
    }
    for (; n + 8 <= n1; n += 8) {
        __m256 acc = _mm256_setzero_ps();
        for (int k = 0; k < K; k++) {
            __m256 a = _mm256_set1_ps(h2f(A[k]));
            __m256 b = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(B + (size_t)k * N + n)));
            acc = _mm256_fmadd_ps(a, b, acc);
        }
        _mm_storeu_si128((__m128i*)(C + n), _mm256_cvtps_ph(acc, _MM_FROUND_TO_NEAREST_INT));
    }
    for (; n < n1; n++) {
        float s = 0.0f;
        for (int k = 0; k < K; k++) s = fmaf(h2f(A[k]), h2f(B[(size_t)k * N + n]), s);
        C[n] = f2h(s);
    }
}

static void gemv_kn_range(void* c, int64_t b, int64_t e) {
    gemv_ctx* g = (gemv_ctx*)c;
    gemv_kn_cols(g->A, g->B, g->C, g->N, g->K, b, e);
}

void orc_hgemv_kn(const f16* A, const f16* B, f16* C, int N, int K, int nthreads) {
    gemv_ctx g = {A, B, C, N, K, 1};
    par_for_once(nthreads, N, 64, gemv_kn_range, &g);
}

static void gemv_nk_range(void* c, int64_t b, int64_t e) {
    gemv_ctx* g = (gemv_ctx*)c;
    for (int64_t n = b; n < e; n++) {
        const f16* w = g->B + (size_t)n * g->K;
        float s = 0.0f;
        for (int k = 0; k < g->K; k++) s = fmaf(h2f(g->A[k]), h2f(w[k]), s);
        g->C[n] = f2h(s);
    }
}

void orc_gemv_nk(const f16* x, const f16* W, f16* y, int N, int K, int nthreads) {
    gemv_ctx g = {x, W, y, N, K, 1};
    par_for_once(nthreads, N, 16, gemv_nk_range, &g);
}

/* GEMM C[M,N] = A[M,K] B[K,N]: the prefill product of
 * kernels/hgemm_mma_swizzle.cuh:414-439, restated with an fp32 chain per
 * output (the reference accumulates in fp16 mma; see the header). */
static void gemm_kn_range(void* c, int64_t b, int64_t e) {
    gemv_ctx* g = (gemv_ctx*)c;
    int64_t cols_blocks = (g->N + 63) / 64;
    for (int64_t u = b; u < e; u++) {
        int64_t r = u / cols_blocks, cb = u % cols_blocks;
        int64_t n0 = cb * 64, n1 = n0 + 64 > g->N ? g->N : n0 + 64;
        gemv_kn_cols(g->A + (size_t)r * g->K, g->B, g->C + (size_t)r * g->N, g->N, g->K, n0, n1);
    }
}

void orc_hgemm_kn(const f16* A, const f16* B, f16* C, int M, int N, int K, int nthreads) {
    gemv_ctx g = {A, B, C, N, K, M};
    int64_t units = (int64_t)M * ((N + 63) / 64);
    par_for_once(nthreads, units, 1, gemm_kn_range, &g);
}

/* ------------------------------------------------------------------------ */
/* ArgMax — kernels/argmax.cuh:7-72 launched <<<1,512>>>.                    */
/* Thread t scans [t*ipt, t*ipt+ipt) keeping the first strictly greater      */
/* value; two xor butterflies keep the partner only when strictly greater.   */
/* ------------------------------------------------------------------------ */
static void butterfly_argmax32(float* v, int* ix) {
    float tv[32]; int ti[32];
    for (int mask = 16; mask >= 1; mask >>= 1) {
        for (int l = 0; l < 32; l++) {
            int p = l ^ mask;
            if (v[p] > v[l]) { tv[l] = v[p]; ti[l] = ix[p]; }
            else { tv[l] = v[l]; ti[l] = ix[l]; }
        }
        memcpy(v, tv, sizeof(tv)); memcpy(ix, ti, sizeof(ti));
    }
}

int orc_argmax(const f16* logits, int V) {
    enum { T = 512 };
    int ipt = (V + T - 1) / T;
    float lv[T]; int li[T];
    for (int t = 0; t < T; t++) {
        float best = -INFINITY; int bi = -1;
        for (int i = 0; i < ipt; i++) {
            int idx = t * ipt + i;
            if (idx < V) {
                float v = h2f(logits[idx]);
                if (v > best) { best = v; bi = idx; }
            }
        }
        lv[t] = best; li[t] = bi;
    }
    float wv[32]; int wi[32];
    for (int w = 0; w < T / 32; w++) {
        butterfly_argmax32(lv + w * 32, li + w * 32);
        wv[w] = lv[w * 32]; wi[w] = li[w * 32];
    }
    for (int l = T / 32; l < 32; l++) { wv[l] = -INFINITY; wi[l] = -1; }
    butterfly_argmax32(wv, wi);
    return wi[0];
}

/* ------------------------------------------------------------------------ */
/* Attention                                                                  */
/* ------------------------------------------------------------------------ */
/* exact single-query softmax attention (kernels/unit_tests/run_tests.cu:502-527) */
void orc_attention_q1(const f16* q, const f16* K, const f16* V, f16* O, int L, int stride, int hd) {
    float scale = 1.0f / sqrtf((float)hd);
    float* sc = (float*)malloc(sizeof(float) * (size_t)(L > 0 ? L : 1));
    float mx = -INFINITY;
    for (int i = 0; i < L; i++) {
        float dot = 0.0f;
        for (int j = 0; j < hd; j++) dot += h2f(q[j]) * h2f(K[(size_t)i * stride + j]);
        sc[i] = dot * scale;
        if (sc[i] > mx) mx = sc[i];
    }
    float sum = 0.0f;
    for (int i = 0; i < L; i++) { sc[i] = expf(sc[i] - mx); sum += sc[i]; }
    for (int i = 0; i < L; i++) sc[i] /= sum;
    for (int j = 0; j < hd; j++) {
        float o = 0.0f;
        for (int i = 0; i < L; i++) o += sc[i] * h2f(V[(size_t)i * stride + j]);
        O[j] = f2h(o);
    }
    free(sc);
}

/* one 256-row chunk of flash_decode_q1_opt.cuh:548-656: normalised fp16
 * partial and LSE = log(sum) + max over the scaled scores */
static void fd_chunk(const f16* q, const f16* K, const f16* V, int r0, int r1, int stride,
                     f16* opart, float* lse) {
    enum { D = 128 };
    float scale = 1.0f / sqrtf((float)D);
    float sc[256];
    float mx = -INFINITY;
    for (int i = r0; i < r1; i++) {
        float dot = 0.0f;
        for (int j = 0; j < D; j++) dot += h2f(q[j]) * h2f(K[(size_t)i * stride + j]);
        sc[i - r0] = dot * scale;
        if (sc[i - r0] > mx) mx = sc[i - r0];
    }
    float sum = 0.0f;
    for (int i = 0; i < r1 - r0; i++) { sc[i] = expf(sc[i] - mx); sum += sc[i]; }
    for (int j = 0; j < D; j++) {
        float o = 0.0f;
        for (int i = r0; i < r1; i++) o += sc[i - r0] * h2f(V[(size_t)i * stride + j]);
        opart[j] = f2h(o / sum);
    }
    *lse = logf(sum) + mx;
}

void orc_fd_split_stage1(const f16* q, const f16* K, const f16* V, f16* Opart, float* LSE,
                         int L, int num_chunks, int stride) {
    for (int c = 0; c < num_chunks; c++) {
        int r0 = c * 256, r1 = r0 + 256 < L ? r0 + 256 : L;
        if (r0 >= r1) {  /* an empty chunk leaves max=-inf, sum=0 in the reference */
            for (int j = 0; j < 128; j++) Opart[c * 128 + j] = f2h(NAN);
            LSE[c] = -INFINITY;
            continue;
        }
        fd_chunk(q, K, V, r0, r1, stride, Opart + c * 128, LSE + c);
    }
}

/* flash_decode_q1_opt.cuh:666-724 */
void orc_fd_stage2(const f16* Opart, const float* LSE, f16* O, int num_chunks) {
    float mx = -INFINITY;
    for (int c = 0; c < num_chunks; c++) mx = fmaxf(mx, LSE[c]);
    float sw = 0.0f, o[128];
    for (int j = 0; j < 128; j++) o[j] = 0.0f;
    for (int c = 0; c < num_chunks; c++) {
        float w = expf(LSE[c] - mx);
        sw += w;
        for (int j = 0; j < 128; j++) o[j] = fmaf(w, h2f(Opart[c * 128 + j]), o[j]);
    }
    float inv = 1.0f / sw;
    for (int j = 0; j < 128; j++) O[j] = f2h(o[j] * inv);
}

/* framework_src/qwen_infer.cu:646-677: fused path for L <= 256, else split + merge */
void orc_fd_engine(const f16* q, const f16* K, const f16* V, f16* O, int L, int stride) {
    if (L <= 256) { orc_attention_q1(q, K, V, O, L, stride, 128); return; }
    int nc = (L + 255) / 256;
    f16* part = (f16*)malloc(sizeof(f16) * 128 * (size_t)nc);
    float* lse = (float*)malloc(sizeof(float) * (size_t)nc);
    orc_fd_split_stage1(q, K, V, part, lse, L, nc, stride);
    orc_fd_stage2(part, lse, O, nc);
    free(part); free(lse);
}

void orc_fd_partial_mlo(const f16* q, const f16* K, const f16* V, float* m, float* l, float* o,
                        int L, int stride, int hd) {
    float scale = 1.0f / sqrtf((float)hd);
    float mx = -INFINITY;
    float* sc = (float*)malloc(sizeof(float) * (size_t)(L > 0 ? L : 1));
    for (int i = 0; i < L; i++) {
        float dot = 0.0f;
        for (int j = 0; j < hd; j++) dot += h2f(q[j]) * h2f(K[(size_t)i * stride + j]);
        sc[i] = dot * scale;
        if (sc[i] > mx) mx = sc[i];
    }
    float sum = 0.0f;
    for (int j = 0; j < hd; j++) o[j] = 0.0f;
    for (int i = 0; i < L; i++) {
        float p = expf(sc[i] - mx);
        sum += p;
        for (int j = 0; j < hd; j++) o[j] += p * h2f(V[(size_t)i * stride + j]);
    }
    *m = mx; *l = sum;
    free(sc);
}

typedef struct { const f16 *Q, *K, *V; f16* O; int N, sq, skv, hd; } causal_ctx;

static void causal_rows(void* c, int64_t b, int64_t e) {
    causal_ctx* g = (causal_ctx*)c;
    for (int64_t i = b; i < e; i++)
        orc_attention_q1(g->Q + (size_t)i * g->sq, g->K, g->V, g->O + (size_t)i * g->sq,
                         (int)i + 1, g->skv, g->hd);
}

/* causal attention: row i attends keys 0..i (flash_attn.cu:2016-2031 mask) */
void orc_causal_attention(const f16* Q, const f16* K, const f16* V, f16* O, int N,
                          int stride_q, int stride_kv, int head_dim, int nthreads) {
    causal_ctx g = {Q, K, V, O, N, stride_q, stride_kv, head_dim};
    par_for_once(nthreads, N, 8, causal_rows, &g);
}

/* ------------------------------------------------------------------------ */
/* Whole model — framework_src/qwen_infer.cu:69-738                          */
/* ------------------------------------------------------------------------ */
struct orc_model {
    orc_config cfg;
    pool_t* pool;
    f16 *wte, *ln_f, *lm_head;                 /* lm_head transposed to [H,V] */
    f16 **ln1, **qkv_w, **qkv_b, **proj_w, **ln2, **w1, **w2, **cproj;  /* matrices [K,N] */
    f16 *kc, *vc;                              /* [layers][max_seqlen][H] */
    f16 *x, *xn, *qkv, *att, *tmp, *a, *b, *act, *logits;
};

static int read_exact(FILE* f, void* p, size_t n) { return fread(p, 1, n, f) == n; }

/* [rows, cols] -> [cols, rows] (kernels/transpose.cuh:6-30 at load time, qwen_infer.cu:233-242) */
static f16* load_transposed(FILE* f, int rows, int cols, int* ok) {
    f16* tmp = (f16*)malloc(sizeof(f16) * (size_t)rows * cols);
    f16* out = (f16*)malloc(sizeof(f16) * (size_t)rows * cols);
    if (!tmp || !out || !read_exact(f, tmp, sizeof(f16) * (size_t)rows * cols)) { *ok = 0; free(tmp); return out; }
    const int B = 64;
    for (int r0 = 0; r0 < rows; r0 += B)
        for (int c0 = 0; c0 < cols; c0 += B)
            for (int r = r0; r < r0 + B && r < rows; r++)
                for (int c = c0; c < c0 + B && c < cols; c++)
                    out[(size_t)c * rows + r] = tmp[(size_t)r * cols + c];
    free(tmp);
    return out;
}

static f16* load_plain(FILE* f, size_t n, int* ok) {
    f16* p = (f16*)malloc(sizeof(f16) * n);
    if (!p || !read_exact(f, p, sizeof(f16) * n)) *ok = 0;
    return p;
}

orc_model* orc_model_load(const char* path, int nthreads) {
    FILE* f = fopen(path, "rb");
    if (!f) return NULL;
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    if (!read_exact(f, &m->cfg, sizeof(orc_config)) || m->cfg.magic != 0x46445751u) {
        fclose(f); free(m); return NULL;
    }
    orc_config c = m->cfg;
    int H = (int)c.hidden_size, IM = (int)c.intermediate_size, V = (int)c.vocab_size, NL = (int)c.num_layers;
    int ok = 1;
    m->wte = load_plain(f, (size_t)V * H, &ok);
    m->ln1 = calloc(NL, sizeof(f16*)); m->qkv_w = calloc(NL, sizeof(f16*)); m->qkv_b = calloc(NL, sizeof(f16*));
    m->proj_w = calloc(NL, sizeof(f16*)); m->ln2 = calloc(NL, sizeof(f16*)); m->w1 = calloc(NL, sizeof(f16*));
    m->w2 = calloc(NL, sizeof(f16*)); m->cproj = calloc(NL, sizeof(f16*));
    for (int l = 0; l < NL && ok; l++) {
        m->ln1[l] = load_plain(f, H, &ok);
        m->qkv_w[l] = load_transposed(f, 3 * H, H, &ok);
        m->qkv_b[l] = load_plain(f, 3 * (size_t)H, &ok);
        m->proj_w[l] = load_transposed(f, H, H, &ok);
        m->ln2[l] = load_plain(f, H, &ok);
        m->w1[l] = load_transposed(f, IM, H, &ok);
        m->w2[l] = load_transposed(f, IM, H, &ok);
        m->cproj[l] = load_transposed(f, H, IM, &ok);
    }
    if (ok) m->ln_f = load_plain(f, H, &ok);
    if (ok) m->lm_head = load_transposed(f, V, H, &ok);
    fclose(f);
    if (!ok) { orc_model_free(m); return NULL; }
    size_t kv = (size_t)NL * c.max_seqlen * H;
    m->kc = (f16*)calloc(kv, sizeof(f16));
    m->vc = (f16*)calloc(kv, sizeof(f16));
    size_t big = (size_t)(IM > 3 * H ? IM : 3 * H);
    m->x = calloc(H, sizeof(f16)); m->xn = calloc(H, sizeof(f16)); m->qkv = calloc(3 * (size_t)H, sizeof(f16));
    m->att = calloc(H, sizeof(f16)); m->tmp = calloc(big, sizeof(f16));
    m->a = calloc(IM, sizeof(f16)); m->b = calloc(IM, sizeof(f16)); m->act = calloc(IM, sizeof(f16));
    m->logits = calloc(V, sizeof(f16));
    m->pool = pool_new(nthreads);
    return m;
}

void orc_model_free(orc_model* m) {
    if (!m) return;
    int NL = (int)m->cfg.num_layers;
    for (int l = 0; l < NL; l++) {
        if (m->ln1) free(m->ln1[l]);
        if (m->qkv_w) free(m->qkv_w[l]);
        if (m->qkv_b) free(m->qkv_b[l]);
        if (m->proj_w) free(m->proj_w[l]);
        if (m->ln2) free(m->ln2[l]);
        if (m->w1) free(m->w1[l]);
        if (m->w2) free(m->w2[l]);
        if (m->cproj) free(m->cproj[l]);
    }
    free(m->ln1); free(m->qkv_w); free(m->qkv_b); free(m->proj_w); free(m->ln2); free(m->w1); free(m->w2); free(m->cproj);
    free(m->wte); free(m->ln_f); free(m->lm_head); free(m->kc); free(m->vc);
    free(m->x); free(m->xn); free(m->qkv); free(m->att); free(m->tmp); free(m->a); free(m->b); free(m->act); free(m->logits);
    pool_free(m->pool);
    free(m);
}

void orc_model_config(const orc_model* m, orc_config* out) { *out = m->cfg; }

void orc_model_reset(orc_model* m) {
    size_t kv = (size_t)m->cfg.num_layers * m->cfg.max_seqlen * m->cfg.hidden_size;
    memset(m->kc, 0, kv * sizeof(f16));
    memset(m->vc, 0, kv * sizeof(f16));
}

const f16* orc_model_kcache(const orc_model* m, int layer) {
    return m->kc + (size_t)layer * m->cfg.max_seqlen * m->cfg.hidden_size;
}
const f16* orc_model_vcache(const orc_model* m, int layer) {
    return m->vc + (size_t)layer * m->cfg.max_seqlen * m->cfg.hidden_size;
}

static void mgemv(orc_model* m, const f16* A, const f16* B, f16* C, int N, int K) {
    gemv_ctx g = {A, B, C, N, K, 1};
    par_for(m->pool, N, 64, gemv_kn_range, &g);
}

typedef struct { orc_model* m; int layer, L; const f16* q; f16* out; } head_ctx;

static void heads_range(void* c, int64_t b, int64_t e) {
    head_ctx* g = (head_ctx*)c;
    int H = (int)g->m->cfg.hidden_size;
    const f16* kcl = orc_model_kcache(g->m, g->layer);
    const f16* vcl = orc_model_vcache(g->m, g->layer);
    for (int64_t h = b; h < e; h++)
        orc_fd_engine(g->q + h * 128, kcl + h * 128, vcl + h * 128, g->out + h * 128, g->L, H);
}

/* QwenEngine::step, qwen_infer.cu:614-737 */
int orc_model_step(orc_model* m, int token, int pos, f16* logits_out, f16* trace_out) {
    orc_config c = m->cfg;
    int H = (int)c.hidden_size, IM = (int)c.intermediate_size, V = (int)c.vocab_size, NH = (int)c.num_heads;
    const float eps = 1e-6f;
    memcpy(m->x, m->wte + (size_t)token * H, sizeof(f16) * H);                  /* :617 */
    if (trace_out) memcpy(trace_out, m->x, sizeof(f16) * H);
    for (int l = 0; l < (int)c.num_layers; l++) {
        f16* kcl = m->kc + (size_t)l * c.max_seqlen * H;
        f16* vcl = m->vc + (size_t)l * c.max_seqlen * H;
        orc_rmsnorm(m->xn, m->x, m->ln1[l], H, eps);                              /* :626 */
        mgemv(m, m->xn, m->qkv_w[l], m->qkv, 3 * H, H);                           /* :629 */
        orc_add_bias(m->qkv, m->qkv_b[l], 3 * H);                                 /* :631 */
        orc_fused_qkv_rope_cache(m->qkv, kcl, vcl, pos, (int)c.max_seqlen, NH, 128); /* :634 */
        head_ctx hc = {m, l, pos + 1, m->qkv, m->att};                             /* :646-677 */
        par_for(m->pool, NH, 1, heads_range, &hc);
        mgemv(m, m->att, m->proj_w[l], m->tmp, H, H);                             /* :701 */
        orc_add_bias(m->x, m->tmp, H);                                            /* :704 */
        orc_rmsnorm(m->xn, m->x, m->ln2[l], H, eps);                              /* :708 */
        mgemv(m, m->xn, m->w1[l], m->a, IM, H);                                   /* :711 */
        mgemv(m, m->xn, m->w2[l], m->b, IM, H);                                   /* :712 */
        orc_swiglu(m->act, m->a, m->b, IM);                                       /* :715 */
        mgemv(m, m->act, m->cproj[l], m->tmp, H, IM);                             /* :718 */
        orc_add_bias(m->x, m->tmp, H);                                            /* :721 */
        if (trace_out) memcpy(trace_out + (size_t)(l + 1) * H, m->x, sizeof(f16) * H);
    }
    orc_rmsnorm(m->xn, m->x, m->ln_f, H, eps);                                    /* :725 */
    mgemv(m, m->xn, m->lm_head, m->logits, V, H);                                 /* :728 */
    if (logits_out) memcpy(logits_out, m->logits, sizeof(f16) * V);
    return orc_argmax(m->logits, V);                                              /* :731 */
}

typedef struct { const f16* A; const f16* B; f16* C; int M, N, K; } mgemm_ctx;

static void mgemm(orc_model* m, const f16* A, const f16* B, f16* C, int M, int N, int K) {
    gemv_ctx g = {A, B, C, N, K, M};
    int64_t units = (int64_t)M * ((N + 63) / 64);
    par_for(m->pool, units, 1, gemm_kn_range, &g);
}

typedef struct { orc_model* m; int layer, N; const f16* qkv; f16* out; } pf_head_ctx;

static void pf_rows(void* c, int64_t b, int64_t e) {
    pf_head_ctx* g = (pf_head_ctx*)c;
    int H = (int)g->m->cfg.hidden_size, NH = (int)g->m->cfg.num_heads;
    const f16* kcl = orc_model_kcache(g->m, g->layer);
    const f16* vcl = orc_model_vcache(g->m, g->layer);
    for (int64_t u = b; u < e; u++) {
        int i = (int)(u / NH), h = (int)(u % NH);
        orc_attention_q1(g->qkv + (size_t)i * 3 * H + h * 128, kcl + h * 128, vcl + h * 128,
                         g->out + (size_t)i * H + h * 128, i + 1, H, 128);
    }
}

/* QwenEngine::prefill, qwen_infer.cu:372-611 (row semantics; fp32 GEMM chains) */
void orc_model_prefill(orc_model* m, const int* tokens, int n) {
    if (n <= 0) return;
    orc_config c = m->cfg;
    int H = (int)c.hidden_size, IM = (int)c.intermediate_size, NH = (int)c.num_heads;
    const float eps = 1e-6f;
    f16* X = malloc(sizeof(f16) * (size_t)n * H);
    f16* XN = malloc(sizeof(f16) * (size_t)n * H);
    f16* QKV = malloc(sizeof(f16) * (size_t)n * 3 * H);
    f16* ATT = malloc(sizeof(f16) * (size_t)n * H);
    f16* T = malloc(sizeof(f16) * (size_t)n * H);
    f16* A = malloc(sizeof(f16) * (size_t)n * IM);
    f16* B = malloc(sizeof(f16) * (size_t)n * IM);
    for (int i = 0; i < n; i++) memcpy(X + (size_t)i * H, m->wte + (size_t)tokens[i] * H, sizeof(f16) * H); /* :440-444 */
    for (int l = 0; l < (int)c.num_layers; l++) {
        f16* kcl = m->kc + (size_t)l * c.max_seqlen * H;
        f16* vcl = m->vc + (size_t)l * c.max_seqlen * H;
        for (int i = 0; i < n; i++) orc_rmsnorm(XN + (size_t)i * H, X + (size_t)i * H, m->ln1[l], H, eps); /* :455 */
        mgemm(m, XN, m->qkv_w[l], QKV, n, 3 * H, H);                                                      /* :462 */
        for (int i = 0; i < n; i++) {                                                                     /* :471-477 */
            orc_add_bias(QKV + (size_t)i * 3 * H, m->qkv_b[l], 3 * H);
            orc_fused_qkv_rope_cache(QKV + (size_t)i * 3 * H, kcl, vcl, i, (int)c.max_seqlen, NH, 128);
        }
        pf_head_ctx hc = {m, l, n, QKV, ATT};                                                             /* :486-528 */
        par_for(m->pool, (int64_t)n * NH, 4, pf_rows, &hc);
        mgemm(m, ATT, m->proj_w[l], T, n, H, H);                                                          /* :542 */
        for (int i = 0; i < n; i++) orc_add_bias(X + (size_t)i * H, T + (size_t)i * H, H);               /* :551 */
        for (int i = 0; i < n; i++) orc_rmsnorm(XN + (size_t)i * H, X + (size_t)i * H, m->ln2[l], H, eps); /* :562 */
        mgemm(m, XN, m->w1[l], A, n, IM, H);                                                              /* :573 */
        mgemm(m, XN, m->w2[l], B, n, IM, H);                                                              /* :574 */
        for (int i = 0; i < n; i++) orc_swiglu(A + (size_t)i * IM, A + (size_t)i * IM, B + (size_t)i * IM, IM); /* :583 */
        mgemm(m, A, m->cproj[l], T, n, H, IM);                                                            /* :593 */
        for (int i = 0; i < n; i++) orc_add_bias(X + (size_t)i * H, T + (size_t)i * H, H);               /* :600 */
    }
    free(X); free(XN); free(QKV); free(ATT); free(T); free(A); free(B);
}

/* main() turn, qwen_infer.cu:786-818 */
int orc_model_generate(orc_model* m, const int* prompt, int n, int max_new, int stop_on_eos, int* out) {
    if (n <= 0) return 0;
    int pos = 0;
    if (n > 1) { orc_model_prefill(m, prompt, n - 1); pos = n - 1; }
    int last = prompt[n - 1], cnt = 0;
    for (int s = 0; s < max_new; s++) {
        int next = orc_model_step(m, last, pos, NULL, NULL);
        pos++;
        if (stop_on_eos && (next == 151645 || next == 151643)) break;
        out[cnt++] = next;
        last = next;
    }
    return cnt;
}

/* ------------------------------------------------------------------------ */
/* Seeded random QWDF file: the synthetic weights of the benchmark configs.  */
/* The reference has no such writer; this restates the generator of the     */
/* library under test (per tensor id a splitmix64 key, Box-Muller pairs in   */
/* double, then double -> float -> fp16 RNE; norm weights 1.0), so the       */
/* reference arm of the bench and the tests produce the same bytes without   */
/* loading that library.  Layout: model_weights/convert_weights.py:107-185.   */
/* ------------------------------------------------------------------------ */
static uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

typedef struct { uint64_t key; double sd; uint64_t first; f16* out; } rnd_ctx;

/* elements [first + b, first + e) of a tensor; pair p holds elements 2p (cos) and 2p+1 (sin) */
static void rnd_range(void* c, int64_t b, int64_t e) {
    rnd_ctx* g = (rnd_ctx*)c;
    for (int64_t i = b; i < e; i++) {
        const uint64_t gi = g->first + (uint64_t)i, p = gi / 2;
        const uint64_t u = splitmix64(g->key + 2 * p), v = splitmix64(g->key + 2 * p + 1);
        const double u1 = (double)((u >> 11) + 1) * (1.0 / 9007199254740992.0);
        const double u2 = (double)(v >> 11) * (1.0 / 9007199254740992.0);
        const double r = sqrt(-2.0 * log(u1)), a = 6.283185307179586476925286766559 * u2;
        const double z = (gi & 1) ? r * sin(a) : r * cos(a);
        g->out[i] = f2h((float)(z * g->sd));
    }
}

int orc_write_random_bin(const char* path, const orc_config* cfg, uint64_t seed, float std_dev, int nthreads) {
    FILE* f = fopen(path, "wb");
    if (!f) return -1;
    orc_config h = *cfg;
    h.magic = 0x46445751u;
    int ok = fwrite(&h, sizeof(h), 1, f) == 1;
    const uint64_t H = h.hidden_size, IM = h.intermediate_size, V = h.vocab_size;
    const int NL = (int)h.num_layers, nt = 1 + 8 * NL + 2;
    const size_t chunk = (size_t)1 << 24;
    f16* buf = (f16*)malloc(sizeof(f16) * chunk);
    pool_t* pool = pool_new(nthreads);
    for (int id = 0; ok && id < nt; id++) {
        uint64_t n;
        int norm = 0;
        if (id == 0 || id == nt - 1) n = V * H;
        else if (id == nt - 2) { n = H; norm = 1; }
        else switch ((id - 1) % 8) {
            case 0: case 4: n = H; norm = 1; break;          /* ln_1, ln_2 */
            case 1: n = 3 * H * H; break;                    /* qkv_w */
            case 2: n = 3 * H; break;                        /* qkv_b */
            case 3: n = H * H; break;                        /* attn_proj_w */
            case 5: case 6: n = IM * H; break;               /* ffn_w1, ffn_w2 */
            default: n = H * IM; break;                      /* ffn_proj_w */
        }
        const uint64_t key = splitmix64(seed ^ (0xD1B54A32D192ED03ull * (uint64_t)(id + 1)));
        for (uint64_t i = 0; ok && i < n; i += chunk) {
            const size_t m = (size_t)(n - i < chunk ? n - i : chunk);
            if (norm) {
                for (size_t k = 0; k < m; k++) buf[k] = f2h(1.0f);
            } else {
                rnd_ctx rc = {key, (double)std_dev, i, buf};
                par_for(pool, (int64_t)m, 1 << 16, rnd_range, &rc);
            }
            ok = fwrite(buf, sizeof(f16), m, f) == m;
        }
    }
    pool_free(pool);
    free(buf);
    ok = (fclose(f) == 0) && ok;
    return ok ? 0 : -1;
}
