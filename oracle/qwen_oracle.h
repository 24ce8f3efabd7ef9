/*
 * qwen_oracle.h — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, fp32 restatement of the LLM-inference-DIY decode path
 * (framework_src/qwen_infer.cu and the kernels it launches), used as the
 * parity checker for the sm_100a kernels and as the timed CPU baseline.
 * Nothing in the product library links, loads or calls this code.
 *
 * Numerics follow the reference: fp16 storage (IEEE binary16, round to
 * nearest even) at every point where the reference stores a `half`, fp32
 * arithmetic in between, the same fused-multiply-add chains where nvcc
 * contracts the reference's `sum += a * b`, and the same reduction trees
 * where the reference's order decides the bits (RMSNorm, ArgMax).  libm
 * replaces the fast-math intrinsics the reference is built with
 * (framework_src/Makefile:58 `--use_fast_math`), so transcendental results
 * differ in the last float bits; tests carry tolerances for that.
 *
 * Pinning: tests/golden/ holds outputs of the reference's own kernels
 * (built from its sources into oracle/_ref/ and JIT-run on a B200); the
 * CPU test suite checks every function here against them.
 */
#ifndef QWEN_ORACLE_H
#define QWEN_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t orc_f16;

/* ---- conversions (IEEE binary16, RNE) ---- */
float   orc_h2f(orc_f16 h);
orc_f16 orc_f2h(float f);
void    orc_f32_to_f16(const float* in, orc_f16* out, int64_t n);
void    orc_f16_to_f32(const orc_f16* in, float* out, int64_t n);

/* ---- per-op restatements (argument order = the reference kernels') ---- */
/* kernels/rmsnorm.cuh:6-57, launched <<<1,512>>> */
void orc_rmsnorm(orc_f16* out, const orc_f16* in, const orc_f16* w, int d, float eps);
/* kernels/bias.cuh:6-11 */
void orc_add_bias(orc_f16* out, const orc_f16* bias, int n);
/* kernels/swiglu.cuh:6-15 (silu applied to the w2 output) */
void orc_swiglu(orc_f16* out, const orc_f16* w1o, const orc_f16* w2o, int n);
/* kernels/fused_qkv_rope_cache.cuh:6-55, launched <<<num_heads,64>>> */
void orc_fused_qkv_rope_cache(orc_f16* qkv, orc_f16* kc, orc_f16* vc, int pos,
                              int max_seqlen, int num_heads, int head_dim);
/* kernels/hgemm_final.cuh:274-295: C[n] = sum_k A[k]*B[k*N+n] (sequential fp32 FMA chain) */
void orc_hgemv_kn(const orc_f16* A, const orc_f16* B, orc_f16* C, int N, int K, int nthreads);
/* same product with the weight in [N,K] (file) layout, sequential chain over k */
void orc_gemv_nk(const orc_f16* x, const orc_f16* W, orc_f16* y, int N, int K, int nthreads);
/* kernels/hgemm_mma_swizzle.cuh:414-439 semantics C[M,N] = A[M,K]*B[K,N], fp32 accumulation */
void orc_hgemm_kn(const orc_f16* A, const orc_f16* B, orc_f16* C, int M, int N, int K, int nthreads);
/* kernels/argmax.cuh:7-72 launched <<<1,512>>>: greedy argmax with the reference tie rule */
int  orc_argmax(const orc_f16* logits, int V);
/* single-query attention, exact fp32 softmax (kernels/unit_tests/run_tests.cu:502-527) */
void orc_attention_q1(const orc_f16* q, const orc_f16* K, const orc_f16* V, orc_f16* O,
                      int L, int stride, int head_dim);
/* the engine's attention for one head (framework_src/qwen_infer.cu:646-677):
 * L <= 256 -> one softmax; else 256-row chunks with fp16-normalised partials,
 * fp32 LSE, and the LSE-weighted merge of flash_decode_q1_opt.cuh:666-724 */
void orc_fd_engine(const orc_f16* q, const orc_f16* K, const orc_f16* V, orc_f16* O,
                   int L, int stride);
/* flash_decode_q1_opt.cuh:548-656 (one call = all chunks) */
void orc_fd_split_stage1(const orc_f16* q, const orc_f16* K, const orc_f16* V,
                         orc_f16* Opart, float* LSE, int L, int num_chunks, int stride);
/* flash_decode_q1_opt.cuh:666-724 */
void orc_fd_stage2(const orc_f16* Opart, const float* LSE, orc_f16* O, int num_chunks);
/* causal prefill attention for one head, rows/keys at `stride` (flash_attn.cu:1854-2179 semantics) */
void orc_causal_attention(const orc_f16* Q, const orc_f16* K, const orc_f16* V, orc_f16* O,
                          int N, int stride_q, int stride_kv, int head_dim, int nthreads);
/* split-KV partials over positions [0,L): per head unnormalised (m, l, o[128]) in fp32 */
void orc_fd_partial_mlo(const orc_f16* q, const orc_f16* K, const orc_f16* V,
                        float* m, float* l, float* o, int L, int stride, int head_dim);

/* ---- whole-model restatement of QwenEngine (framework_src/qwen_infer.cu:69-738) ---- */
typedef struct {
    uint32_t magic, vocab_size, hidden_size, num_layers, num_heads, intermediate_size, max_seqlen;
} orc_config;

typedef struct orc_model orc_model;

/* Reads a QWDF .bin (model_weights/convert_weights.py:107-185). Returns NULL on error. */
orc_model* orc_model_load(const char* path, int nthreads);
void orc_model_free(orc_model* m);
void orc_model_config(const orc_model* m, orc_config* out);
void orc_model_reset(orc_model* m);
/* QwenEngine::step: returns the greedy next token; optional logits [V] and
 * residual stream after each layer [(layers+1) * H] (entry 0 = embedding). */
int  orc_model_step(orc_model* m, int token, int pos, orc_f16* logits_out, orc_f16* trace_out);
/* QwenEngine::prefill over tokens[0..n-1] at positions 0..n-1 (no lm_head). */
void orc_model_prefill(orc_model* m, const int* tokens, int n);
/* main()'s turn (qwen_infer.cu:786-818): prefill all but the last prompt token,
 * then up to max_new greedy steps.  stop_on_eos: stop at 151643/151645.
 * Returns the number of tokens written to out. */
int  orc_model_generate(orc_model* m, const int* prompt, int n, int max_new, int stop_on_eos, int* out);
/* Writes a QWDF file of seeded N(0, std_dev) fp16 weights (norm weights 1) with the
 * header *cfg (magic filled in): the synthetic model of the benchmark configs, byte for
 * byte the one the library under test generates for the same (cfg, seed, std_dev).
 * Returns 0, or -1 on an I/O error. */
int  orc_write_random_bin(const char* path, const orc_config* cfg, uint64_t seed, float std_dev, int nthreads);
/* read-only views used by tests */
const orc_f16* orc_model_kcache(const orc_model* m, int layer);
const orc_f16* orc_model_vcache(const orc_model* m, int layer);

#ifdef __cplusplus
}
#endif
#endif
