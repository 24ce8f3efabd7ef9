/*
 * llmdiy_engine.h — C ABI of the B200 decode engine (libllmdiy_b200.so).
 *
 * A drop-in for the reference engine object and its host driver:
 *   QwenEngine(path)              framework_src/qwen_infer.cu:117-284  -> llmdiy_engine_create
 *   QwenEngine::reset()           framework_src/qwen_infer.cu:318-356  -> llmdiy_engine_reset
 *   QwenEngine::prefill(tokens)   framework_src/qwen_infer.cu:372-611  -> llmdiy_engine_prefill
 *   QwenEngine::step(token, pos)  framework_src/qwen_infer.cu:614-737  -> llmdiy_engine_step
 *   main() turn loop              framework_src/qwen_infer.cu:786-818  -> llmdiy_engine_generate[_stream]
 * The weight file is the reference's QWDF .bin (model_weights/convert_weights.py:107-185).
 *
 * All functions return 0 (LLMDIY_OK) on success, a positive cudaError_t
 * value on a CUDA failure, or a negative LLMDIY_ERR_* code; the engine keeps
 * a readable message (llmdiy_engine_last_error).  Token buffers are host
 * memory.  One engine per device; calls on one engine are not thread-safe.
 */
#ifndef LLMDIY_ENGINE_H
#define LLMDIY_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    LLMDIY_OK = 0,
    LLMDIY_ERR_ARG = -1,          /* invalid argument (bad token id, position beyond max_seqlen, ...) */
    LLMDIY_ERR_FILE = -2,         /* weight file missing or unreadable */
    LLMDIY_ERR_FORMAT = -3,       /* bad magic / truncated file (qwen_infer.cu:126-130) */
    LLMDIY_ERR_UNSUPPORTED = -4,  /* config outside what the sm_100a kernels are built for */
    LLMDIY_ERR_DEVICE = -5,       /* a kernel recorded an error (bounded wait expired, ...) */
    LLMDIY_ERR_NOMEM = -6
};

/* Header of the .bin file (qwen_infer.cu:24-32 without the magic). */
typedef struct {
    uint32_t vocab_size, hidden_size, num_layers, num_heads, intermediate_size, max_seqlen;
} llmdiy_config;

typedef struct llmdiy_engine llmdiy_engine;
typedef void (*llmdiy_token_cb)(int token, void* user);

/* ---- QWDF file tooling ---- */
int llmdiy_qwdf_read_config(const char* path, llmdiy_config* out);
/* Check a .bin against the format (convert_weights.py:107-185 writes it, qwen_infer.cu:117-242 reads it):
 * the magic, a non-zero config, a length covering every tensor, every fp16 value finite, and then
 * whether the engine runs the config.  Returns 0 (valid), LLMDIY_ERR_FILE, LLMDIY_ERR_FORMAT or
 * LLMDIY_ERR_UNSUPPORTED; the header goes to *cfg, the count of non-finite values to *nonfinite
 * and a one-line verdict to msg (either pointer may be NULL). */
int llmdiy_qwdf_validate(const char* path, llmdiy_config* cfg, uint64_t* nonfinite, char* msg, size_t msg_len);
/* Seeded random weights: matrices, biases and wte ~ N(0, std_dev), RMSNorm weights = 1. */
int llmdiy_qwdf_write_random(const char* path, const llmdiy_config* cfg, uint64_t seed, float std_dev, int nthreads);
/* Elements [first, first+n) of tensor `tensor_id` (file order) of that random source, as fp16 bits. */
int llmdiy_qwdf_fill_tensor(const llmdiy_config* cfg, int tensor_id, uint64_t seed, float std_dev, size_t first,
                            size_t n, uint16_t* out, int nthreads);

/* ---- engine lifecycle ---- */
int  llmdiy_engine_create(const char* bin_path, int device, llmdiy_engine** out);
/* Same weights as llmdiy_qwdf_write_random(cfg, seed, std_dev) would write, without a file. */
int  llmdiy_engine_create_random(const llmdiy_config* cfg, uint64_t seed, float std_dev, int device,
                                 llmdiy_engine** out);
void llmdiy_engine_destroy(llmdiy_engine* e);
int  llmdiy_engine_get_config(const llmdiy_engine* e, llmdiy_config* out);
const char* llmdiy_engine_last_error(const llmdiy_engine* e);

/* ---- the reference engine's operations ---- */
int llmdiy_engine_reset(llmdiy_engine* e);
/* Prompt forward over tokens[0..n-1] at positions 0..n-1 (fills the KV cache; no lm_head). */
int llmdiy_engine_prefill(llmdiy_engine* e, const int* tokens, int n);
/* One greedy decode step at position pos; *next = argmax of the logits. */
int llmdiy_engine_step(llmdiy_engine* e, int token, int pos, int* next);
/* A full turn: prefill prompt[0..n-2], then up to max_new greedy steps from prompt[n-1].
 * stop_on_eos stops at 151645/151643 (not written to out).  *n_out = tokens written. */
int llmdiy_engine_generate(llmdiy_engine* e, const int* prompt, int n, int max_new, int stop_on_eos, int* out,
                           int* n_out);
/* As llmdiy_engine_generate, calling cb(token) as each token is produced (streaming). */
int llmdiy_engine_generate_stream(llmdiy_engine* e, const int* prompt, int n, int max_new, int stop_on_eos,
                                  llmdiy_token_cb cb, void* user, int* n_out);

/* ---- device-resident decode (benchmarks): no host synchronisation inside ---- */
/* Enqueue n_steps greedy steps from (first_token, pos) on `stream` (NULL = the engine's stream). */
int llmdiy_engine_decode_async(llmdiy_engine* e, int first_token, int pos, int n_steps, int stop_on_eos,
                               void* stream);
/* After the stream is synchronised: kernel status of the last launch and steps completed. */
int llmdiy_engine_status(llmdiy_engine* e, int* n_done);

/* Timing probes of one decode launch (development aid): out[(cta*cap + i)*2] = %globaltimer ns at
 * the i-th phase boundary of CTA `cta`; prod[((cta*6 + phase)*8 + warp)*4 + {0..3}] = SM cycles waiting
 * for weight chunks, computing, issuing copies; chunks (phase 0..5 = qkv, att, o, w12, c, lm_head). */
int llmdiy_engine_profile(llmdiy_engine* e, int first_token, int pos, int n_steps, int cap, uint64_t* out,
                          uint64_t* prod);

/* ---- inspection (tests) ---- */
int llmdiy_engine_copy_tokens(llmdiy_engine* e, int* out, int n);          /* last decode's tokens */
int llmdiy_engine_copy_logits(llmdiy_engine* e, uint16_t* out);            /* [vocab] fp16 of the last step */
int llmdiy_engine_copy_hidden(llmdiy_engine* e, uint16_t* out);            /* residual stream x [hidden] */
int llmdiy_engine_copy_kv(llmdiy_engine* e, int layer, int pos0, int n, uint16_t* k, uint16_t* v);
int llmdiy_engine_num_sms(const llmdiy_engine* e);

#ifdef __cplusplus
}
#endif
#endif
