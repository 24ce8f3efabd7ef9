/*
 * llmdiy_batch.h — batched greedy decode of independent sequences on one engine's weights.
 *
 * No counterpart in the reference, which serves one sequence at a time (QwenEngine::step,
 * framework_src/qwen_infer.cu:614-737); each row here follows that step's arithmetic.  A batch
 * owns one KV cache region per sequence ([max_len][hidden] per layer, the engine's row format),
 * shares the engine's weights and stream, and runs one step for B sequences as tensor-core GEMMs
 * with M = B plus a ragged split-KV attention over every sequence's own rows.
 *
 * Returns follow llmdiy_engine.h (0, a positive cudaError_t, or a negative LLMDIY_ERR_*).
 */
#ifndef LLMDIY_BATCH_H
#define LLMDIY_BATCH_H

#include <stdint.h>

#include "llmdiy_engine.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct llmdiy_batch llmdiy_batch;

/* At most 64 sequences of at most max_len positions each. */
int  llmdiy_batch_create(llmdiy_engine* e, int max_batch, int max_len, llmdiy_batch** out);
void llmdiy_batch_destroy(llmdiy_batch* b);
const char* llmdiy_batch_last_error(const llmdiy_batch* b);

/* Sequence seq: cache rows [0, len) of every layer filled with seeded N(0,1) fp16 (benchmarks). */
int llmdiy_batch_fill_random(llmdiy_batch* b, int seq, int len, uint64_t seed);
/* Sequence seq: prompt forward of tokens[0..n-1] at positions 0..n-1 into its cache (no lm_head). */
int llmdiy_batch_prefill(llmdiy_batch* b, int seq, const int* tokens, int n);
/* n_steps greedy steps of sequences 0..B-1, sequence s starting from tokens[s] at position pos[s]
 * (host arrays); tokens_out is [n_steps][B] (host).  The first call for a given B captures one step in
 * a CUDA graph; later steps and calls replay it on `stream` (NULL = the engine's stream). */
int llmdiy_batch_decode(llmdiy_batch* b, int B, const int* tokens, const int* pos, int n_steps, int* tokens_out,
                        void* stream);

/* ---- inspection (tests) ---- */
int llmdiy_batch_copy_logits(llmdiy_batch* b, int seq, uint16_t* out);  /* [vocab] of the last step */
int llmdiy_batch_copy_kv(llmdiy_batch* b, int seq, int layer, int pos0, int n, uint16_t* k, uint16_t* v);

#ifdef __cplusplus
}
#endif
#endif
