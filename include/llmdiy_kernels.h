/*
 * llmdiy_kernels.h — C ABI of the sm_100a kernels (libllmdiy_b200.so) that
 * replace the reference's kernel launches one for one.
 *
 * Each launcher keeps the parameter list (names, order, meaning) of the
 * reference kernel or host helper it replaces, cited below as
 * file:line in SeaTheDestiny/LLM-inference-DIY, and adds:
 *   - a trailing `stream` (NULL = the legacy default stream the reference uses);
 *   - an int return: the cudaError_t of the launch (0 = success), instead of
 *     the reference's silent void launch + later cudaGetLastError.
 * Buffers are device pointers to IEEE fp16 bit patterns (uint16_t) or fp32;
 * no launcher allocates, except llmdiy_transpose_weight_gpu, which keeps
 * the reference helper's allocate / transpose / free / swap contract.
 * Launch shapes are the launchers' own choice (B200: 148 SMs).
 */
#ifndef LLMDIY_KERNELS_H
#define LLMDIY_KERNELS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* kernels/rmsnorm.cuh:6 rmsnorm_kernel(out, in, weight, d, epsilon), launched <<<1,512>>>
 * (framework_src/qwen_infer.cu:626). Same reduction tree, bit-identical output. d >= 512. */
int llmdiy_rmsnorm(uint16_t* out, const uint16_t* in, const uint16_t* weight, int d, float eps, void* stream);

/* kernels/bias.cuh:6 add_bias_kernel(out, bias, size): out = half(out + bias)
 * (qwen_infer.cu:631 QKV bias, :704 and :721 residual adds). */
int llmdiy_add_bias(uint16_t* out, const uint16_t* bias, int size, void* stream);

/* kernels/swiglu.cuh:6 swiglu_kernel(out, w1_out, w2_out, size): out = w1 * silu(w2) (qwen_infer.cu:715). */
int llmdiy_swiglu(uint16_t* out, const uint16_t* w1o, const uint16_t* w2o, int size, void* stream);

/* kernels/fused_qkv_rope_cache.cuh:6 fused_qkv_rope_cache_kernel(d_qkv, d_kv_cache_k, d_kv_cache_v,
 * pos, max_seqlen, num_heads, head_dim), launched <<<num_heads,64>>> (qwen_infer.cu:634-642). */
int llmdiy_fused_qkv_rope_cache(uint16_t* qkv, uint16_t* kc, uint16_t* vc, int pos, int max_seqlen, int num_heads,
                                int head_dim, void* stream);

/* kernels/flash_decode_q1_opt.cuh:434 fd_v5_fused_kernel<128,8,32>(Q, K, V, O_final, KV_seqlen, stride),
 * <<<1,256>>> per head (qwen_infer.cu:666-668).  Like the reference it attends rows [0, min(L,256)). */
int llmdiy_fd_v5_fused(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O, int L, int stride,
                       void* stream);

/* kernels/flash_decode_q1_opt.cuh:548 fd_v5_split_stage1_kernel<128,256,8>(Q, K, V, O_partial, LSE,
 * KV_seqlen, num_chunks, stride), <<<num_chunks,256>>> (qwen_infer.cu:671-673). */
int llmdiy_fd_v5_split_stage1(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* Opart, float* LSE,
                              int L, int num_chunks, int stride, void* stream);

/* kernels/flash_decode_q1_opt.cuh:666 fd_opt_stage2_kernel<128>(O_partial, LSE, O_final, num_chunks),
 * <<<1,128>>> (qwen_infer.cu:674-676). */
int llmdiy_fd_opt_stage2(const uint16_t* Opart, const float* LSE, uint16_t* O, int num_chunks, void* stream);

/* ---- tensor-core GEMM (new entry point: the reference's prefill GEMM is hgemm_swizzle_nn with the
 * weights transposed to [K,N] and fp16 accumulation, kernels/hgemm_mma_swizzle.cuh:414).
 * C[M,N] = A[M,K] * W[N,K]^T with W in the .bin file's [out,in] layout, fp16 operands, fp32
 * accumulation on the tcgen05 tensor cores (TMEM accumulators, TMA-staged 128x256x64 tiles), fp16 C.
 * K must be a multiple of 8 and the pointers 16-byte aligned. */
int llmdiy_gemm_tc(const uint16_t* A, const uint16_t* W, uint16_t* C, int M, int N, int K, void* stream);
/* As llmdiy_gemm_tc with B[K,N] row-major (the reference's transposed-weight layout; N a multiple of 64),
 * staged as an MN-major tcgen05 operand. */
int llmdiy_gemm_tc_kn(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K, void* stream);
/* After synchronising: 0, or 1 if a tensor-core GEMM on this device had a pipeline wait expire since the
 * last call (its output is then not valid). */
int llmdiy_gemm_tc_status(void);

/* ---- multi-head split-KV flash decoding (new entry points: the reference attends one head per
 * launch with fd_v5_split_stage1 + fd_opt_stage2, kernels/flash_decode_q1_opt.cuh:548-724, called per
 * head at qwen_infer.cu:650-677).  Q is [num_heads][128] fp16; K and V are the engine's cache layout,
 * row r of head h at r*stride + h*128 (stride >= num_heads*128, a multiple of 8); O is [num_heads][128].
 * Scale 1/sqrt(128), fp32 accumulation, fast-math exponentials like the reference.  `work` is caller
 * scratch of llmdiy_fd_mh_work_bytes(L, num_heads) bytes (device memory, 16-byte aligned, zero-filled once
 * before its first use: its first word is the error word, which the kernels only set, at the same
 * place for every L, so a workspace sized for the longest L serves every shorter one); nothing is
 * allocated.  A partial is 130 fp32: o[128] (unnormalised), m (max score), l (sum of e^{s-m}). */
size_t llmdiy_fd_mh_work_bytes(int L, int num_heads);
/* O = softmax(q k^T / sqrt(128)) v for every head over rows [0, L).  L <= 2048: one launch, a cluster of
 * 8 CTAs per head merging through distributed shared memory (the workspace only carries the error word);
 * longer caches: the persistent split kernel and a merge kernel. */
int llmdiy_fd_multihead(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O, int L, int stride,
                        int num_heads, float* work, size_t work_bytes, void* stream);
/* One merged partial per head over rows [0, L) of this K/V shard: part is [num_heads][130] fp32. */
int llmdiy_fd_mh_partials(const uint16_t* Q, const uint16_t* K, const uint16_t* V, int L, int stride,
                          int num_heads, float* part, float* work, size_t work_bytes, void* stream);
/* Log-sum-exp merge of G shards' partials, parts = [G][num_heads][130] in shard order, into O. */
int llmdiy_fd_mh_merge(const float* parts, int G, int num_heads, uint16_t* O, void* stream);
/* After the stream is synchronised: 0, or -5 when a pipeline wait of a call with this workspace expired
 * since the last status query (that output is then not valid); the query clears the word. */
int llmdiy_fd_mh_status(const float* work, int L, int num_heads);

/* Multi-GPU exchange of the shards' partials over peer memory (no counterpart in the reference,
 * which has no multi-GPU path; replaces an all-gather + llmdiy_fd_mh_merge).  Every rank owns a
 * receive buffer of llmdiy_p2p_buffer_bytes(world, num_heads) bytes (two regions, used by calls of odd
 * and even tag, each [world][num_heads][130] 8-byte words: an fp32 value in the low half, the call's
 * tag in the high half; so a rank may start the next call while a slower rank still merges the last
 * one), allocated with llmdiy_p2p_alloc (zero-filled), whose CUDA IPC handle (64 bytes) the other
 * ranks open with llmdiy_p2p_open.  llmdiy_fd_p2p_merge, called by every rank with the same tag (a
 * call counter starting at 1, never 0), stores this rank's [num_heads][130] partial as tagged words
 * into slot `rank` of every rank's buffer (peers[] = device array of the world buffer pointers in rank
 * order, this rank's own included; one 8-byte store per value, no fence), waits (bounded) until every
 * rank's words in its own buffer carry the tag, and merges the partials in rank order into O.
 * world <= 16.  *err (device int) becomes 1 when a wait expired.  The ranks' kernels must run on
 * different GPUs. */
size_t llmdiy_p2p_buffer_bytes(int world, int num_heads);
int llmdiy_p2p_alloc(size_t bytes, void** ptr, uint8_t* ipc_handle /* 64 bytes out */);
int llmdiy_p2p_open(const uint8_t* ipc_handle /* 64 bytes */, void** ptr);
int llmdiy_p2p_close(void* peer_ptr);
int llmdiy_p2p_free(void* ptr);
int llmdiy_fd_p2p_merge(const float* part, const uint64_t* peers, int world, int rank, int num_heads, uint32_t tag,
                        uint16_t* O, int* err, void* stream);
/* The shard's partials and the exchange in two launches (no counterpart in the reference): the split
 * kernel of llmdiy_fd_mh_partials over this rank's L rows, then llmdiy_fd_p2p_merge's kernel, which
 * merges each head's split partials itself before pushing them (no separate merge launch).  `work`
 * as for llmdiy_fd_mh_partials; the other arguments as for llmdiy_fd_p2p_merge. */
int llmdiy_fd_mh_p2p(const uint16_t* Q, const uint16_t* K, const uint16_t* V, int L, int stride, int num_heads,
                     float* work, size_t work_bytes, const uint64_t* peers, int world, int rank, uint32_t tag,
                     uint16_t* O, int* err, void* stream);

/* No counterpart in the reference.  Split-KV flash decoding of one head in a single launch that
 * allocates nothing: the same result, bit for bit, as llmdiy_fd_v5_split_stage1 + llmdiy_fd_opt_stage2
 * with num_chunks = ceil(L/256), but the chunk partials live in a file-scope device array (33,536 bytes)
 * instead of caller buffers.  L may be at most 32768 rows (128 chunks); a larger L returns -1 before
 * anything is launched.  The first call on each device looks the array up with cudaGetSymbolAddress and
 * should come before any stream capture; so should the first call after a cudaDeviceReset (the address
 * is cached per device and CUDA context, and looked up again when the context changes).  Every call
 * on a device shares the array: calls whose work overlaps on the GPU race; calls ordered on one stream
 * do not. */
int llmdiy_fd_split_noalloc(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O, int L, int stride,
                            void* stream);

/* kernels/argmax.cuh:7 argmax_kernel(out_token, logits, vocab_size), <<<1,512>>> (qwen_infer.cu:731).
 * Reproduces the reference winner among tied maxima; -1 when no value is > -inf. */
int llmdiy_argmax(int* out, const uint16_t* logits, int V, void* stream);

/* kernels/hgemm_final.cuh:274 hgemv_kernel(A, B, C, N, K): C[n] = sum_k A[k] * B[k*N+n],
 * B in the reference's transposed [K,N] layout (qwen_infer.cu:359-363). */
int llmdiy_hgemv(const uint16_t* A, const uint16_t* B, uint16_t* C, int N, int K, void* stream);

/* kernels/hgemm_mma_swizzle.cuh:414 hgemm_swizzle_nn(A, B, C, M, N, K): row-major C[M,N] = A[M,K] * B[K,N]
 * (qwen_infer.cu:364-366).  Accumulates in fp32 (the reference accumulates in fp16).  Runs on the tcgen05
 * tensor cores when N and K are multiples of 8 and the pointers 16-byte aligned (the row pitches a TMA
 * descriptor can address), else on CUDA cores. */
int llmdiy_hgemm_swizzle_nn(uint16_t* A, uint16_t* B, uint16_t* C, int M, int N, int K, void* stream);
/* Which kernel llmdiy_hgemm_swizzle_nn runs for these arguments, without running it (host only, no CUDA
 * call): 1 = tcgen05 tensor cores, 0 = CUDA cores, -1 = invalid shape.  No counterpart in the reference. */
int llmdiy_hgemm_swizzle_nn_path(const uint16_t* A, const uint16_t* B, const uint16_t* C, int M, int N, int K);

/* kernels/flash_attn.cu:1854 flash_attn_tuned_A_kernel<128,...>(Q, K, V, O, QKV_seqlen, QKV_head,
 * stride_Q, stride_KV, K_ofs_override, V_ofs_override, Q_ofs_override, O_ofs_override) with the causal
 * mask the engine compiles in (FLASH_ATTN_CAUSAL, qwen_infer.cu:62, launched per head at :501-516).
 * Offsets < 0 mean "derive from QKV_head" exactly as the reference does.  Runs the tcgen05 flash
 * attention of the engine's prefill on the one head (P in fp16, fp32 accumulation); row pitches must be
 * multiples of 8 elements and the rows 16-byte aligned. */
int llmdiy_flash_attn_tuned_A(uint16_t* Q, uint16_t* K, uint16_t* V, uint16_t* O, int N, int QKV_head,
                              int stride_Q, int stride_KV, int K_ofs, int V_ofs, int Q_ofs, int O_ofs, void* stream);

/* kernels/gather_qkv.cuh:63 gather_q_from_qkv(d_qkv, d_buf, N, numHeads, kHeadDim, stream) */
int llmdiy_gather_q_from_qkv(const uint16_t* qkv, uint16_t* buf, int N, int num_heads, int head_dim, void* stream);
/* kernels/gather_qkv.cuh:75 gather_kv_from_cache(d_cache, d_buf, N, numHeads, kHeadDim, stream) */
int llmdiy_gather_kv_from_cache(const uint16_t* cache, uint16_t* buf, int N, int num_heads, int head_dim,
                                void* stream);
/* kernels/gather_qkv.cuh:39 scatter_interleaved_kernel<128,256>(src, dst, N, numHeads, dst_stride_cols)
 * (qwen_infer.cu:527-528) */
int llmdiy_scatter_interleaved(const uint16_t* src, uint16_t* dst, int N, int num_heads, int dst_cols, void* stream);

/* kernels/transpose.cuh:6 transpose_weight_kernel(out, in, rows, cols): out[c*rows+r] = in[r*cols+c] */
int llmdiy_transpose_weight(uint16_t* out, const uint16_t* in, int rows, int cols, void* stream);
/* kernels/transpose.cuh:17 transpose_weight_gpu(half*& w, rows, cols): allocates, transposes, frees the
 * old buffer and replaces *w (qwen_infer.cu:233-242). Synchronous. */
int llmdiy_transpose_weight_gpu(uint16_t** w, int rows, int cols);

#ifdef __cplusplus
}
#endif
#endif
