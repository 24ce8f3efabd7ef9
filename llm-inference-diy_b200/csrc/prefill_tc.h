// prefill_tc.h — the tensor-core prompt forward used by llmdiy_engine_prefill.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "decode.h"

namespace llmdiy {

constexpr int kPrefillChunk = 2048;  // prompt rows per pass (scratch is sized for this many)

struct PrefillArgs {
    const LayerPtrs* layers;  // host array [NL] of device pointers
    const half* wte;
    half* kc;                  // layer l of the cache at kc + l * layer_stride, row r at + r * H
    half* vc;
    size_t layer_stride;       // elements between layers of the cache
    int NL, IM, max_seqlen;
    // scratch, kPrefillChunk rows each: x, xn, q, att [rows][H]; act [rows][IM]
    half *x, *xn, *q, *att, *act;
    half* hidden;  // [H] receives the residual stream of the prompt's last row
};

// Causal attention on the tcgen05 tensor cores (flash_tc.cuh) of n query rows at positions
// p0 .. p0+n-1 over key/value rows [0, p0+n): q [n] rows of ldq elements, k / v [kv_rows] rows of
// ldkv elements, o [n] rows of ldo elements; `heads` heads of 128 columns side by side in each row.
// Pointers 16-byte aligned, row pitches multiples of 8 elements.  Returns a cudaError_t value.
int flash_tc_causal(const half* q, int ldq, const half* k, const half* v, int ldkv, int kv_rows, half* o, int ldo,
                    int n, int p0, int heads, cudaStream_t st);

// Forward of prompt tokens (device array, n of them) at positions p0 .. p0+n-1:
// fills the KV cache rows; no lm_head.  Returns a cudaError_t value.
int prefill_tc(const PrefillArgs& p, const int* tokens_dev, int n, int p0, cudaStream_t st);

}  // namespace llmdiy
