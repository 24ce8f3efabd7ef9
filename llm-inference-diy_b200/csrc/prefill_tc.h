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

// Forward of prompt tokens (device array, n of them) at positions p0 .. p0+n-1:
// fills the KV cache rows; no lm_head.  Returns a cudaError_t value.
int prefill_tc(const PrefillArgs& p, const int* tokens_dev, int n, int p0, cudaStream_t st);

}  // namespace llmdiy
