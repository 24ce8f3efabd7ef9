// engine_internal.h — what other translation units of the library (the
// batched decode) read of an engine: its config, device, stream and the
// device addresses of its weights.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "decode.h"
#include "llmdiy_engine.h"

namespace llmdiy {
struct EngineView {
    llmdiy_config cfg;
    int device, num_sms;
    cudaStream_t stream;
    const LayerPtrs* layers;  // host array [NL] of device pointers
    const half* wte;
    const half* lnf;
    const half* lm_head;
};
EngineView engine_view(const llmdiy_engine* e);
}  // namespace llmdiy
