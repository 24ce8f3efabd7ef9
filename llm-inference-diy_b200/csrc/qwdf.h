// qwdf.h — the QWDF weight file (model_weights/convert_weights.py:107-185,
// read by framework_src/qwen_infer.cu:117-242) and a seeded random-weight
// source that produces the same tensors whether they are written to a file
// or generated straight into memory.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include "llmdiy_engine.h"

namespace llmdiy {

constexpr uint32_t kQwdfMagic = 0x46445751u;  // "QWDF", qwen_infer.cu:21

struct QwdfHeader {
    uint32_t magic, vocab_size, hidden_size, num_layers, num_heads, intermediate_size, max_seqlen;
};
static_assert(sizeof(QwdfHeader) == 28, "QWDF header is 7 little-endian u32");

// Tensors in file order: 0 = wte, then per layer 8 tensors, then ln_f, lm_head.
enum LayerTensor { T_LN1 = 0, T_QKV_W, T_QKV_B, T_PROJ_W, T_LN2, T_W1, T_W2, T_CPROJ, T_PER_LAYER };

struct TensorDesc {
    int id;          // sequential id in file order
    size_t rows, cols;
    bool is_norm;    // RMSNorm weight (set to 1.0 by the random source)
};

// Number of tensors and the descriptor of tensor `id` for a config.
int qwdf_num_tensors(const llmdiy_config& c);
TensorDesc qwdf_tensor(const llmdiy_config& c, int id);
size_t qwdf_file_bytes(const llmdiy_config& c);

// Nullptr when the engine's kernels run this config, else why not (the
// decode kernel is built for hidden 2048 = 16 heads x 128, intermediate a
// multiple of 32 up to 6144, at most 64 layers, an even vocabulary).
const char* qwdf_unsupported(const llmdiy_config& c);

// Name of tensor `id` in file order ("wte", "layer 3 qkv_w", ..., "lm_head").
void qwdf_tensor_name(const llmdiy_config& c, int id, char* out, size_t len);

// Fill n consecutive elements [first, first+n) of tensor `id` with the
// seeded values (fp16 bits): N(0, std) from a counter-based Box-Muller
// stream, or 1.0 for RMSNorm weights.
void qwdf_fill(const llmdiy_config& c, int id, uint64_t seed, float std_dev, size_t first, size_t n, uint16_t* out,
               int nthreads);

}  // namespace llmdiy
