// qwdf.cpp — QWDF format helpers and the seeded random-weight source.
#include "qwdf.h"

#include <cuda_fp16.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

namespace llmdiy {

int qwdf_num_tensors(const llmdiy_config& c) { return 1 + T_PER_LAYER * (int)c.num_layers + 2; }

TensorDesc qwdf_tensor(const llmdiy_config& c, int id) {
    const size_t H = c.hidden_size, IM = c.intermediate_size, V = c.vocab_size;
    const int last = qwdf_num_tensors(c) - 1;
    if (id == 0) return {id, V, H, false};
    if (id == last) return {id, V, H, false};
    if (id == last - 1) return {id, 1, H, true};
    switch ((id - 1) % T_PER_LAYER) {
        case T_LN1: return {id, 1, H, true};
        case T_QKV_W: return {id, 3 * H, H, false};
        case T_QKV_B: return {id, 1, 3 * H, false};
        case T_PROJ_W: return {id, H, H, false};
        case T_LN2: return {id, 1, H, true};
        case T_W1: return {id, IM, H, false};
        case T_W2: return {id, IM, H, false};
        default: return {id, H, IM, false};
    }
}

const char* qwdf_unsupported(const llmdiy_config& c) {
    if (c.hidden_size != 2048u || c.num_heads != 16u)
        return "fused decode kernel is built for hidden_size 2048 / 16 heads x 128";
    if (c.intermediate_size == 0 || c.intermediate_size % 32 || c.intermediate_size > 6144)
        return "intermediate_size must be a multiple of 32 and <= 6144";
    if (c.num_layers > 64u) return "at most 64 layers";
    if (c.vocab_size == 0 || c.vocab_size % 2 || c.num_layers == 0 || c.max_seqlen == 0)
        return "vocab_size must be even; layers and max_seqlen non-zero";
    return nullptr;
}

void qwdf_tensor_name(const llmdiy_config& c, int id, char* out, size_t len) {
    static const char* kLayer[T_PER_LAYER] = {"ln_1", "qkv_w", "qkv_b", "attn_proj_w", "ln_2", "ffn_w1", "ffn_w2",
                                              "ffn_proj_w"};
    const int last = qwdf_num_tensors(c) - 1;
    if (id == 0) std::snprintf(out, len, "wte");
    else if (id == last) std::snprintf(out, len, "lm_head");
    else if (id == last - 1) std::snprintf(out, len, "ln_f");
    else std::snprintf(out, len, "layer %d %s", (id - 1) / T_PER_LAYER, kLayer[(id - 1) % T_PER_LAYER]);
}

size_t qwdf_file_bytes(const llmdiy_config& c) {
    size_t n = sizeof(QwdfHeader);
    for (int i = 0; i < qwdf_num_tensors(c); ++i) {
        TensorDesc d = qwdf_tensor(c, i);
        n += d.rows * d.cols * 2;
    }
    return n;
}

namespace {

inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// Box-Muller pair p of tensor `id`: elements 2p and 2p+1.
inline void normal_pair(uint64_t key, uint64_t p, double* z0, double* z1) {
    const uint64_t u = splitmix64(key + 2 * p), v = splitmix64(key + 2 * p + 1);
    const double u1 = (double)((u >> 11) + 1) * (1.0 / 9007199254740992.0);  // (0, 1]
    const double u2 = (double)(v >> 11) * (1.0 / 9007199254740992.0);        // [0, 1)
    const double r = std::sqrt(-2.0 * std::log(u1));
    const double a = 6.283185307179586476925286766559 * u2;
    *z0 = r * std::cos(a);
    *z1 = r * std::sin(a);
}

inline uint16_t to_half_bits(float f) {
    __half h = __float2half_rn(f);
    uint16_t b;
    std::memcpy(&b, &h, 2);
    return b;
}

}  // namespace

void qwdf_fill(const llmdiy_config& c, int id, uint64_t seed, float std_dev, size_t first, size_t n, uint16_t* out,
               int nthreads) {
    TensorDesc d = qwdf_tensor(c, id);
    if (d.is_norm) {
        const uint16_t one = to_half_bits(1.0f);
        for (size_t i = 0; i < n; ++i) out[i] = one;
        return;
    }
    const uint64_t key = splitmix64(seed ^ (0xD1B54A32D192ED03ull * (uint64_t)(id + 1)));
    auto work = [&](size_t b, size_t e) {
        size_t i = b;
        while (i < e) {
            const size_t g = first + i, p = g / 2;
            double z0, z1;
            normal_pair(key, p, &z0, &z1);
            if ((g & 1) == 0) {
                out[i++] = to_half_bits((float)(z0 * std_dev));
                if (i < e) out[i++] = to_half_bits((float)(z1 * std_dev));
            } else {
                out[i++] = to_half_bits((float)(z1 * std_dev));
            }
        }
    };
    if (nthreads <= 1 || n < (1u << 16)) { work(0, n); return; }
    std::vector<std::thread> th;
    const size_t per = ((n + nthreads - 1) / nthreads + 1) & ~(size_t)1;  // even split keeps pairs together
    for (int t = 0; t < nthreads; ++t) {
        size_t b = per * t, e = b + per < n ? b + per : n;
        if (b >= e) break;
        th.emplace_back(work, b, e);
    }
    for (auto& x : th) x.join();
}

}  // namespace llmdiy

using namespace llmdiy;

extern "C" {

int llmdiy_qwdf_read_config(const char* path, llmdiy_config* out) {
    FILE* f = std::fopen(path, "rb");
    if (!f) return LLMDIY_ERR_FILE;
    QwdfHeader h;
    size_t got = std::fread(&h, 1, sizeof(h), f);
    std::fseek(f, 0, SEEK_END);
    long long size = std::ftell(f);
    std::fclose(f);
    if (got != sizeof(h) || h.magic != kQwdfMagic) return LLMDIY_ERR_FORMAT;
    out->vocab_size = h.vocab_size;
    out->hidden_size = h.hidden_size;
    out->num_layers = h.num_layers;
    out->num_heads = h.num_heads;
    out->intermediate_size = h.intermediate_size;
    out->max_seqlen = h.max_seqlen;
    if (h.vocab_size == 0 || h.hidden_size == 0 || h.num_layers == 0 || h.num_heads == 0 ||
        h.intermediate_size == 0)
        return LLMDIY_ERR_FORMAT;
    if ((unsigned long long)size < (unsigned long long)qwdf_file_bytes(*out)) return LLMDIY_ERR_FORMAT;
    return LLMDIY_OK;
}

int llmdiy_qwdf_validate(const char* path, llmdiy_config* cfg, uint64_t* nonfinite, char* msg, size_t msg_len) {
    char scratch[8];
    if (!msg || msg_len == 0) { msg = scratch; msg_len = sizeof(scratch); }
    msg[0] = '\0';
    if (nonfinite) *nonfinite = 0;
    FILE* f = std::fopen(path, "rb");
    if (!f) {
        std::snprintf(msg, msg_len, "cannot open %s", path);
        return LLMDIY_ERR_FILE;
    }
    QwdfHeader h{};
    const size_t got = std::fread(&h, 1, sizeof(h), f);
    if (got != sizeof(h) || h.magic != kQwdfMagic) {
        std::fclose(f);
        std::snprintf(msg, msg_len, "not a QWDF file (magic 0x%08x, expected 0x%08x)", h.magic, kQwdfMagic);
        return LLMDIY_ERR_FORMAT;
    }
    const llmdiy_config c{h.vocab_size, h.hidden_size, h.num_layers, h.num_heads, h.intermediate_size, h.max_seqlen};
    if (cfg) *cfg = c;
    if (!c.vocab_size || !c.hidden_size || !c.num_layers || !c.num_heads || !c.intermediate_size) {
        std::fclose(f);
        std::snprintf(msg, msg_len, "header has a zero dimension");
        return LLMDIY_ERR_FORMAT;
    }
    std::fseek(f, 0, SEEK_END);
    const unsigned long long size = (unsigned long long)std::ftell(f);
    const unsigned long long want = qwdf_file_bytes(c);
    if (size < want) {
        std::fclose(f);
        std::snprintf(msg, msg_len, "truncated: %llu bytes, the header's config needs %llu", size, want);
        return LLMDIY_ERR_FORMAT;
    }
    // every fp16 value finite (exponent bits not all ones), counted per tensor
    std::fseek(f, (long)sizeof(QwdfHeader), SEEK_SET);
    const size_t chunk = (size_t)1 << 22;
    std::vector<uint16_t> buf(chunk);
    uint64_t bad_total = 0;
    int first_bad = -1;
    uint64_t first_bad_count = 0;
    for (int id = 0; id < qwdf_num_tensors(c); ++id) {
        const TensorDesc d = qwdf_tensor(c, id);
        const size_t n = d.rows * d.cols;
        uint64_t bad = 0;
        for (size_t i = 0; i < n; i += chunk) {
            const size_t m = n - i < chunk ? n - i : chunk;
            if (std::fread(buf.data(), 2, m, f) != m) {
                std::fclose(f);
                std::snprintf(msg, msg_len, "read error in tensor %d", id);
                return LLMDIY_ERR_FILE;
            }
            for (size_t k = 0; k < m; ++k) bad += (buf[k] & 0x7C00u) == 0x7C00u;
        }
        if (bad && first_bad < 0) { first_bad = id; first_bad_count = bad; }
        bad_total += bad;
    }
    std::fclose(f);
    if (nonfinite) *nonfinite = bad_total;
    if (bad_total) {
        char name[64];
        qwdf_tensor_name(c, first_bad, name, sizeof(name));
        std::snprintf(msg, msg_len, "%llu non-finite fp16 values (first in %s: %llu)", (unsigned long long)bad_total,
                      name, (unsigned long long)first_bad_count);
        return LLMDIY_ERR_FORMAT;
    }
    if (const char* why = qwdf_unsupported(c)) {
        std::snprintf(msg, msg_len, "valid QWDF file, not supported by the engine: %s", why);
        return LLMDIY_ERR_UNSUPPORTED;
    }
    if (size > want)
        std::snprintf(msg, msg_len, "valid; %llu trailing bytes after lm_head are ignored", size - want);
    else
        std::snprintf(msg, msg_len, "valid");
    return LLMDIY_OK;
}

int llmdiy_qwdf_write_random(const char* path, const llmdiy_config* cfg, uint64_t seed, float std_dev, int nthreads) {
    FILE* f = std::fopen(path, "wb");
    if (!f) return LLMDIY_ERR_FILE;
    QwdfHeader h{kQwdfMagic, cfg->vocab_size, cfg->hidden_size, cfg->num_layers, cfg->num_heads,
                 cfg->intermediate_size, cfg->max_seqlen};
    bool ok = std::fwrite(&h, 1, sizeof(h), f) == sizeof(h);
    const size_t chunk = (size_t)1 << 24;
    std::vector<uint16_t> buf(chunk);
    for (int id = 0; ok && id < qwdf_num_tensors(*cfg); ++id) {
        TensorDesc d = qwdf_tensor(*cfg, id);
        const size_t n = d.rows * d.cols;
        for (size_t i = 0; ok && i < n; i += chunk) {
            const size_t m = n - i < chunk ? n - i : chunk;
            qwdf_fill(*cfg, id, seed, std_dev, i, m, buf.data(), nthreads);
            ok = std::fwrite(buf.data(), 2, m, f) == m;
        }
    }
    ok = (std::fclose(f) == 0) && ok;
    return ok ? LLMDIY_OK : LLMDIY_ERR_FILE;
}

int llmdiy_qwdf_fill_tensor(const llmdiy_config* cfg, int tensor_id, uint64_t seed, float std_dev, size_t first,
                            size_t n, uint16_t* out, int nthreads) {
    if (tensor_id < 0 || tensor_id >= qwdf_num_tensors(*cfg)) return LLMDIY_ERR_ARG;
    qwdf_fill(*cfg, tensor_id, seed, std_dev, first, n, out, nthreads);
    return LLMDIY_OK;
}

}  // extern "C"
