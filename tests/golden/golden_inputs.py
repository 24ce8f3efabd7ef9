"""Seeded inputs of the golden fixtures (shared by make_golden.py and the tests)."""
import numpy as np

ROPE_POS = (3, 300)
FDF_L, FDF_STRIDE = 200, 256
FDS_L = 1024
FA_N = 100
# max_seqlen leaves room for the reference's fixed 512 new tokens after a 16-token prompt
# (framework_src/qwen_infer.cu:798 never checks the KV capacity).
ENGINE_CFG = dict(vocab_size=8192, hidden_size=2048, num_layers=2, num_heads=16, intermediate_size=5504,
                  max_seqlen=1024)
ENGINE_SEED = 2024


def _h(x):
    return np.asarray(x, np.float32).astype(np.float16)


def ops_inputs():
    r = np.random.default_rng(20241201)
    u = lambda *s: _h(r.random(s) - 0.5)  # run_tests.cu: rand()%1000/1000 - 0.5 style values
    n = lambda *s: _h(r.standard_normal(s))
    return {
        "rms_x": u(2048), "rms_w": _h(r.random(2048) + 0.5),
        "bias_out": u(6144), "bias_b": u(6144),
        "sw_a": n(4096), "sw_b": n(4096),
        "rope_qkv": n(3 * 2048),
        "gemv_A": n(256), "gemv_B": _h(r.standard_normal((256, 512)) * 0.05),
        "fd_q": n(128), "fdf_K": n(FDF_L * FDF_STRIDE), "fdf_V": n(FDF_L * FDF_STRIDE),
        "fds_K": u(FDS_L * 128), "fds_V": u(FDS_L * 128),
        "gemm_A": _h((r.random((128, 128)) - 0.5) * 0.1), "gemm_B": _h((r.random((128, 128)) - 0.5) * 0.1),
        "fa_Q": n(FA_N * 128), "fa_K": n(FA_N * 128), "fa_V": n(FA_N * 128),
    }


def argmax_cases():
    r = np.random.default_rng(7)
    V = 151936
    ipt = (V + 511) // 512
    cases = {}
    a = _h(r.standard_normal(10000))
    a[4321] = 100.0  # run_tests.cu:371-402
    cases["unique_10000"] = a
    b = np.full(V, 0.5, np.float16)
    cases["all_equal"] = b
    c = _h(r.standard_normal(V))
    c[8 * ipt + 3] = c[16 * ipt + 1] = c[24 * ipt] = 9.0
    cases["lanes"] = c
    d = _h(r.standard_normal(V))
    d[(3 * 32) * ipt] = d[(8 * 32) * ipt] = d[(12 * 32 + 5) * ipt] = 9.0
    cases["warps"] = d
    e = _h(np.round(r.standard_normal(V) * 2) / 2)
    cases["random_ties"] = e
    f = _h(r.standard_normal(V))
    f[11] = np.nan
    f[5000] = f[90000] = np.inf
    cases["nan_inf"] = f
    return cases


def engine_prompts():
    """Prompts of the recorded ref_engine.json: a one-token prompt (pure decode
    path) and a 16-token prompt (exercises the reference's prefill)."""
    r = np.random.default_rng(31)
    return [[77], r.integers(0, ENGINE_CFG["vocab_size"], 16).tolist()]


def engine_prompts_rerun():
    """Prompts make_golden.py --engine may run again on the reference engine."""
    return [[77]]
