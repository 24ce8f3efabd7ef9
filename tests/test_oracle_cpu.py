"""CPU checks of the C oracle (oracle/qwen_oracle.c) against independent
numpy restatements of the reference formulas, the reference's own unit-test
thresholds (kernels/unit_tests/run_tests.cu), and the ArgMax tie rule."""
import os
import tempfile

import numpy as np
import pytest

import refmath


def f16_ulp(x):
    x = np.abs(np.asarray(x, np.float32))
    e = np.floor(np.log2(np.maximum(x, 2.0 ** -14)))
    return 2.0 ** (e - 10)


# ---------------------------------------------------------------- small ops
def test_rmsnorm_matches_formula(oracle, rng):
    # run_tests.cu:55-99: d=2048, eps 1e-6, threshold 1e-2
    x = refmath.h(rng.random(2048) - 0.5)
    w = refmath.h(rng.random(2048) + 0.5)
    got = oracle.rmsnorm(x, w).astype(np.float32)
    ref = refmath.rmsnorm(x, w).astype(np.float32)
    assert np.max(np.abs(got - ref)) < 1e-2
    assert np.all(np.abs(got - ref) <= f16_ulp(ref) + 1e-7)


def test_add_bias_exact(oracle, rng):
    o = refmath.h(rng.random(6144) - 0.5)
    b = refmath.h(rng.random(6144) - 0.5)
    got = oracle.add_bias(o, b)
    ref = refmath.h(o.astype(np.float32) + b.astype(np.float32))
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))


def test_swiglu(oracle, rng):
    a = refmath.h(rng.random(4096) - 0.5)
    b = refmath.h(rng.random(4096) - 0.5)
    got = oracle.swiglu(a, b).astype(np.float32)
    bf = b.astype(np.float64)
    ref = a.astype(np.float64) * bf / (1 + np.exp(-bf))
    assert np.max(np.abs(got - ref)) < 1e-3


@pytest.mark.parametrize("pos", [0, 3, 5, 383])
def test_rope_cache(oracle, rng, pos):
    S, H = 400, 2048
    qkv = refmath.h(rng.random(3 * H) - 0.5)
    kc = np.zeros(S * H, np.float16)
    vc = np.zeros(S * H, np.float16)
    q1, k1, v1 = oracle.fused_qkv_rope_cache(qkv, kc, vc, pos, S)
    q2, k2, v2 = refmath.rope_cache(qkv, kc, vc, pos)
    assert np.max(np.abs(q1.astype(np.float32) - q2.astype(np.float32))) < 1e-3
    assert np.max(np.abs(k1.astype(np.float32) - k2.astype(np.float32))) < 1e-3
    assert np.array_equal(v1.view(np.uint16), v2.view(np.uint16))
    # only row `pos` of the caches is written
    mask = np.ones(S, bool)
    mask[pos] = False
    assert not np.any(k1.reshape(S, H)[mask].astype(np.float32))


def test_gemv_chains_agree(oracle, rng):
    # hgemv over [K,N] and gemv over [N,K] both run the reference's sequential chain
    K, N = 2048, 200
    A = refmath.h((rng.random(K) - 0.5))
    W = refmath.h((rng.random((N, K)) - 0.5) * 0.1)
    y1 = oracle.hgemv_kn(A, np.ascontiguousarray(W.T))
    y2 = oracle.gemv_nk(A, W)
    assert np.array_equal(y1.view(np.uint16), y2.view(np.uint16))
    ref = W.astype(np.float64) @ A.astype(np.float64)
    assert np.max(np.abs(y1.astype(np.float64) - ref)) < 1e-3  # run_tests.cu:848


def test_hgemm(oracle, rng):
    # run_tests.cu:700-725: 128^3, values x0.1, threshold 2e-2
    A = refmath.h((rng.random((128, 128)) - 0.5) * 0.1)
    B = refmath.h((rng.random((128, 128)) - 0.5) * 0.1)
    C = oracle.hgemm_kn(A, B).astype(np.float64)
    assert np.max(np.abs(C - A.astype(np.float64) @ B.astype(np.float64))) < 2e-2


# ---------------------------------------------------------------- argmax tie rule
def test_argmax_unique(oracle, rng):
    lg = refmath.h(rng.random(10000) * 10 - 5)
    lg[1234] = 100.0  # run_tests.cu:380-382
    assert oracle.argmax(lg) == 1234 == refmath.argmax_reference(lg)


@pytest.mark.parametrize("case", ["all_equal", "lanes_8_16", "warps", "within_thread", "nan_inf", "neg_zero",
                                  "all_neg_inf", "random_ties"])
def test_argmax_tie_rule(oracle, rng, case):
    V = 151936
    ipt = (V + 511) // 512
    lg = refmath.h(rng.random(V) - 0.5)
    if case == "all_equal":
        lg[:] = 0.25
    elif case == "lanes_8_16":
        lg[8 * ipt + 3] = 7.0      # thread 8 (lane 8)
        lg[16 * ipt + 1] = 7.0     # thread 16 (lane 16) -> wins: bitrev5(16)=1 < bitrev5(8)=2
    elif case == "warps":
        lg[(3 * 32) * ipt] = 9.0   # warp 3
        lg[(8 * 32) * ipt] = 9.0   # warp 8 -> wins: bitrev5(8)=2 < bitrev5(3)=24
        lg[(12 * 32) * ipt] = 9.0  # warp 12: bitrev5(12)=6
    elif case == "within_thread":
        lg[5 * ipt + 10] = 3.0
        lg[5 * ipt + 2] = 3.0      # same thread: first index wins
    elif case == "nan_inf":
        lg[100] = np.nan
        lg[200] = np.inf
        lg[300] = np.inf
    elif case == "neg_zero":
        lg[:] = -1.0
        lg[40 * ipt] = -0.0
        lg[64 * ipt] = 0.0
    elif case == "all_neg_inf":
        lg[:] = -np.inf
        lg[7] = np.nan
    elif case == "random_ties":
        lg = refmath.h(np.round((rng.random(V) - 0.5) * 8) / 4)  # many exact ties
    assert oracle.argmax(lg) == refmath.argmax_reference(lg)


# ---------------------------------------------------------------- attention
@pytest.mark.parametrize("L,stride", [(1, 128), (31, 128), (256, 128), (256, 2048), (257, 2048), (1024, 128),
                                      (1024, 2048)])
def test_fd_engine(oracle, rng, L, stride):
    hd = 128
    q = refmath.h(rng.standard_normal(hd))
    K = refmath.h(rng.standard_normal(L * stride))
    V = refmath.h(rng.standard_normal(L * stride))
    got = oracle.fd_engine(q, K, V, L, stride).astype(np.float64)
    ref = refmath.attention(q, K, V, L, stride)
    assert np.max(np.abs(got - ref)) < 1e-3


def test_split_stage_matches_exact(oracle, rng):
    # run_tests.cu:626-694: L=1024, Bc=256, 4 chunks, contiguous stride 128
    L, nc = 1024, 4
    q = refmath.h(rng.random(128) - 0.5)
    K = refmath.h(rng.random(L * 128) - 0.5)
    V = refmath.h(rng.random(L * 128) - 0.5)
    Op, lse = oracle.fd_split_stage1(q, K, V, L, nc, 128)
    O = oracle.fd_stage2(Op, lse).astype(np.float64)
    assert np.max(np.abs(O - refmath.attention(q, K, V, L, 128))) < 5e-3


def test_causal_attention(oracle, rng):
    N, st = 40, 128
    Q = refmath.h(rng.standard_normal(N * st))
    K = refmath.h(rng.standard_normal(N * st))
    V = refmath.h(rng.standard_normal(N * st))
    O = oracle.causal_attention(Q, K, V, N, st, st).astype(np.float64)
    for i in (0, 1, 17, N - 1):
        ref = refmath.attention(Q[i * st:], K, V, i + 1, st)
        assert np.max(np.abs(O[i * st:(i + 1) * st] - ref)) < 1e-3


def test_partial_mlo_merge(oracle, rng):
    L, st = 600, 2048
    q = refmath.h(rng.standard_normal(128))
    K = refmath.h(rng.standard_normal(L * st))
    V = refmath.h(rng.standard_normal(L * st))
    parts = [oracle.fd_partial_mlo(q, K[a * st:], V[a * st:], b - a, st) for a, b in ((0, 200), (200, 450), (450, 600))]
    M = max(p[0] for p in parts)
    Lsum = sum(p[1] * np.exp(p[0] - M) for p in parts)
    O = sum(p[2] * np.exp(p[0] - M) for p in parts) / Lsum
    assert np.max(np.abs(O - refmath.attention(q, K, V, L, st))) < 1e-4


# ---------------------------------------------------------------- whole model
TINY = dict(vocab_size=1024, hidden_size=512, num_layers=2, num_heads=4, intermediate_size=384, max_seqlen=64)


@pytest.fixture(scope="module")
def tiny_bin():
    import llmdiy_b200 as L
    d = tempfile.mkdtemp()
    path = os.path.join(d, "tiny.bin")
    L.write_random_bin(path, L.make_config(**TINY), seed=7)
    yield path
    os.remove(path)


def test_tiny_model_step_matches_numpy(tiny_bin):
    import oracle as orc
    W, cfg = refmath.read_bin(tiny_bin)
    m = orc.OracleModel(tiny_bin, nthreads=4)
    S, H = cfg["max_seqlen"], cfg["hidden_size"]
    kc = np.zeros((cfg["num_layers"], S, H), np.float16)
    vc = np.zeros_like(kc)
    tok = 5
    for pos in range(6):
        nxt, lg, _ = m.step(tok, pos, want_logits=True)
        ref_lg, _ = refmath.model_step(W, kc, vc, tok, pos, cfg)
        err = np.max(np.abs(lg.astype(np.float32) - ref_lg.astype(np.float32)))
        assert err < 2e-2, (pos, err)
        assert nxt == refmath.argmax_reference(lg)
        tok = nxt
    k0, v0 = m.kv(0, 0, 6)
    assert np.max(np.abs(k0.astype(np.float32) - kc[0, :6].astype(np.float32))) < 2e-2


def test_tiny_model_prefill_equals_steps(tiny_bin):
    """prefill(tokens) leaves the same KV cache as stepping the same tokens."""
    import oracle as orc
    prompt = [3, 17, 250, 999, 4, 42, 7]
    a = orc.OracleModel(tiny_bin, nthreads=4)
    a.prefill(prompt)
    b = orc.OracleModel(tiny_bin, nthreads=4)
    for i, t in enumerate(prompt):
        b.step(t, i)
    for layer in range(TINY["num_layers"]):
        ka, va = a.kv(layer, 0, len(prompt))
        kb, vb = b.kv(layer, 0, len(prompt))
        assert np.array_equal(ka.view(np.uint16), kb.view(np.uint16))
        assert np.array_equal(va.view(np.uint16), vb.view(np.uint16))


def test_tiny_generate_protocol_semantics(tiny_bin):
    import oracle as orc
    m = orc.OracleModel(tiny_bin, nthreads=4)
    toks = m.generate([1, 2, 3], 10)
    m2 = orc.OracleModel(tiny_bin, nthreads=4)
    m2.prefill([1, 2])
    t, pos, ref = 3, 2, []
    for _ in range(10):
        t, _, _ = m2.step(t, pos)
        pos += 1
        ref.append(t)
    assert toks == ref
