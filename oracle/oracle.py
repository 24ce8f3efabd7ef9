"""TEST INFRASTRUCTURE ONLY -- ctypes wrappers of the CPU oracle and of the
reference's own kernels.

* `Oracle` wraps oracle/_build/libqwen_oracle.so, the C restatement of the
  reference decode path (oracle/qwen_oracle.c).  Used by tests/, by
  __graft_entry__.smoke() as the checker, and by bench.py's cpu_baseline /
  --impl reference legs.  Never by the product.
* `RefKernels` wraps oracle/_ref/libref_kernels.so: the reference's kernels
  (kernels/*.cuh of LLM-inference-DIY) compiled from its sources to
  compute_89 PTX by `make -C oracle ref` and JIT-run on the B200; used to
  produce and check golden fixtures.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "_build", "libqwen_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref_kernels.so")
REF_ENGINE = os.path.join(HERE, "_ref", "qwen_infer_ref")
# The reference checkout: $LLMDIY_REFERENCE_TREE, else a `reference` directory beside this repository.
REFERENCE_TREE = os.environ.get("LLMDIY_REFERENCE_TREE",
                                os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))


def build(reference: bool = True) -> None:
    """Compile the oracle (and, when the reference tree is present, the reference kernels)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if reference and os.path.isdir(os.path.join(REFERENCE_TREE, "kernels")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={REFERENCE_TREE}"], check=True)


def f16(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float16))


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


class OrcConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in
                ("magic", "vocab_size", "hidden_size", "num_layers", "num_heads", "intermediate_size", "max_seqlen")]


class Oracle:
    def __init__(self, path: str = ORACLE_LIB):
        if not os.path.exists(path):
            build(reference=False)
        L = ctypes.CDLL(path)
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        sig = {
            "orc_rmsnorm": ([P, P, P, I, F], None),
            "orc_add_bias": ([P, P, I], None),
            "orc_swiglu": ([P, P, P, I], None),
            "orc_fused_qkv_rope_cache": ([P, P, P, I, I, I, I], None),
            "orc_hgemv_kn": ([P, P, P, I, I, I], None),
            "orc_gemv_nk": ([P, P, P, I, I, I], None),
            "orc_hgemm_kn": ([P, P, P, I, I, I, I], None),
            "orc_argmax": ([P, I], I),
            "orc_attention_q1": ([P, P, P, P, I, I, I], None),
            "orc_fd_engine": ([P, P, P, P, I, I], None),
            "orc_fd_split_stage1": ([P, P, P, P, P, I, I, I], None),
            "orc_fd_stage2": ([P, P, P, I], None),
            "orc_causal_attention": ([P, P, P, P, I, I, I, I, I], None),
            "orc_fd_partial_mlo": ([P, P, P, P, P, P, I, I, I], None),
            "orc_model_load": ([ctypes.c_char_p, I], P),
            "orc_model_free": ([P], None),
            "orc_model_config": ([P, ctypes.POINTER(OrcConfig)], None),
            "orc_model_reset": ([P], None),
            "orc_model_step": ([P, I, I, P, P], I),
            "orc_model_prefill": ([P, P, I], None),
            "orc_model_generate": ([P, P, I, I, I, P], I),
            "orc_model_kcache": ([P, I], P),
            "orc_write_random_bin": ([ctypes.c_char_p, ctypes.POINTER(OrcConfig), ctypes.c_uint64, F, I], I),
            "orc_model_vcache": ([P, I], P),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        self.L = L

    # ---- ops (numpy in, numpy out) ----
    def rmsnorm(self, x, w, eps=1e-6):
        x, w = f16(x), f16(w)
        out = np.zeros_like(x)
        self.L.orc_rmsnorm(_ptr(out), _ptr(x), _ptr(w), x.size, eps)
        return out

    def add_bias(self, out, b):
        out, b = f16(out).copy(), f16(b)
        self.L.orc_add_bias(_ptr(out), _ptr(b), out.size)
        return out

    def swiglu(self, a, b):
        a, b = f16(a), f16(b)
        out = np.zeros_like(a)
        self.L.orc_swiglu(_ptr(out), _ptr(a), _ptr(b), a.size)
        return out

    def fused_qkv_rope_cache(self, qkv, kc, vc, pos, max_seqlen, nh=16, hd=128):
        qkv, kc, vc = f16(qkv).copy(), f16(kc).copy(), f16(vc).copy()
        self.L.orc_fused_qkv_rope_cache(_ptr(qkv), _ptr(kc), _ptr(vc), pos, max_seqlen, nh, hd)
        return qkv, kc, vc

    def hgemv_kn(self, A, B, nthreads=8):
        A, B = f16(A), f16(B)
        K, N = B.shape
        C = np.zeros(N, np.float16)
        self.L.orc_hgemv_kn(_ptr(A), _ptr(B), _ptr(C), N, K, nthreads)
        return C

    def gemv_nk(self, x, W, nthreads=8):
        x, W = f16(x), f16(W)
        N, K = W.shape
        y = np.zeros(N, np.float16)
        self.L.orc_gemv_nk(_ptr(x), _ptr(W), _ptr(y), N, K, nthreads)
        return y

    def hgemm_kn(self, A, B, nthreads=8):
        A, B = f16(A), f16(B)
        M, K = A.shape
        N = B.shape[1]
        C = np.zeros((M, N), np.float16)
        self.L.orc_hgemm_kn(_ptr(A), _ptr(B), _ptr(C), M, N, K, nthreads)
        return C

    def argmax(self, logits):
        logits = f16(logits)
        return int(self.L.orc_argmax(_ptr(logits), logits.size))

    def attention_q1(self, q, K, V, L, stride, hd=128):
        q, K, V = f16(q), f16(K), f16(V)
        O = np.zeros(hd, np.float16)
        self.L.orc_attention_q1(_ptr(q), _ptr(K), _ptr(V), _ptr(O), L, stride, hd)
        return O

    def fd_engine(self, q, K, V, L, stride):
        q, K, V = f16(q), f16(K), f16(V)
        O = np.zeros(128, np.float16)
        self.L.orc_fd_engine(_ptr(q), _ptr(K), _ptr(V), _ptr(O), L, stride)
        return O

    def fd_split_stage1(self, q, K, V, L, nc, stride):
        q, K, V = f16(q), f16(K), f16(V)
        Op = np.zeros(nc * 128, np.float16)
        lse = np.zeros(nc, np.float32)
        self.L.orc_fd_split_stage1(_ptr(q), _ptr(K), _ptr(V), _ptr(Op), _ptr(lse), L, nc, stride)
        return Op, lse

    def fd_stage2(self, Op, lse):
        Op, lse = f16(Op), np.ascontiguousarray(lse, dtype=np.float32)
        O = np.zeros(128, np.float16)
        self.L.orc_fd_stage2(_ptr(Op), _ptr(lse), _ptr(O), lse.size)
        return O

    def write_random_bin(self, path, vocab_size, hidden_size, num_layers, num_heads, intermediate_size,
                         max_seqlen, seed, std_dev=0.02, nthreads=8):
        """Seeded random QWDF file (the benchmark's synthetic model), without the product library."""
        c = OrcConfig(0x46445751, vocab_size, hidden_size, num_layers, num_heads, intermediate_size, max_seqlen)
        rc = self.L.orc_write_random_bin(path.encode(), ctypes.byref(c), seed, std_dev, nthreads)
        if rc != 0:
            raise OSError(f"could not write {path}")

    def causal_attention(self, Q, K, V, N, stride_q, stride_kv, hd=128, nthreads=8):
        Q, K, V = f16(Q), f16(K), f16(V)
        O = np.zeros_like(Q)
        self.L.orc_causal_attention(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), N, stride_q, stride_kv, hd, nthreads)
        return O

    def fd_partial_mlo(self, q, K, V, L, stride, hd=128):
        q, K, V = f16(q), f16(K), f16(V)
        m = np.zeros(1, np.float32)
        l = np.zeros(1, np.float32)
        o = np.zeros(hd, np.float32)
        self.L.orc_fd_partial_mlo(_ptr(q), _ptr(K), _ptr(V), _ptr(m), _ptr(l), _ptr(o), L, stride, hd)
        return float(m[0]), float(l[0]), o


class OracleModel:
    """The whole-model restatement of QwenEngine (CPU, fp32 with fp16 stores)."""

    def __init__(self, bin_path: str, nthreads: int = 8, oracle: Oracle | None = None):
        self.o = oracle or Oracle()
        self.h = self.o.L.orc_model_load(bin_path.encode(), nthreads)
        if not self.h:
            raise RuntimeError(f"oracle could not load {bin_path}")
        c = OrcConfig()
        self.o.L.orc_model_config(self.h, ctypes.byref(c))
        self.config = c

    def close(self):
        if self.h:
            self.o.L.orc_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        self.o.L.orc_model_reset(self.h)

    def step(self, token, pos, want_logits=False, want_trace=False):
        lg = np.zeros(self.config.vocab_size, np.float16) if want_logits else None
        tr = np.zeros((self.config.num_layers + 1, self.config.hidden_size), np.float16) if want_trace else None
        nxt = self.o.L.orc_model_step(self.h, token, pos, None if lg is None else _ptr(lg),
                                      None if tr is None else _ptr(tr))
        return nxt, lg, tr

    def prefill(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        self.o.L.orc_model_prefill(self.h, _ptr(t), t.size)

    def generate(self, prompt, max_new, stop_on_eos=True):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(1, max_new), np.int32)
        n = self.o.L.orc_model_generate(self.h, _ptr(p), p.size, max_new, int(stop_on_eos), _ptr(out))
        return out[:n].tolist()

    def kv(self, layer, pos0, n):
        H, S = self.config.hidden_size, self.config.max_seqlen
        kp = self.o.L.orc_model_kcache(self.h, layer)
        vp = self.o.L.orc_model_vcache(self.h, layer)
        k = np.ctypeslib.as_array(ctypes.cast(kp, ctypes.POINTER(ctypes.c_uint16)), shape=(S * H,))
        v = np.ctypeslib.as_array(ctypes.cast(vp, ctypes.POINTER(ctypes.c_uint16)), shape=(S * H,))
        sl = slice(pos0 * H, (pos0 + n) * H)
        return k[sl].copy().view(np.float16).reshape(n, H), v[sl].copy().view(np.float16).reshape(n, H)


class RefKernels:
    """The reference's own kernels (compute_89 PTX, JIT-run on the GPU); device addresses in, status out."""

    def __init__(self, path: str = REF_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = ctypes.CDLL(path)
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        sig = {
            "ref_rmsnorm": [P, P, P, I, F],
            "ref_add_bias": [P, P, I],
            "ref_swiglu": [P, P, P, I],
            "ref_fused_qkv_rope_cache": [P, P, P, I, I, I, I],
            "ref_hgemv": [P, P, P, I, I],
            "ref_fd_v5_fused": [P, P, P, P, I, I],
            "ref_fd_v5_split_stage1": [P, P, P, P, P, I, I, I],
            "ref_fd_opt_stage2": [P, P, P, I],
            "ref_argmax": [P, P, I],
            "ref_hgemm_swizzle_nn": [P, P, P, I, I, I],
            "ref_flash_attn_causal_head": [P, P, P, P, I],
            "ref_gather_q_from_qkv": [P, P, I, I],
            "ref_gather_kv_from_cache": [P, P, I, I],
            "ref_scatter_interleaved": [P, P, I, I, I],
            "ref_transpose": [P, P, I, I],
            "ref_fd_layer": [P, P, P, P, P, P, I, I, I, P],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        self.L = L

    def __getattr__(self, name):
        fn = getattr(self.L, "ref_" + name)

        def call(*args):
            conv = [ctypes.c_void_p(a) if isinstance(a, int) and a > 2 ** 31 else a for a in args]
            rc = fn(*conv)
            if rc != 0:
                raise RuntimeError(f"ref_{name} returned {rc}")
        return call
