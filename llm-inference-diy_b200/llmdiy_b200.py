"""ctypes binding of libllmdiy_b200.so (include/llmdiy_kernels.h, include/llmdiy_engine.h).

Host-side mirror of the reference's interfaces for Python callers: the
`Engine` class follows QwenEngine (framework_src/qwen_infer.cu:69-738) --
construct from a .bin path, reset(), prefill(tokens), step(token, pos) --
plus generate() for the driver's turn loop (qwen_infer.cu:786-818).  The
kernel launchers take device addresses (ints, e.g. torch.Tensor.data_ptr())
and an optional CUDA stream handle, keeping the reference parameter order.

The library is required: importing this module never falls back to another
implementation, and every call raises LlmdiyError on a non-zero status.
"""
from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "libllmdiy_b200.so")
LIB_PATH = os.environ.get("LLMDIY_LIB", LIB_PATH)  # an alternative build of the library (A/B timing)
DRIVER_PATH = os.path.join(_HERE, "_build", "qwen_infer_b200")
INCLUDE_DIR = os.path.join(os.path.dirname(_HERE), "include")

STOP_IDS = (151645, 151643)  # qwen_infer.cu:808
ERR_ARG, ERR_FILE, ERR_FORMAT, ERR_UNSUPPORTED, ERR_DEVICE, ERR_NOMEM = -1, -2, -3, -4, -5, -6  # llmdiy_engine.h


class LlmdiyError(RuntimeError):
    pass


class Config(ctypes.Structure):
    _fields_ = [
        ("vocab_size", ctypes.c_uint32),
        ("hidden_size", ctypes.c_uint32),
        ("num_layers", ctypes.c_uint32),
        ("num_heads", ctypes.c_uint32),
        ("intermediate_size", ctypes.c_uint32),
        ("max_seqlen", ctypes.c_uint32),
    ]

    def as_dict(self):
        return {k: int(getattr(self, k)) for k, _ in self._fields_}


def make_config(vocab_size=151936, hidden_size=2048, num_layers=24, num_heads=16, intermediate_size=5504,
                max_seqlen=2048) -> Config:
    return Config(vocab_size, hidden_size, num_layers, num_heads, intermediate_size, max_seqlen)


QWEN_1_8B = dict(vocab_size=151936, hidden_size=2048, num_layers=24, num_heads=16, intermediate_size=5504)

_lib = None


def lib() -> ctypes.CDLL:
    """Load the sm_100a library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise LlmdiyError(f"{LIB_PATH} is missing: build it with `make -C llm-inference-diy_b200`")
    L = ctypes.CDLL(LIB_PATH)
    P, I, F, U64, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_uint64, ctypes.c_size_t
    IP = ctypes.POINTER(ctypes.c_int)
    sig = {
        "llmdiy_rmsnorm": [P, P, P, I, F, P],
        "llmdiy_add_bias": [P, P, I, P],
        "llmdiy_swiglu": [P, P, P, I, P],
        "llmdiy_fused_qkv_rope_cache": [P, P, P, I, I, I, I, P],
        "llmdiy_fd_v5_fused": [P, P, P, P, I, I, P],
        "llmdiy_fd_v5_split_stage1": [P, P, P, P, P, I, I, I, P],
        "llmdiy_fd_opt_stage2": [P, P, P, I, P],
        "llmdiy_gemm_tc": [P, P, P, I, I, I, P],
        "llmdiy_gemm_tc_kn": [P, P, P, I, I, I, P],
        "llmdiy_gemm_tc_status": [],
        "llmdiy_fd_multihead": [P, P, P, P, I, I, I, P, SZ, P],
        "llmdiy_fd_mh_partials": [P, P, P, I, I, I, P, P, SZ, P],
        "llmdiy_fd_mh_merge": [P, I, I, P, P],
        "llmdiy_fd_mh_status": [P, I, I],
        "llmdiy_p2p_alloc": [SZ, ctypes.POINTER(P), P],
        "llmdiy_p2p_open": [P, ctypes.POINTER(P)],
        "llmdiy_p2p_close": [P],
        "llmdiy_p2p_free": [P],
        "llmdiy_fd_p2p_merge": [P, P, I, I, I, ctypes.c_uint32, P, P, P],
        "llmdiy_fd_mh_p2p": [P, P, P, I, I, I, P, SZ, P, I, I, ctypes.c_uint32, P, P, P],
        "llmdiy_argmax": [P, P, I, P],
        "llmdiy_hgemv": [P, P, P, I, I, P],
        "llmdiy_hgemm_swizzle_nn": [P, P, P, I, I, I, P],
        "llmdiy_hgemm_swizzle_nn_path": [P, P, P, I, I, I],
        "llmdiy_flash_attn_tuned_A": [P, P, P, P, I, I, I, I, I, I, I, I, P],
        "llmdiy_gather_q_from_qkv": [P, P, I, I, I, P],
        "llmdiy_gather_kv_from_cache": [P, P, I, I, I, P],
        "llmdiy_scatter_interleaved": [P, P, I, I, I, P],
        "llmdiy_transpose_weight": [P, P, I, I, P],
        "llmdiy_transpose_weight_gpu": [ctypes.POINTER(ctypes.c_void_p), I, I],
        "llmdiy_qwdf_read_config": [ctypes.c_char_p, ctypes.POINTER(Config)],
        "llmdiy_qwdf_validate": [ctypes.c_char_p, ctypes.POINTER(Config), ctypes.POINTER(U64), ctypes.c_char_p, SZ],
        "llmdiy_qwdf_write_random": [ctypes.c_char_p, ctypes.POINTER(Config), U64, F, I],
        "llmdiy_qwdf_fill_tensor": [ctypes.POINTER(Config), I, U64, F, SZ, SZ, P, I],
        "llmdiy_engine_create": [ctypes.c_char_p, I, ctypes.POINTER(P)],
        "llmdiy_engine_create_random": [ctypes.POINTER(Config), U64, F, I, ctypes.POINTER(P)],
        "llmdiy_engine_get_config": [P, ctypes.POINTER(Config)],
        "llmdiy_engine_reset": [P],
        "llmdiy_engine_prefill": [P, IP, I],
        "llmdiy_engine_step": [P, I, I, IP],
        "llmdiy_engine_generate": [P, IP, I, I, I, IP, IP],
        "llmdiy_engine_decode_async": [P, I, I, I, I, P],
        "llmdiy_engine_status": [P, IP],
        "llmdiy_engine_copy_tokens": [P, IP, I],
        "llmdiy_engine_copy_logits": [P, P],
        "llmdiy_engine_copy_hidden": [P, P],
        "llmdiy_engine_copy_kv": [P, I, I, I, P, P],
        "llmdiy_engine_num_sms": [P],
        "llmdiy_engine_profile": [P, I, I, I, I, P, P],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    L.llmdiy_p2p_buffer_bytes.argtypes = [I, I]
    L.llmdiy_p2p_buffer_bytes.restype = SZ
    L.llmdiy_engine_destroy.argtypes = [P]
    L.llmdiy_engine_destroy.restype = None
    L.llmdiy_engine_last_error.argtypes = [P]
    L.llmdiy_engine_last_error.restype = ctypes.c_char_p
    bsig = {
        "llmdiy_batch_create": [P, I, I, ctypes.POINTER(ctypes.c_void_p)],
        "llmdiy_batch_fill_random": [P, I, I, U64],
        "llmdiy_batch_prefill": [P, I, IP, I],
        "llmdiy_batch_decode": [P, I, IP, IP, I, IP, P],
        "llmdiy_batch_copy_logits": [P, I, P],
        "llmdiy_batch_copy_kv": [P, I, I, I, I, P, P],
    }
    for name, args in bsig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    L.llmdiy_batch_destroy.argtypes = [P]
    L.llmdiy_batch_destroy.restype = None
    L.llmdiy_batch_last_error.argtypes = [P]
    L.llmdiy_batch_last_error.restype = ctypes.c_char_p
    L.llmdiy_fd_mh_work_bytes.argtypes = [I, I]
    L.llmdiy_fd_mh_work_bytes.restype = SZ
    _lib = L
    return L


def declared_symbols() -> list[str]:
    """Every function declared in include/*.h (for the export check)."""
    names = []
    for fn in sorted(os.listdir(INCLUDE_DIR)):
        if fn.endswith(".h"):
            text = open(os.path.join(INCLUDE_DIR, fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"\b(llmdiy_\w+)\s*\(", text)
    return sorted(set(names))


def _check(rc: int, what: str, engine=None):
    if rc != 0:
        msg = ""
        if engine is not None:
            m = lib().llmdiy_engine_last_error(engine)
            msg = m.decode() if m else ""
        raise LlmdiyError(f"{what} failed with status {rc} {msg}".strip())


# ----------------------------------------------------------------- kernels
def _p(x):
    return None if x is None else ctypes.c_void_p(int(x))


def rmsnorm(out, inp, weight, d, eps=1e-6, stream=None):
    _check(lib().llmdiy_rmsnorm(_p(out), _p(inp), _p(weight), d, eps, _p(stream)), "rmsnorm")


def add_bias(out, bias, size, stream=None):
    _check(lib().llmdiy_add_bias(_p(out), _p(bias), size, _p(stream)), "add_bias")


def swiglu(out, w1o, w2o, size, stream=None):
    _check(lib().llmdiy_swiglu(_p(out), _p(w1o), _p(w2o), size, _p(stream)), "swiglu")


def fused_qkv_rope_cache(qkv, kc, vc, pos, max_seqlen, num_heads, head_dim, stream=None):
    _check(lib().llmdiy_fused_qkv_rope_cache(_p(qkv), _p(kc), _p(vc), pos, max_seqlen, num_heads, head_dim,
                                             _p(stream)), "fused_qkv_rope_cache")


def fd_v5_fused(Q, K, V, O, L, stride, stream=None):
    _check(lib().llmdiy_fd_v5_fused(_p(Q), _p(K), _p(V), _p(O), L, stride, _p(stream)), "fd_v5_fused")


def fd_v5_split_stage1(Q, K, V, Opart, LSE, L, num_chunks, stride, stream=None):
    _check(lib().llmdiy_fd_v5_split_stage1(_p(Q), _p(K), _p(V), _p(Opart), _p(LSE), L, num_chunks, stride,
                                           _p(stream)), "fd_v5_split_stage1")


def fd_opt_stage2(Opart, LSE, O, num_chunks, stream=None):
    _check(lib().llmdiy_fd_opt_stage2(_p(Opart), _p(LSE), _p(O), num_chunks, _p(stream)), "fd_opt_stage2")


def gemm_tc(A, W, C, M, N, K, stream=None):
    """C[M,N] = A[M,K] @ W[N,K]^T on the tcgen05 tensor cores (fp16 in/out, fp32 accumulation)."""
    _check(lib().llmdiy_gemm_tc(_p(A), _p(W), _p(C), M, N, K, _p(stream)), "gemm_tc")


def gemm_tc_kn(A, B, C, M, N, K, stream=None):
    """C[M,N] = A[M,K] @ B[K,N] (B in the reference's [K,N] layout) on the tcgen05 tensor cores."""
    _check(lib().llmdiy_gemm_tc_kn(_p(A), _p(B), _p(C), M, N, K, _p(stream)), "gemm_tc_kn")


def gemm_tc_status():
    return lib().llmdiy_gemm_tc_status()


def fd_mh_work_bytes(L, num_heads):
    return int(lib().llmdiy_fd_mh_work_bytes(L, num_heads))


def fd_multihead(Q, K, V, O, L, stride, num_heads, work, work_bytes, stream=None):
    _check(lib().llmdiy_fd_multihead(_p(Q), _p(K), _p(V), _p(O), L, stride, num_heads, _p(work), work_bytes,
                                     _p(stream)), "fd_multihead")


def fd_mh_partials(Q, K, V, L, stride, num_heads, part, work, work_bytes, stream=None):
    _check(lib().llmdiy_fd_mh_partials(_p(Q), _p(K), _p(V), L, stride, num_heads, _p(part), _p(work), work_bytes,
                                       _p(stream)), "fd_mh_partials")


def fd_mh_merge(parts, G, num_heads, O, stream=None):
    _check(lib().llmdiy_fd_mh_merge(_p(parts), G, num_heads, _p(O), _p(stream)), "fd_mh_merge")


def fd_mh_status(work, L, num_heads):
    return lib().llmdiy_fd_mh_status(_p(work), L, num_heads)


def p2p_buffer_bytes(world, num_heads):
    return int(lib().llmdiy_p2p_buffer_bytes(world, num_heads))


def p2p_alloc(nbytes):
    """Device buffer for llmdiy_fd_p2p_merge: (pointer, 64-byte CUDA IPC handle)."""
    ptr = ctypes.c_void_p()
    h = (ctypes.c_uint8 * 64)()
    _check(lib().llmdiy_p2p_alloc(nbytes, ctypes.byref(ptr), h), "p2p_alloc")
    return ptr.value, bytes(h)


def p2p_open(handle: bytes):
    ptr = ctypes.c_void_p()
    buf = (ctypes.c_uint8 * 64).from_buffer_copy(handle)
    _check(lib().llmdiy_p2p_open(buf, ctypes.byref(ptr)), "p2p_open")
    return ptr.value


def p2p_close(ptr):
    _check(lib().llmdiy_p2p_close(_p(ptr)), "p2p_close")


def p2p_free(ptr):
    _check(lib().llmdiy_p2p_free(_p(ptr)), "p2p_free")


def fd_p2p_merge(part, peers, world, rank, num_heads, tag, O, err, stream=None):
    _check(lib().llmdiy_fd_p2p_merge(_p(part), _p(peers), world, rank, num_heads, tag, _p(O), _p(err), _p(stream)),
           "fd_p2p_merge")


def fd_mh_p2p(Q, K, V, L, stride, num_heads, work, work_bytes, peers, world, rank, tag, O, err, stream=None):
    """This rank's split partials over its L rows, then the peer exchange and merge (two launches)."""
    _check(lib().llmdiy_fd_mh_p2p(_p(Q), _p(K), _p(V), L, stride, num_heads, _p(work), work_bytes, _p(peers), world,
                                  rank, tag, _p(O), _p(err), _p(stream)), "fd_mh_p2p")


def argmax(out, logits, V, stream=None):
    _check(lib().llmdiy_argmax(_p(out), _p(logits), V, _p(stream)), "argmax")


def hgemv(A, B, C, N, K, stream=None):
    _check(lib().llmdiy_hgemv(_p(A), _p(B), _p(C), N, K, _p(stream)), "hgemv")


def hgemm_swizzle_nn(A, B, C, M, N, K, stream=None):
    _check(lib().llmdiy_hgemm_swizzle_nn(_p(A), _p(B), _p(C), M, N, K, _p(stream)), "hgemm_swizzle_nn")


def hgemm_swizzle_nn_path(A, B, C, M, N, K) -> int:
    """Which kernel hgemm_swizzle_nn runs for these arguments: 1 tcgen05, 0 CUDA cores, -1 invalid."""
    return int(lib().llmdiy_hgemm_swizzle_nn_path(_p(A), _p(B), _p(C), M, N, K))


def flash_attn_tuned_A(Q, K, V, O, N, QKV_head, stride_Q, stride_KV, K_ofs=-1, V_ofs=-1, Q_ofs=-1, O_ofs=-1,
                       stream=None):
    _check(lib().llmdiy_flash_attn_tuned_A(_p(Q), _p(K), _p(V), _p(O), N, QKV_head, stride_Q, stride_KV, K_ofs,
                                           V_ofs, Q_ofs, O_ofs, _p(stream)), "flash_attn_tuned_A")


def gather_q_from_qkv(qkv, buf, N, num_heads, head_dim=128, stream=None):
    _check(lib().llmdiy_gather_q_from_qkv(_p(qkv), _p(buf), N, num_heads, head_dim, _p(stream)), "gather_q")


def gather_kv_from_cache(cache, buf, N, num_heads, head_dim=128, stream=None):
    _check(lib().llmdiy_gather_kv_from_cache(_p(cache), _p(buf), N, num_heads, head_dim, _p(stream)), "gather_kv")


def scatter_interleaved(src, dst, N, num_heads, dst_cols, stream=None):
    _check(lib().llmdiy_scatter_interleaved(_p(src), _p(dst), N, num_heads, dst_cols, _p(stream)), "scatter")


def transpose_weight(out, inp, rows, cols, stream=None):
    _check(lib().llmdiy_transpose_weight(_p(out), _p(inp), rows, cols, _p(stream)), "transpose_weight")


# ----------------------------------------------------------------- QWDF files
def write_random_bin(path: str, cfg: Config, seed: int, std_dev: float = 0.02, nthreads: int = 8):
    _check(lib().llmdiy_qwdf_write_random(path.encode(), ctypes.byref(cfg), seed, std_dev, nthreads),
           "qwdf_write_random")


def read_bin_config(path: str) -> Config:
    c = Config()
    _check(lib().llmdiy_qwdf_read_config(path.encode(), ctypes.byref(c)), "qwdf_read_config")
    return c


def validate_bin(path: str) -> dict:
    """Check a .bin against the QWDF format (llmdiy_qwdf_validate): {"status": 0 | LLMDIY_ERR_*,
    "ok": bool, "config": dict or None, "nonfinite": int, "message": str}.  Never raises on a bad file."""
    c = Config()
    bad = ctypes.c_uint64(0)
    msg = ctypes.create_string_buffer(512)
    rc = lib().llmdiy_qwdf_validate(path.encode(), ctypes.byref(c), ctypes.byref(bad), msg, len(msg))
    has_header = rc in (ERR_FORMAT, ERR_UNSUPPORTED, 0) and c.vocab_size != 0
    return {"status": rc, "ok": rc == 0, "config": c.as_dict() if has_header else None,
            "nonfinite": int(bad.value), "message": msg.value.decode()}


def fill_tensor(cfg: Config, tensor_id: int, seed: int, first: int, n: int, std_dev: float = 0.02, nthreads=8):
    import numpy as np
    out = np.empty(n, dtype=np.uint16)
    _check(lib().llmdiy_qwdf_fill_tensor(ctypes.byref(cfg), tensor_id, seed, std_dev, first, n,
                                         out.ctypes.data_as(ctypes.c_void_p), nthreads), "qwdf_fill_tensor")
    return out


# ----------------------------------------------------------------- engine
def _ints(seq):
    arr = (ctypes.c_int * max(1, len(seq)))(*seq)
    return arr


class Engine:
    """QwenEngine on one B200 (framework_src/qwen_infer.cu:69-738)."""

    def __init__(self, bin_path: str | None = None, device: int = 0, *, config: Config | None = None,
                 seed: int = 0, std_dev: float = 0.02):
        self._h = ctypes.c_void_p()
        L = lib()
        if bin_path is not None:
            rc = L.llmdiy_engine_create(bin_path.encode(), device, ctypes.byref(self._h))
        else:
            if config is None:
                raise ValueError("either bin_path or config is required")
            rc = L.llmdiy_engine_create_random(ctypes.byref(config), seed, std_dev, device, ctypes.byref(self._h))
        if rc != 0:
            raise LlmdiyError(f"engine create failed with status {rc}")
        c = Config()
        L.llmdiy_engine_get_config(self._h, ctypes.byref(c))
        self.config = c

    def close(self):
        if self._h:
            lib().llmdiy_engine_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _chk(self, rc, what):
        _check(rc, what, self._h)

    def reset(self):
        self._chk(lib().llmdiy_engine_reset(self._h), "reset")

    def prefill(self, tokens):
        self._chk(lib().llmdiy_engine_prefill(self._h, _ints(tokens), len(tokens)), "prefill")

    def step(self, token: int, pos: int) -> int:
        nxt = ctypes.c_int()
        self._chk(lib().llmdiy_engine_step(self._h, token, pos, ctypes.byref(nxt)), "step")
        return nxt.value

    def generate(self, prompt, max_new: int, stop_on_eos: bool = True) -> list[int]:
        out = (ctypes.c_int * max(1, max_new))()
        n = ctypes.c_int()
        self._chk(lib().llmdiy_engine_generate(self._h, _ints(prompt), len(prompt), max_new, int(stop_on_eos), out,
                                               ctypes.byref(n)), "generate")
        return list(out[: n.value])

    def decode_async(self, first_token: int, pos: int, n_steps: int, stop_on_eos=False, stream=None):
        self._chk(lib().llmdiy_engine_decode_async(self._h, first_token, pos, n_steps, int(stop_on_eos), _p(stream)),
                  "decode_async")

    def status(self) -> int:
        n = ctypes.c_int()
        self._chk(lib().llmdiy_engine_status(self._h, ctypes.byref(n)), "status")
        return n.value

    def tokens(self, n: int) -> list[int]:
        out = (ctypes.c_int * max(1, n))()
        self._chk(lib().llmdiy_engine_copy_tokens(self._h, out, n), "copy_tokens")
        return list(out[:n])

    def logits(self):
        import numpy as np
        out = np.empty(self.config.vocab_size, dtype=np.uint16)
        self._chk(lib().llmdiy_engine_copy_logits(self._h, out.ctypes.data_as(ctypes.c_void_p)), "copy_logits")
        return out.view(np.float16)

    def hidden(self):
        import numpy as np
        out = np.empty(self.config.hidden_size, dtype=np.uint16)
        self._chk(lib().llmdiy_engine_copy_hidden(self._h, out.ctypes.data_as(ctypes.c_void_p)), "copy_hidden")
        return out.view(np.float16)

    def kv(self, layer: int, pos0: int, n: int):
        import numpy as np
        H = self.config.hidden_size
        k = np.empty((n, H), dtype=np.uint16)
        v = np.empty((n, H), dtype=np.uint16)
        self._chk(lib().llmdiy_engine_copy_kv(self._h, layer, pos0, n, k.ctypes.data_as(ctypes.c_void_p),
                                              v.ctypes.data_as(ctypes.c_void_p)), "copy_kv")
        return k.view(np.float16), v.view(np.float16)

    def profile(self, first_token: int, pos: int, n_steps: int, cap: int = 4096):
        """Timing probes of one decode launch (development aid): (probe times [cta, cap, 2] in
        %globaltimer ns -- per CTA and phase boundary, warp 0's and the last warp's arrival -- and
        per-chunk accounting [cta, 6 phases, 8 warps, 4] in SM cycles: chunk wait, compute, refill
        issue, longest single wait)."""
        import numpy as np
        G = self.num_sms
        out = np.zeros((G, cap, 2), dtype=np.uint64)
        prod = np.zeros((G, 6, 8, 4), dtype=np.uint64)
        self._chk(lib().llmdiy_engine_profile(self._h, first_token, pos, n_steps, cap,
                                              out.ctypes.data_as(ctypes.c_void_p),
                                              prod.ctypes.data_as(ctypes.c_void_p)), "profile")
        return out, prod

    @property
    def num_sms(self) -> int:
        return lib().llmdiy_engine_num_sms(self._h)


class Batch:
    """Batched greedy decode of independent sequences on an Engine's weights (include/llmdiy_batch.h)."""

    def __init__(self, engine: "Engine", max_batch: int, max_len: int):
        self.engine = engine  # keeps the weights alive
        self._h = ctypes.c_void_p()
        self.max_batch, self.max_len = max_batch, max_len
        rc = lib().llmdiy_batch_create(engine._h, max_batch, max_len, ctypes.byref(self._h))
        if rc:
            raise LlmdiyError(f"batch create failed with status {rc}")

    def _chk(self, rc, what):
        if rc:
            m = lib().llmdiy_batch_last_error(self._h)
            raise LlmdiyError(f"{what} failed with status {rc} {m.decode() if m else ''}".strip())

    def close(self):
        if self._h:
            lib().llmdiy_batch_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def fill_random(self, seq: int, length: int, seed: int):
        self._chk(lib().llmdiy_batch_fill_random(self._h, seq, length, seed), "batch fill_random")

    def prefill(self, seq: int, tokens):
        self._chk(lib().llmdiy_batch_prefill(self._h, seq, _ints(tokens), len(tokens)), "batch prefill")

    def decode(self, tokens, pos, n_steps: int, stream=None):
        """n_steps greedy steps of len(tokens) sequences; returns an int array [n_steps][B]."""
        import numpy as np
        B = len(tokens)
        out = (ctypes.c_int * max(1, n_steps * B))()
        self._chk(lib().llmdiy_batch_decode(self._h, B, _ints(tokens), _ints(pos), n_steps, out, _p(stream)),
                  "batch decode")
        return np.frombuffer(out, dtype=np.int32)[: n_steps * B].reshape(n_steps, B).copy()

    def logits(self, seq: int):
        import numpy as np
        V = self.engine.config.vocab_size
        out = np.zeros(V, dtype=np.uint16)
        self._chk(lib().llmdiy_batch_copy_logits(self._h, seq, out.ctypes.data_as(ctypes.c_void_p)), "batch logits")
        return out.view(np.float16)

    def kv(self, seq: int, layer: int, pos0: int, n: int):
        import numpy as np
        H = self.engine.config.hidden_size
        k = np.zeros(n * H, dtype=np.uint16)
        v = np.zeros(n * H, dtype=np.uint16)
        self._chk(lib().llmdiy_batch_copy_kv(self._h, seq, layer, pos0, n, k.ctypes.data_as(ctypes.c_void_p),
                                             v.ctypes.data_as(ctypes.c_void_p)), "batch kv")
        return k.view(np.float16).reshape(n, H), v.view(np.float16).reshape(n, H)


def _main(argv=None) -> int:
    """QWDF file tooling: `validate FILE` checks a .bin (exit 0 when the engine can run it);
    `write-random FILE [--layers N] [--vocab V] [--intermediate I] [--max-seqlen S] [--seed K]` writes
    seeded random weights (N(0, 0.02), RMSNorm weights 1) in the same format."""
    import argparse
    import json
    ap = argparse.ArgumentParser(prog="llmdiy_b200", description=_main.__doc__)
    sub = ap.add_subparsers(dest="cmd", required=True)
    v = sub.add_parser("validate")
    v.add_argument("file")
    w = sub.add_parser("write-random")
    w.add_argument("file")
    w.add_argument("--layers", type=int, default=QWEN_1_8B["num_layers"])
    w.add_argument("--vocab", type=int, default=QWEN_1_8B["vocab_size"])
    w.add_argument("--intermediate", type=int, default=QWEN_1_8B["intermediate_size"])
    w.add_argument("--max-seqlen", type=int, default=2048)
    w.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    if a.cmd == "validate":
        r = validate_bin(a.file)
        print(json.dumps(r))
        return 0 if r["ok"] else 1
    cfg = make_config(vocab_size=a.vocab, num_layers=a.layers, intermediate_size=a.intermediate,
                      max_seqlen=a.max_seqlen)
    write_random_bin(a.file, cfg, seed=a.seed, nthreads=os.cpu_count() or 8)
    print(json.dumps({"written": a.file, "config": cfg.as_dict()}))
    return 0


if __name__ == "__main__":
    raise SystemExit(_main())
