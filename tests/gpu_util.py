"""Helpers for the GPU tests: torch supplies device memory only; every
computation under test runs through the C ABI of libllmdiy_b200.so."""
import os

import numpy as np

import llmdiy_b200 as L

ORACLE_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle")


def torch():
    import torch as t
    return t


def dev(a, dtype=None):
    t = torch()
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return t.from_numpy(a.view(np.int16).copy()).cuda().view(t.float16)
    return t.from_numpy(a.copy()).cuda()


def host(t_):
    t = torch()
    t.cuda.synchronize()
    if t_.dtype == t.float16:
        return t_.view(t.int16).cpu().numpy().view(np.float16)
    return t_.cpu().numpy()


def zeros16(n):
    t = torch()
    return t.zeros(n, dtype=t.float16, device="cuda")


def ref_kernels():
    """The reference's own kernels (oracle/_ref, compute_89 PTX JIT) or None when not built."""
    try:
        import oracle as orc
        return orc.RefKernels()
    except (FileNotFoundError, OSError):
        return None


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(a) else 0.0


def f16_ulp(x):
    x = np.abs(np.asarray(x, np.float32))
    e = np.floor(np.log2(np.maximum(x, 2.0 ** -14)))
    return 2.0 ** (e - 10)
