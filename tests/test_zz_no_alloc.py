"""The allocation-free split-KV flash-decoding entry point
(llmdiy_fd_split_noalloc) against the two-launch pair it stands in for
(llmdiy_fd_v5_split_stage1 + llmdiy_fd_opt_stage2), through the C ABI, on two
calls in a row that share its scratch array.  Collected last on purpose: it
must pass both alone in a fresh process and after every other test."""
import ctypes

import numpy as np
import pytest

import llmdiy_b200 as L

MAX_ROWS = 32768  # scratch limit stated in include/llmdiy_kernels.h


def _noalloc():
    f = L.lib().llmdiy_fd_split_noalloc
    f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def _pair(q, K, V, L_, stride):
    import torch
    nc = (L_ + 255) // 256
    Op = torch.empty(nc * 128, dtype=torch.float16, device="cuda")
    lse = torch.empty(nc, dtype=torch.float32, device="cuda")
    O = torch.empty(128, dtype=torch.float16, device="cuda")
    L.fd_v5_split_stage1(q.data_ptr(), K.data_ptr(), V.data_ptr(), Op.data_ptr(), lse.data_ptr(), L_, nc, stride)
    L.fd_opt_stage2(Op.data_ptr(), lse.data_ptr(), O.data_ptr(), nc)
    return O


@pytest.mark.gpu
def test_fd_split_noalloc_matches_pair_twice():
    import torch
    fn = _noalloc()
    rng = np.random.default_rng(20261201)
    # (rows, row stride in halves), all through the same scratch array back to back on one stream:
    # a long cache, a short ragged one, one chunk (the only CTA also merges), an exact multiple of
    # the 256-row chunk, and the stated maximum (every scratch slot and the full merge loop)
    cases = [(9000, 2048), (333, 128), (200, 2048), (512, 128), (MAX_ROWS, 128)]
    outs = []
    for L_, stride in cases:
        q = torch.from_numpy(rng.standard_normal(128).astype(np.float16)).cuda()
        K = torch.from_numpy(rng.standard_normal(L_ * stride).astype(np.float16)).cuda()
        V = torch.from_numpy(rng.standard_normal(L_ * stride).astype(np.float16)).cuda()
        O = torch.full((128,), float("nan"), dtype=torch.float16, device="cuda")
        rc = fn(q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), L_, stride, None)
        assert rc == 0, rc
        outs.append((O, _pair(q, K, V, L_, stride)))
    torch.cuda.synchronize()
    for got, want in outs:
        g = got.view(torch.int16).cpu().numpy()
        w = want.view(torch.int16).cpu().numpy()
        assert np.array_equal(g, w)
    # beyond the scratch maximum: rejected before any launch
    dummy = torch.zeros(128, dtype=torch.float16, device="cuda")
    p = dummy.data_ptr()
    assert fn(p, p, p, p, MAX_ROWS + 1, 128, None) == -1
