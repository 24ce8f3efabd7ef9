"""The tcgen05 tensor-core GEMM (llmdiy_gemm_tc: C = A W^T, fp16 operands, fp32
accumulation) against a float64 numpy product of the same fp16 inputs.  The
bound is the fp16 rounding of the output plus fp32 accumulation error:
|C - C64| <= 2^-10 |C64| + 1e-3 (values scaled to O(1))."""
import numpy as np
import pytest

import llmdiy_b200 as L
from gpu_util import dev, host, zeros16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 384, 2048), (200, 136, 5504), (1, 128, 64),
                                   (127, 6144, 2048), (2048, 2048, 2048), (333, 11008, 2048), (2048, 2048, 5504),
                                   (2048, 6144, 2048), (1000, 4736, 320)])
def test_gemm_tc(rng, M, N, K):
    """M > 128 with at least as many 256 x 256 tiles as SM pairs takes the persistent 2-CTA kernel
    (several tiles per pair, ragged M and N edges, K shorter than its pipeline); the rest the
    single-SM kernel."""
    A = (rng.standard_normal((M, K)) * 0.5).astype(np.float16)
    W = (rng.standard_normal((N, K)) * (1.0 / np.sqrt(K))).astype(np.float16)
    dA, dW, C = dev(A), dev(W), zeros16(M * N)  # keep the inputs alive during the call
    L.gemm_tc(dA.data_ptr(), dW.data_ptr(), C.data_ptr(), M, N, K)
    got = host(C).reshape(M, N).astype(np.float64)
    assert L.gemm_tc_status() == 0
    exp = A.astype(np.float64) @ W.astype(np.float64).T
    err = np.abs(got - exp) - (np.abs(exp) * 2.0 ** -10 + 1e-3)
    assert err.max() <= 0, (float(err.max()), np.unravel_index(err.argmax(), err.shape))


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (200, 384, 2048), (127, 5504, 2048), (64, 2048, 5504)])
def test_gemm_tc_kn(rng, M, N, K):
    """B in the reference's [K,N] layout (MN-major tcgen05 operand)."""
    A = (rng.standard_normal((M, K)) * 0.5).astype(np.float16)
    B = (rng.standard_normal((K, N)) * (1.0 / np.sqrt(K))).astype(np.float16)
    dA, dB, C = dev(A), dev(B), zeros16(M * N)
    L.gemm_tc_kn(dA.data_ptr(), dB.data_ptr(), C.data_ptr(), M, N, K)
    got = host(C).reshape(M, N).astype(np.float64)
    assert L.gemm_tc_status() == 0
    exp = A.astype(np.float64) @ B.astype(np.float64)
    err = np.abs(got - exp) - (np.abs(exp) * 2.0 ** -10 + 1e-3)
    assert err.max() <= 0, (float(err.max()), np.unravel_index(err.argmax(), err.shape))


def test_gemm_tc_rejects_bad_arguments():
    import torch
    x = torch.zeros(4096, dtype=torch.float16, device="cuda")
    p = x.data_ptr()
    with pytest.raises(L.LlmdiyError):
        L.gemm_tc(p + 2, p, p, 8, 8, 64)  # misaligned A
    with pytest.raises(L.LlmdiyError):
        L.gemm_tc(p, p, p, 8, 8, 12)  # K not a multiple of 8
    with pytest.raises(L.LlmdiyError):
        L.gemm_tc(p, p, p, 0, 8, 64)
