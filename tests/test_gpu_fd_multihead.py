"""Multi-head split-KV flash decoding (llmdiy_fd_multihead / _partials / _merge)
against the CPU oracle per head (orc_attention_q1, orc_fd_partial_mlo) and,
where oracle/_ref is built, against the reference's own per-head split kernels
(fd_v5_split_stage1 + fd_opt_stage2) run on the same inputs.

Inputs follow BASELINE configs 1 and 5: q, K, V ~ N(0, 1) fp16 in the engine
cache layout (row r of head h at r*stride + h*128).  Tolerance: 1e-3 abs on
the fp16 outputs (north_star attention tolerance)."""
import numpy as np
import pytest

import llmdiy_b200 as L
import refmath
from gpu_util import dev, host, max_abs, ref_kernels, torch, zeros16

pytestmark = pytest.mark.gpu


def _inputs(rng, L_, H, stride):
    q = refmath.h(rng.standard_normal(H * 128))
    K = refmath.h(rng.standard_normal(L_ * stride))
    V = refmath.h(rng.standard_normal(L_ * stride))
    return q, K, V


def _work(L_, H):
    t = torch()
    n = L.fd_mh_work_bytes(L_, H)
    assert n > 0
    return t.zeros((n + 3) // 4, dtype=t.float32, device="cuda"), n


def _multihead(q, K, V, L_, H, stride):
    dq, dK, dV, O = dev(q), dev(K), dev(V), zeros16(H * 128)
    w, n = _work(L_, H)
    L.fd_multihead(dq.data_ptr(), dK.data_ptr(), dV.data_ptr(), O.data_ptr(), L_, stride, H, w.data_ptr(), n)
    got = host(O).reshape(H, 128)
    assert L.fd_mh_status(w.data_ptr(), L_, H) == 0
    return got, (dq, dK, dV)


@pytest.mark.parametrize("L_,H,stride", [(1024, 16, 2048), (1, 16, 2048), (63, 16, 2048), (65, 4, 512),
                                         (1000, 16, 2048), (520, 16, 2048), (2048, 16, 2048), (2049, 8, 1024),
                                         (4097, 2, 256), (32768, 16, 2048)])
def test_fd_multihead_vs_oracle(oracle, rng, L_, H, stride):
    """L <= 2048: the one-launch cluster kernel (L = 520 leaves three CTAs of each cluster without rows,
    2048 fills all four tiles of every CTA); longer caches: the persistent split kernel + merge."""
    q, K, V = _inputs(rng, L_, H, stride)
    got, _ = _multihead(q, K, V, L_, H, stride)
    for h in range(H):
        exp = oracle.attention_q1(q[h * 128:(h + 1) * 128], K[h * 128:], V[h * 128:], L_, stride)
        assert max_abs(got[h], exp) < 1e-3, h


def test_fd_multihead_workspace_reused_across_lengths(oracle, rng):
    """One workspace sized for the longest cache serves shorter ones: the split kernel's partials of a
    40000-row call occupy the place where a shorter cache's split count would otherwise have put its
    error word, and every call still reads back a clean status and the oracle's attention."""
    t = torch()
    H, stride = 16, 2048
    w, nb = _work(40000, H)
    for n in (40000, 5000, 3000, 40000):
        q, K, V = _inputs(rng, n, H, stride)
        dq, dK, dV, O = dev(q), dev(K), dev(V), zeros16(H * 128)
        L.fd_multihead(dq.data_ptr(), dK.data_ptr(), dV.data_ptr(), O.data_ptr(), n, stride, H, w.data_ptr(), nb)
        t.cuda.synchronize()
        assert L.fd_mh_status(w.data_ptr(), n, H) == 0, n
        got = host(O).reshape(H, 128)
        for h in (0, H - 1):
            exp = oracle.attention_q1(q[h * 128:(h + 1) * 128], K[h * 128:], V[h * 128:], n, stride)
            assert max_abs(got[h], exp) < 1e-3, (n, h)


def test_fd_multihead_vs_reference_split(oracle, rng):
    """Config 1 against the reference's split kernels run head by head."""
    ref = ref_kernels()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    t = torch()
    L_, H, stride = 1024, 16, 2048
    q, K, V = _inputs(rng, L_, H, stride)
    got, (dq, dK, dV) = _multihead(q, K, V, L_, H, stride)
    nc = (L_ + 255) // 256
    for h in range(H):
        Op = zeros16(nc * 128)
        lse = t.zeros(nc, dtype=t.float32, device="cuda")
        r = zeros16(128)
        off = h * 128 * 2  # bytes
        ref.fd_v5_split_stage1(dq.data_ptr() + off, dK.data_ptr() + off, dV.data_ptr() + off, Op.data_ptr(),
                               lse.data_ptr(), L_, nc, stride)
        ref.fd_opt_stage2(Op.data_ptr(), lse.data_ptr(), r.data_ptr(), nc)
        assert max_abs(got[h], host(r)) < 1e-3, h


@pytest.mark.parametrize("shards", [[5000], [1234, 2000, 1766], [1, 4095], [777, 777, 777, 777]])
def test_fd_shard_partials_merge(oracle, rng, shards):
    """Config 5's data path on one GPU: contiguous KV shards -> one partial per head each
    -> log-sum-exp merge in shard order == attention over the whole cache."""
    t = torch()
    H, stride = 16, 2048
    Lt = sum(shards)
    q, K, V = _inputs(rng, Lt, H, stride)
    dq, dK, dV = dev(q), dev(K), dev(V)
    parts = t.zeros((len(shards), H, 130), dtype=t.float32, device="cuda")
    r0 = 0
    for g, n in enumerate(shards):
        w, nb = _work(n, H)
        off = r0 * stride * 2
        L.fd_mh_partials(dq.data_ptr(), dK.data_ptr() + off, dV.data_ptr() + off, n, stride, H,
                         parts[g].data_ptr(), w.data_ptr(), nb)
        r0 += n
    O = zeros16(H * 128)
    L.fd_mh_merge(parts.data_ptr(), len(shards), H, O.data_ptr())
    got = host(O).reshape(H, 128)
    hp = host(parts)
    r0 = 0
    for g, n in enumerate(shards):
        for h in (0, H - 1):
            m, l, o = oracle.fd_partial_mlo(q[h * 128:(h + 1) * 128], K[r0 * stride + h * 128:],
                                            V[r0 * stride + h * 128:], n, stride)
            assert abs(hp[g, h, 128] - m) < 1e-4 * max(1.0, abs(m))
            assert abs(hp[g, h, 129] - l) < 1e-4 * max(1.0, abs(l))
            assert max_abs(hp[g, h, :128] / hp[g, h, 129], o / l) < 1e-4
        r0 += n
    for h in range(H):
        exp = oracle.attention_q1(q[h * 128:(h + 1) * 128], K[h * 128:], V[h * 128:], Lt, stride)
        assert max_abs(got[h], exp) < 1e-3, h


def test_fd_multihead_rejects_bad_arguments(rng):
    t = torch()
    x = t.zeros(4096, dtype=t.float16, device="cuda")
    w = t.zeros(1 << 16, dtype=t.float32, device="cuda")
    p = x.data_ptr()
    with pytest.raises(L.LlmdiyError):
        L.fd_multihead(p, p, p, p, 16, 1000, 16, w.data_ptr(), 1 << 18)  # stride < heads * 128
    with pytest.raises(L.LlmdiyError):
        L.fd_multihead(p + 2, p, p, p, 16, 2048, 16, w.data_ptr(), 1 << 18)  # misaligned q
    with pytest.raises(L.LlmdiyError):
        L.fd_multihead(p, p, p, p, 16, 2048, 16, w.data_ptr(), 4)  # workspace too small


def test_fd_p2p_exchange_single_rank(oracle, rng):
    """The peer-memory exchange kernel (llmdiy_fd_p2p_merge) with one rank on one GPU: the partial
    goes through the rank's own IPC-exported buffer as tagged 8-byte words, and the merge equals the
    attention over the shard; later calls (new tags) reuse the buffer.  The multi-rank run is the
    2-GPU `bench.py --workload fd-op`, which checks it against the NCCL all-gather path."""
    import llmdiy_dist as D
    t = torch()
    H, stride, n = 16, 2048, 3000
    ex = D.P2PExchange(None, H, t.device("cuda"))

    class _View:  # the exchange's own receive buffer as an int64 tensor of its words (no copy)
        def __init__(self, ptr, n):
            self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i8", "data": (ptr, False), "version": 2}

    region = H * 130  # words per region: [1][H][130], value in the low half, tag in the high half
    words = t.as_tensor(_View(ex.own, 2 * region), device="cuda")

    def region_values(r):  # (values [H][130] as float32, tags [H][130])
        w = words[r * region:(r + 1) * region]
        return ((w & 0xFFFFFFFF).to(t.int32).view(t.float32).view(H, 130), (w >> 32).view(H, 130))
    parts = []
    try:
        for call in range(3):
            q, K, V = _inputs(rng, n, H, stride)
            dq, dK, dV = dev(q), dev(K), dev(V)
            part = t.zeros((H, 130), dtype=t.float32, device="cuda")
            w, nb = _work(n, H)
            L.fd_mh_partials(dq.data_ptr(), dK.data_ptr(), dV.data_ptr(), n, stride, H, part.data_ptr(),
                             w.data_ptr(), nb)
            O = zeros16(H * 128)
            ex(part, O, None)
            t.cuda.synchronize()
            assert ex.status() == 0 and ex.tag == call + 1
            got = host(O).reshape(H, 128)
            for h in (0, 7, H - 1):
                exp = oracle.attention_q1(q[h * 128:(h + 1) * 128], K[h * 128:], V[h * 128:], n, stride)
                assert max_abs(got[h], exp) < 1e-3, (call, h)
            # call `tag` writes region (tag & 1); the other region keeps the previous call's partial
            parts.append(part.clone())
            vals, tags = region_values((call + 1) & 1)
            assert t.equal(vals, part) and bool((tags == call + 1).all())
            if call:
                vals, tags = region_values(call & 1)
                assert t.equal(vals, parts[call - 1]) and bool((tags == call).all())
    finally:
        ex.close()


def test_fd_p2p_wait_expires_without_a_peer():
    """Failure detection without a GPU fault: a rank of a two-rank exchange whose peer never runs.
    The partner's buffer is a second local buffer, and nothing writes rank 1's tagged words into this
    rank's buffer, so the kernel's bounded wait for them runs out; the kernel reports it in the error
    word and returns, and the context stays usable for a normal call afterwards."""
    import time
    t = torch()
    H = 16
    nb = L.p2p_buffer_bytes(2, H)
    own, _ = L.p2p_alloc(nb)
    other, _ = L.p2p_alloc(nb)
    try:
        peers = t.tensor([own, other], dtype=t.int64, device="cuda")
        part = t.zeros((H, 130), dtype=t.float32, device="cuda")
        part[:, 129] = 1.0
        O = zeros16(H * 128)
        err = t.zeros(1, dtype=t.int32, device="cuda")
        t0 = time.time()
        L.fd_p2p_merge(part.data_ptr(), peers.data_ptr(), 2, 0, H, 1, O.data_ptr(), err.data_ptr())
        t.cuda.synchronize()
        assert int(err.item()) == 1
        assert time.time() - t0 < 60
        # the same buffer as a one-rank exchange afterwards: completes normally
        err.zero_()
        one = t.tensor([own], dtype=t.int64, device="cuda")
        L.fd_p2p_merge(part.data_ptr(), one.data_ptr(), 1, 0, H, 2, O.data_ptr(), err.data_ptr())
        t.cuda.synchronize()
        assert int(err.item()) == 0
    finally:
        L.p2p_free(own)
        L.p2p_free(other)


def test_fd_mh_p2p_single_rank(oracle, rng):
    """The one-call shard path (llmdiy_fd_mh_p2p through SplitKVAttention with the peer exchange):
    the split kernel, then the exchange kernel merging each head's splits itself, one rank on one GPU,
    against the oracle; two calls in a row (both buffer regions)."""
    import llmdiy_dist as D
    t = torch()
    H, stride, n = 16, 2048, 5000
    att = D.SplitKVAttention(None, H, stride, exchange="p2p")
    try:
        for call in range(2):
            q, K, V = _inputs(rng, n, H, stride)
            dq, dK, dV = dev(q), dev(K), dev(V)
            O = zeros16(H * 128)
            att(dq, dK, dV, n, O)
            t.cuda.synchronize()
            assert att._p2p.status() == 0
            assert L.fd_mh_status(att._work.data_ptr(), n, H) == 0
            got = host(O).reshape(H, 128)
            for h in (0, 5, H - 1):
                exp = oracle.attention_q1(q[h * 128:(h + 1) * 128], K[h * 128:], V[h * 128:], n, stride)
                assert max_abs(got[h], exp) < 1e-3, (call, h)
    finally:
        att.close()
