"""The multi-GPU split-KV decode path's host logic (llmdiy_dist) on world-size-2
gloo ranks on the CPU: contiguous sharding of the cache positions, the rank-order
all-gather of per-head partials, and the log-sum-exp merge.  The GPU kernels are
replaced by the CPU oracle's partial (orc_fd_partial_mlo) and a numpy merge of
the same contracts; the result must equal the oracle's attention over the whole
cache within 1e-3 (the attention tolerance)."""
import os
import socket
import sys
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _np_merge(parts):
    """[G][H][130] -> [H][128]: O = sum_j e^{m_j-M} o_j / sum_j e^{m_j-M} l_j (rank order)."""
    m = parts[:, :, 128]
    M = m.max(axis=0)
    w = np.where(np.isneginf(m), 0.0, np.exp(m - M[None, :]))
    num = (w[:, :, None] * parts[:, :, :128]).sum(axis=0)
    den = (w * parts[:, :, 129]).sum(axis=0)
    return num / den[:, None]


def _worker(rank, world, port, L_total, H, stride, seed, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "llm-inference-diy_b200"))
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
    import llmdiy_dist as D
    import oracle as orc
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rng = np.random.default_rng(seed)
        q = rng.standard_normal(H * 128).astype(np.float16)
        K = rng.standard_normal(L_total * stride).astype(np.float16)
        V = rng.standard_normal(L_total * stride).astype(np.float16)
        o = orc.Oracle()

        def partials(qt, Kt, Vt, rows, part):
            qn, Kn, Vn = qt.numpy(), Kt.numpy(), Vt.numpy()
            for h in range(H):
                if rows == 0:
                    part[h].zero_()
                    part[h, 128] = float("-inf")
                    continue
                m, l, ov = o.fd_partial_mlo(qn[h * 128:(h + 1) * 128], Kn[h * 128:], Vn[h * 128:], rows, stride)
                part[h, :128] = torch.from_numpy(ov)
                part[h, 128] = m
                part[h, 129] = l

        def merge(parts, out):
            out.copy_(torch.from_numpy(_np_merge(parts.numpy()).reshape(-1).astype(np.float16)))

        att = D.SplitKVAttention(dist.group.WORLD, H, stride, partials=partials, merge=merge)
        r0, r1 = att.rows(L_total)
        Ks = torch.from_numpy(K[r0 * stride:r1 * stride].copy())
        Vs = torch.from_numpy(V[r0 * stride:r1 * stride].copy())
        out = torch.empty(H * 128, dtype=torch.float16)
        att(torch.from_numpy(q), Ks, Vs, L_total, out)
        err = 0.0
        for h in range(H):
            exp = o.attention_q1(q[h * 128:(h + 1) * 128], K[h * 128:], V[h * 128:], L_total, stride)
            err = max(err, float(np.max(np.abs(out.numpy()[h * 128:(h + 1) * 128].astype(np.float64) -
                                               exp.astype(np.float64)))))
        with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{r0} {r1} {err}\n{out.numpy().view(np.uint16).tobytes().hex()}\n")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("L_total", [1000, 1001, 1])
def test_split_kv_two_gloo_ranks(L_total):
    world, H, stride = 2, 4, 512
    outdir = tempfile.mkdtemp()
    mp.spawn(_worker, args=(world, _free_port(), L_total, H, stride, 11, outdir), nprocs=world, join=True)
    lines = [open(os.path.join(outdir, f"rank{r}.txt")).read().split("\n") for r in range(world)]
    ranges = [tuple(int(x) for x in ln[0].split()[:2]) for ln in lines]
    assert ranges[0][0] == 0 and ranges[-1][1] == L_total
    assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
    for ln in lines:
        assert float(ln[0].split()[2]) < 1e-3
    assert lines[0][1] == lines[1][1]  # every rank holds the same merged output


def test_shard_range():
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "llm-inference-diy_b200"))
    import llmdiy_dist as D
    for L_total in (0, 1, 7, 131072):
        for world in (1, 2, 3, 8):
            rs = [D.shard_range(L_total, world, r) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == L_total
            assert all(rs[i][1] == rs[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in rs) - min(b - a for a, b in rs) <= 1
    with pytest.raises(ValueError):
        D.shard_range(10, 2, 2)
