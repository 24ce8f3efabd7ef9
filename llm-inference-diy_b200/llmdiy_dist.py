"""Multi-GPU split-KV decode attention (one query token over a very long KV cache).

The cache's positions are sharded contiguously over the ranks of a process group
(one process per GPU).  Each rank computes one partial per head over its shard
-- o[128] unnormalised, m (max score), l (sum of e^{s - m}) as 130 fp32 --
with llmdiy_fd_mh_partials; then either the partials are all-gathered (NCCL over
NVLink) and every rank merges them in rank order with llmdiy_fd_mh_merge, or one
kernel per rank stores its partial straight into every rank's buffer over peer
memory as tagged words and merges once every rank's words carry the call's tag
(P2PExchange, llmdiy_fd_p2p_merge).  This is the
only exchange on the path: 130 x num_heads fp32 per rank.

The reference has no multi-GPU path; its single-GPU counterpart is the per-head
split-KV pair fd_v5_split_stage1 + fd_opt_stage2
(kernels/flash_decode_q1_opt.cuh:548-724), whose log-sum-exp merge this
generalises from chunks within one GPU to shards across GPUs.
"""
from __future__ import annotations

PART = 130  # o[128], m, l


def shard_range(L: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of an L-row cache held by `rank` (contiguous, sizes differ by at most one)."""
    if L < 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError("bad shard request")
    return L * rank // world, L * (rank + 1) // world


def gather_partials(group, part, world: int, out=None):
    """All-gather this rank's [num_heads, 130] partial into [world, num_heads, 130] in rank order."""
    import torch
    import torch.distributed as dist
    if out is None:
        out = torch.empty((world,) + tuple(part.shape), dtype=part.dtype, device=part.device)
    if world == 1:
        out[0].copy_(part)
        return out
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, part.contiguous(), group=group)
    else:
        bufs = list(out.unbind(0))
        dist.all_gather(bufs, part.contiguous(), group=group)
    return out


class P2PExchange:
    """The partials exchange over peer memory (llmdiy_fd_p2p_merge): every rank allocates a receive
    buffer, the ranks swap its CUDA IPC handle through the process group once, and each call is one
    kernel per rank that stores the rank's partial into every buffer as 8-byte words carrying the
    call's tag and merges when every rank's words in its own buffer carry it.  Up to 16 ranks.
    Collective: every rank constructs it and calls it in the same order."""

    def __init__(self, group, num_heads: int, device):
        import torch
        import torch.distributed as dist
        import llmdiy_b200 as L
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        self.num_heads = num_heads
        self.own, handle = L.p2p_alloc(L.p2p_buffer_bytes(self.world, num_heads))
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=group)
        else:
            handles = [handle]
        self.opened = []
        ptrs = []
        for r in range(self.world):
            if r == self.rank:
                ptrs.append(self.own)
            else:
                p = L.p2p_open(handles[r])
                self.opened.append(p)
                ptrs.append(p)
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.tag = 0

    def __call__(self, part, out, stream):
        import llmdiy_b200 as L
        self.tag += 1
        L.fd_p2p_merge(part.data_ptr(), self.peers.data_ptr(), self.world, self.rank, self.num_heads, self.tag,
                       out.data_ptr(), self.err.data_ptr(), stream=stream)

    def shard(self, q, K, V, rows, stride, work, out, stream):
        """This rank's split partials over its `rows` cached rows and the exchange, in two launches
        (llmdiy_fd_mh_p2p: the exchange kernel merges the head's split partials itself)."""
        import llmdiy_b200 as L
        self.tag += 1
        L.fd_mh_p2p(q.data_ptr(), K.data_ptr(), V.data_ptr(), rows, stride, self.num_heads, work.data_ptr(),
                    work.numel() * 4, self.peers.data_ptr(), self.world, self.rank, self.tag, out.data_ptr(),
                    self.err.data_ptr(), stream=stream)

    def status(self) -> int:
        """0, or 1 when a wait for another rank's words expired (after synchronising)."""
        return int(self.err.item())

    def close(self):
        import llmdiy_b200 as L
        for p in self.opened:
            L.p2p_close(p)
        self.opened = []
        if self.own:
            L.p2p_free(self.own)
            self.own = 0


class SplitKVAttention:
    """Distributed decode attention over a sharded cache.

    `partials(q, K, V, rows, part)` and `merge(parts, out)` default to the sm_100a
    kernels (llmdiy_fd_mh_partials / llmdiy_fd_mh_merge on the current CUDA
    stream); CPU tests substitute other implementations of the same contracts to
    exercise the sharding and exchange logic on gloo ranks.
    """

    def __init__(self, group, num_heads: int, stride: int, partials=None, merge=None, exchange: str = "nccl"):
        """exchange: "nccl" (all-gather of the partials, then a merge kernel) or "p2p" (one kernel per
        rank that exchanges over peer memory and merges: P2PExchange; CUDA devices only)."""
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        self.num_heads = num_heads
        self.stride = stride
        self._partials = partials or self._gpu_partials
        self._merge = merge or self._gpu_merge
        if exchange not in ("nccl", "p2p"):
            raise ValueError(exchange)
        self.exchange = exchange
        self._p2p = None
        self._work = None
        self._bufs = None  # (part, parts) reused across calls on one device

    def rows(self, L: int) -> tuple[int, int]:
        return shard_range(L, self.world, self.rank)

    def __call__(self, q, K_shard, V_shard, L: int, out):
        """q: [num_heads*128] fp16; K_shard/V_shard: this rank's rows of the cache (row stride
        `stride`); L: total rows over all ranks; out: [num_heads*128] fp16, the same on every rank."""
        import torch
        r0, r1 = self.rows(L)
        if self._bufs is None or self._bufs[0].device != q.device:
            self._bufs = (torch.empty((self.num_heads, PART), dtype=torch.float32, device=q.device),
                          torch.empty((self.world, self.num_heads, PART), dtype=torch.float32, device=q.device))
        part, parts = self._bufs
        if self.exchange == "p2p":
            if self._p2p is None:
                self._p2p = P2PExchange(self.group, self.num_heads, q.device)
            st = torch.cuda.current_stream(q.device).cuda_stream
            if self._partials == self._gpu_partials and r1 > r0:
                # the split kernel then the exchange kernel, which merges the splits itself
                self._p2p.shard(q, K_shard, V_shard, r1 - r0, self.stride, self._workspace(r1 - r0, q.device), out,
                                st)
            else:
                self._partials(q, K_shard, V_shard, r1 - r0, part)
                self._p2p(part, out, st)
            return out
        self._partials(q, K_shard, V_shard, r1 - r0, part)
        gather_partials(self.group, part, self.world, parts)
        self._merge(parts, out)
        return out

    def close(self):
        if self._p2p is not None:
            self._p2p.close()
            self._p2p = None

    def _workspace(self, rows, device):
        """The split kernel's workspace for `rows` rows (zero-filled once: its error word)."""
        import torch
        import llmdiy_b200 as L
        nb = L.fd_mh_work_bytes(rows, self.num_heads)
        if self._work is None or self._work.numel() * 4 < nb:
            self._work = torch.zeros((nb + 3) // 4, dtype=torch.float32, device=device)
        return self._work

    # ---- default implementations: the sm_100a kernels
    def _gpu_partials(self, q, K, V, rows, part):
        import torch
        import llmdiy_b200 as L
        if rows <= 0:
            # an empty shard contributes nothing: m = -inf, l = 0, o = 0
            part.zero_()
            part[:, 128] = float("-inf")
            return
        self._workspace(rows, q.device)
        nb = L.fd_mh_work_bytes(rows, self.num_heads)
        st = torch.cuda.current_stream(q.device).cuda_stream
        L.fd_mh_partials(q.data_ptr(), K.data_ptr(), V.data_ptr(), rows, self.stride, self.num_heads,
                         part.data_ptr(), self._work.data_ptr(), nb, stream=st)

    def _gpu_merge(self, parts, out):
        import torch
        import llmdiy_b200 as L
        st = torch.cuda.current_stream(parts.device).cuda_stream
        L.fd_mh_merge(parts.data_ptr(), parts.shape[0], self.num_heads, out.data_ptr(), stream=st)
