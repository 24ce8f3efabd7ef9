"""Benchmark of the decode hot path (BASELINE.json metric, configs[1]).

Workload: Qwen-1.8B (24 layers, hidden 2048, 16x128 MHA, SwiGLU 5504,
vocab 151936) with seeded random fp16 weights N(0, 0.02) (RMSNorm weights 1),
a 128-token prompt of uniform random ids, 256 greedy decode tokens at batch 1.

One step = the 256 greedy decode steps that follow the prompt (positions
127..382; the prompt's first 127 tokens are prefilled once before timing,
the KV rows they fill stay valid, and each step rewrites rows 127..382).
`value` = decode tokens/s with everything resident in HBM (CUDA events on
the launching stream).  `e2e` = the same metric through the public C API
llmdiy_engine_generate(): prompt ids from host memory, prefill, 256 decode
steps, generated ids back to host, all inside the timed region.

Multi-GPU (torchrun): one engine replica per GPU, independent requests, no
collective on the data path ("scaling": "weak"); timing is the max over ranks.

--impl reference: the reference has no CPU path of its own; this arm times
the C restatement of its decode path (oracle/, multi-threaded fp32) on the
host cores on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "llm-inference-diy_b200"))

QWEN = dict(vocab_size=151936, hidden_size=2048, num_layers=24, num_heads=16, intermediate_size=5504)
PROMPT_LEN, GEN_LEN, SEED, PROMPT_SEED = 128, 256, 1234, 99
MAX_SEQLEN = 512


def weight_bytes(c=QWEN):
    """Algorithmic bytes of weights read per decode token (every GEMV matrix,
    the QKV bias, the RMSNorm weights and one embedding row)."""
    H, IM, V, NL = c["hidden_size"], c["intermediate_size"], c["vocab_size"], c["num_layers"]
    per_layer = 3 * H * H + H * H + 2 * IM * H + H * IM + 3 * H + 2 * H
    return 2 * (NL * per_layer + V * H + H + H)


def kv_bytes(L, c=QWEN):
    """KV bytes per token at L attended positions: read L rows of K and V, write one row of each."""
    H, NL = c["hidden_size"], c["num_layers"]
    return NL * 2 * H * 2 * (L + 1)


def bytes_per_step():
    return sum(weight_bytes() + kv_bytes(PROMPT_LEN + t) for t in range(GEN_LEN))


def prompt_ids():
    import numpy as np
    return np.random.default_rng(PROMPT_SEED).integers(0, QWEN["vocab_size"], PROMPT_LEN).tolist()


class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.p = None
        self.lines = []

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.p = None
        return self

    def _read(self):
        for line in self.p.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic_ratio():
    """DRAM bytes (read + write) over algorithmic bytes of decode_kernel, from the committed ncu
    capture of the small case (profiles/decode_kernel_traffic.json), if present."""
    p = os.path.join(ROOT, "profiles", "decode_kernel_traffic.json")
    if os.path.exists(p):
        return float(json.load(open(p))["traffic_over_algorithmic"])
    return None


def dist_setup(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist
    return rank, world, local, pg


def max_over_ranks(pg, x, local):
    if pg is None:
        return x
    import torch
    t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def barrier(pg, local):
    if pg is not None:
        import torch
        pg.barrier(device_ids=[local])
        torch.cuda.synchronize()


# ------------------------------------------------------------------ CPU baseline (oracle port)
def cpu_decode_sample(n_tokens, threads, warm_tokens=1):
    """Time n_tokens decode steps of the CPU restatement on the same weights (tokens/s), after
    warm_tokens untimed steps."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import llmdiy_b200 as L
    import oracle as orc
    d = tempfile.mkdtemp()
    path = os.path.join(d, "qwen_random.bin")
    L.write_random_bin(path, L.make_config(**QWEN, max_seqlen=MAX_SEQLEN), seed=SEED, nthreads=threads)
    try:
        m = orc.OracleModel(path, nthreads=threads)
    finally:
        os.remove(path)
    # The sample times decode steps at the workload's positions (127..); the KV
    # rows it attends over are the zero-initialised cache, which costs the same work.
    p = prompt_ids()
    tok, pos = p[-1], PROMPT_LEN - 1
    for i in range(max(1, warm_tokens)):
        m.step(p[i % len(p)], i % PROMPT_LEN)  # touch every weight page; untimed
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        tok, _, _ = m.step(tok, pos)
        pos += 1
    dt = time.perf_counter() - t0
    m.close()
    return n_tokens / dt, dt


def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    n_per = 8  # decode tokens per step: a bounded sample of the 256-token workload
    rate, dt = cpu_decode_sample(n_per * args.steps, threads, warm_tokens=n_per * max(1, args.warmup))
    line = {
        "impl": "reference", "metric": "decode_tokens_per_s", "value": round(rate, 4), "unit": "tok/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * dt / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (fp16 storage)",
        "data": "synthetic: seeded N(0,0.02) fp16 weights, uniform random prompt ids",
        "config": {"workload": "Qwen-1.8B bs1 greedy decode: prompt 128, 256 new tokens (BASELINE configs[1])",
                   "sample": f"{n_per} decode tokens per step at positions 127.., {n_per * max(1, args.warmup)} "
                             f"untimed warm-up tokens"},
        "cpu_baseline": {"value": round(rate, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{n_per * args.steps} decode tokens of the Qwen-1.8B workload, fp32 C "
                                   f"restatement (oracle/qwen_oracle.c), {threads} threads"},
        "e2e": {"value": round(rate, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def run_ours(args, rank, world, local, pg):
    import torch
    import llmdiy_b200 as L

    torch.cuda.set_device(local)
    cfg = L.make_config(**QWEN, max_seqlen=MAX_SEQLEN)
    eng = L.Engine(config=cfg, seed=SEED, device=local)
    prompt = prompt_ids()
    eng.reset()
    eng.prefill(prompt[:-1])
    stream = torch.cuda.Stream(device=local)
    sh = stream.cuda_stream
    first, pos0 = prompt[-1], PROMPT_LEN - 1

    def one_step():
        eng.decode_async(first, pos0, GEN_LEN, stop_on_eos=False, stream=sh)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            one_step()
    torch.cuda.synchronize()
    n_done = eng.status()
    assert n_done == GEN_LEN, n_done
    ref_tokens = eng.tokens(GEN_LEN)

    barrier(pg, local)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                one_step()
            ev1.record(stream)
        torch.cuda.synchronize()
    barrier(pg, local)
    ms = ev0.elapsed_time(ev1)
    eng.status()
    assert eng.tokens(GEN_LEN) == ref_tokens, "decode is not deterministic across steps"
    ms_max = max_over_ranks(pg, ms, local)
    ms_per_step = ms_max / args.steps
    value = world * GEN_LEN * args.steps / (ms_max / 1000.0)

    # roofline of the (only) kernel in the timed region: one launch per step
    peak, peak_kind = measured_peaks()
    bps = bytes_per_step()
    achieved = bps / (ms / args.steps / 1000.0) / 1e9
    traffic_ratio = profile_traffic_ratio()

    # e2e through the public API with host buffers (includes prefill of the 127 prompt tokens)
    for _ in range(max(1, args.warmup // 2)):
        eng.generate(prompt, GEN_LEN, stop_on_eos=False)
    barrier(pg, local)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = eng.generate(prompt, GEN_LEN, stop_on_eos=False)
    e2e_s = time.perf_counter() - t0
    barrier(pg, local)
    assert out == ref_tokens, "generate() differs from the device-resident decode"
    e2e_max = max_over_ranks(pg, e2e_s, local)
    e2e_val = world * GEN_LEN * args.steps / e2e_max

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate, dt = cpu_decode_sample(args.cpu_tokens, threads)
        cpu = {"value": round(rate, 4), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{args.cpu_tokens} decode tokens of the same Qwen-1.8B workload, fp32 C restatement "
                         f"(oracle/qwen_oracle.c), {threads} threads, {dt:.1f} s"}

    if rank == 0:
        line = {
            "metric": "decode_tokens_per_s", "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
            "data": "synthetic: seeded N(0,0.02) fp16 weights (RMSNorm=1), uniform random prompt ids",
            "config": {"workload": "Qwen-1.8B bs1 greedy decode: prompt 128, 256 new tokens (BASELINE configs[1])",
                       "global_batch": world, "seq_len": PROMPT_LEN + GEN_LEN,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2: 3.05 GB of weights streamed per token"},
            "gpu_launches": args.steps,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": (round(traffic_ratio * bps) if traffic_ratio else None),
                         "traffic_source": "ncu dram bytes / algorithmic bytes of the 4-layer case, scaled",
                         "algorithmic_bytes_per_launch": bps, "kernel": "decode_kernel (persistent, 256 tokens)"},
            "e2e": {"value": round(e2e_val, 3), "unit": "tok/s", "h2d_bytes_per_step": 4 * PROMPT_LEN,
                    "d2h_bytes_per_step": 4 * GEN_LEN},
            "clocks": clk.summary(),
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    eng.close()


# ------------------------------------------------------------------ flash-decoding op (configs 1 and 5)
FD_HEADS, FD_STRIDE = 16, 2048


def fd_bytes(L):
    """Algorithmic bytes of one multi-head decode-attention call: K and V rows read, q read, O written."""
    return 2 * L * FD_HEADS * 128 * 2 + 2 * FD_HEADS * 128 * 2


def run_fd_op(args, rank, world, local, pg):
    """Config 1 (L=1024) and config 5 (L=131072 split over the ranks' GPUs): 16 heads x 128, one query
    token, K/V ~ N(0,1) fp16 in the engine cache layout.  Config 1 rotates over enough K/V copies
    (> 2x L2) that every call reads from HBM, and times a CUDA graph of the calls; config 5 shards
    the 131072 positions contiguously over the ranks (each rank's partials -> exchange over peer
    memory + LSE merge in one kernel; the NCCL all-gather path is timed beside it) and times on device
    with the max over ranks."""
    import torch
    import llmdiy_b200 as L
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    peak, peak_kind = measured_peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    lines = []
    if world == 1:
        # ---- config 1: 16 x 128, L = 1024
        Lc = 1024
        nset = 40  # 40 x 8.4 MB = 336 MB > 2 x L2
        q = torch.randn(FD_HEADS * 128, generator=g, device=dev).half()
        Ks = [torch.randn(Lc * FD_STRIDE, generator=g, device=dev).half() for _ in range(nset)]
        Vs = [torch.randn(Lc * FD_STRIDE, generator=g, device=dev).half() for _ in range(nset)]
        O = torch.empty(FD_HEADS * 128, dtype=torch.float16, device=dev)
        nb = L.fd_mh_work_bytes(Lc, FD_HEADS)
        work = torch.empty((nb + 3) // 4, dtype=torch.float32, device=dev)
        st = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(st):
            for i in range(nset):  # warm-up (also loads the module)
                L.fd_multihead(q.data_ptr(), Ks[i].data_ptr(), Vs[i].data_ptr(), O.data_ptr(), Lc, FD_STRIDE,
                               FD_HEADS, work.data_ptr(), nb, stream=st.cuda_stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            for i in range(nset):
                L.fd_multihead(q.data_ptr(), Ks[i].data_ptr(), Vs[i].data_ptr(), O.data_ptr(), Lc, FD_STRIDE,
                               FD_HEADS, work.data_ptr(), nb, stream=st.cuda_stream)
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(1, args.steps)
        e0.record(st)
        with torch.cuda.stream(st):
            for _ in range(reps):
                graph.replay()
        e1.record(st)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / (reps * nset)
        gbs = fd_bytes(Lc) / (us * 1e-6) / 1e9
        lines.append({"metric": "flash_decode_GBps", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1,
                      "us_per_call": round(us, 3), "higher_is_better": True, "dtype": "fp16 (fp32 accumulate)",
                      "data": "synthetic N(0,1)", "config": {"workload": "BASELINE configs[0]: 16x128, L=1024, "
                      "engine layout stride 2048", "l2": f"cold: {nset} K/V copies rotated, CUDA graph of the calls"},
                      "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                                   "frac": round(gbs / peak, 4), "peak_kind": peak_kind}})
        del graph, Ks, Vs
        torch.cuda.empty_cache()
    # ---- config 5: L = 131072 over the ranks
    Lt = 131072
    import llmdiy_dist as D
    q = torch.randn(FD_HEADS * 128, generator=g, device=dev).half()
    if pg is not None:
        pg.broadcast(q, src=0)
    att = D.SplitKVAttention(pg.group.WORLD if pg is not None else None, FD_HEADS, FD_STRIDE)
    r0, r1 = att.rows(Lt)
    Lr = r1 - r0
    K = torch.randn(Lr * FD_STRIDE, generator=g, device=dev).half()
    V = torch.randn(Lr * FD_STRIDE, generator=g, device=dev).half()
    O = torch.empty(FD_HEADS * 128, dtype=torch.float16, device=dev)
    nb = L.fd_mh_work_bytes(Lr, FD_HEADS)
    work = torch.empty((nb + 3) // 4, dtype=torch.float32, device=dev)
    st = torch.cuda.current_stream(dev)

    # multi-GPU: the exchange over peer memory (one kernel per rank: push partials, flags, merge) is
    # the measured path; the NCCL all-gather path is timed beside it and must agree
    att_p2p = D.SplitKVAttention(pg.group.WORLD, FD_HEADS, FD_STRIDE, exchange="p2p") if world > 1 else None

    def call(a=None):
        if world == 1:
            L.fd_multihead(q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), Lr, FD_STRIDE, FD_HEADS,
                           work.data_ptr(), nb, stream=st.cuda_stream)
        else:
            (a or att_p2p)(q, K, V, Lt, O)  # partials -> exchange -> merge, all on the current stream

    def timed(a=None):
        for _ in range(max(3, args.warmup)):
            call(a)
        barrier(pg, local)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(1, args.steps) * 4
        e0.record(st)
        for _ in range(reps):
            call(a)
        e1.record(st)
        torch.cuda.synchronize()
        barrier(pg, local)
        return max_over_ranks(pg, e0.elapsed_time(e1) / reps, local)

    nccl_ms = None
    if world > 1:
        call(att)
        ref = O.clone()
        call(att_p2p)
        torch.cuda.synchronize()
        assert att_p2p._p2p.status() == 0, "peer exchange wait expired"
        diff = float((O.float() - ref.float()).abs().max())
        assert diff < 1e-3, f"peer exchange differs from the all-gather path by {diff}"
        nccl_ms = timed(att)
    ms = timed(att_p2p)
    gbs = fd_bytes(Lt) / (ms * 1e-3) / 1e9
    wk = work if world == 1 else att_p2p._work
    assert L.fd_mh_status(wk.data_ptr(), Lr, FD_HEADS) == 0
    if att_p2p is not None:
        assert att_p2p._p2p.status() == 0
        att_p2p.close()
    lines.append({"metric": "flash_decode_GBps", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world,
                  "us_per_call": round(ms * 1000, 2), "higher_is_better": True, "scaling": "strong",
                  "dtype": "fp16 (fp32 accumulate)", "data": "synthetic N(0,1)",
                  "config": {"workload": "BASELINE configs[4]: 16x128, L=131072 split over the GPUs",
                             "rows_per_gpu": Lr, "exchange": "16x130 fp32 per rank stored into every rank's "
                             "buffer over NVLink peer memory, flags, merge (one kernel)" if world > 1 else "none",
                             "nccl_allgather_us_per_call": round(nccl_ms * 1000, 2) if nccl_ms else None,
                             "l2": "inputs larger than L2 (1 GiB of K+V)"},
                  "roofline": {"bound": "hbm", "achieved_per_gpu": round(gbs / world, 1), "peak": peak,
                               "unit": "GB/s", "frac": round(gbs / world / peak, 4), "peak_kind": peak_kind}})
    if rank == 0:
        for ln in lines:
            print(json.dumps(ln), flush=True)


# ------------------------------------------------------------------ prefill (config 3)
def prefill_flops(N, c=QWEN):
    """GEMM FLOPs of an N-token prompt forward (no lm_head) plus causal attention (QK^T and PV)."""
    H, IM, NL = c["hidden_size"], c["intermediate_size"], c["num_layers"]
    gemm = 2 * N * (3 * H * H + H * H + 2 * IM * H + H * IM) * NL
    attn = 2 * 2 * H * (N * (N + 1) // 2) * NL
    return gemm, attn


def run_prefill(args, rank, world, local, pg):
    """Qwen-1.8B prompt forward of 2048 uniform-random ids through the public
    API (llmdiy_engine_prefill: ids uploaded from host, KV cache filled, synchronised), wall-clock
    per prefill, TFLOP/s against the measured dense fp16/bf16 tensor peak."""
    import numpy as np
    import torch
    import llmdiy_b200 as L
    torch.cuda.set_device(local)
    N = 2048
    cfg = L.make_config(**QWEN, max_seqlen=N + 64)
    eng = L.Engine(config=cfg, seed=SEED, device=local)
    ids = np.random.default_rng(PROMPT_SEED + rank).integers(0, QWEN["vocab_size"], N).tolist()
    for _ in range(max(1, args.warmup)):
        eng.prefill(ids)
    barrier(pg, local)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.prefill(ids)
    dt = (time.perf_counter() - t0) / args.steps
    barrier(pg, local)
    dt = max_over_ranks(pg, dt, local)
    gemm, attn = prefill_flops(N)
    tf = (gemm + attn) / dt / 1e12
    peak = 1665.2
    mp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(mp):
        peak = float(json.load(open(mp))["bf16_tflops"])
    if rank == 0:
        print(json.dumps({"metric": "prefill_ms", "value": round(dt * 1e3, 3), "unit": "ms", "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
                          "scaling": "weak", "dtype": "fp16 (fp32 accumulate)",
                          "data": "synthetic: seeded N(0,0.02) fp16 weights, uniform random prompt ids",
                          "config": {"workload": "BASELINE configs[2]: Qwen-1.8B prefill of 2048 tokens "
                                     "(no lm_head; the last prompt token goes through decode)",
                                     "timing": "wall clock around llmdiy_engine_prefill (host ids in, synchronised)"},
                          "tflops": round(tf, 1), "gemm_tflop": round(gemm / 1e12, 3),
                          "attention_tflop": round(attn / 1e12, 3),
                          "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak,
                                       "unit": "TFLOP/s", "frac": round(tf / peak, 4), "peak_kind": "measured"}}),
              flush=True)
    eng.close()


# ------------------------------------------------------------------ batched ragged decode (config 4)
def run_batch(args, rank, world, local, pg):
    """64 independent sequences with KV lengths uniform in [128, 4096] (seeded),
    their caches pre-filled with N(0,1) fp16, 128 greedy steps each; the sequences are partitioned
    over the ranks' per-GPU weight replicas with no collective (total work fixed: "strong").
    Timed on the device per rank (CUDA events around llmdiy_batch_decode, which uploads the start
    tokens/positions and reads the generated ids back), max over ranks."""
    import numpy as np
    import torch
    import llmdiy_b200 as L
    torch.cuda.set_device(local)
    NSEQ, STEPS, LO, HI = 64, 128, 128, 4096
    rng = np.random.default_rng(17)
    lens_all = rng.integers(LO, HI + 1, NSEQ)
    toks_all = rng.integers(0, QWEN["vocab_size"], NSEQ)
    mine = [i for i in range(NSEQ) if i % world == rank]
    B = len(mine)
    cfg = L.make_config(**QWEN, max_seqlen=256)
    eng = L.Engine(config=cfg, seed=SEED, device=local)
    bt = L.Batch(eng, max_batch=B, max_len=HI + STEPS + 1)
    for j, i in enumerate(mine):
        bt.fill_random(j, int(lens_all[i]), seed=1000 + i)
    toks = [int(toks_all[i]) for i in mine]
    pos = [int(lens_all[i]) for i in mine]
    bt.decode(toks, pos, max(1, args.warmup))  # captures the step
    barrier(pg, local)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    out = bt.decode(toks, pos, STEPS, stream=st.cuda_stream)
    e1.record(st)
    torch.cuda.synchronize()
    ms = max_over_ranks(pg, e0.elapsed_time(e1), local)
    assert out.shape == (STEPS, B) and (out >= 0).all()
    value = NSEQ * STEPS / (ms / 1e3)
    kv_bytes = sum(2 * 2 * 2048 * 24 * (int(lens_all[i]) + s + 1) for i in range(NSEQ) for s in range(STEPS))
    w_bytes = weight_bytes() * STEPS * world
    peak, peak_kind = measured_peaks()
    gbs = (kv_bytes + w_bytes) / (ms / 1e3) / 1e9
    if rank == 0:
        print(json.dumps({"metric": "batched_decode_tokens_per_s", "value": round(value, 1), "unit": "tok/s",
                          "n_gpus": world, "steps": STEPS, "higher_is_better": True, "scaling": "strong",
                          "ms_per_step": round(ms / STEPS, 3), "dtype": "fp16 (fp32 accumulate)",
                          "data": "synthetic: seeded N(0,0.02) weights; caches pre-filled N(0,1)",
                          "config": {"workload": "BASELINE configs[3]: 64 sequences, KV lengths U[128,4096], "
                                     "128 greedy steps", "sequences_per_gpu": B, "parallelism": f"replicas x{world}"},
                          "roofline": {"bound": "hbm", "achieved_per_gpu": round(gbs / world, 1), "peak": peak,
                                       "unit": "GB/s", "frac": round(gbs / world / peak, 4),
                                       "peak_kind": peak_kind,
                                       "algorithmic_bytes": kv_bytes + w_bytes}}), flush=True)
    bt.close()
    eng.close()


# ------------------------------------------------------------------ tensor-core GEMM shapes of configs 3/4
def run_gemm(args, rank, world, local, pg):
    """llmdiy_gemm_tc (tcgen05, fp16 in, fp32 accumulate) on the prefill's GEMM shapes, CUDA events,
    against the measured dense fp16/bf16 peak; cuBLAS (torch.matmul) on the same shapes for context."""
    import torch
    import llmdiy_b200 as L
    torch.cuda.set_device(local)
    peak = 1665.2
    mp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(mp):
        peak = float(json.load(open(mp))["bf16_tflops"])
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    for (M, N, K) in [(2048, 6144, 2048), (2048, 2048, 2048), (2048, 11008, 2048), (2048, 2048, 5504),
                      (8192, 8192, 8192)]:
        A = (torch.randn(M, K, generator=g, device="cuda") * 0.5).half()
        W = (torch.randn(N, K, generator=g, device="cuda") / K ** 0.5).half()
        C = torch.empty(M, N, device="cuda", dtype=torch.half)
        st = torch.cuda.current_stream().cuda_stream

        def ours():
            L.gemm_tc(A.data_ptr(), W.data_ptr(), C.data_ptr(), M, N, K, stream=st)

        def timed(fn, n=20):
            for _ in range(max(3, args.warmup)):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(n):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / n

        ms = timed(ours)
        ms_cublas = timed(lambda: torch.matmul(A, W.t()))
        tf = 2 * M * N * K / ms / 1e9
        if rank == 0:
            print(json.dumps({"metric": "gemm_tflops", "value": round(tf, 1), "unit": "TFLOP/s",
                              "config": {"workload": f"C[{M},{N}] = A[{M},{K}] W[{N},{K}]^T fp16, fp32 accumulate"},
                              "us": round(ms * 1e3, 1), "cublas_tflops": round(2 * M * N * K / ms_cublas / 1e9, 1),
                              "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak,
                                           "unit": "TFLOP/s", "frac": round(tf / peak, 4), "peak_kind": "measured"}}),
                  flush=True)


def run_ncu_case():
    """Small case for ncu captures of decode_kernel: the Qwen-1.8B shapes with 4 layers (full vocab,
    0.95 GB of weights, larger than L2), a tensor-core prefill of 127 tokens, then one decode_kernel
    launch of 2 tokens (capture it with `-k regex:decode_kernel -c 1`)."""
    import torch
    import llmdiy_b200 as L
    cfg = L.make_config(**dict(QWEN, num_layers=4), max_seqlen=MAX_SEQLEN)
    eng = L.Engine(config=cfg, seed=SEED, device=0)
    prompt = prompt_ids()
    eng.reset()
    eng.prefill(prompt[:-1])
    eng.decode_async(prompt[-1], PROMPT_LEN - 1, 2, stop_on_eos=False)
    torch.cuda.synchronize()
    n = eng.status()
    eng.close()
    print(json.dumps({"ncu_case": "qwen-1.8b-4layer decode 2 tokens", "n_done": n}), flush=True)
    if n != 2:
        sys.exit(1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=256,
                    help="decode tokens of the CPU baseline sample (256 = the whole workload, ~15 s on 16 cores)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu-case", action="store_true", help="run the small decode case used for ncu captures")
    ap.add_argument("--workload", default="decode", choices=["decode", "fd-op", "prefill", "gemm", "batch"],
                    help="decode: the headline config-2 line; fd-op: flash-decoding op lines (configs 1 and 5); "
                         "prefill: 2048-token prompt forward (config 3)")
    args = ap.parse_args()
    if args.ncu_case:
        run_ncu_case()
        return
    rank, world, local, pg = dist_setup(args.gpus)
    try:
        if args.workload == "batch":
            if args.impl == "reference":
                if rank == 0:
                    print(json.dumps({"impl": "reference", "workload": "batch", "unavailable":
                                      "the reference has no batched path; see the decode arm"}))
            else:
                run_batch(args, rank, world, local, pg)
        elif args.workload == "gemm":
            if args.impl == "reference":
                if rank == 0:
                    print(json.dumps({"impl": "reference", "workload": "gemm", "unavailable":
                                      "the reference has no CPU GEMM path; see the decode arm"}))
            else:
                run_gemm(args, rank, world, local, pg)
        elif args.workload == "prefill":
            if args.impl == "reference":
                if rank == 0:
                    print(json.dumps({"impl": "reference", "workload": "prefill", "unavailable":
                                      "the reference has no CPU prefill path; see the decode arm"}))
            else:
                run_prefill(args, rank, world, local, pg)
        elif args.workload == "fd-op":
            if args.impl == "reference":
                if rank == 0:
                    print(json.dumps({"impl": "reference", "workload": "fd-op", "unavailable":
                                      "the reference has no CPU flash-decoding path; see the decode arm"}))
            else:
                run_fd_op(args, rank, world, local, pg)
        elif args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_ours(args, rank, world, local, pg)
    finally:
        if pg is not None:
            pg.destroy_process_group()


if __name__ == "__main__":
    main()
