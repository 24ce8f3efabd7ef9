"""Benchmark of the decode hot path (BASELINE.json metric, configs[1] as the headline).

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

The same line carries the other configurations, measured in the same run:
  "batch"   configs[3]: 64 ragged sequences, 128 greedy steps, split over the ranks' replicas;
  "fd_op"   configs[0]: 16x128 flash decoding at L=1024 (1 GPU), with the reference's own
            per-head kernels timed beside it; configs[4]: L=131072 sharded over the ranks,
            partials exchanged over NVLink peer memory and merged (NCCL all-gather path timed
            beside it);
  "prefill" configs[2]: a 2048-token prompt forward (1 GPU);
  "reference_gpu" (1 GPU): the reference engine itself (its sources built to compute_89 PTX,
            JIT-run on this GPU) through its stdin protocol, next to this repository's drop-in
            driver on the same weights and the same protocol input;
  "cpu_baseline" (1 GPU): the C restatement of the reference's decode path on the host cores.

Multi-GPU (torchrun): one engine replica per GPU, independent requests, no
collective on the data path ("scaling": "weak"); timing is the max over ranks.

--impl reference: the reference has no CPU path of its own; this arm times
the C restatement of its decode path (oracle/, multi-threaded fp32) on the
host cores over the same positions 127..382 after the same prompt prefill.
It never loads this repository's library.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "llm-inference-diy_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")

QWEN = dict(vocab_size=151936, hidden_size=2048, num_layers=24, num_heads=16, intermediate_size=5504)
PROMPT_LEN, GEN_LEN, SEED, PROMPT_SEED = 128, 256, 1234, 99
MAX_SEQLEN = 512            # .bin header of the CPU / reference-engine runs (every position they reach is < 512)
ENGINE_MAX_SEQLEN = 2112    # our engine: the decode positions (< 384) and the 2048-token prefill


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


def measured_tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


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


def oracle_mod():
    if ORACLE_DIR not in sys.path:
        sys.path.insert(0, ORACLE_DIR)
    import oracle as orc
    return orc


def product_mod():
    if PKG not in sys.path:
        sys.path.insert(0, PKG)
    import llmdiy_b200 as L
    return L


def write_model_bin(path, threads):
    """The benchmark's seeded model as a QWDF file, written by the oracle's copy of the generator
    (byte-identical to the library's), so the CPU and reference-engine legs never load the library."""
    oracle_mod().Oracle().write_random_bin(path, **QWEN, max_seqlen=MAX_SEQLEN, seed=SEED, nthreads=threads)


# ------------------------------------------------------------------ CPU restatement (oracle port)
def cpu_decode(path, threads, warm_steps, steps, tokens_per_step):
    """The C restatement on the host cores: prefill the workload's 127 prompt tokens (untimed), then
    greedy decode `tokens_per_step` tokens per step over the workload's positions 127..382 (cyclic:
    after 382 the next step restarts at 127), warm_steps untimed steps, then `steps` timed ones.
    Returns (tokens/s, timed seconds)."""
    orc = oracle_mod()
    m = orc.OracleModel(path, nthreads=threads)
    p = prompt_ids()
    m.prefill(p[:-1])
    tok, k = p[-1], 0

    def run(n):
        nonlocal tok, k
        for _ in range(n):
            tok, _, _ = m.step(tok, PROMPT_LEN - 1 + k)
            k = (k + 1) % GEN_LEN

    run(warm_steps * tokens_per_step)
    t0 = time.perf_counter()
    run(steps * tokens_per_step)
    dt = time.perf_counter() - t0
    m.close()
    return steps * tokens_per_step / dt, dt


def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    t_per = math.ceil(GEN_LEN / max(1, args.steps))  # the timed steps cover all 256 positions
    d = tempfile.mkdtemp()
    path = os.path.join(d, "qwen_random.bin")
    write_model_bin(path, threads)
    try:
        rate, dt = cpu_decode(path, threads, max(1, args.warmup), args.steps, t_per)
    finally:
        os.remove(path)
    sample = (f"{t_per} greedy decode tokens per step at positions 127..382 (cyclic; the {args.steps} timed steps "
              f"cover all 256) after an untimed prefill of the 127 prompt tokens, {t_per * max(1, args.warmup)} "
              f"untimed warm-up tokens")
    line = {
        "impl": "reference", "metric": "decode_tokens_per_s", "value": round(rate, 4), "unit": "tok/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * dt / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (fp16 storage)",
        "data": "synthetic: seeded N(0,0.02) fp16 weights (RMSNorm=1), uniform random prompt ids",
        "config": {"workload": "Qwen-1.8B bs1 greedy decode: prompt 128, 256 new tokens (BASELINE configs[1])",
                   "sample": sample},
        "cpu_baseline": {"value": round(rate, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{t_per * args.steps} decode tokens of the Qwen-1.8B workload, fp32 C "
                                   f"restatement (oracle/qwen_oracle.c), {threads} threads"},
        "e2e": {"value": round(rate, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ an engine through its stdin protocol
def protocol_rate(exe, bin_path, ids, env=None, timeout=900):
    """Drives a qwen_infer-protocol engine (framework_src/qwen_infer.cu:743-822): waits for
    [ENGINE_READY], sends one turn, and wall-times [GENERATION_START]..[GENERATION_END] while
    counting the generated ids.  Returns {"tokens", "seconds", "rate", "load_s", "stream"}."""
    t_start = time.perf_counter()
    p = subprocess.Popen([exe, bin_path], stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                         text=True, bufsize=1, env=env)
    timer = threading.Timer(timeout, p.kill)
    timer.start()
    try:
        for line in p.stdout:
            if "[ENGINE_READY]" in line:
                break
        load_s = time.perf_counter() - t_start
        p.stdin.write(" ".join(map(str, ids)) + "\n")
        p.stdin.flush()
        toks, t0, t1 = [], None, None
        for line in p.stdout:
            s = line.strip()
            if s == "[GENERATION_START]":
                t0 = time.perf_counter()
            elif s == "[GENERATION_END]":
                t1 = time.perf_counter()
                break
            elif t0 is not None and s.lstrip("-").isdigit():
                toks.append(int(s))
        p.stdin.write("exit\n")
        p.stdin.flush()
        p.wait(timeout=60)
    finally:
        timer.cancel()
        if p.poll() is None:
            p.kill()
    if t0 is None or t1 is None:
        return None
    return {"tokens": len(toks), "seconds": t1 - t0, "rate": len(toks) / (t1 - t0), "load_s": load_s,
            "stream": toks}


def reference_gpu_leg(bin_path, first_token):
    """The reference engine (oracle/_ref/qwen_infer_ref, its own sources as compute_89 PTX) and our
    drop-in driver on the same .bin, one-token prompt (the reference's multi-token prefill is not
    usable), each through the stdin protocol on this GPU."""
    orc = oracle_mod()
    L = product_mod()
    out = {"workload": "Qwen-1.8B greedy decode, one-token prompt, until EOS or the protocol's 512-token cap, "
                       "through the qwen_infer stdin/stdout protocol on the same seeded .bin",
           "timing": "wall clock from [GENERATION_START] to [GENERATION_END]"}
    if not os.path.exists(orc.REF_ENGINE):
        out["unavailable"] = "oracle/_ref/qwen_infer_ref not built (needs the reference tree at build time)"
        return out
    ref = protocol_rate(orc.REF_ENGINE, bin_path, [first_token])
    ours = protocol_rate(L.DRIVER_PATH, bin_path, [first_token])
    if ref is None or ours is None:
        out["unavailable"] = "an engine did not complete the turn"
        return out
    n_same = next((i for i, (a, b) in enumerate(zip(ours["stream"], ref["stream"])) if a != b),
                  min(len(ours["stream"]), len(ref["stream"])))
    out.update({
        "reference": {"value": round(ref["rate"], 2), "unit": "tok/s", "tokens": ref["tokens"],
                      "load_s": round(ref["load_s"], 1),
                      "kind": "reference engine qwen_infer.cu built from its sources (compute_89 PTX, JIT on B200)"},
        "ours": {"value": round(ours["rate"], 2), "unit": "tok/s", "tokens": ours["tokens"],
                 "load_s": round(ours["load_s"], 1), "kind": "qwen_infer_b200 (this repository's driver)"},
        "speedup": round(ours["rate"] / ref["rate"], 2),
        "identical_leading_tokens": n_same,
    })
    return out


# ------------------------------------------------------------------ batched ragged decode (config 4)
def batch_leg(eng, args, rank, world, local, pg):
    """64 independent sequences with KV lengths uniform in [128, 4096] (seeded),
    their caches pre-filled with N(0,1) fp16, 128 greedy steps each; the sequences are partitioned
    over the ranks' per-GPU weight replicas with no collective (total work fixed: "strong").
    Timed on the device per rank (CUDA events around llmdiy_batch_decode, which uploads the start
    tokens/positions and reads the generated ids back), max over ranks."""
    import numpy as np
    import torch
    L = product_mod()
    NSEQ, STEPS, LO, HI = 64, 128, 128, 4096
    rng = np.random.default_rng(17)
    lens_all = rng.integers(LO, HI + 1, NSEQ)
    toks_all = rng.integers(0, QWEN["vocab_size"], NSEQ)
    mine = [i for i in range(NSEQ) if i % world == rank]
    B = len(mine)
    bt = L.Batch(eng, max_batch=B, max_len=HI + STEPS + 1)
    for j, i in enumerate(mine):
        bt.fill_random(j, int(lens_all[i]), seed=1000 + i)
    toks = [int(toks_all[i]) for i in mine]
    pos = [int(lens_all[i]) for i in mine]
    bt.decode(toks, pos, max(3, args.warmup))  # captures the step
    barrier(pg, local)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    out = bt.decode(toks, pos, STEPS, stream=st.cuda_stream)
    e1.record(st)
    torch.cuda.synchronize()
    ms = max_over_ranks(pg, e0.elapsed_time(e1), local)
    assert out.shape == (STEPS, B) and (out >= 0).all()
    bt.close()
    value = NSEQ * STEPS / (ms / 1e3)
    kv = sum(2 * 2 * 2048 * 24 * (int(lens_all[i]) + s + 1) for i in range(NSEQ) for s in range(STEPS))
    w = weight_bytes() * STEPS * world
    peak, peak_kind = measured_peaks()
    gbs = (kv + w) / (ms / 1e3) / 1e9
    return {"metric": "batched_decode_tokens_per_s", "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
            "steps": STEPS, "higher_is_better": True, "scaling": "strong", "ms_per_step": round(ms / STEPS, 3),
            "data": "synthetic: seeded N(0,0.02) weights; caches pre-filled N(0,1)",
            "config": {"workload": "BASELINE configs[3]: 64 sequences, KV lengths U[128,4096], 128 greedy steps",
                       "sequences_per_gpu": B, "parallelism": f"replicas x{world}",
                       "l2": "inputs larger than L2 (3.05 GB of weights + ~27 GB of KV per step)"},
            "roofline": {"bound": "hbm", "achieved_per_gpu": round(gbs / world, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / world / peak, 4), "peak_kind": peak_kind,
                         "algorithmic_bytes": kv + w}}


# ------------------------------------------------------------------ flash-decoding op (configs 1 and 5)
FD_HEADS, FD_STRIDE = 16, 2048


def fd_bytes(L):
    """Algorithmic bytes of one multi-head decode-attention call: K and V rows read, q read, O written."""
    return 2 * L * FD_HEADS * 128 * 2 + 2 * FD_HEADS * 128 * 2


def _graph_us(torch, st, capture, reps, warmup):
    """Captures `capture()` into a CUDA graph on stream st and returns µs per replay (CUDA events)."""
    with torch.cuda.stream(st):
        capture()  # eager warm-up (loads modules)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        capture()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    with torch.cuda.stream(st):
        for _ in range(reps):
            g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / reps
    del g
    return us


def fd_op_leg(args, rank, world, local, pg):
    """Config 1 (L=1024, 1 GPU) and config 5 (L=131072 split over the ranks' GPUs): 16 heads x 128,
    one query token, K/V ~ N(0,1) fp16 in the engine cache layout.  Config 1 rotates over enough
    K/V copies (> 2x L2) that every call reads from HBM and times CUDA graphs of the calls; the
    reference's own per-head launches of the decode step (qwen_infer.cu:646-677: split stage 1 over
    4 chunks + stage 2 per head at L=1024) are captured and timed the same way.  Config 5 shards the
    131072 positions contiguously over the ranks (each rank's partials -> exchange over peer memory
    + LSE merge in one kernel; the NCCL all-gather path is timed beside it) and times on device with
    the max over ranks."""
    import torch
    L = product_mod()
    dev = torch.device("cuda", local)
    peak, peak_kind = measured_peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    res = {}
    refk = None
    if world == 1:
        try:
            refk = oracle_mod().RefKernels()
        except (FileNotFoundError, OSError):
            refk = None
    if world == 1:
        Lc, nset = 1024, 40  # 40 x 8.4 MB = 336 MB > 2 x L2
        q = torch.randn(FD_HEADS * 128, generator=g, device=dev).half()
        Ks = [torch.randn(Lc * FD_STRIDE, generator=g, device=dev).half() for _ in range(nset)]
        Vs = [torch.randn(Lc * FD_STRIDE, generator=g, device=dev).half() for _ in range(nset)]
        O = torch.empty(FD_HEADS * 128, dtype=torch.float16, device=dev)
        nb = L.fd_mh_work_bytes(Lc, FD_HEADS)
        work = torch.zeros((nb + 3) // 4, dtype=torch.float32, device=dev)
        st = torch.cuda.Stream(device=dev)

        def ours():
            for i in range(nset):
                L.fd_multihead(q.data_ptr(), Ks[i].data_ptr(), Vs[i].data_ptr(), O.data_ptr(), Lc, FD_STRIDE,
                               FD_HEADS, work.data_ptr(), nb, stream=st.cuda_stream)

        reps = max(1, args.steps)
        us = _graph_us(torch, st, ours, reps, args.warmup) / nset
        gbs = fd_bytes(Lc) / (us * 1e-6) / 1e9
        c1 = {"metric": "flash_decode_GBps", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1,
              "us_per_call": round(us, 3), "higher_is_better": True,
              "config": {"workload": "BASELINE configs[0]: 16x128, L=1024, engine layout stride 2048",
                         "l2": f"cold: {nset} K/V copies rotated, CUDA graph of the calls"},
              "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                           "frac": round(gbs / peak, 4), "peak_kind": peak_kind}}
        if refk is not None:
            Op = torch.empty(8 * 128, dtype=torch.float16, device=dev)
            lse = torch.empty(8, dtype=torch.float32, device=dev)
            Or = torch.empty(FD_HEADS * 128, dtype=torch.float16, device=dev)

            def ref():
                for i in range(nset):
                    refk.fd_layer(q.data_ptr(), Ks[i].data_ptr(), Vs[i].data_ptr(), Or.data_ptr(), Op.data_ptr(),
                                  lse.data_ptr(), Lc, FD_HEADS, FD_STRIDE, ctypes.c_void_p(st.cuda_stream))

            rus = _graph_us(torch, st, ref, reps, args.warmup) / nset
            diff = float((O.float() - Or.float()).abs().max())
            c1["reference_v5"] = {"us_per_call": round(rus, 3), "GBps": round(fd_bytes(Lc) / (rus * 1e-6) / 1e9, 1),
                                  "launches_per_call": 2 * FD_HEADS, "max_abs_diff_vs_ours": diff,
                                  "kind": "the reference's fd_v5_split_stage1 + fd_opt_stage2 per head "
                                          "(compute_89 PTX JIT), CUDA graph of the same calls"}
            c1["speedup_vs_reference"] = round(rus / us, 2)
        res["config1"] = c1
        del Ks, Vs
        torch.cuda.empty_cache()

    # ---- config 5: L = 131072 over the ranks
    Lt = 131072
    if PKG not in sys.path:
        sys.path.insert(0, PKG)
    import llmdiy_dist as D
    q = torch.randn(FD_HEADS * 128, generator=g, device=dev).half()
    q2 = torch.randn(FD_HEADS * 128, generator=g, device=dev).half()
    if pg is not None:
        pg.broadcast(q, src=0)
        pg.broadcast(q2, src=0)
    att = D.SplitKVAttention(pg.group.WORLD if pg is not None else None, FD_HEADS, FD_STRIDE)
    r0, r1 = att.rows(Lt)
    Lr = r1 - r0
    K = torch.randn(Lr * FD_STRIDE, generator=g, device=dev).half()
    V = torch.randn(Lr * FD_STRIDE, generator=g, device=dev).half()
    O = torch.empty(FD_HEADS * 128, dtype=torch.float16, device=dev)
    nb = L.fd_mh_work_bytes(Lr, FD_HEADS)
    work = torch.zeros((nb + 3) // 4, dtype=torch.float32, device=dev)
    st = torch.cuda.current_stream(dev)
    att_p2p = D.SplitKVAttention(pg.group.WORLD, FD_HEADS, FD_STRIDE, exchange="p2p") if world > 1 else None

    def call(a=None, qq=q, out=O):
        if world == 1:
            L.fd_multihead(qq.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), Lr, FD_STRIDE, FD_HEADS,
                           work.data_ptr(), nb, stream=st.cuda_stream)
        else:
            (a or att_p2p)(qq, K, V, Lt, out)  # partials -> exchange -> merge, all on the current stream

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

    nccl_ms, p2p_diff = None, None
    if world > 1:
        # two different queries back to back through the peer exchange (no host sync between the
        # calls, so a fast rank's second call overlaps a slow rank's first merge), each checked
        # against the all-gather path
        ref1, ref2 = torch.empty_like(O), torch.empty_like(O)
        call(att, q, ref1)
        call(att, q2, ref2)
        O1, O2 = torch.empty_like(O), torch.empty_like(O)
        call(att_p2p, q, O1)
        call(att_p2p, q2, O2)
        torch.cuda.synchronize()
        assert att_p2p._p2p.status() == 0, "peer exchange wait expired"
        p2p_diff = max(float((O1.float() - ref1.float()).abs().max()), float((O2.float() - ref2.float()).abs().max()))
        assert p2p_diff < 1e-3, f"peer exchange differs from the all-gather path by {p2p_diff}"
        nccl_ms = timed(att)
    ms = timed(att_p2p)
    gbs = fd_bytes(Lt) / (ms * 1e-3) / 1e9
    wk = work if world == 1 else att_p2p._work
    assert L.fd_mh_status(wk.data_ptr(), Lr, FD_HEADS) == 0
    c5 = {"metric": "flash_decode_GBps", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world,
          "us_per_call": round(ms * 1000, 2), "higher_is_better": True, "scaling": "strong",
          "config": {"workload": "BASELINE configs[4]: 16x128, L=131072 split over the GPUs", "rows_per_gpu": Lr,
                     "exchange": "16x130 fp32 per rank stored into every rank's buffer over NVLink peer memory, "
                                 "flags, merge (one kernel)" if world > 1 else "none",
                     "nccl_allgather_us_per_call": round(nccl_ms * 1000, 2) if nccl_ms else None,
                     "p2p_vs_allgather_max_abs_diff": p2p_diff,
                     "l2": "inputs larger than L2 (1 GiB of K+V in total)"},
          "roofline": {"bound": "hbm", "achieved_per_gpu": round(gbs / world, 1), "peak": peak, "unit": "GB/s",
                       "frac": round(gbs / world / peak, 4), "peak_kind": peak_kind}}
    if world == 1 and refk is not None:
        nc = (Lt + 255) // 256
        Op = torch.empty(nc * 128, dtype=torch.float16, device=dev)
        lse = torch.empty(nc, dtype=torch.float32, device=dev)
        Or = torch.empty(FD_HEADS * 128, dtype=torch.float16, device=dev)

        rs = torch.cuda.Stream(device=dev)

        def ref():
            refk.fd_layer(q.data_ptr(), K.data_ptr(), V.data_ptr(), Or.data_ptr(), Op.data_ptr(), lse.data_ptr(),
                          Lt, FD_HEADS, FD_STRIDE, ctypes.c_void_p(rs.cuda_stream))

        rus = _graph_us(torch, rs, ref, max(1, args.steps), max(1, args.warmup))
        call()
        torch.cuda.synchronize()
        c5["reference_v5"] = {"us_per_call": round(rus, 1), "GBps": round(fd_bytes(Lt) / (rus * 1e-6) / 1e9, 1),
                              "max_abs_diff_vs_ours": float((O.float() - Or.float()).abs().max()),
                              "kind": "the reference's fd_v5_split_stage1 (512 chunks) + fd_opt_stage2 per head "
                                      "(compute_89 PTX JIT), CUDA graph"}
        c5["speedup_vs_reference"] = round(rus / (ms * 1000), 2)
    if att_p2p is not None:
        assert att_p2p._p2p.status() == 0
        att_p2p.close()
    res["config5"] = c5
    del K, V
    torch.cuda.empty_cache()
    return res


# ------------------------------------------------------------------ prefill (config 3)
def prefill_flops(N, c=QWEN):
    """GEMM FLOPs of an N-token prompt forward (no lm_head) plus causal attention (QK^T and PV)."""
    H, IM, NL = c["hidden_size"], c["intermediate_size"], c["num_layers"]
    gemm = 2 * N * (3 * H * H + H * H + 2 * IM * H + H * IM) * NL
    attn = 2 * 2 * H * (N * (N + 1) // 2) * NL
    return gemm, attn


def prefill_leg(eng, args, rank, world, local, pg):
    """Qwen-1.8B prompt forward of 2048 uniform-random ids through the public
    API (llmdiy_engine_prefill: ids uploaded from host, KV cache filled, synchronised), wall-clock
    per prefill, TFLOP/s against the measured dense fp16/bf16 tensor peak."""
    import numpy as np
    N = 2048
    ids = np.random.default_rng(PROMPT_SEED + rank).integers(0, QWEN["vocab_size"], N).tolist()
    for _ in range(max(3, args.warmup)):
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
    peak, kind = measured_tensor_peak()
    return {"metric": "prefill_ms", "value": round(dt * 1e3, 3), "unit": "ms", "n_gpus": world,
            "higher_is_better": False,
            "config": {"workload": "BASELINE configs[2]: Qwen-1.8B prefill of 2048 tokens "
                                   "(no lm_head; the last prompt token goes through decode)",
                       "timing": "wall clock around llmdiy_engine_prefill (host ids in, synchronised)"},
            "tflops": round(tf, 1), "gemm_tflop": round(gemm / 1e12, 3), "attention_tflop": round(attn / 1e12, 3),
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tf / peak, 4), "peak_kind": kind}}


# ------------------------------------------------------------------ our arm
def run_ours(args, rank, world, local, pg):
    import torch
    L = product_mod()

    torch.cuda.set_device(local)
    cfg = L.make_config(**QWEN, max_seqlen=ENGINE_MAX_SEQLEN)
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

    # the other configurations, in the same run (same collective order on every rank)
    extra = {}
    if not args.headline_only:
        extra["batch"] = batch_leg(eng, args, rank, world, local, pg)
        if world == 1:
            extra["prefill"] = prefill_leg(eng, args, rank, world, local, pg)
    eng.close()
    torch.cuda.empty_cache()
    if not args.headline_only:
        extra["fd_op"] = fd_op_leg(args, rank, world, local, pg)

    cpu, refgpu = None, None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        d = tempfile.mkdtemp()
        path = os.path.join(d, "qwen_random.bin")
        write_model_bin(path, threads)
        try:
            if not args.headline_only:
                refgpu = reference_gpu_leg(path, first)
            t_per = 8
            rate, dt = cpu_decode(path, threads, 1, args.cpu_tokens // t_per, t_per)
        finally:
            os.remove(path)
        cpu = {"value": round(rate, 4), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{args.cpu_tokens} greedy decode tokens at positions 127..382 after the 127-token "
                         f"prompt prefill, same weights, fp32 C restatement (oracle/qwen_oracle.c), {threads} "
                         f"threads, {dt:.1f} s"}

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
        if refgpu:
            line["reference_gpu"] = refgpu
        line.update(extra)
        print(json.dumps(line), flush=True)


def run_ncu_case():
    """Small case for ncu captures of decode_kernel: the Qwen-1.8B shapes with 4 layers (full vocab,
    0.95 GB of weights, larger than L2), a tensor-core prefill of 127 tokens, then one decode_kernel
    launch of 2 tokens (capture it with `-k regex:decode_kernel -c 1`)."""
    import torch
    L = product_mod()
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


def run_single_leg(args, rank, world, local, pg):
    """One configuration on its own (development and ncu captures): prints its object as a line."""
    import torch
    L = product_mod()
    torch.cuda.set_device(local)
    if args.workload == "fd-op":
        res = fd_op_leg(args, rank, world, local, pg)
        lines = list(res.values())
    else:
        eng = L.Engine(config=L.make_config(**QWEN, max_seqlen=ENGINE_MAX_SEQLEN), seed=SEED, device=local)
        lines = [batch_leg(eng, args, rank, world, local, pg) if args.workload == "batch"
                 else prefill_leg(eng, args, rank, world, local, pg)]
        eng.close()
    if rank == 0:
        for ln in lines:
            print(json.dumps(ln), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=256,
                    help="decode tokens of the CPU baseline sample (256 = the whole workload, ~15 s on 16 cores)")
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the host-side legs (CPU baseline and the reference engine on the GPU)")
    ap.add_argument("--headline-only", action="store_true", help="only the config-2 decode numbers")
    ap.add_argument("--ncu-case", action="store_true", help="run the small decode case used for ncu captures")
    ap.add_argument("--workload", default="decode", choices=["decode", "fd-op", "prefill", "batch"],
                    help="decode: the full line (headline config 2 plus the other configs' objects); "
                         "fd-op / prefill / batch: that configuration alone")
    args = ap.parse_args()
    if args.ncu_case:
        run_ncu_case()
        return
    rank, world, local, pg = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            if args.workload == "decode":
                run_reference(args, rank, world)
            elif rank == 0:
                print(json.dumps({"impl": "reference", "workload": args.workload, "unavailable":
                                  "the reference has no CPU path for this configuration; see the decode arm"}))
        elif args.workload == "decode":
            run_ours(args, rank, world, local, pg)
        else:
            run_single_leg(args, rank, world, local, pg)
    finally:
        if pg is not None:
            pg.destroy_process_group()


if __name__ == "__main__":
    main()
