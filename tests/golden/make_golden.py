"""Generates the golden fixtures in tests/golden/ from the reference's own
kernels and engine (LLM-inference-DIY), compiled from their sources by
`make -C oracle ref` into oracle/_ref as compute_89 PTX and JIT-run on a B200.

Run on a GPU box from the repository root:
    python tests/golden/make_golden.py OUTPUT_DIR [--engine]
It writes ref_ops.npz (seeded inputs and the reference kernels' outputs) and
ref_engine.json (token streams of the reference engine qwen_infer on a
seeded random-weight QWDF file).  Inputs are regenerated from the stored
seeds by the tests; the arrays stored are the reference outputs plus the
small inputs.
"""
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "llm-inference-diy_b200"))

import golden_inputs as gi  # noqa: E402


def main(outdir, engine=False):
    import torch

    import oracle as orc
    ref = orc.RefKernels()
    os.makedirs(outdir, exist_ok=True)

    keep = []  # device inputs stay referenced so the caching allocator cannot alias them

    def dev(a):
        a = np.ascontiguousarray(a)
        if a.dtype == np.float16:
            t = torch.from_numpy(a.view(np.int16).copy()).cuda()
        else:
            t = torch.from_numpy(a.copy()).cuda()
        keep.append(t)
        return t

    def host16(t):
        torch.cuda.synchronize()
        return t.cpu().numpy().view(np.float16)

    def z16(n):
        t = torch.zeros(n, dtype=torch.int16, device="cuda")
        keep.append(t)
        return t

    out = {}
    inp = gi.ops_inputs()
    # rmsnorm (run_tests.cu:55-99 shapes)
    x, w = inp["rms_x"], inp["rms_w"]
    o = z16(x.size)
    ref.rmsnorm(o.data_ptr(), dev(x).data_ptr(), dev(w).data_ptr(), x.size, 1e-6)
    out["rms_out"] = host16(o)
    # add_bias
    b_o, b_b = dev(inp["bias_out"]), dev(inp["bias_b"])
    ref.add_bias(b_o.data_ptr(), b_b.data_ptr(), inp["bias_out"].size)
    out["bias_res"] = host16(b_o)
    # swiglu
    o = z16(inp["sw_a"].size)
    ref.swiglu(o.data_ptr(), dev(inp["sw_a"]).data_ptr(), dev(inp["sw_b"]).data_ptr(), inp["sw_a"].size)
    out["sw_out"] = host16(o)
    # fused qkv rope cache, pos 3 and 300, max_seqlen 512
    for pos in gi.ROPE_POS:
        q = dev(inp["rope_qkv"])
        kc, vc = z16(512 * 2048), z16(512 * 2048)
        ref.fused_qkv_rope_cache(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos, 512, 16, 128)
        out[f"rope_q_{pos}"] = host16(q)
        out[f"rope_k_{pos}"] = host16(kc).reshape(512, 2048)[pos].copy()
        out[f"rope_v_{pos}"] = host16(vc).reshape(512, 2048)[pos].copy()
    # argmax cases
    for name, lg in gi.argmax_cases().items():
        r = torch.zeros(1, dtype=torch.int32, device="cuda")
        ref.argmax(r.data_ptr(), dev(lg).data_ptr(), lg.size)
        torch.cuda.synchronize()
        out[f"argmax_{name}"] = np.array([int(r.item())], np.int32)
    # hgemv, weight [K,N]
    o = z16(inp["gemv_B"].shape[1])
    ref.hgemv(dev(inp["gemv_A"]).data_ptr(), dev(inp["gemv_B"]).data_ptr(), o.data_ptr(), inp["gemv_B"].shape[1],
              inp["gemv_B"].shape[0])
    out["gemv_C"] = host16(o)
    # flash decoding: fused (L=200, stride 256) and split (L=1024, stride 128)
    o = z16(128)
    ref.fd_v5_fused(dev(inp["fd_q"]).data_ptr(), dev(inp["fdf_K"]).data_ptr(), dev(inp["fdf_V"]).data_ptr(),
                    o.data_ptr(), gi.FDF_L, gi.FDF_STRIDE)
    out["fdf_O"] = host16(o)
    nc = (gi.FDS_L + 255) // 256
    op, lse, o = z16(nc * 128), torch.zeros(nc, dtype=torch.float32, device="cuda"), z16(128)
    dq, dK, dV = dev(inp["fd_q"]), dev(inp["fds_K"]), dev(inp["fds_V"])
    ref.fd_v5_split_stage1(dq.data_ptr(), dK.data_ptr(), dV.data_ptr(), op.data_ptr(), lse.data_ptr(), gi.FDS_L, nc,
                           128)
    ref.fd_opt_stage2(op.data_ptr(), lse.data_ptr(), o.data_ptr(), nc)
    out["fds_Opart"] = host16(op)
    out["fds_LSE"] = lse.cpu().numpy()
    out["fds_O"] = host16(o)
    # hgemm 128^3 x0.1 (run_tests.cu:700-725)
    o = z16(128 * 128)
    ref.hgemm_swizzle_nn(dev(inp["gemm_A"]).data_ptr(), dev(inp["gemm_B"]).data_ptr(), o.data_ptr(), 128, 128, 128)
    out["gemm_C"] = host16(o).reshape(128, 128)
    # causal flash attention, one head, N=100
    n = gi.FA_N
    o = z16(n * 128)
    ref.flash_attn_causal_head(dev(inp["fa_Q"]).data_ptr(), dev(inp["fa_K"]).data_ptr(), dev(inp["fa_V"]).data_ptr(),
                               o.data_ptr(), n)
    out["fa_O"] = host16(o)
    np.savez_compressed(os.path.join(outdir, "ref_ops.npz"), **out)
    print("op fixtures written to", outdir)
    if not engine:
        return

    # Engine level: the reference engine binary on a seeded QWDF file.  Only
    # one-token prompts are run: with a longer prompt the reference's prefill
    # attention produced NaN on a B200, its argmax returned -1, and the next
    # step read the embedding row at index -1 (outside the wte allocation);
    # that recorded turn is kept in ref_engine.json and is not re-run.
    assert all(len(p) == 1 for p in gi.engine_prompts_rerun())
    import llmdiy_b200 as L
    d = tempfile.mkdtemp()
    path = os.path.join(d, "golden.bin")
    L.write_random_bin(path, L.make_config(**gi.ENGINE_CFG), seed=gi.ENGINE_SEED)
    lines = ["reset"] + [" ".join(map(str, p)) for p in gi.engine_prompts_rerun()] + ["exit"]
    r = subprocess.run([orc.REF_ENGINE, path], input="\n".join(lines) + "\n", capture_output=True, text=True,
                       timeout=1200)
    os.remove(path)
    turns, cur = [], None
    for line in r.stdout.splitlines():
        line = line.strip()
        if line == "[GENERATION_START]":
            cur = []
        elif line == "[GENERATION_END]":
            turns.append(cur)
            cur = None
        elif cur is not None and line.lstrip("-").isdigit():
            cur.append(int(line))
    res = {"config": gi.ENGINE_CFG, "seed": gi.ENGINE_SEED, "prompts": gi.engine_prompts_rerun(), "tokens": turns,
           "returncode": r.returncode, "engine": "oracle/_ref/qwen_infer_ref (compute_89 PTX, JIT on B200)"}
    json.dump(res, open(os.path.join(outdir, "ref_engine.json"), "w"))
    print("golden fixtures written to", outdir, "turns:", [len(t) for t in turns])


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    if len(args) != 1:
        sys.exit("usage: make_golden.py OUTPUT_DIR [--engine]")
    main(args[0], engine="--engine" in sys.argv)
