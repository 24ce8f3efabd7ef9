"""Engine-level parity: the persistent decode kernel (through the C ABI)
against the CPU oracle model on the same seeded QWDF weights, plus the
reference engine itself (oracle/_ref/qwen_infer_ref, compute_89 PTX) when it
is built.  Bar (north_star): logits within 2e-2 abs, identical greedy
token streams (a divergence is accepted only at a near-tie, reported with
its top-2 margin)."""
import os
import subprocess
import tempfile

import numpy as np
import pytest

import llmdiy_b200 as L

pytestmark = pytest.mark.gpu

SMALL = dict(vocab_size=8192, hidden_size=2048, num_layers=2, num_heads=16, intermediate_size=5504, max_seqlen=1024)
SEED = 2024


@pytest.fixture(scope="module")
def small_bin():
    d = tempfile.mkdtemp()
    p = os.path.join(d, "small.bin")
    L.write_random_bin(p, L.make_config(**SMALL), seed=SEED)
    yield p
    os.remove(p)


@pytest.fixture(scope="module")
def engine(small_bin):
    e = L.Engine(small_bin)
    yield e
    e.close()


@pytest.fixture(scope="module")
def omodel(small_bin):
    import oracle as orc
    return orc.OracleModel(small_bin, nthreads=os.cpu_count() or 8)


def test_random_engine_equals_file_engine(small_bin, engine):
    e2 = L.Engine(config=L.make_config(**SMALL), seed=SEED)
    engine.reset()
    e2.reset()
    a = engine.step(11, 0)
    la = engine.logits().copy()
    b = e2.step(11, 0)
    assert a == b
    assert np.array_equal(la.view(np.uint16), e2.logits().view(np.uint16))
    e2.close()


def test_step_matches_oracle(engine, omodel):
    """40 teacher-forced steps: both sides get the oracle's token at every step, so a near-tie
    cannot end the check early; a differing argmax is accepted only where the oracle's logits of
    the two candidates are at most one fp16 ulp apart."""
    from gpu_util import f16_ulp
    engine.reset()
    omodel.reset()
    tok, n_diff = 123, 0
    for pos in range(40):
        g = engine.step(tok, pos)
        lg = engine.logits().astype(np.float32)
        o, olg, _ = omodel.step(tok, pos, want_logits=True)
        olg = olg.astype(np.float32)
        err = float(np.max(np.abs(lg - olg)))
        assert err < 2e-2, (pos, err)
        if g != o:
            n_diff += 1
            assert olg[o] - olg[g] <= f16_ulp(olg[o]), (pos, g, o, float(olg[o] - olg[g]))
        tok = o
    assert n_diff <= 2, n_diff
    k, v = engine.kv(1, 0, 40)
    ok_, ov = omodel.kv(1, 0, 40)
    assert float(np.max(np.abs(k.astype(np.float32) - ok_.astype(np.float32)))) < 2e-2
    assert float(np.max(np.abs(v.astype(np.float32) - ov.astype(np.float32)))) < 2e-2


def test_prefill_matches_oracle(engine, omodel):
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, SMALL["vocab_size"], 100).tolist()
    engine.reset()
    omodel.reset()
    engine.prefill(prompt)
    omodel.prefill(prompt)
    for layer in (0, 1):
        k, v = engine.kv(layer, 0, 100)
        ok_, ov = omodel.kv(layer, 0, 100)
        assert float(np.max(np.abs(k.astype(np.float32) - ok_.astype(np.float32)))) < 2e-2
        assert float(np.max(np.abs(v.astype(np.float32) - ov.astype(np.float32)))) < 2e-2


def test_long_prefill_matches_oracle(engine, omodel):
    """A prompt spanning several 64-row query tiles and key tiles of the prefill's flash attention
    and several 128-row GEMM tiles: the KV rows of the last layer (which depend on every earlier
    layer's attention) against the oracle's prefill."""
    rng = np.random.default_rng(15)
    prompt = rng.integers(0, SMALL["vocab_size"], 333).tolist()
    engine.reset()
    omodel.reset()
    engine.prefill(prompt)
    omodel.prefill(prompt)
    k, v = engine.kv(1, 0, 333)
    ok_, ov = omodel.kv(1, 0, 333)
    assert float(np.max(np.abs(k.astype(np.float32) - ok_.astype(np.float32)))) < 2e-2
    assert float(np.max(np.abs(v.astype(np.float32) - ov.astype(np.float32)))) < 2e-2


def test_generate_stream_matches_oracle(engine, omodel):
    rng = np.random.default_rng(6)
    prompt = rng.integers(0, SMALL["vocab_size"], 64).tolist()
    got = engine.generate(prompt, 96, stop_on_eos=False)
    ref = omodel.generate(prompt, 96, stop_on_eos=False)
    assert len(got) == 96
    n_same = next((i for i, (a, b) in enumerate(zip(got, ref)) if a != b), len(got))
    assert n_same >= 64, (n_same, got[:n_same + 1], ref[:n_same + 1])


def test_step_api_equals_generate(engine):
    prompt = [5, 6, 7, 8]
    g = engine.generate(prompt, 12, stop_on_eos=False)
    engine.reset()
    engine.prefill(prompt[:-1])
    t, pos, s = prompt[-1], len(prompt) - 1, []
    for _ in range(12):
        t = engine.step(t, pos)
        pos += 1
        s.append(t)
    assert s == g


def test_decode_async_status(engine):
    engine.reset()
    engine.prefill([1, 2, 3])
    engine.decode_async(4, 3, 20)
    torch = __import__("torch")
    torch.cuda.synchronize()
    assert engine.status() == 20
    toks = engine.tokens(20)
    assert all(0 <= t < SMALL["vocab_size"] for t in toks)


def test_position_bounds_rejected(engine):
    with pytest.raises(L.LlmdiyError):
        engine.step(1, SMALL["max_seqlen"])
    with pytest.raises(L.LlmdiyError):
        engine.step(SMALL["vocab_size"], 0)
    # the engine stays usable after a rejected call
    assert 0 <= engine.step(1, 0) < SMALL["vocab_size"]


def _run_driver(exe, bin_path, lines, env=None, timeout=300):
    p = subprocess.run([exe, bin_path], input="\n".join(lines) + "\n", capture_output=True, text=True,
                       timeout=timeout, env=env)
    return p


def _parse_turns(stdout):
    turns, cur = [], None
    for line in stdout.splitlines():
        line = line.strip()
        if line == "[GENERATION_START]":
            cur = []
        elif line == "[GENERATION_END]":
            turns.append(cur)
            cur = None
        elif cur is not None and (line.isdigit() or (line.startswith("-") and line[1:].isdigit())):
            cur.append(int(line))
    return turns


def test_driver_protocol(small_bin, engine):
    env = dict(os.environ, LLMDIY_MAX_NEW_TOKENS="24")
    p = _run_driver(L.DRIVER_PATH, small_bin, ["reset", "5 6 7 8", "reset", "9", "12 x 3", "exit"], env=env)
    assert p.returncode == 0, p.stderr
    assert "[ENGINE_READY]" in p.stdout
    assert p.stdout.count("[RESET_DONE]") == 2
    turns = _parse_turns(p.stdout)
    assert len(turns) == 3
    assert turns[0] == engine.generate([5, 6, 7, 8], 24, stop_on_eos=True)
    assert turns[1] == engine.generate([9], 24, stop_on_eos=True)
    assert turns[2] == []  # malformed id: empty turn, process keeps serving
    assert "invalid token id" in p.stderr


def _oracle_stream_agrees(omodel, prompt, got):
    """The oracle's greedy stream for `prompt` against `got`: equal, or first different at a step
    where the oracle's logits of its token and of ours are at most one fp16 ulp apart (a near tie).
    Returns the number of equal leading tokens."""
    from gpu_util import f16_ulp
    omodel.reset()
    ref = omodel.generate(prompt, len(got), stop_on_eos=False)
    first = next((i for i, (a, b) in enumerate(zip(got, ref)) if a != b), len(got))
    if first < len(got):
        omodel.reset()
        omodel.prefill(prompt[:-1])
        tok, pos = prompt[-1], len(prompt) - 1
        for i in range(first + 1):
            o, lg, _ = omodel.step(tok, pos, want_logits=True)
            tok, pos = o, pos + 1
        margin = float(lg[o]) - float(lg[got[first]])
        assert margin <= float(f16_ulp(lg[o])), (prompt, first, got, ref, margin)
    return first


def test_driver_batch_verb(small_bin, engine, omodel):
    """The driver's "batch" verb (continuous batching, two slots for six requests): every request
    gets its own turn's tokens, each request's stream equals the CPU oracle's greedy stream for its
    prompt (or first differs at a near tie), a malformed request is rejected, and plain turns still
    work after."""
    env = dict(os.environ, LLMDIY_MAX_NEW_TOKENS="12", LLMDIY_IGNORE_EOS="1", LLMDIY_MAX_BATCH="2",
               LLMDIY_BATCH_MAX_LEN="256")
    prompts = [[5, 6, 7, 8], [9], [100, 200, 300], [11, 12], [1, 2, 3, 4, 5, 6, 7], [40, 41]]
    lines = ["batch"] + [" ".join(map(str, q)) for q in prompts] + ["12 x", "end", "5 6 7 8", "exit"]
    p = _run_driver(L.DRIVER_PATH, small_bin, lines, env=env)
    assert p.returncode == 0, p.stderr
    out = p.stdout.splitlines()
    i0, i1 = out.index("[BATCH_START] 7"), out.index("[BATCH_END]")
    got, done = {r: [] for r in range(7)}, []
    for line in out[i0 + 1:i1]:
        if line.startswith("[DONE] "):
            done.append(int(line.split()[1]))
        else:
            r, t = map(int, line.split())
            assert r not in done
            got[r].append(t)
    assert sorted(done) == list(range(7))
    for r, q in enumerate(prompts):
        assert len(got[r]) == 12, (r, got[r])
        n_same = _oracle_stream_agrees(omodel, q, got[r])
        print(f"batch request {r}: {n_same} of 12 tokens equal to the oracle's stream")
    assert got[6] == [] and "invalid token id" in p.stderr
    turns = _parse_turns("\n".join(out[i1 + 1:]))
    assert turns == [engine.generate([5, 6, 7, 8], 12, stop_on_eos=False)]


def test_reference_engine_stream(small_bin, engine):
    """The reference engine, built from its sources as compute_89 PTX, on the same weights."""
    import oracle as orc
    if not os.path.exists(orc.REF_ENGINE):
        pytest.skip("reference engine not built")
    p = _run_driver(orc.REF_ENGINE, small_bin, ["reset", "77", "exit"], timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    ref = _parse_turns(p.stdout)[0]
    ours = engine.generate([77], len(ref), stop_on_eos=True)
    n_same = next((i for i, (a, b) in enumerate(zip(ours, ref)) if a != b), min(len(ours), len(ref)))
    # one-token prompt: the reference runs only its decode path (no fp16-accumulating prefill)
    assert n_same >= min(64, len(ref)), (n_same, ours[:70], ref[:70])


def test_chunked_prefill_matches_oracle():
    """A prompt longer than the prefill's 2048-row chunk: the second chunk (700 rows at positions
    2048..2747, six q tiles of 34 to 44 key tiles each) attends over the first chunk's cached rows.
    KV rows of the last layer, which depend on the first layer's attention, against the oracle
    across both chunks."""
    import oracle as orc
    cfg = dict(SMALL, max_seqlen=2800)
    d = tempfile.mkdtemp()
    p = os.path.join(d, "chunk.bin")
    L.write_random_bin(p, L.make_config(**cfg), seed=SEED + 1)
    e = L.Engine(p)
    m = orc.OracleModel(p, nthreads=os.cpu_count() or 8)
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, cfg["vocab_size"], 2748).tolist()
    e.prefill(prompt)
    m.prefill(prompt)
    for lo, n in ((0, 16), (1000, 64), (1900, 148), (2040, 60), (2300, 64), (2680, 68)):
        k, v = e.kv(1, lo, n)
        ok_, ov = m.kv(1, lo, n)
        assert float(np.max(np.abs(k.astype(np.float32) - ok_.astype(np.float32)))) < 2e-2, lo
        assert float(np.max(np.abs(v.astype(np.float32) - ov.astype(np.float32)))) < 2e-2, lo
    e.close()
    m.close()
    os.remove(p)
