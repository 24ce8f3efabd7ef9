"""Batched greedy decode (include/llmdiy_batch.h) against the CPU oracle run one
sequence at a time (QwenEngine::prefill + step semantics): sequences with ragged
prompt lengths are prefilled into their own cache regions, then decoded together.
Bars (north_star): greedy streams identical for the first tokens of every
sequence, KV rows and logits within 2e-2 of the oracle."""
import os
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


def test_batch_matches_oracle_per_sequence(engine, omodel):
    rng = np.random.default_rng(41)
    lens = [5, 37, 100, 1, 600]
    prompts = [rng.integers(0, SMALL["vocab_size"], n).tolist() for n in lens]
    steps = 24
    b = L.Batch(engine, max_batch=len(prompts), max_len=700)
    for s, p in enumerate(prompts):
        b.prefill(s, p[:-1])
    toks = b.decode([p[-1] for p in prompts], [len(p) - 1 for p in prompts], steps)
    assert toks.shape == (steps, len(prompts))
    for s, p in enumerate(prompts):
        omodel.reset()
        ref = omodel.generate(p, steps, stop_on_eos=False)
        got = toks[:, s].tolist()
        n_same = next((i for i, (a, c) in enumerate(zip(got, ref)) if a != c), steps)
        assert n_same >= 16, (s, n_same, got, ref)
        if n_same == steps:
            # the cache rows written by prefill and by the batched steps
            n = len(p) - 1 + steps
            k, v = b.kv(s, 1, 0, n)
            ok_, ov = omodel.kv(1, 0, n)
            assert float(np.max(np.abs(k.astype(np.float32) - ok_.astype(np.float32)))) < 2e-2
            assert float(np.max(np.abs(v.astype(np.float32) - ov.astype(np.float32)))) < 2e-2
    b.close()


def test_batch_decode_twice_and_logits(engine, omodel):
    """A second decode call on the same batch (replaying its captured step) continues correctly,
    and the last step's logits match the oracle's step within 2e-2."""
    rng = np.random.default_rng(43)
    prompts = [rng.integers(0, SMALL["vocab_size"], n).tolist() for n in (9, 70)]
    b = L.Batch(engine, max_batch=2, max_len=200)
    for s, p in enumerate(prompts):
        b.prefill(s, p[:-1])
    t1 = b.decode([p[-1] for p in prompts], [len(p) - 1 for p in prompts], 4)
    t2 = b.decode(t1[-1].tolist(), [len(p) + 3 for p in prompts], 4)
    for s, p in enumerate(prompts):
        omodel.reset()
        ref = omodel.generate(p, 8, stop_on_eos=False)
        assert t1[:, s].tolist() + t2[:, s].tolist() == ref, s
        # the oracle's last step (token ref[-2] at position len+6) against the batch's logits
        _, lg, _ = omodel.step(ref[-2], len(p) + 6, want_logits=True)
        got = b.logits(s).astype(np.float32)
        assert float(np.max(np.abs(got - lg.astype(np.float32)))) < 2e-2
    b.close()


def test_batch_rejects_bad_arguments(engine):
    b = L.Batch(engine, max_batch=2, max_len=16)
    with pytest.raises(L.LlmdiyError):
        b.decode([1, 2, 3], [0, 0, 0], 1)  # more sequences than max_batch
    with pytest.raises(L.LlmdiyError):
        b.decode([1, 2], [10, 0], 8)  # positions beyond max_len
    with pytest.raises(L.LlmdiyError):
        b.decode([SMALL["vocab_size"], 2], [0, 0], 1)  # token id out of range
    with pytest.raises(L.LlmdiyError):
        b.prefill(2, [1, 2])  # sequence index out of range
    b.close()
    with pytest.raises(L.LlmdiyError):
        L.Batch(engine, max_batch=65, max_len=16)


def test_batch_weight_row_gemms_match_splitk_at_64(engine, monkeypatch):
    """The step's GEMMs at the full batch of 64 rows: the weight-row GEMMs (K split over a
    thread-block cluster, partials summed in shared memory; LLMDIY_BATCH_WROWS=1) against the
    split-K path (per-slice partials in HBM and a reduce launch) on the same caches
    and tokens.  Both accumulate in fp32; logits within 2e-2, greedy tokens equal except
    where the two logits' top-2 are within that tolerance."""
    rng = np.random.default_rng(47)
    B, steps = 64, 1
    lens = rng.integers(1, 300, B).tolist()
    toks = rng.integers(0, SMALL["vocab_size"], B).tolist()
    out = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("LLMDIY_BATCH_WROWS", mode)
        b = L.Batch(engine, max_batch=B, max_len=320)
        for s in range(B):
            b.fill_random(s, lens[s], seed=500 + s)
        t = b.decode(toks, lens, steps)
        out[mode] = (t, np.stack([b.logits(s).astype(np.float32) for s in range(B)]))
        b.close()
    (t0, l0), (t1, l1) = out["0"], out["1"]
    assert float(np.max(np.abs(l0 - l1))) < 2e-2
    for s in range(B):
        if t0[-1, s] != t1[-1, s]:
            top = np.sort(l1[s])[-2:]
            assert top[1] - top[0] < 2e-2, s


def test_batch_overlapped_launch_matches_serial(engine, monkeypatch):
    """The batched step with programmatic dependent launch (the default: every step kernel may
    start before the previous one ends and waits on it in every CTA) against plain serial
    launches (LLMDIY_BATCH_PDL=0) on the same caches and tokens: identical tokens and logits
    bit for bit, over several steps at a ragged batch."""
    rng = np.random.default_rng(53)
    B, steps = 24, 6
    lens = rng.integers(1, 900, B).tolist()
    toks = rng.integers(0, SMALL["vocab_size"], B).tolist()
    out = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("LLMDIY_BATCH_PDL", mode)
        b = L.Batch(engine, max_batch=B, max_len=920)
        for s in range(B):
            b.fill_random(s, lens[s], seed=900 + s)
        t = b.decode(toks, lens, steps)
        out[mode] = (t, np.stack([b.logits(s).view(np.uint16) for s in range(B)]))
        b.close()
    assert np.array_equal(out["0"][0], out["1"][0])
    assert np.array_equal(out["0"][1], out["1"][1])


@pytest.mark.parametrize("B", [5, 64])
def test_batch_fused_residual_norm_matches_separate(engine, monkeypatch, B):
    """o_proj and c_proj slice sums fused with the following RMSNorm (the default: one launch that
    sums the split-K slices of a row in slice order, adds the residual and normalises the row)
    against the reduce kernel + RMSNorm kernel pair (LLMDIY_BATCH_FUSED_NORM=0): the same arithmetic
    in the same order, so identical tokens and logits bit for bit over several steps."""
    rng = np.random.default_rng(67 + B)
    steps = 4
    lens = rng.integers(1, 600, B).tolist()
    toks = rng.integers(0, SMALL["vocab_size"], B).tolist()
    out = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("LLMDIY_BATCH_FUSED_NORM", mode)
        b = L.Batch(engine, max_batch=B, max_len=620)
        for s in range(B):
            b.fill_random(s, lens[s], seed=800 + s)
        t = b.decode(toks, lens, steps)
        out[mode] = (t, np.stack([b.logits(s).view(np.uint16) for s in range(B)]))
        b.close()
    assert np.array_equal(out["0"][0], out["1"][0])
    assert np.array_equal(out["0"][1], out["1"][1])
