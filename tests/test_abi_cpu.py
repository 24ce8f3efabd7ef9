"""CPU checks of the product library: it loads without a GPU, exports every
symbol include/*.h declares, its QWDF tooling round-trips, and the drop-in
driver fails cleanly on bad inputs (no GPU compute is called here)."""
import ctypes
import os
import subprocess
import tempfile

import numpy as np
import pytest

import llmdiy_b200 as L


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    names = L.declared_symbols()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_kernel_header_cites_reference():
    text = open(os.path.join(L.INCLUDE_DIR, "llmdiy_kernels.h")).read()
    for ref in ("rmsnorm.cuh:6", "bias.cuh:6", "swiglu.cuh:6", "fused_qkv_rope_cache.cuh:6",
                "flash_decode_q1_opt.cuh:434", "flash_decode_q1_opt.cuh:548", "flash_decode_q1_opt.cuh:666",
                "argmax.cuh:7", "hgemm_final.cuh:274", "hgemm_mma_swizzle.cuh:414", "flash_attn.cu:1854",
                "gather_qkv.cuh", "transpose.cuh:6"):
        assert ref in text, ref


SMALL = L.make_config(vocab_size=256, hidden_size=2048, num_layers=1, num_heads=16, intermediate_size=64,
                      max_seqlen=16)


def test_qwdf_writer_layout_and_determinism():
    d = tempfile.mkdtemp()
    p1, p2 = os.path.join(d, "a.bin"), os.path.join(d, "b.bin")
    L.write_random_bin(p1, SMALL, seed=11)
    L.write_random_bin(p2, SMALL, seed=11, nthreads=3)
    b1, b2 = open(p1, "rb").read(), open(p2, "rb").read()
    assert b1 == b2  # thread count does not change the values
    c = L.read_bin_config(p1)
    assert c.as_dict() == SMALL.as_dict()
    H, V, IM = 2048, 256, 64
    expect = 28 + 2 * (V * H + (H + 3 * H * H + 3 * H + H * H + H + 2 * IM * H + H * IM) + H + V * H)
    assert len(b1) == expect
    hdr = np.frombuffer(b1[:28], "<u4")
    assert hdr[0] == 0x46445751
    # tensor 0 = wte: N(0, 0.02); tensor 1 = ln_1: all ones; fill_tensor reproduces the file bytes
    wte = np.frombuffer(b1[28:28 + 2 * V * H], np.float16)
    assert abs(float(wte.astype(np.float64).std()) - 0.02) < 1e-3
    assert np.array_equal(L.fill_tensor(SMALL, 0, 11, 0, V * H).view(np.float16), wte)
    ln1 = np.frombuffer(b1[28 + 2 * V * H: 28 + 2 * V * H + 2 * H], np.float16)
    assert np.all(ln1 == 1.0)
    part = L.fill_tensor(SMALL, 0, 11, 1001, 77)  # odd offset keeps Box-Muller pairs aligned
    assert np.array_equal(part.view(np.float16), wte[1001:1078])
    assert not np.array_equal(L.fill_tensor(SMALL, 0, 12, 0, 64), L.fill_tensor(SMALL, 0, 11, 0, 64))
    os.remove(p1)
    os.remove(p2)


def test_qwdf_rejects_bad_files():
    d = tempfile.mkdtemp()
    bad = os.path.join(d, "bad.bin")
    with open(bad, "wb") as f:
        f.write(b"\x00" * 64)
    with pytest.raises(L.LlmdiyError):
        L.read_bin_config(bad)
    trunc = os.path.join(d, "trunc.bin")
    L.write_random_bin(trunc, SMALL, seed=1)
    data = open(trunc, "rb").read()
    with open(trunc, "wb") as f:
        f.write(data[: len(data) // 2])
    with pytest.raises(L.LlmdiyError):
        L.read_bin_config(trunc)
    with pytest.raises(L.LlmdiyError):
        L.read_bin_config(os.path.join(d, "missing.bin"))


def test_qwdf_validate_verdicts():
    """The validator (llmdiy_qwdf_validate) accepts a well-formed file and names what is wrong with
    bad ones: magic, length, a non-finite value (with its tensor), an unsupported config, a missing file."""
    import json
    import sys
    d = tempfile.mkdtemp()
    good = os.path.join(d, "good.bin")
    L.write_random_bin(good, SMALL, seed=5)
    r = L.validate_bin(good)
    assert r["ok"] and r["status"] == 0 and r["nonfinite"] == 0, r
    assert r["config"] == SMALL.as_dict()

    data = bytearray(open(good, "rb").read())
    magic = os.path.join(d, "magic.bin")
    open(magic, "wb").write(b"XXXX" + bytes(data[4:]))
    r = L.validate_bin(magic)
    assert r["status"] == L.ERR_FORMAT and "magic" in r["message"], r

    trunc = os.path.join(d, "trunc.bin")
    open(trunc, "wb").write(bytes(data[:-2]))
    r = L.validate_bin(trunc)
    assert r["status"] == L.ERR_FORMAT and "truncated" in r["message"], r

    # plant a NaN and an Inf in layer 0's qkv_w (tensor 2: after wte and ln_1)
    H, V = SMALL.hidden_size, SMALL.vocab_size
    off = 28 + 2 * (V * H + H) + 2 * 1000
    nan = bytearray(data)
    nan[off:off + 2] = (0x7E00).to_bytes(2, "little")
    nan[off + 2:off + 4] = (0x7C00).to_bytes(2, "little")
    pn = os.path.join(d, "nan.bin")
    open(pn, "wb").write(bytes(nan))
    r = L.validate_bin(pn)
    assert r["status"] == L.ERR_FORMAT and r["nonfinite"] == 2 and "layer 0 qkv_w" in r["message"], r

    trail = os.path.join(d, "trail.bin")
    open(trail, "wb").write(bytes(data) + b"\0" * 6)
    r = L.validate_bin(trail)
    assert r["ok"] and "trailing" in r["message"], r

    odd = L.make_config(vocab_size=64, hidden_size=256, num_layers=1, num_heads=2, intermediate_size=64,
                        max_seqlen=8)
    po = os.path.join(d, "odd.bin")
    L.write_random_bin(po, odd, seed=1)
    r = L.validate_bin(po)
    assert r["status"] == L.ERR_UNSUPPORTED and "hidden_size 2048" in r["message"], r

    r = L.validate_bin(os.path.join(d, "missing.bin"))
    assert r["status"] == L.ERR_FILE and r["config"] is None, r

    # the command-line form
    cli = L.__file__
    out = subprocess.run([sys.executable, cli, "validate", good], capture_output=True, text=True)
    assert out.returncode == 0 and json.loads(out.stdout)["ok"], out
    out = subprocess.run([sys.executable, cli, "validate", pn], capture_output=True, text=True)
    assert out.returncode == 1 and not json.loads(out.stdout)["ok"], out
    for f in (good, magic, trunc, pn, trail, po):
        os.remove(f)


def test_driver_reports_missing_weights():
    # qwen_infer.cu:121-124: an unreadable model file ends the process with status 1
    if not os.path.exists(L.DRIVER_PATH):
        pytest.skip("driver not built")
    r = subprocess.run([L.DRIVER_PATH, "/nonexistent/model.bin"], capture_output=True, text=True, timeout=60,
                       stdin=subprocess.DEVNULL)
    assert r.returncode == 1
    assert "[ENGINE_READY]" not in r.stdout


def test_engine_create_fails_cleanly_without_valid_config():
    cfg = L.make_config(hidden_size=1024, num_heads=8)  # not the 2048/16x128 the fused kernel is built for
    with pytest.raises(L.LlmdiyError):
        L.Engine(config=cfg)


def test_oracle_random_writer_matches_library():
    """The oracle's seeded writer (used where the product library must not be loaded: the bench's
    reference arm) produces the library's file byte for byte, here with two layers and a ragged
    intermediate size."""
    import oracle as orc
    cfg = L.make_config(vocab_size=300, hidden_size=2048, num_layers=2, num_heads=16, intermediate_size=96,
                        max_seqlen=32)
    d = tempfile.mkdtemp()
    p1, p2 = os.path.join(d, "lib.bin"), os.path.join(d, "orc.bin")
    L.write_random_bin(p1, cfg, seed=1234, nthreads=4)
    orc.Oracle().write_random_bin(p2, **cfg.as_dict(), seed=1234, nthreads=3)
    assert open(p1, "rb").read() == open(p2, "rb").read()
    os.remove(p1)
    os.remove(p2)


def test_hgemm_dispatch_rule():
    """llmdiy_hgemm_swizzle_nn_path (host only): the tcgen05 kernel whenever a TMA descriptor can
    address the row pitches (N, K multiples of 8 elements, 16-byte aligned pointers)."""
    a = 1 << 20
    assert L.hgemm_swizzle_nn_path(a, a, a, 2048, 5504, 2048) == 1
    assert L.hgemm_swizzle_nn_path(a, a, a, 300, 200, 104) == 1
    assert L.hgemm_swizzle_nn_path(a, a, a, 300, 200, 100) == 0
    assert L.hgemm_swizzle_nn_path(a, a, a, 8, 12, 8) == 0
    assert L.hgemm_swizzle_nn_path(a + 8, a, a, 64, 64, 64) == 0
    assert L.hgemm_swizzle_nn_path(a, a, a, 0, 64, 64) == -1
