"""The reference's own T2S test files, compiled against this repository's drop-in headers.

GPT-SoVITS.cpp's tests/t2s/test_t2s_infer.cpp (the end-to-end prefill + decode loop,
:158-472) and tests/t2s/test_t2s_loader.cpp are compiled unchanged against
include/gpt_sovits/t2s.h and the ggml type shim, linked to libt2sx.so.  Two helpers are swapped:
GoogleTest (absent here) by the minimal stand-in in tests/cpp/gtest_min, and the backend helper
tests/common/test_backend.h by tests/cpp/gtest_min/test_backend.h, whose one line creates a CUDA
backend (ggml_backend_cuda_init(0)) instead of ggml's CPU one -- the only change a caller makes.

The CPU test builds the binaries into tests/cpp/_ref_bin (only where the reference sources are
present; nothing is copied from them).  The GPU test runs those binaries on synthetic GGUF files
of the reference's model shapes: every loader test passes, and in the infer suite the three
F16-KV configurations pass (prefill, 200 stochastic decode steps, token checks) while the nine
others fail at t2s_session_init, which refuses KV types other than F16 (this path keeps an
f16 cache).
"""
import os
import re
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gpt-sovits.cpp_b200")
GMIN = os.path.join(ROOT, "tests", "cpp", "gtest_min")
BIN = os.path.join(ROOT, "tests", "cpp", "_ref_bin")
REF = "/root/reference"
SUITES = ("test_t2s_infer", "test_t2s_loader")


def test_reference_t2s_tests_build_against_the_drop_in(t2sx_mod):
    srcs = [os.path.join(REF, "tests", "t2s", s + ".cpp") for s in SUITES]
    if not all(os.path.exists(s) for s in srcs):
        pytest.skip("the reference sources are not present on this machine")
    gxx = shutil.which("g++")
    assert gxx, "g++ is required"
    os.makedirs(BIN, exist_ok=True)
    for name, src in zip(SUITES, srcs):
        out = os.path.join(BIN, name)
        cmd = [gxx, "-std=c++17", "-O1", "-Wall", "-Wno-unused-function", "-Wno-unused-variable", "-include", "cstring",
               "-I", GMIN, "-I", os.path.join(ROOT, "include"), "-I", os.path.join(REF, "tests", "common"),
               '-DT2S_TEST_DIR="t2s_test_data/"', src, os.path.join(REF, "tests", "common", "cnpy.cpp"),
               os.path.join(GMIN, "gtest_main.cpp"), "-L", PKG, "-lt2sx", "-lz", f"-Wl,-rpath,{PKG}", "-o", out]
        r = subprocess.run(cmd, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        assert os.path.exists(out)


def _save_npy_f32(path, a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    np.save(path, a)


def _results(stdout):
    return dict(re.findall(r"^RESULT (\S+) (PASSED|FAILED|SKIPPED)$", stdout, flags=re.M))


@pytest.mark.gpu
def test_reference_t2s_tests_run_on_the_gpu(t2sx_mod, orc, tmp_path):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required")
    bins = [os.path.join(BIN, s) for s in SUITES]
    if not all(os.path.exists(b) for b in bins):
        pytest.skip("reference test binaries were not built (their sources are not on this machine)")
    import synth
    data = tmp_path / "t2s_test_data"
    (data / "models").mkdir(parents=True)
    (data / "ref").mkdir()
    models = {"s1v3-s2Gv2ProPlus-f16.gguf": "f16", "s1v3-s2Gv2Pro-f16.gguf": "f16", "s1v3-s2Gv2Pro-q8.gguf": "q8_0",
              "s1v3-s2Gv2Pro-q4.gguf": "q4_0"}
    for name, wt in models.items():
        os.symlink(synth.ensure_gguf(wt, 0, n_layer=24), data / "models" / name)
    # the prefill input the infer suite reads: [52 reference + 28 input text rows | 113 prompt rows]
    m = orc.Model(synth.ensure_gguf("f16", 0, n_layer=24))
    ph, bert, sem = synth.session_inputs(7, 80, 113)
    x = m.embed_prefill(ph, bert, sem)
    m.close()
    _save_npy_f32(data / "ref" / "xy_pos.npy", x[None])
    _save_npy_f32(data / "ref" / "xy_dec.npy", np.zeros_like(x)[None])   # compared only with an F32 cache
    _save_npy_f32(data / "ref" / "k_cache.npy", np.zeros((24, 193, 512), np.float32))
    _save_npy_f32(data / "ref" / "v_cache.npy", np.zeros((24, 193, 512), np.float32))

    r = subprocess.run([bins[1]], cwd=tmp_path, capture_output=True, text=True, timeout=600)
    res = _results(r.stdout)
    assert r.returncode == 0 and len(res) == 3 and set(res.values()) == {"PASSED"}, r.stdout + r.stderr

    r = subprocess.run([bins[0]], cwd=tmp_path, capture_output=True, text=True, timeout=1200)
    res = _results(r.stdout)
    assert len(res) == 12, r.stdout + r.stderr
    for name, outcome in res.items():
        want = "PASSED" if name.endswith("_kv_f16") else "FAILED"
        assert outcome == want, (name, outcome, r.stdout[-4000:], r.stderr[-2000:])
    for suffix in ("f16", "q8", "q4"):
        toks = np.load(data / "ref" / f"sampled_tokens_{suffix}_kvf16.npy")
        assert toks.size > 1 and toks.min() >= 0 and toks.max() < 1025
    assert "kv_cache_type f32 is not supported" in r.stderr
