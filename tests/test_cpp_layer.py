"""The reference-compatible C++ interface (include/gpt_sovits/t2s.h + the ggml type shim) as a
C++ host uses it.

tests/cpp/t2s_decode_loop.cpp is the reference's decode loop (test_t2s_infer.cpp:204-421: flex-plan
prefill, persistent decode graph driven through ggml_backend_tensor_set / decode_advance /
ggml_backend_graph_compute / ggml_backend_tensor_get, then a mixed prefill/decode plan) written
against that header; it is compiled with g++ and linked to libt2sx.so.  On a GPU its tokens, the
flex graph's y rows and the layer-0 K cache read through the tensor views must equal the oracle's;
illegal slot transitions must abort through GGML_ASSERT, as in the reference (death-tested in
test_t2s_session.cpp:1008-1031).
"""
import json
import os
import shutil
import signal
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gpt-sovits.cpp_b200")
SRC = os.path.join(ROOT, "tests", "cpp", "t2s_decode_loop.cpp")


def _compile(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.fail("g++ is required to build the C++ host program")
    exe = str(tmp_path / "t2s_decode_loop")
    cmd = [gxx, "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"), SRC,
           "-L", PKG, "-lt2sx", f"-Wl,-rpath,{PKG}", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_cpp_layer_compiles_and_links(t2sx_mod, tmp_path):
    """The header compiles warning-free under -Wall -Wextra -Werror and links against the library."""
    exe = _compile(tmp_path)
    assert os.path.exists(exe)


def _write_inputs(path, prompts):
    with open(path, "wb") as f:
        np.array([len(prompts)], dtype=np.int32).tofile(f)
        for ph, bert, sem in prompts:
            np.array([ph.size, sem.size], dtype=np.int32).tofile(f)
            ph.astype(np.int32).tofile(f)
            bert.astype(np.float32).tofile(f)
            sem.astype(np.int32).tofile(f)


def _case(tmp_path):
    import synth
    path = synth.ensure_gguf("q4_k", seed=5, n_layer=2)
    specs = [(40, 30, 101), (25, 50, 102), (60, 20, 103)]   # two sessions, then the refill of slot 0
    prompts = [synth.session_inputs(seed, tt, tp) for tt, tp, seed in specs]
    inp = str(tmp_path / "inputs.bin")
    _write_inputs(inp, prompts)
    return path, prompts, inp


def _oracle(orc, path, prompts, n_steps):
    m = orc.Model(path)
    n = len(prompts) - 1
    cap = max(p[0].size + p[2].size for p in prompts) + 2 * n_steps + 2
    s = orc.Session(m, n, cap)
    first, y0, k0 = [], None, None
    for i in range(n):
        ph, bert, sem = prompts[i]
        tok, _, y = s.prefill(i, m.embed_prefill(ph, bert, sem), sem.size, eos_mask=True, want_y=(i == 0))
        first.append(tok)
        if i == 0:
            y0, k0 = y, s.read_kv(0, 0, 0)
    steps, cur = [], list(first)
    for _ in range(n_steps):
        out, _ = s.decode(np.arange(n), cur, eos_mask=True)
        steps.append([int(t) for t in out]); cur = list(out)
    # mixed plan: slot 0 released and refilled, the other slots decode one step
    s.release(0)
    out, _ = s.decode(np.arange(1, n), cur[1:], eos_mask=True)
    ph, bert, sem = prompts[n]
    refill, _, _ = s.prefill(0, m.embed_prefill(ph, bert, sem), sem.size, eos_mask=True)
    mixed = [refill] + [int(t) for t in out]
    cur = list(mixed)
    for _ in range(n_steps):
        out, _ = s.decode(np.arange(n), cur, eos_mask=True)
        steps.append([int(t) for t in out]); cur = list(out)
    n_pos0 = s.n_pos(0)
    s.close(); m.close()
    return {"first": [int(t) for t in first], "mixed": mixed, "steps": steps, "n_pos_slot0": n_pos0}, y0, k0


@pytest.mark.gpu
def test_cpp_decode_loop_matches_oracle(t2sx_mod, orc, tmp_path):
    exe = _compile(tmp_path)
    path, prompts, inp = _case(tmp_path)
    n_steps = 6
    prefix = str(tmp_path / "out")
    r = subprocess.run([exe, path, inp, str(n_steps), prefix], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.returncode, r.stderr)
    got = json.loads(r.stdout)
    want, y0, k0 = _oracle(orc, path, prompts, n_steps)
    assert got["first"] == want["first"] and got["mixed"] == want["mixed"] and got["steps"] == want["steps"]
    assert got["n_pos_slot0"] == want["n_pos_slot0"] == got["mask_visible_slot0"]
    y = np.fromfile(prefix + ".y", dtype=np.float32).reshape(y0.shape)
    assert np.array_equal(y.view(np.uint32), y0.view(np.uint32)), "flex graph y differs"
    k = np.fromfile(prefix + ".k0", dtype=np.uint16).reshape(k0.shape)
    assert np.array_equal(k, k0), "layer-0 K cache view differs"


@pytest.mark.gpu
@pytest.mark.parametrize("mode,msg", [("release_bad", "slot_id < session.slots.size()"),
                                      ("decode_idle", "n_pos[i] > 0"),
                                      ("prefill_busy", "n_pos[i] == 0")])
def test_cpp_illegal_transitions_abort(t2sx_mod, tmp_path, mode, msg):
    exe = _compile(tmp_path)
    path, _, inp = _case(tmp_path)
    r = subprocess.run([exe, path, inp, "2", str(tmp_path / "out"), mode], capture_output=True, text=True, timeout=600)
    assert r.returncode == -signal.SIGABRT, (r.returncode, r.stderr)
    assert "GGML_ASSERT" in r.stderr and msg in r.stderr, r.stderr


@pytest.mark.gpu
def test_cpp_compute_ref_emb_matches_oracle(t2sx_mod, orc, tmp_path):
    """t2s_session_compute_ref_emb: prompt codes extracted from HuBERT frames on the device, the
    input text embedded after the reference text (session.cpp:881-1044 flow), first token of the
    prefill; the token and the cached reference embeddings equal the oracle's."""
    exe = _compile(tmp_path)
    path, prompts, inp = _case(tmp_path)
    rng = np.random.default_rng(21)
    T_hub = 57
    hub = rng.standard_normal((T_hub, 768), dtype=np.float32)
    hub_path = str(tmp_path / "hubert.bin")
    with open(hub_path, "wb") as f:
        np.array([T_hub], np.int32).tofile(f)
        hub.tofile(f)
    emb = str(tmp_path / "refemb")
    r = subprocess.run([exe, path, inp, "2", emb, "ref", hub_path], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.returncode, r.stderr)
    got = json.loads(r.stdout)

    m = orc.Model(path)
    codes = m.extract_latent(hub)
    ref_ph, ref_bert, _ = prompts[0]
    in_ph, in_bert, _ = prompts[1]
    ph = np.concatenate([ref_ph, in_ph])
    bert = np.concatenate([ref_bert, in_bert])
    n = len(prompts) - 1
    s = orc.Session(m, n, ph.size + codes.size + 8)
    tok, _, _ = s.prefill(0, m.embed_prefill(ph, bert, codes), codes.size, eos_mask=True)
    s.close()
    assert got["T_prompt"] == codes.size
    assert got["tokens"] == [int(tok)]
    # t2s_session_get_ref_text_emb / get_ref_audio_emb: the reference rows of the prefill input
    x_ref = m.embed_prefill(ref_ph, ref_bert, codes)
    m.close()
    text = np.fromfile(emb + ".text", dtype=np.float32).reshape(-1, 512)
    audio = np.fromfile(emb + ".audio", dtype=np.float32).reshape(-1, 512)
    assert text.shape == (ref_ph.size, 512) and audio.shape == (codes.size, 512)
    assert np.array_equal(text.view(np.uint32), x_ref[:ref_ph.size].view(np.uint32))
    assert np.array_equal(audio.view(np.uint32), x_ref[ref_ph.size:].view(np.uint32))
