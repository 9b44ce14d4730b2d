"""GPU parity: libt2sx (through its C ABI) against the CPU oracle, bit for bit.

Every kernel reproduces the oracle's evaluation order, so the comparisons below are exact
(array_equal on the raw bits), well inside the logit tolerance (1e-2 abs /
1e-3 rel), and greedy token streams must be identical.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def _weights(fmt, N, K, seed):
    import gguf
    import synth
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    if fmt == "q8_0":
        return 8, gguf.quantize(w, gguf.GGMLQuantizationType.Q8_0)
    if fmt == "q4_0":
        return 2, gguf.quantize(w, gguf.GGMLQuantizationType.Q4_0)
    if fmt == "q5_0":
        return 6, gguf.quantize(w, gguf.GGMLQuantizationType.Q5_0)
    if fmt == "q4_k":
        return 12, synth.quantize_q4_k(w)
    if fmt == "f16":
        return 1, w.astype(np.float16).view(np.uint8)
    return 0, w.view(np.uint8)


def same_bits(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("fmt", ["q8_0", "q5_0", "q4_0", "q4_k", "f16", "f32"])
@pytest.mark.parametrize("NK", [(1536, 512), (512, 2048), (1025, 512)])
@pytest.mark.parametrize("M", [1, 7, 8, 16, 17, 32, 33, 64, 65, 130, 255, 2048])
def test_matmul_bit_exact(t2sx_mod, orc, fmt, NK, M):
    _need_gpu()
    if fmt in ("f16", "f32") and M > 33:
        M = 40
    N, K = NK
    wt, wb = _weights(fmt, N, K, seed=N * 7 + K + M)
    x = np.random.default_rng(M).standard_normal((M, K), dtype=np.float32)
    ref = orc.matmul(wt, wb.reshape(-1), N, K, x)
    w = t2sx_mod.Weight(wt, wb, N, K)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((M, N), dtype=torch.float32, device="cuda")
    w.matmul(xd.data_ptr(), M, yd.data_ptr(), stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = yd.cpu().numpy()
    assert np.isfinite(got).all()
    if not same_bits(got, ref):
        d = np.abs(got - ref)
        pytest.fail(f"{fmt} {NK} M={M}: {int((got != ref).sum())} mismatches, max abs {d.max():.3e}")


def _run_pair(t2sx_mod, orc, path, lengths, steps, rep_penalty=1.0, eos_mask=True, check_kv=True):
    """Prefill + `steps` greedy decode steps on both; returns the token arrays."""
    import synth
    m_gpu = t2sx_mod.Model(path)
    m_orc = orc.Model(path)
    cap = max(tt + tp for tt, tp, _ in lengths) + steps + 1
    n = len(lengths)
    s_gpu = t2sx_mod.Session(m_gpu, n, cap, repetition_penalty=rep_penalty, eos_mask=eos_mask)
    s_orc = orc.Session(m_orc, n, cap)
    xs, nq, tps = [], [], []
    first_orc = []
    for i, (tt, tp, seed) in enumerate(lengths):
        ph, bert, sem = synth.session_inputs(seed, tt, tp)
        x_ref = m_orc.embed_prefill(ph, bert, sem)
        x_gpu = s_gpu.embed_prefill(ph, bert, sem)
        assert same_bits(x_gpu, x_ref), "prefill embedding differs"
        xs.append(x_ref); nq.append(tt + tp); tps.append(tp)
        tok, lg, _ = s_orc.prefill(i, x_ref, tp, eos_mask=eos_mask, want_logits=True)
        first_orc.append((tok, lg))
    toks_gpu = s_gpu.prefill(np.arange(n), nq, tps, np.concatenate(xs))
    lg_gpu = s_gpu.read_logits(n)
    for i in range(n):
        assert same_bits(lg_gpu[i], first_orc[i][1]), f"prefill logits of slot {i} differ"
        assert toks_gpu[i] == first_orc[i][0]
        assert s_gpu.slot_n_pos(i) == nq[i] and s_gpu.slot_audio_offset(i) == nq[i] - tps[i]
    if check_kv:
        for layer in (0, m_orc.n_layer - 1):
            for which in (0, 1):
                assert np.array_equal(s_gpu.read_kv(0, layer, which), s_orc.read_kv(0, layer, which))
    V = m_orc.vocab
    seen = np.zeros((n, V), dtype=np.float32)
    cur = np.array([t for t, _ in first_orc], dtype=np.int32)
    seen[np.arange(n), cur] = 1.0
    ref_tokens = []
    ref_last_logits = None
    for step in range(steps):
        out, lg = s_orc.decode(np.arange(n), cur, seen=seen if rep_penalty != 1.0 else None,
                               rep_penalty=rep_penalty, eos_mask=eos_mask, want_logits=(step == steps - 1))
        ref_tokens.append(out.copy())
        seen[np.arange(n), out] = 1.0
        cur = out
        if lg is not None:
            ref_last_logits = lg
    gpu_tokens = s_gpu.decode(steps)
    ref_tokens = np.stack(ref_tokens)
    assert np.array_equal(gpu_tokens, ref_tokens), (
        f"token streams differ at step {int(np.argmax((gpu_tokens != ref_tokens).any(axis=1)))}")
    assert same_bits(s_gpu.read_logits(n), ref_last_logits), "last-step logits differ"
    if check_kv:
        for which in (0, 1):
            assert np.array_equal(s_gpu.read_kv(n - 1, m_orc.n_layer - 1, which), s_orc.read_kv(n - 1, m_orc.n_layer - 1, which))
    return gpu_tokens


@pytest.mark.parametrize("fmt", ["q8_0", "q5_0", "q4_0", "q4_k", "f16"])
def test_decode_small_model_bit_exact(t2sx_mod, orc, fmt):
    _need_gpu()
    import synth
    path = synth.ensure_gguf(fmt, 7, n_layer=2)
    lengths = [(40, 30, 11), (17, 50, 12), (64, 3, 13)]
    _run_pair(t2sx_mod, orc, path, lengths, steps=70)


@pytest.mark.parametrize("n", [12, 24])
@pytest.mark.parametrize("fmt", ["q8_0", "q5_0", "q4_0", "q4_k", "f16"])
def test_decode_8_to_32_sessions_bit_exact(t2sx_mod, orc, fmt, n):
    """8-32 rows per step: split-K matmul tiles (16 activation rows per tile, partly filled; the
    int8 tiles for the quantised formats, the f16-pair tiles for F16), the four-threads-per-lane
    attention and programmatic launches."""
    _need_gpu()
    import synth
    path = synth.ensure_gguf(fmt, 7, n_layer=2)
    rng = np.random.default_rng(40 + n)
    lengths = [(int(rng.integers(8, 70)), int(rng.integers(2, 60)), 100 + i) for i in range(n)]
    _run_pair(t2sx_mod, orc, path, lengths, steps=40)


@pytest.mark.parametrize("n", [1, 2])
@pytest.mark.parametrize("fmt", ["q8_0", "q5_0", "q4_0", "q4_k", "f16"])
def test_decode_one_or_two_sessions_bit_exact(t2sx_mod, orc, fmt, n):
    """One or two rows per step: Q8_0/Q4_0 (and Q5_0, held as Q8_0) weights run each LayerNorm at
    the start of the matmul that consumes it, Q4_K/F16 in the last CTA of the preceding matmul."""
    _need_gpu()
    import synth
    path = synth.ensure_gguf(fmt, 7, n_layer=2)
    lengths = [(40, 30, 31), (17, 50, 32)][:n]
    _run_pair(t2sx_mod, orc, path, lengths, steps=40)


def test_decode_repetition_penalty_bit_exact(t2sx_mod, orc):
    _need_gpu()
    import synth
    path = synth.ensure_gguf("q8_0", 7, n_layer=2)
    _run_pair(t2sx_mod, orc, path, [(20, 20, 21), (33, 9, 22)], steps=40, rep_penalty=1.35, eos_mask=False)


def test_decode_full_model_bs1_bit_exact(t2sx_mod, orc):
    """The one-session workload at its real size: Q8_0 weights seed 0, 24 layers, 128 phonemes +
    150 prompt tokens, all 500 greedy steps (EOS masked); tokens, last logits and KV bit-exact."""
    _need_gpu()
    import synth
    path = synth.ensure_gguf("q8_0", 0, n_layer=24)
    _run_pair(t2sx_mod, orc, path, synth.workload_lengths("bs1_q8_0"), steps=500)


def test_decode_32_sessions_q4_0_full_size_bit_exact(t2sx_mod, orc):
    """The 32-session workload at its real size: Q4_0 weights seed 1, 24 layers, 32 sessions with
    phoneme lengths U[64,256] and prompt lengths U[50,300] (inputs from seed 1 + session), all 500
    greedy steps on the GPU in one call; every step's tokens, the last logits and the KV equal
    the oracle's."""
    _need_gpu()
    import synth
    orc.set_threads(os.cpu_count() or 1)
    path = synth.ensure_gguf("q4_0", 1, n_layer=24)
    lengths = synth.workload_lengths("bs32_q4_0")
    assert len(lengths) == 32
    _run_pair(t2sx_mod, orc, path, lengths, steps=500)


def test_decode_many_rows_q4_k_24_layers_bit_exact(t2sx_mod, orc):
    """Many rows on the 24-layer Q4_K model (seed 3, the box-scale workload's weights): 96
    sessions, so every matmul of the step runs on the tcgen05 kernel (64 rows and more) and the
    attention on the many-row kernel; short ragged prompts keep the oracle's share small."""
    _need_gpu()
    import synth
    orc.set_threads(os.cpu_count() or 1)
    path = synth.ensure_gguf("q4_k", 3, n_layer=24)
    rng = np.random.default_rng(96)
    lengths = [(int(rng.integers(8, 40)), int(rng.integers(4, 30)), 5000 + i) for i in range(96)]
    _run_pair(t2sx_mod, orc, path, lengths, steps=40)


def test_model_load_rejects_wide_ffn(t2sx_mod, tmp_path):
    """A GGUF whose FFN is wider than 2048 (the bound of the few-row matmul's per-row block sums)
    is refused at load with a format error, not run."""
    _need_gpu()
    import synth
    path = synth.write_gguf(str(tmp_path / "wide_ffn.gguf"), 8, 5, n_layer=1, ff=2304)
    with pytest.raises(t2sx_mod.T2SXError) as e:
        t2sx_mod.Model(path)
    assert e.value.code == t2sx_mod.ERR_FORMAT and "FFN width 2304" in str(e.value)


def test_model_load_rejects_large_vocabulary(t2sx_mod, tmp_path):
    """A semantic vocabulary above 2048 (the sampler sorts a row's logits in a 2048-entry shared
    array) is refused at load with a format error, before any kernel runs."""
    _need_gpu()
    import synth
    path = synth.write_gguf(str(tmp_path / "big_vocab.gguf"), 8, 5, n_layer=1, vocab=2049, eos=2048)
    with pytest.raises(t2sx_mod.T2SXError) as e:
        t2sx_mod.Model(path)
    assert e.value.code == t2sx_mod.ERR_FORMAT and "vocabulary size 2049" in str(e.value)


def test_slot_reuse_and_errors(t2sx_mod):
    _need_gpu()
    import synth
    T = t2sx_mod
    path = synth.ensure_gguf("q8_0", 7, n_layer=2)
    m = T.Model(path)
    s = T.Session(m, 2, 64, eos_mask=True)
    assert s.find_free_slot() == 0
    x = np.random.default_rng(0).standard_normal((10, 512), dtype=np.float32)
    s.prefill([0], [10], [4], x)
    assert s.find_free_slot() == 1
    with pytest.raises(T.T2SXError) as e:
        s.prefill([0], [10], [4], x)           # prefill on an active slot
    assert e.value.code == T.ERR_STATE
    with pytest.raises(T.T2SXError) as e:
        s.prefill([1], [3], [4], x[:3])        # n_query < ref_T_prompt
    assert e.value.code == T.ERR_INVALID
    s.decode(5)
    assert s.slot_n_pos(0) == 15
    with pytest.raises(T.T2SXError) as e:
        s.decode(60)                           # would run past slot_size
    assert e.value.code == T.ERR_BOUNDS
    s.slot_release(0)
    assert s.slot_n_pos(0) == 0 and s.find_free_slot() == 0
    with pytest.raises(T.T2SXError):
        s.decode(1)                            # no active slot
    s.prefill([0], [10], [4], x)
    s.decode(3)
    with pytest.raises(T.T2SXError) as e:
        T.Model("/nonexistent/path.gguf")
    assert e.value.code == T.ERR_IO


SAMPLER_CONFIGS = [
    dict(top_k=15, top_p=1.0, temperature=1.0, repetition_penalty=1.35),   # reference defaults
    dict(top_k=0, top_p=0.95, temperature=1.0, repetition_penalty=1.0),
    dict(top_k=1, top_p=1.0, temperature=1.0, repetition_penalty=1.0),
    dict(top_k=1025, top_p=0.5, temperature=0.7, repetition_penalty=1.35),
    dict(top_k=5, top_p=0.8, temperature=0.0, repetition_penalty=1.0),
]


@pytest.mark.parametrize("cfg", SAMPLER_CONFIGS, ids=lambda c: "k{top_k}-p{top_p}-t{temperature}-rp{repetition_penalty}".format(**c))
def test_stochastic_sampler_stream_bit_exact(t2sx_mod, orc, cfg):
    """Full sampler chain (block.cpp:52-348) with caller-supplied Exp(1) noise: sampled and greedy
    tokens equal the oracle's at every step, with the sampled token fed back."""
    _need_gpu()
    import synth
    path = synth.ensure_gguf("q8_0", 7, n_layer=2)
    m_gpu, m_orc = t2sx_mod.Model(path), orc.Model(path)
    lengths = [(30, 20, 31), (12, 40, 32), (50, 5, 33)]
    n, steps, V = len(lengths), 24, m_orc.vocab
    cap = max(tt + tp for tt, tp, _ in lengths) + steps + 2
    s_gpu = t2sx_mod.Session(m_gpu, n, cap, eos_mask=True, **cfg)
    s_orc = orc.Session(m_orc, n, cap)
    xs, nq, tps, cur = [], [], [], []
    for i, (tt, tp, seed) in enumerate(lengths):
        ph, bert, sem = synth.session_inputs(seed, tt, tp)
        x = m_orc.embed_prefill(ph, bert, sem)
        xs.append(x); nq.append(tt + tp); tps.append(tp)
        cur.append(s_orc.prefill(i, x, tp, eos_mask=True)[0])
    first = s_gpu.prefill(np.arange(n), nq, tps, np.concatenate(xs))
    assert list(first) == cur
    cur = np.array(cur, dtype=np.int32)
    seen = np.zeros((n, V), dtype=np.float32)
    seen[np.arange(n), cur] = 1.0
    rng = np.random.default_rng(42)
    for step in range(steps):
        noise = rng.exponential(size=(n, V)).astype(np.float32)
        s_gpu.set_exp_noise(noise)
        got = s_gpu.decode_step_host(cur)
        got_greedy = s_gpu.read_greedy(n)
        ref, ref_greedy = s_orc.decode_sampled(np.arange(n), cur, noise,
                                               seen=seen if cfg["repetition_penalty"] != 1.0 else None,
                                               top_k=cfg["top_k"], top_p=cfg["top_p"], temperature=cfg["temperature"],
                                               rep_penalty=cfg["repetition_penalty"], eos_mask=True)
        assert np.array_equal(got_greedy, ref_greedy), (step, got_greedy, ref_greedy)
        assert np.array_equal(got, ref), (step, got, ref)
        seen[np.arange(n), ref] = 1.0
        cur = ref
    s_gpu.set_exp_noise(None)


def test_model_freed_before_session(t2sx_mod):
    """Freeing the model first (e.g. Python's cyclic GC finalising in any order) defers the release
    until its last session is freed; the session keeps working and no CUDA error is left pending."""
    _need_gpu()
    import synth
    T = t2sx_mod
    path = synth.ensure_gguf("q8_0", 7, n_layer=2)
    m = T.Model(path)
    s = T.Session(m, 1, 64, repetition_penalty=1.0, eos_mask=True)
    x = np.random.default_rng(1).standard_normal((12, 512), dtype=np.float32)
    s.prefill([0], [12], [6], x)
    m.close()
    toks = s.decode(4)
    assert toks.shape == (4, 1)
    s.close()
    m2 = T.Model(path)
    s2 = T.Session(m2, 1, 64, repetition_penalty=1.0, eos_mask=True)
    s2.prefill([0], [12], [6], x)
    assert np.array_equal(s2.decode(4), toks)


# ---- isolated batched attention over a paged f16 KV cache (one layer) ----

def _kv_case(n_seqs, max_len, seed):
    rng = np.random.default_rng(seed)
    scale = np.float32(1.0 / np.sqrt(32.0))
    k = (rng.standard_normal((n_seqs, max_len, 16, 32), dtype=np.float32) * scale).astype(np.float16).view(np.uint16)
    v = (rng.standard_normal((n_seqs, max_len, 16, 32), dtype=np.float32) * scale).astype(np.float16).view(np.uint16)
    return rng, k, v


def _kv_fill(t2sx_mod, k, v, lens, chunks=1):
    n_seqs, max_len = k.shape[:2]
    c = t2sx_mod.KVCache(n_seqs, max_len)
    for s in range(n_seqs):
        L = int(lens[s])
        cuts = np.linspace(0, L, chunks + 1).astype(int)
        for a, b in zip(cuts[:-1], cuts[1:]):
            if b > a:
                c.write(s, int(a), k[s, a:b], v[s, a:b])
    return c


def _kv_run(c, mode, seqs, lens, q16):
    qd = torch.from_numpy(q16.view(np.int16)).cuda()
    od = torch.full((len(seqs), 512), float("nan"), dtype=torch.float32, device="cuda")
    fn = c.attn_decode if mode == 0 else c.attn_prefill
    fn(seqs, lens, qd.data_ptr(), od.data_ptr(), stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return od.cpu().numpy()


def test_kvcache_decode_batched_shape(t2sx_mod, orc):
    """Decode attention at the batched-attention shape: 256 sequences, prefixes uniform in
    [200, 1500], K/V ~ N(0,1)/sqrt(32) in f16, one query per sequence: bit-exact to the oracle."""
    _need_gpu()
    n, max_len = 256, 1500
    rng, k, v = _kv_case(n, max_len, seed=30)
    lens = rng.integers(200, 1501, size=n).astype(np.int32)
    q16 = rng.standard_normal((n, 512), dtype=np.float32).astype(np.float16).view(np.uint16)
    c = _kv_fill(t2sx_mod, k, v, lens, chunks=2)
    seqs = np.arange(n, dtype=np.int32)
    got = _kv_run(c, 0, seqs, lens, q16)
    ref = orc.attn_rows(seqs, lens, q16, k, v)
    c.close()
    assert same_bits(got, ref), f"{int((got != ref).sum())} mismatches, max abs {np.nanmax(np.abs(got - ref)):.3e}"


def test_kvcache_prefill_causal(t2sx_mod, orc):
    """Causal prefill rows (each query attends to its own prefix), empty and non-empty prefixes,
    page-boundary lengths, rows of several sequences interleaved: bit-exact to the oracle."""
    _need_gpu()
    n_seqs, max_len = 6, 300
    rng, k, v = _kv_case(n_seqs, max_len, seed=31)
    full = np.array([256, 256, 64, 65, 129, 300], dtype=np.int32)
    c = _kv_fill(t2sx_mod, k, v, full, chunks=3)
    prefix = np.array([0, 100, 0, 1, 63, 44], dtype=np.int32)   # cached before the new rows
    seqs, lens = [], []
    for s in range(n_seqs):
        for L in range(prefix[s] + 1, full[s] + 1):
            seqs.append(s); lens.append(L)
    seqs = np.array(seqs, dtype=np.int32); lens = np.array(lens, dtype=np.int32)
    perm = rng.permutation(len(seqs))
    seqs, lens = seqs[perm], lens[perm]
    q16 = rng.standard_normal((len(seqs), 512), dtype=np.float32).astype(np.float16).view(np.uint16)
    got = _kv_run(c, 1, seqs, lens, q16)
    ref = orc.attn_rows(seqs, lens, q16, k, v)
    assert same_bits(got, ref), f"{int((got != ref).sum())} mismatches"
    # the decode entry point on the same rows: the same computation
    assert same_bits(_kv_run(c, 0, seqs, lens, q16), got)
    c.close()


def test_kvcache_prefill_grouped_rows(t2sx_mod, orc):
    """Prompt rows in order (the grouped prefill kernel: up to 16 consecutive rows of a sequence
    share the staged K/V), text rows with one common prefix followed by causal rows, prompts of
    1, 15, 16, 17 and 300 rows, prefixes crossing pages: bit-exact to the oracle and to the
    per-row entry point."""
    _need_gpu()
    n_seqs, max_len = 6, 400
    rng, k, v = _kv_case(n_seqs, max_len, seed=34)
    c = _kv_fill(t2sx_mod, k, v, np.full(n_seqs, max_len), chunks=2)
    spec = [(0, 1, 0), (1, 15, 3), (2, 16, 0), (3, 17, 40), (4, 300, 120), (5, 70, 64)]   # (seq, rows, text rows)
    seqs, lens = [], []
    for s, nq, tt in spec:
        for j in range(nq):
            seqs.append(s); lens.append(tt if j < tt else j + 1 + 10)
    seqs = np.array(seqs, dtype=np.int32); lens = np.minimum(np.array(lens, dtype=np.int32), max_len)
    q16 = rng.standard_normal((len(seqs), 512), dtype=np.float32).astype(np.float16).view(np.uint16)
    got = _kv_run(c, 1, seqs, lens, q16)
    ref = orc.attn_rows(seqs, lens, q16, k, v)
    assert same_bits(got, ref), f"{int((got != ref).sum())} mismatches"
    assert same_bits(_kv_run(c, 0, seqs, lens, q16), got)
    c.close()


def test_kvcache_edge_lengths_and_errors(t2sx_mod, orc):
    """Length 1, exact page multiples, a single sequence repeated across rows, small batches
    (the pipelined decode variant), and host-side rejection of bad rows and writes."""
    _need_gpu()
    n_seqs, max_len = 3, 200
    rng, k, v = _kv_case(n_seqs, max_len, seed=32)
    c = _kv_fill(t2sx_mod, k, v, np.full(n_seqs, max_len))
    seqs = np.array([0, 1, 2, 1, 1, 0, 2], dtype=np.int32)
    lens = np.array([1, 64, 128, 192, 200, 2, 63], dtype=np.int32)
    q16 = rng.standard_normal((len(seqs), 512), dtype=np.float32).astype(np.float16).view(np.uint16)
    for mode in (0, 1):
        assert same_bits(_kv_run(c, mode, seqs, lens, q16), orc.attn_rows(seqs, lens, q16, k, v)), mode
    qd = torch.zeros((1, 512), dtype=torch.int16, device="cuda")
    od = torch.zeros((1, 512), dtype=torch.float32, device="cuda")
    for bad_seq, bad_len in ((3, 10), (-1, 10), (0, 0), (0, 201)):
        with pytest.raises(t2sx_mod.T2SXError) as e:
            c.attn_decode([bad_seq], [bad_len], qd.data_ptr(), od.data_ptr())
        assert e.value.code == t2sx_mod.ERR_INVALID
    with pytest.raises(t2sx_mod.T2SXError):
        c.write(0, 190, k[0, :20], v[0, :20])   # past max_len
    c.close()


def test_kvcache_long_prefixes_many_rows(t2sx_mod, orc):
    """Many rows (the persistent kernel) with prefixes past 32 pages (2048 positions), where the
    page numbers held one per lane are reloaded: lengths at and around 2048 and 4096."""
    _need_gpu()
    n_seqs, max_len = 4, 4500
    rng, k, v = _kv_case(n_seqs, max_len, seed=33)
    c = _kv_fill(t2sx_mod, k, v, np.full(n_seqs, max_len), chunks=3)
    fixed = [2047, 2048, 2049, 2112, 4095, 4096, 4097, 4500, 1, 64, 65]
    lens = np.concatenate([fixed, rng.integers(1, max_len + 1, size=80 - len(fixed))]).astype(np.int32)
    seqs = rng.integers(0, n_seqs, size=lens.size).astype(np.int32)
    q16 = rng.standard_normal((lens.size, 512), dtype=np.float32).astype(np.float16).view(np.uint16)
    got = _kv_run(c, 0, seqs, lens, q16)
    ref = orc.attn_rows(seqs, lens, q16, k, v)
    c.close()
    assert same_bits(got, ref), f"{int((got != ref).sum())} mismatches"


def test_decode_many_sessions_q4_k_bit_exact(t2sx_mod, orc):
    """72 sessions of a Q4_K model: the many-row decode path (tcgen05 matmuls, persistent
    attention with the Q8_K output) against the oracle for 8 steps."""
    _need_gpu()
    import synth
    path = synth.ensure_gguf("q4_k", 7, n_layer=2)
    rng = np.random.default_rng(50)
    lengths = [(int(rng.integers(5, 40)), int(rng.integers(3, 30)), 500 + i) for i in range(72)]
    _run_pair(t2sx_mod, orc, path, lengths, steps=8)


@pytest.mark.parametrize("n", [40, 100, 400])
@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "q4_k", "f16"])
def test_decode_between_paths_bit_exact(t2sx_mod, orc, fmt, n):
    """33-63 rows (two-head attention CTAs with cp.async rings, mma.sync matmuls for Q8_0/Q4_0),
    64-384 rows (the attention with each lane's next position in flight; Q4_K: eight-head CTAs
    writing the Q8_K row in place) and above 384 rows (five one-deep CTAs per SM); F16 weights:
    split-K tiles up to 256 rows, the tiled kernel above."""
    _need_gpu()
    import synth
    path = synth.ensure_gguf(fmt, 7, n_layer=2)
    rng = np.random.default_rng(60 + n)
    lengths = [(int(rng.integers(5, 40)), int(rng.integers(3, 30)), 700 + i) for i in range(n)]
    _run_pair(t2sx_mod, orc, path, lengths, steps=6, check_kv=False)


@pytest.mark.parametrize("fmt", ["q8_0", "f32"])
def test_extract_latent_bit_exact(t2sx_mod, orc, fmt):
    """Prompt codes from HuBERT frames (Conv1d k=2 s=2 + nearest codebook entry), GPU against the
    oracle, for even and odd frame counts from the minimum of 2 frames up."""
    _need_gpu()
    import synth
    path = synth.ensure_gguf(fmt, seed=6, n_layer=2)
    m_gpu = t2sx_mod.Model(path)
    s = t2sx_mod.Session(m_gpu, 1, 64)
    m_orc = orc.Model(path)
    rng = np.random.default_rng(11)
    for T in (2, 3, 64, 101, 999):
        h = rng.standard_normal((T, 768), dtype=np.float32)
        got = s.extract_latent(h)
        want = m_orc.extract_latent(h)
        assert got.shape == ((T - 2) // 2 + 1,)
        assert np.array_equal(got, want), (fmt, T, int((got != want).sum()))
    with pytest.raises(t2sx_mod.T2SXError):
        s.extract_latent(np.zeros((1, 768), np.float32))
    s.close(); m_gpu.close(); m_orc.close()


@pytest.mark.parametrize("rp,refill", [(1.0, (25, 25, 44)), (1.35, (25, 25, 44)), (1.0, (60, 70, 45))],
                         ids=["greedy-50rows", "penalty-50rows", "greedy-130rows"])
def test_flex_step_mixed_plan_bit_exact(t2sx_mod, orc, rp, refill):
    """t2sx_flex_step (session.cpp:461-859 with decode and prefill slots in one plan): a decode of a
    subset of the active slots, then a released slot prefilled in the same pass as the others'
    decode step, then ordinary decode steps.  Tokens, logits and the refilled slot's KV equal the
    oracle's separate decode and prefill; the repetition penalty applies to the decode rows only.
    A 130-row refill runs its rows on the grouped prefill attention, the decode rows per row."""
    _need_gpu()
    import synth
    path = synth.ensure_gguf("q4_k", 7, n_layer=2)
    m_gpu, m_orc = t2sx_mod.Model(path), orc.Model(path)
    lengths = [(30, 20, 41), (12, 40, 42), (50, 5, 43)]
    n, cap, V = len(lengths), 160, m_orc.vocab
    s_gpu = t2sx_mod.Session(m_gpu, n, cap, eos_mask=True, repetition_penalty=rp)
    s_orc = orc.Session(m_orc, n, cap)
    seen = np.zeros((n, V), dtype=np.float32)
    xs, nq, tps, cur = [], [], [], np.zeros(n, np.int32)
    for i, (tt, tp, seed) in enumerate(lengths):
        ph, bert, sem = synth.session_inputs(seed, tt, tp)
        x = m_orc.embed_prefill(ph, bert, sem)
        xs.append(x); nq.append(tt + tp); tps.append(tp)
        cur[i] = s_orc.prefill(i, x, tp, eos_mask=True)[0]
    assert np.array_equal(s_gpu.prefill(np.arange(n), nq, tps, np.concatenate(xs)), cur)
    seen[np.arange(n), cur] = 1.0

    def orc_decode(slots, toks, want_logits=False):
        slots = np.asarray(slots, np.int32)
        out, lg = s_orc.decode(slots, toks, seen=seen[slots] if rp != 1.0 else None, rep_penalty=rp,
                               eos_mask=True, want_logits=want_logits)
        seen[slots, out] = 1.0
        return out, lg

    for _ in range(3):
        got = s_gpu.decode_step_host(cur)
        cur, _ = orc_decode(np.arange(n), cur)
        assert np.array_equal(got, cur)
    # decode of a subset (slot 1 waits)
    got = s_gpu.flex_step([2, 0], cur[[2, 0]])
    ref, lg = orc_decode([2, 0], cur[[2, 0]], want_logits=True)
    assert np.array_equal(got, ref)
    assert same_bits(s_gpu.read_logits(2), lg)
    cur[[2, 0]] = ref
    assert s_gpu.slot_n_pos(1) == nq[1] + 3 and s_gpu.slot_n_pos(0) == nq[0] + 4
    # slot 1 released and prefilled again while slots 0 and 2 decode, in one pass
    s_gpu.slot_release(1); s_orc.release(1)
    tt, tp, seed = refill
    ph, bert, sem = synth.session_inputs(seed, tt, tp)
    x = m_orc.embed_prefill(ph, bert, sem)
    got = s_gpu.flex_step([0, 2], cur[[0, 2]], [1], [tt + tp], [tp], x)
    lg_gpu = s_gpu.read_logits(3)
    ref, lg = orc_decode([0, 2], cur[[0, 2]], want_logits=True)
    tok1, lg1, _ = s_orc.prefill(1, x, tp, eos_mask=True, want_logits=True)
    assert list(got) == list(ref) + [tok1]
    assert same_bits(lg_gpu[:2], lg) and same_bits(lg_gpu[2], lg1)
    assert s_gpu.slot_n_pos(1) == tt + tp and s_gpu.slot_audio_offset(1) == tt
    for which in (0, 1):
        assert np.array_equal(s_gpu.read_kv(1, m_orc.n_layer - 1, which), s_orc.read_kv(1, m_orc.n_layer - 1, which))
    cur[[0, 2]] = ref
    cur[1] = tok1
    seen[1] = 0.0
    seen[1, tok1] = 1.0
    for _ in range(4):
        got = s_gpu.decode_step_host(cur)
        cur, _ = orc_decode(np.arange(n), cur)
        assert np.array_equal(got, cur)
    s_gpu.close(); s_orc.close(); m_gpu.close(); m_orc.close()


def test_flex_step_errors(t2sx_mod):
    """Plans the reference rejects (session.cpp:461-540) fail before any device work."""
    _need_gpu()
    import synth
    T = t2sx_mod
    path = synth.ensure_gguf("q8_0", 7, n_layer=2)
    m = T.Model(path)
    s = T.Session(m, 3, 64, eos_mask=True)
    x = np.random.default_rng(0).standard_normal((10, 512), dtype=np.float32)
    s.prefill([0], [10], [4], x)
    for args, code in [(([1], [5]), T.ERR_STATE),                          # decode of an idle slot
                       (([0], [5], [0], [10], [4], x), T.ERR_INVALID),     # slot both decoded and prefilled
                       (([0], [5], [1], [10], [4], x), None),              # legal
                       (([0], [5], [1], [10], [4], x), T.ERR_STATE),       # slot 1 is busy now
                       (([0], [5], [2], [3], [4], x[:3]), T.ERR_INVALID),  # n_query < ref_T_prompt
                       (([0, 0], [5, 5]), T.ERR_INVALID),                  # repeated slot
                       (([0], [m.vocab + 5]), T.ERR_INVALID)]:             # token out of range
        if code is None:
            s.flex_step(*args)
            continue
        with pytest.raises(T.T2SXError) as e:
            s.flex_step(*args)
        assert e.value.code == code, args
    assert s.slot_n_pos(0) == 11 and s.slot_n_pos(1) == 10 and s.slot_n_pos(2) == 0
    s.close(); m.close()


def test_tc_wait_timeout_reported_and_recovered(t2sx_mod, orc):
    """The tensor-core matmul's barrier waits are bounded.  The test hook makes each CTA's fold
    warps first wait on a barrier that nothing completes, bounded by 100k cycles (about 50 us):
    the wait runs out, the CTA gives up, drains the copies it issued, frees its TMEM and stores
    NaN, and the failure reaches the host as T2SX_ERR_TIMEOUT -- through t2sx_weight_sync for
    the isolated matmul and through the call's status for a session prefill.  With the hook off,
    the same weight and a new session give bit-exact results again: the context stays usable."""
    _need_gpu()
    import synth
    T = t2sx_mod
    N, K, M = 512, 2048, 256            # Q4_K, 64 rows and more: the tcgen05 kernel
    wt, wb = _weights("q4_k", N, K, seed=77)
    x = np.random.default_rng(77).standard_normal((M, K), dtype=np.float32)
    ref = orc.matmul(wt, wb.reshape(-1), N, K, x)
    w = T.Weight(wt, wb, N, K)
    xd = torch.from_numpy(x).cuda()
    yd = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    path = synth.ensure_gguf("q4_k", 7, n_layer=2)
    m = T.Model(path)
    lengths = [(20, 12, 41 + i) for i in range(4)]   # 128 prefill rows: the tcgen05 kernel
    prompts = [synth.session_inputs(seed, tt, tp) for tt, tp, seed in lengths]
    try:
        T.test_set_tc_wait_cycles(100_000)
        w.matmul(xd.data_ptr(), M, yd.data_ptr(), stream=stream)
        with pytest.raises(T.T2SXError) as e:
            w.sync(stream)
        assert e.value.code == T.ERR_TIMEOUT
        assert np.isnan(yd.cpu().numpy()).any()
        s = T.Session(m, 4, 64, repetition_penalty=1.0, eos_mask=True)
        xs = np.concatenate([s.embed_prefill(*p) for p in prompts])
        with pytest.raises(T.T2SXError) as e:
            s.prefill(np.arange(4), [tt + tp for tt, tp, _ in lengths], [tp for _, tp, _ in lengths], xs)
        assert e.value.code == T.ERR_TIMEOUT
        s.close()
    finally:
        T.test_set_tc_wait_cycles(0)
    w.sync(stream)                      # the state was cleared by the failed check
    for _ in range(2):
        yd.zero_()
        w.matmul(xd.data_ptr(), M, yd.data_ptr(), stream=stream)
        w.sync(stream)
        assert same_bits(yd.cpu().numpy(), ref)
    w.close()
    s = T.Session(m, 4, 64, repetition_penalty=1.0, eos_mask=True)
    om = orc.Model(path)
    os_ = orc.Session(om, 4, 64)
    xs = [om.embed_prefill(*p) for p in prompts]
    first = s.prefill(np.arange(4), [tt + tp for tt, tp, _ in lengths], [tp for _, tp, _ in lengths], np.concatenate(xs))
    assert list(first) == [os_.prefill(i, xs[i], lengths[i][1])[0] for i in range(4)]
    s.close()
    m.close()


def test_roofline_probes_measure_the_device(t2sx_mod):
    """The measured roofline denominators run and give figures of the B200's class: the L2 read
    of an L2-resident 32 MiB buffer (about 6 TB/s, the two dies' L2 halves seen from every SM) and
    the dense int8 tcgen05 loop (nominal 4.5 POP/s)."""
    _need_gpu()
    l2 = t2sx_mod.probe_l2_read_gbs(0, 32 << 20, 50)
    tops = t2sx_mod.probe_i8_mma_tops(0, 4000, 1)
    assert 1000.0 < l2 < 100000.0, l2
    assert 500.0 < tops < 10000.0, tops
