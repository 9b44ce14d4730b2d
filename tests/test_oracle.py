"""CPU checks of the oracle (no GPU): pins against gguf-py and the reference's own known
answers, and cross-checks of the float pipeline against an independent float64 restatement."""
import numpy as np
import pytest


def test_f16_conversion_matches_ieee(orc):
    L = orc.lib()
    allh = np.arange(65536, dtype=np.uint16)
    back = np.array([L.orc_f16_to_f32(int(h)) for h in allh], dtype=np.float32)
    ref = allh.view(np.float16).astype(np.float32)
    assert np.array_equal(np.isnan(back), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.array_equal(back[ok].view(np.uint32), ref[ok].view(np.uint32))
    rng = np.random.default_rng(0)
    v = (rng.standard_normal(40000) * 10.0 ** rng.uniform(-9, 4.5, 40000)).astype(np.float32)
    v = np.concatenate([v, np.float32([0, -0.0, 65504, 65519.99, 2 ** -24, 2 ** -25, 3 * 2 ** -26, 6.1e-5])])
    mine = np.array([L.orc_f32_to_f16(float(x)) for x in v], dtype=np.uint16)
    with np.errstate(over="ignore"):
        ref16 = v.astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, ref16)


def test_expf_accuracy(orc):
    L = orc.lib()
    rng = np.random.default_rng(1)
    xs = np.concatenate([-np.abs(rng.standard_normal(20000)).astype(np.float32) * 25, np.float32([0.0, -86.5, -1e-7])])
    got = np.array([L.orc_expf(float(x)) for x in xs], dtype=np.float64)
    ref = np.exp(xs.astype(np.float64))
    ulp = np.abs(got - ref) / np.spacing(ref.astype(np.float32)).astype(np.float64)
    live = xs > -87.0                       # below -87 the softmax weight is flushed to 0
    assert ulp[live].max() <= 1.0
    assert (got[~live] == 0).all()
    assert L.orc_expf(0.0) == 1.0
    assert L.orc_expf(float("-inf")) == 0.0 and L.orc_expf(-200.0) == 0.0


@pytest.mark.parametrize("fmt", ["q8_0", "q5_0", "q4_0", "q4_k", "f16"])
def test_dequant_bit_exact_vs_gguf_py(orc, fmt):
    import gguf
    import synth
    from gguf import GGUFReader
    path = synth.ensure_gguf(fmt, 7, n_layer=2)
    rd = GGUFReader(path)
    assert len(rd.tensors) == 2 * 12 + 10
    for t in rd.tensors:
        raw = np.asarray(t.data)
        n = int(np.prod(t.shape))
        mine = orc.dequantize(int(t.tensor_type), raw.view(np.uint8).ravel(), n)
        ref = gguf.dequantize(raw, t.tensor_type).astype(np.float32).ravel()
        assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32)), t.name


def test_gguf_layout_matches_converter(orc):
    """Tensor names, shapes and types follow python/convert_t2s_to_gguf.py (and the shapes the
    reference loader test expects, tests/t2s/test_t2s_loader.cpp:42-88)."""
    import synth
    from gguf import GGUFReader
    rd = GGUFReader(synth.ensure_gguf("q8_0", 7, n_layer=2))
    t = {x.name: x for x in rd.tensors}
    shape = lambda n: tuple(int(v) for v in t[n].shape)
    assert shape("attention.0.qkv_w") == (512, 1536) and int(t["attention.0.qkv_w"].tensor_type) == 8
    assert shape("attention.1.ffn_down_w") == (2048, 512)
    assert shape("encoder.text_embedding") == (512, 732) and int(t["encoder.text_embedding"].tensor_type) == 1
    assert shape("encoder.audio_embedding") == (512, 1025)
    assert shape("encoder.bert_proj_w") == (1024, 512) and int(t["encoder.bert_proj_w"].tensor_type) == 8
    assert shape("sampler.lm_head_w") == (512, 1025) and int(t["sampler.lm_head_w"].tensor_type) == 8
    assert shape("extract_latent.ssl_proj_w") == (2, 768, 768) and int(t["extract_latent.ssl_proj_w"].tensor_type) == 1
    assert shape("extract_latent.codebook") == (768, 1024) and int(t["extract_latent.codebook"].tensor_type) == 0
    assert int(t["attention.0.ln1_w"].tensor_type) == 0 and shape("encoder.text_pos_alpha") == (1,)
    m = orc.Model(synth.ensure_gguf("q8_0", 7, n_layer=2))
    assert list(m.hp) == [512, 512, 16, 2048, 2, 1025, 732, 1024, 192]


def test_q4_k_encoder_roundtrip():
    import gguf
    import synth
    w = np.random.default_rng(3).standard_normal((32, 512)).astype(np.float32) * 0.02
    q = synth.quantize_q4_k(w)
    assert q.shape == (32, 2 * 144)
    deq = gguf.dequantize(q, gguf.GGMLQuantizationType.Q4_K).reshape(32, 512)
    assert np.sqrt(((deq - w) ** 2).mean()) / w.std() < 0.1


# ---- independent float64 restatement ----------------------------------------------------------

def q8_0_act(x):
    """x86 AVX2 rule of ggml quantize_row_q8_0 in numpy float32 arithmetic."""
    b = x.astype(np.float32).reshape(-1, 32)
    amax = np.abs(b).max(axis=1)
    d16 = (amax / np.float32(127)).astype(np.float32).astype(np.float16).astype(np.float32)
    with np.errstate(divide="ignore"):
        idd = np.where(amax != 0, np.float32(127) / amax, np.float32(0)).astype(np.float32)
    q = np.rint((b * idd[:, None]).astype(np.float32)).clip(-128, 127)
    return q, d16


def q8_k_act(x):
    b = x.astype(np.float32).reshape(-1, 256)
    i = np.abs(b).argmax(axis=1)
    mx = b[np.arange(b.shape[0]), i]
    with np.errstate(divide="ignore", invalid="ignore"):
        isc = np.where(mx != 0, np.float32(-127) / mx, 0).astype(np.float32)
        q = np.minimum(np.rint((isc[:, None] * b).astype(np.float32)), 127)
        d = np.where(mx != 0, np.float32(1) / isc, 0).astype(np.float32)
    return q, d


def f64_matmul(wtype, wbytes, N, K, x, orc):
    wd = orc.dequantize(wtype, wbytes.reshape(-1), N * K).astype(np.float64).reshape(N, K)
    if wtype in (8, 6, 2):   # Q8_0, Q5_0, Q4_0 weights: Q8_0 activations
        q, d = q8_0_act(x)
        xa = (q * d[:, None]).reshape(x.shape).astype(np.float64)
    elif wtype == 12:
        q, d = q8_k_act(x)
        xa = (q * d[:, None]).reshape(x.shape).astype(np.float64)
    elif wtype == 1:
        xa = x.astype(np.float16).astype(np.float64)
    else:
        xa = x.astype(np.float64)
    return xa @ wd.T


@pytest.mark.parametrize("fmt,wtype", [("q8_0", 8), ("q5_0", 6), ("q4_0", 2), ("q4_k", 12), ("f16", 1)])
def test_matmul_matches_float64(orc, fmt, wtype):
    import gguf
    import synth
    rng = np.random.default_rng(5)
    N, K, M = 96, 512, 3
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.02
    wb = {"q8_0": lambda: gguf.quantize(w, gguf.GGMLQuantizationType.Q8_0),
          "q4_0": lambda: gguf.quantize(w, gguf.GGMLQuantizationType.Q4_0),
          "q5_0": lambda: gguf.quantize(w, gguf.GGMLQuantizationType.Q5_0),
          "q4_k": lambda: synth.quantize_q4_k(w), "f16": lambda: w.astype(np.float16).view(np.uint8)}[fmt]()
    x = rng.standard_normal((M, K)).astype(np.float32)
    got = orc.matmul(wtype, wb, N, K, x)
    ref = f64_matmul(wtype, wb, N, K, x, orc)
    assert np.abs(got - ref).max() < 1e-5 * max(1.0, np.abs(ref).max())


def test_attention_orders_match_float64(orc):
    L = orc.lib()
    rng = np.random.default_rng(9)
    for n in (1, 5, 127, 128, 129, 700):
        q = rng.standard_normal(32).astype(np.float32)
        k = (rng.standard_normal((n, 32)) / np.sqrt(32)).astype(np.float16)
        v = rng.standard_normal((n, 32)).astype(np.float16)
        qh = q.astype(np.float16).astype(np.float64)
        s = (k.astype(np.float64) @ qh) * float(np.float32(1) / np.sqrt(np.float32(32)))
        p = np.exp(s - s.max())
        ref = (p / p.sum()) @ v.astype(np.float64)
        for fn in (L.orc_attn_decode,):
            out = np.zeros(32, dtype=np.float32)
            fn(orc.ptr(q), orc.ptr(k.view(np.uint16)), orc.ptr(v.view(np.uint16)), n, orc.ptr(out))
            assert np.abs(out - ref).max() < 2e-6 * max(1, np.abs(ref).max()), (n, fn)


def test_layernorm_matches_float64(orc):
    L = orc.lib()
    rng = np.random.default_rng(2)
    x = (rng.standard_normal(512) * 3 + 0.5).astype(np.float32)
    g = rng.standard_normal(512).astype(np.float32)
    b = rng.standard_normal(512).astype(np.float32)
    y = np.zeros(512, dtype=np.float32)
    L.orc_layernorm(orc.ptr(x), orc.ptr(g), orc.ptr(b), 512, 1e-5, orc.ptr(y))
    xd = x.astype(np.float64)
    ref = (xd - xd.mean()) / np.sqrt(xd.var() + 1e-5) * g + b
    assert np.abs(y - ref).max() < 1e-5


def test_prefill_mask_semantics_match_reference_known_answers():
    """Visible key ranges of the prefill rows equal the reference's dense masks
    (tests/t2s/test_t2s_session.cpp:694-855 MaskCorrectness / MaskCorrectnessThreePart):
    text rows see [0, T_text), audio row j sees [0, j]."""
    def visible(nq, t_prompt):
        T_text = nq - t_prompt
        return [set(range(T_text if j < T_text else j + 1)) for j in range(nq)]
    # ref_T_prompt = 0 -> every token is text: all see each other
    assert visible(2, 0) == [{0, 1}, {0, 1}]
    assert visible(3, 0) == [{0, 1, 2}] * 3
    # T_ref=3, T_in=2, T_prompt=4: text cols 0-4 see 0-4, audio col j sees 0..j
    v = visible(9, 4)
    for j in range(5):
        assert v[j] == set(range(5))
    for j in range(5, 9):
        assert v[j] == set(range(j + 1))


def test_oracle_session_bookkeeping(orc):
    import synth
    m = orc.Model(synth.ensure_gguf("q8_0", 7, n_layer=2))
    s = orc.Session(m, 3, 64)
    x = np.random.default_rng(0).standard_normal((9, 512)).astype(np.float32)
    tok, _, _ = s.prefill(2, x, 4)
    assert s.n_pos(2) == 9 and s.n_pos(0) == 0
    out, _ = s.decode([2], [tok])
    assert s.n_pos(2) == 10
    with pytest.raises(RuntimeError):
        s.prefill(2, x, 4)          # prefill on an active slot (session.cpp:738)
    with pytest.raises(RuntimeError):
        s.decode([0], [1])          # decode on an idle slot (session.cpp:735)
    with pytest.raises(RuntimeError):
        s.prefill(1, x[:3], 4)      # n_query < ref_T_prompt (session.cpp:821)


def _np_forward(path, x, T_prompt, orc):
    """Independent float64 restatement of the prefill of one slot (quantisation semantics in
    float32 numpy, all sums in float64); returns last-row logits."""
    from gguf import GGUFReader
    import gguf
    rd = GGUFReader(path)
    T = {t.name: t for t in rd.tensors}

    def W(name):
        t = T[name]
        return int(t.tensor_type), np.asarray(t.data).view(np.uint8), int(t.shape[1]) if len(t.shape) > 1 else 1, int(t.shape[0])

    def vec(name):
        return gguf.dequantize(np.asarray(T[name].data), T[name].tensor_type).astype(np.float64).ravel()

    def mm(name, xx, bias=None):
        wt, wb, N, K = W(name)
        y = f64_matmul(wt, wb, N, K, xx.astype(np.float32), orc)
        return y + vec(bias) if bias else y

    def ln(v, g, b):
        mu = v.mean(axis=1, keepdims=True)
        var = ((v - mu) ** 2).mean(axis=1, keepdims=True)
        return (v - mu) / np.sqrt(var + 1e-5) * vec(g) + vec(b)

    nq = x.shape[0]
    T_text = nq - T_prompt
    h = x.astype(np.float64)
    n_layer = int(rd.fields["t2s.n_layer"].parts[-1][0])
    scale = float(np.float32(1) / np.sqrt(np.float32(32)))
    for l in range(n_layer):
        p = f"attention.{l}."
        qkv = mm(p + "qkv_w", h, p + "qkv_b")
        q = qkv[:, :512].astype(np.float16).astype(np.float64)
        k = qkv[:, 512:1024].astype(np.float16).astype(np.float64)
        v = qkv[:, 1024:].astype(np.float16).astype(np.float64)
        att = np.zeros((nq, 512))
        for hh in range(16):
            sl = slice(32 * hh, 32 * hh + 32)
            s = q[:, sl] @ k[:, sl].T * scale
            for j in range(nq):
                Lj = T_text if j < T_text else j + 1
                e = np.exp(s[j, :Lj] - s[j, :Lj].max())
                att[j, sl] = (e / e.sum()) @ v[:Lj, sl]
        o = mm(p + "out_proj_w", att, p + "out_proj_b")
        l1 = ln(h + o, p + "ln1_w", p + "ln1_b")
        f = np.maximum(mm(p + "ffn_up_w", l1, p + "ffn_up_b"), 0)
        f = mm(p + "ffn_down_w", f, p + "ffn_down_b")
        h = ln(l1 + f, p + "ln2_w", p + "ln2_b")
    return mm("sampler.lm_head_w", h[-1:])[0]


@pytest.mark.parametrize("fmt", ["q8_0", "q4_k"])
def test_prefill_matches_float64_restatement(orc, fmt):
    import synth
    path = synth.ensure_gguf(fmt, 7, n_layer=2)
    m = orc.Model(path)
    ph, bert, sem = synth.session_inputs(4, 24, 20)
    x = m.embed_prefill(ph, bert, sem)
    s = orc.Session(m, 1, 64)
    tok, logits, _ = s.prefill(0, x, 20, want_logits=True)
    ref = _np_forward(path, x, 20, orc)
    # activation quantisation can round a value differently when the float64 and float32
    # paths differ in the last bit; the effect on logits stays far below 1e-2
    assert np.abs(logits - ref).max() < 1e-2
    srt = np.sort(ref[:1024])
    if srt[-1] - srt[-2] > 2e-2:
        assert tok == int(np.argmax(ref[:1024]))


def _np_sample(logits, noise, top_k, top_p, temperature, eos=1024):
    """Independent restatement of the reference sampler chain (block.cpp:52-115,191-271) in
    float64 numpy; returns the sampled token."""
    l = logits.astype(np.float64).copy()
    l[eos] = -1e30
    order = np.lexsort((np.arange(l.size), -l))
    s = l[order]
    if top_p < 1.0:
        p = np.exp(s - s.max()); p /= p.sum()
        cum = np.cumsum(p)
        remove = np.concatenate([[False], cum[:-1] > top_p])
        s = np.where(remove, -1e10, s)
    s = s / max(temperature, 1e-5)
    if 0 < top_k < s.size:
        s = np.where(s < s[top_k - 1], -1e10, s)
    p = np.exp(s - s.max()); p /= p.sum()
    return int(order[np.argmax(p / noise)])


@pytest.mark.parametrize("top_k,top_p,temp", [(15, 1.0, 1.0), (0, 0.9, 1.0), (3, 0.7, 0.5), (1025, 1.0, 2.0)])
def test_sampler_matches_float64_restatement(orc, top_k, top_p, temp):
    import synth
    m = orc.Model(synth.ensure_gguf("q8_0", 7, n_layer=2))
    rng = np.random.default_rng(top_k + 7)
    n = 64
    logits = (rng.standard_normal((n, 1025)) * 3).astype(np.float32)
    noise = rng.exponential(size=(n, 1025)).astype(np.float32)
    sampled, greedy = m.sample(logits, noise=noise, top_k=top_k, top_p=top_p, temperature=temp)
    agree = 0
    for r in range(n):
        lr = logits[r].copy(); lr[1024] = -1e30
        assert greedy[r] == int(np.argmax(lr))
        agree += int(sampled[r] == _np_sample(logits[r], noise[r], top_k, top_p, temp))
    assert agree >= n - 1   # float32 vs float64 rounding can move a near-tie
    s2, g2 = m.sample(logits, noise=None)
    assert np.array_equal(s2, greedy) and np.array_equal(g2, greedy)


def test_attn_rows_matches_per_head_calls(orc):
    """The batched oracle attention (used for the batched-attention parity tests) is the per-head
    restatement applied row by row."""
    rng = np.random.default_rng(0)
    S, Lm = 3, 150
    k = (rng.standard_normal((S, Lm, 16, 32)) / np.sqrt(32)).astype(np.float16).view(np.uint16)
    v = (rng.standard_normal((S, Lm, 16, 32)) / np.sqrt(32)).astype(np.float16).view(np.uint16)
    q = rng.standard_normal((4, 512)).astype(np.float16)
    seqs, lens = [0, 2, 1, 2], [150, 37, 1, 100]
    for fn in ("orc_attn_decode",):
        out = orc.attn_rows(seqs, lens, q.view(np.uint16), k, v)
        for r in range(4):
            for h in range(16):
                kk = np.ascontiguousarray(k[seqs[r], :, h, :])
                vv = np.ascontiguousarray(v[seqs[r], :, h, :])
                qq = np.ascontiguousarray(q[r, h * 32:(h + 1) * 32].astype(np.float32))
                o = np.empty(32, np.float32)
                getattr(orc.lib(), fn)(orc.ptr(qq), orc.ptr(kk), orc.ptr(vv), lens[r], orc.ptr(o))
                assert np.array_equal(o.view(np.uint32), out[r, h * 32:(h + 1) * 32].view(np.uint32)), (r, h)


def test_extract_latent_matches_float64(orc):
    """Oracle extract-latent against an independent float64 restatement of the reference graph
    (block.cpp:140-189: Conv1d k=2 s=2 on f16-rounded frames and kernel, + bias, nearest code by
    x.E - ||E||^2/2): scores agree closely and every code with a clear margin is identical."""
    import synth
    import gguf
    path = synth.ensure_gguf("q8_0", seed=5, n_layer=2)
    r = gguf.GGUFReader(path)
    t = {x.name: x for x in r.tensors}
    w = np.asarray(t["extract_latent.ssl_proj_w"].data).astype(np.float64).reshape(768, 768, 2)   # [oc][ic][k]
    b = np.asarray(t["extract_latent.ssl_proj_b"].data).astype(np.float64)
    E = np.asarray(t["extract_latent.codebook"].data).astype(np.float64).reshape(-1, 768)
    rng = np.random.default_rng(4)
    h = rng.standard_normal((121, 768)).astype(np.float32)
    hq = h.astype(np.float16).astype(np.float64)
    To = (121 - 2) // 2 + 1
    x = np.stack([hq[2 * i:2 * i + 2] for i in range(To)])          # [t][k][ic]
    ssl = np.einsum("tki,oik->to", x, w) + b
    score = ssl @ E.T - 0.5 * (E * E).sum(1)
    want = score.argmax(1)
    m = orc.Model(path)
    got = m.extract_latent(h)
    m.close()
    top2 = np.sort(score, 1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 1e-3 * np.abs(top2[:, 1]).clip(1)
    assert clear.sum() > To // 2
    assert np.array_equal(got[clear], want[clear])


def test_power_of_two_scaling_matches_division():
    """The LayerNorm means divide a double sum by d_model = 512; the kernels multiply by 2^-9
    instead.  Both are the same real number rounded once, so the bits agree, subnormal results
    included."""
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(200_000) * 10.0 ** rng.integers(-30, 30, 200_000),
        np.ldexp(rng.random(50_000) + 0.5, rng.integers(-1074, -1000, 50_000)),   # results in the subnormal range
        np.array([0.0, -0.0, np.inf, -np.inf, 5e-324, -5e-324, 1.7976931348623157e308]),
    ]).astype(np.float64)
    a = x / 512.0
    b = x * (1.0 / 512.0)
    assert np.array_equal(a.view(np.uint64), b.view(np.uint64))
