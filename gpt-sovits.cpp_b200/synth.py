"""Synthetic T2S GGUF files and seeded inputs.

The GGUF layout follows the reference converter exactly (python/convert_t2s_to_gguf.py):
tensor names and order (:95-127, :176-191), KV metadata (:158-168) and the quantisation
policy (:75-88, :209-228: 2-D weights whose row length is a multiple of the block size are
quantised, embeddings and other 2-D tensors are f16, 1-D tensors f32, codebook f32).
Weights are N(0, 0.02) from numpy.random.default_rng(seed) in tensor order, LayerNorm
gamma = 1 and beta = 0, positional alphas = 1.0.  There is no real checkpoint here.

Q8_0, Q5_0 and Q4_0 use gguf-py's own quantizers (the converter's).  Q4_K has no quantizer in
gguf-py, so `quantize_q4_k` below encodes it (any valid Q4_K encoding serves: the oracle and
the GPU consume the same bytes).
"""
from __future__ import annotations

import os
import numpy as np

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q5_0, GGML_Q8_0, GGML_Q4_K = 0, 1, 2, 6, 8, 12
TYPE_NAMES = {"f32": GGML_F32, "f16": GGML_F16, "q4_0": GGML_Q4_0, "q5_0": GGML_Q5_0, "q8_0": GGML_Q8_0, "q4_k": GGML_Q4_K}
BLOCK = {GGML_Q8_0: 32, GGML_Q5_0: 32, GGML_Q4_0: 32, GGML_Q4_K: 256}

ATTN_NAMES = ["qkv_w", "qkv_b", "out_proj_w", "out_proj_b", "ln1_w", "ln1_b",
              "ffn_up_w", "ffn_up_b", "ffn_down_w", "ffn_down_b", "ln2_w", "ln2_b"]
EMBEDDING_NAMES = {"encoder.text_embedding", "encoder.audio_embedding", "extract_latent.codebook"}


def tensor_specs(d=512, ff=2048, n_layer=24, vocab=1025, phone_vocab=732):
    """(name, pytorch shape) in converter order."""
    specs = []
    for i in range(n_layer):
        p = f"attention.{i}."
        specs += [(p + "qkv_w", (3 * d, d)), (p + "qkv_b", (3 * d,)),
                  (p + "out_proj_w", (d, d)), (p + "out_proj_b", (d,)),
                  (p + "ln1_w", (d,)), (p + "ln1_b", (d,)),
                  (p + "ffn_up_w", (ff, d)), (p + "ffn_up_b", (ff,)),
                  (p + "ffn_down_w", (d, ff)), (p + "ffn_down_b", (d,)),
                  (p + "ln2_w", (d,)), (p + "ln2_b", (d,))]
    specs += [("encoder.text_embedding", (phone_vocab, d)), ("encoder.bert_proj_w", (d, 1024)),
              ("encoder.bert_proj_b", (d,)), ("encoder.text_pos_alpha", (1,)),
              ("encoder.audio_embedding", (vocab, d)), ("encoder.audio_pos_alpha", (1,)),
              ("sampler.lm_head_w", (vocab, d)),
              ("extract_latent.ssl_proj_w", (768, 768, 2)), ("extract_latent.ssl_proj_b", (768,)),
              ("extract_latent.codebook", (1024, 768))]
    return specs


def _f16_bits(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def quantize_q4_k(w: np.ndarray) -> np.ndarray:
    """Encode rows of w (multiple of 256 long) as GGUF Q4_K blocks -> uint8 [rows, nb*144].

    Per 32-element sub-block: scale = (max - min')/15 and offset = -min' with min' = min(min, 0);
    the 8 scales and 8 offsets of a super-block are stored as 6-bit multiples of d and dmin
    (d = max scale / 63, dmin = max offset / 63, both f16); quants are round((x + offset)/scale)
    clipped to [0, 15].  Layout per ggml block_q4_K: d, dmin, scales[12], qs[128].
    """
    w = np.asarray(w, dtype=np.float32)
    rows = w.reshape(-1, w.shape[-1])
    nrow, K = rows.shape
    assert K % 256 == 0
    x = rows.reshape(nrow, K // 256, 8, 32)
    mn = np.minimum(x.min(axis=-1), 0.0)
    mx = x.max(axis=-1)
    scale = (mx - mn) / 15.0
    offs = -mn
    d = scale.max(axis=-1) / 63.0
    dmin = offs.max(axis=-1) / 63.0
    d16 = d.astype(np.float16).astype(np.float32)
    dmin16 = dmin.astype(np.float16).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d16[..., None] > 0, np.rint(scale / d16[..., None]), 0).clip(0, 63).astype(np.int32)
        mq = np.where(dmin16[..., None] > 0, np.rint(offs / dmin16[..., None]), 0).clip(0, 63).astype(np.int32)
        eff_s = d16[..., None] * sc
        eff_m = dmin16[..., None] * mq
        q = np.where(eff_s[..., None] > 0, np.rint((x + eff_m[..., None]) / eff_s[..., None]), 0)
    q = q.clip(0, 15).astype(np.uint8)                       # [nrow, nb, 8, 32]
    scales = np.zeros((nrow, K // 256, 12), dtype=np.uint8)
    for j in range(4):
        scales[..., j] = (sc[..., j] & 63) | ((sc[..., j + 4] >> 4) << 6)
        scales[..., j + 4] = (mq[..., j] & 63) | ((mq[..., j + 4] >> 4) << 6)
        scales[..., j + 8] = (sc[..., j + 4] & 0xF) | ((mq[..., j + 4] & 0xF) << 4)
    qs = (q[..., 0::2, :] | (q[..., 1::2, :] << 4)).reshape(nrow, K // 256, 128)
    out = np.concatenate([_f16_bits(d)[..., None].view(np.uint8).reshape(nrow, K // 256, 2),
                          _f16_bits(dmin)[..., None].view(np.uint8).reshape(nrow, K // 256, 2),
                          scales, qs], axis=-1)
    return out.reshape(*w.shape[:-1], K // 256 * 144)


def _should_quantize(name, arr, block):
    return name not in EMBEDDING_NAMES and arr.ndim == 2 and arr.shape[1] % block == 0


def tensor_values(seed: int, n_layer: int = 24, d=512, ff=2048, vocab=1025, phone_vocab=732):
    """(name, f32 array in PyTorch layout) in converter order, before any conversion: LayerNorm
    gamma and the position alphas 1, LayerNorm beta 0, every other tensor N(0, 0.02) drawn from
    numpy.random.default_rng(seed) in this order."""
    rng = np.random.default_rng(seed)
    for name, shape in tensor_specs(d, ff, n_layer, vocab, phone_vocab):
        base = name.split(".")[-1]
        if base in ("ln1_w", "ln2_w") or name.endswith("pos_alpha"):
            arr = np.ones(shape, dtype=np.float32)
        elif base in ("ln1_b", "ln2_b"):
            arr = np.zeros(shape, dtype=np.float32)
        else:
            arr = (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        yield name, arr


def write_gguf(path: str, wtype: int, seed: int, n_layer: int = 24, d=512, ff=2048, n_head=16,
               vocab=1025, phone_vocab=732, eos=1024) -> str:
    import gguf
    # one temporary name per process: several ranks may generate the same file at once; the
    # final rename is atomic and any of the identical results may win
    tmp = f"{path}.tmp.{os.getpid()}"
    writer = gguf.GGUFWriter(tmp, "t2s")
    for k, v in [("t2s.embedding_dim", d), ("t2s.hidden_dim", d), ("t2s.head", n_head),
                 ("t2s.linear_units", ff), ("t2s.n_layer", n_layer), ("t2s.vocab_size", vocab),
                 ("t2s.phoneme_vocab_size", phone_vocab), ("t2s.eos", eos),
                 ("sovits.inter_channels", 192)]:
        writer.add_uint32(k, v)
    qt = gguf.GGMLQuantizationType
    is_quant = wtype in BLOCK
    for name, arr in tensor_values(seed, n_layer, d, ff, vocab, phone_vocab):
        if is_quant and _should_quantize(name, arr, BLOCK[wtype]):
            if wtype == GGML_Q4_K:
                writer.add_tensor(name, quantize_q4_k(arr), raw_dtype=qt.Q4_K)
            else:
                writer.add_tensor(name, gguf.quantize(arr, qt(wtype)), raw_dtype=qt(wtype))
        elif (is_quant or wtype == GGML_F16) and arr.ndim >= 2 and name != "extract_latent.codebook":
            writer.add_tensor(name, arr.astype(np.float16), raw_dtype=qt.F16)
        else:
            writer.add_tensor(name, arr.astype(np.float32), raw_dtype=qt.F32)
    writer.write_header_to_file()
    writer.write_kv_data_to_file()
    writer.write_tensors_to_file()
    writer.close()
    os.replace(tmp, path)
    return path


def cache_dir() -> str:
    d = os.environ.get("T2SX_CACHE", "/tmp/t2sx_cache")
    os.makedirs(d, exist_ok=True)
    return d


def ensure_gguf(wtype_name: str, seed: int, n_layer: int = 24) -> str:
    """Path of the synthetic GGUF for (type, seed, n_layer), generated once per cache dir."""
    path = os.path.join(cache_dir(), f"t2s-synth-{wtype_name}-s{seed}-L{n_layer}.gguf")
    if not os.path.exists(path):
        write_gguf(path, TYPE_NAMES[wtype_name], seed, n_layer=n_layer)
    return path


def session_inputs(seed: int, T_text: int, T_prompt: int, phone_vocab=732, sem_vocab=1024):
    """Seeded prompt of one session: phoneme ids U[0,732), BERT features N(0,1) [T_text, 1024],
    prompt semantic ids U[0,1024)."""
    rng = np.random.default_rng(seed)
    phones = rng.integers(0, phone_vocab, size=T_text, dtype=np.int32)
    bert = rng.standard_normal(size=(T_text, 1024), dtype=np.float32)
    sem = rng.integers(0, sem_vocab, size=T_prompt, dtype=np.int32)
    return phones, bert, sem


# Workload definitions (the reference's benchmark shapes, synthetic data).
WORKLOADS = {
    # one session, Q8_0 seed 0, 128 phonemes + 150 prompt tokens, 500 greedy steps
    "bs1_q8_0": dict(wtype="q8_0", seed=0, sessions=1, text=(128, 128), prompt=(150, 150), steps=500),
    # 32 sessions, Q4_0 seed 1, phonemes U[64,256], prompt U[50,300], 500 steps
    "bs32_q4_0": dict(wtype="q4_0", seed=1, sessions=32, text=(64, 256), prompt=(50, 300), steps=500),
    # 2048 sessions, Q4_K seed 3, 200 phonemes + 150 prompt tokens, 1000 steps
    "bs2048_q4_k": dict(wtype="q4_k", seed=3, sessions=2048, text=(200, 200), prompt=(150, 150), steps=1000),
}


def workload_lengths(name: str, sessions: int | None = None):
    """Per-session (T_text, T_prompt, input_seed) for a workload."""
    w = WORKLOADS[name]
    n = w["sessions"] if sessions is None else sessions
    out = []
    for s in range(n):
        seed = w["seed"] + s if w["sessions"] > 1 else w["seed"]
        rng = np.random.default_rng(10_000 + seed)
        tt = int(rng.integers(w["text"][0], w["text"][1] + 1))
        tp = int(rng.integers(w["prompt"][0], w["prompt"][1] + 1))
        out.append((tt, tp, seed))
    return out
