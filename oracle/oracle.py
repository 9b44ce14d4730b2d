"""ctypes binding of the T2S oracle (liborc.so) -- TEST INFRASTRUCTURE ONLY.

Loaded by tests/, the smoke entry and bench.py's cpu_baseline / reference arm; never by the
product.  `build()` compiles liborc.so with the Makefile beside this file.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liborc.so")
_lib = None

F32, F16, Q4_0, Q5_0, Q8_0, Q4_K = 0, 1, 2, 6, 8, 12


def build(force: bool = False) -> str:
    src = os.path.join(HERE, "t2s_oracle.cpp")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", HERE, "-B" if force else "liborc.so"], check=True,
                       stdout=subprocess.DEVNULL)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, I, I64, F = C.c_void_p, C.c_int, C.c_int64, C.c_float
        sig = {
            "orc_expf": (F, [F]), "orc_f32_to_f16": (C.c_uint16, [F]), "orc_f16_to_f32": (F, [C.c_uint16]),
            "orc_row_bytes": (I64, [I, I64]),
            "orc_quantize_q8_0": (None, [P, I64, P]), "orc_quantize_q8_K": (None, [P, I64, P]),
            "orc_dequantize": (None, [I, P, I64, P]),
            "orc_matmul": (I, [I, P, I64, I64, P, I64, P]),
            "orc_attn_decode": (None, [P, P, P, I, P]),
            "orc_attn_rows": (None, [I, P, P, P, P, P, I, P]),
            "orc_layernorm": (None, [P, P, P, I, F, P]), "orc_pe_row": (None, [I, I, P]),
            "orc_model_load": (P, [C.c_char_p]), "orc_model_free": (None, [P]),
            "orc_model_info": (I, [P, P, P]),
            "orc_session_new": (P, [P, I, I]), "orc_session_free": (None, [P]),
            "orc_set_threads": (None, [I]),
            "orc_embed_prefill": (I, [P, P, P, I, P, I, P]),
            "orc_prefill": (I, [P, I, P, I, I, I, P, P, P]),
            "orc_decode_step": (I, [P, I, P, P, P, F, I, P, P]),
            "orc_slot_n_pos": (I, [P, I]), "orc_slot_release": (I, [P, I]),
            "orc_extract_latent": (I, [P, P, I, P]), "orc_read_kv": (I, [P, I, I, I, P]),
            "orc_sample": (I, [P, I, P, P, P, I, F, F, F, I, P, P]),
            "orc_decode_step2": (I, [P, I, P, P, P, P, I, F, F, F, I, P, P, P]),
            "orc_session_set_mode": (I, [P, I, I]),
            "orc_matmul_ggml": (I, [I, P, I64, I64, P, I64, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def expf(x: float) -> float:
    return lib().orc_expf(x)


def matmul(wtype: int, w_bytes: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    y = np.empty((x.shape[0], N), dtype=np.float32)
    rc = lib().orc_matmul(wtype, ptr(np.ascontiguousarray(w_bytes)), N, K, ptr(x), x.shape[0], ptr(y))
    assert rc == 0
    return y


def matmul_ggml(wtype: int, w_bytes: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
    """The matmul with ggml's generic vec_dot folds instead of the canonical order."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    y = np.empty((x.shape[0], N), dtype=np.float32)
    rc = lib().orc_matmul_ggml(wtype, ptr(np.ascontiguousarray(w_bytes)), N, K, ptr(x), x.shape[0], ptr(y))
    assert rc == 0
    return y


def attn_rows(seqs, lens, q16: np.ndarray, k16: np.ndarray, v16: np.ndarray) -> np.ndarray:
    """Batched attention rows; k16/v16 f16 bits [n_seqs][max_len][16][32], q16 f16 bits [n][512].
    Returns f32 [n][512]."""
    seqs = np.ascontiguousarray(seqs, dtype=np.int32)
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    q16 = np.ascontiguousarray(q16, dtype=np.uint16)
    k16 = np.ascontiguousarray(k16, dtype=np.uint16)
    v16 = np.ascontiguousarray(v16, dtype=np.uint16)
    out = np.empty((len(seqs), 512), dtype=np.float32)
    lib().orc_attn_rows(len(seqs), ptr(seqs), ptr(lens), ptr(q16), ptr(k16), ptr(v16), k16.shape[1], ptr(out))
    return out


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size // 32 * 34, dtype=np.uint8)
    lib().orc_quantize_q8_0(ptr(x), x.size, ptr(out))
    return out


def dequantize(wtype: int, data: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().orc_dequantize(wtype, ptr(np.ascontiguousarray(data)), n, ptr(out))
    return out


class Model:
    def __init__(self, path: str):
        self.h = lib().orc_model_load(path.encode())
        if not self.h:
            raise RuntimeError(f"oracle could not load {path}")
        hp = np.zeros(9, dtype=np.uint32)
        types = np.zeros(4, dtype=np.int32)
        lib().orc_model_info(self.h, ptr(hp), ptr(types))
        self.hp = hp
        (self.embedding_dim, self.d, self.n_head, self.ff, self.n_layer, self.vocab,
         self.phone_vocab, self.eos, _) = [int(v) for v in hp]
        self.types = types

    def embed_prefill(self, phones, bert, sem):
        phones = np.ascontiguousarray(phones, dtype=np.int32)
        sem = np.ascontiguousarray(sem, dtype=np.int32)
        bert = np.ascontiguousarray(bert, dtype=np.float32)
        x = np.empty((phones.size + sem.size, self.d), dtype=np.float32)
        rc = lib().orc_embed_prefill(self.h, ptr(phones), ptr(bert), phones.size, ptr(sem), sem.size, ptr(x))
        assert rc == 0
        return x

    def extract_latent(self, hubert: np.ndarray) -> np.ndarray:
        """Prompt semantic codes of HuBERT frames f32 [T][768]."""
        hubert = np.ascontiguousarray(hubert, dtype=np.float32)
        T = hubert.shape[0]
        out = np.empty((T - 2) // 2 + 1, dtype=np.int32)
        n = lib().orc_extract_latent(self.h, ptr(hubert), T, ptr(out))
        assert n == out.size, n
        return out

    def sample(self, logits, seen=None, noise=None, top_k=15, top_p=1.0, temperature=1.0, rep_penalty=1.0,
               eos_mask=True):
        logits = np.ascontiguousarray(logits, dtype=np.float32).reshape(-1, self.vocab)
        n = logits.shape[0]
        seen_a = None if seen is None else np.ascontiguousarray(seen, dtype=np.float32).reshape(n, self.vocab)
        noise_a = None if noise is None else np.ascontiguousarray(noise, dtype=np.float32).reshape(n, self.vocab)
        sampled = np.zeros(n, dtype=np.int32)
        greedy = np.zeros(n, dtype=np.int32)
        lib().orc_sample(self.h, n, ptr(logits), ptr(seen_a), ptr(noise_a), int(top_k), float(top_p),
                         float(temperature), float(rep_penalty), int(eos_mask), ptr(sampled), ptr(greedy))
        return sampled, greedy

    def close(self):
        if self.h:
            lib().orc_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    def __init__(self, model: Model, n_slots: int, capacity: int):
        self.model = model
        self.h = lib().orc_session_new(model.h, n_slots, capacity)
        if not self.h:
            raise RuntimeError("oracle session init failed")

    def set_mode(self, ggml_order: bool | int = False, kv_f32: bool = False):
        """Evaluation order (before the first prefill): ggml_order=True (or the operator mask 7;
        1 matmuls, 2 LayerNorm, 4 attention) follows ggml's CPU operator definitions; kv_f32
        keeps an F32 KV cache (the reference's default; implies the full ggml order)."""
        mask = 7 if ggml_order is True else int(ggml_order)
        if lib().orc_session_set_mode(self.h, mask, int(kv_f32)) != 0:
            raise RuntimeError("oracle mode must be set before the first prefill")

    def prefill(self, slot: int, x: np.ndarray, T_prompt: int, eos_mask=True, want_logits=False, want_y=False):
        x = np.ascontiguousarray(x, dtype=np.float32)
        tok = np.zeros(1, dtype=np.int32)
        logits = np.empty(self.model.vocab, dtype=np.float32) if want_logits else None
        y = np.empty_like(x) if want_y else None
        rc = lib().orc_prefill(self.h, slot, ptr(x), x.shape[0], T_prompt, int(eos_mask), ptr(tok), ptr(logits), ptr(y))
        if rc != 0:
            raise RuntimeError("oracle prefill rejected")
        return int(tok[0]), logits, y

    def decode(self, slots, tokens, seen=None, rep_penalty=1.0, eos_mask=True, want_logits=False):
        slots = np.ascontiguousarray(slots, dtype=np.int32)
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(slots.size, dtype=np.int32)
        logits = np.empty((slots.size, self.model.vocab), dtype=np.float32) if want_logits else None
        seen_a = None if seen is None else np.ascontiguousarray(seen, dtype=np.float32)
        rc = lib().orc_decode_step(self.h, slots.size, ptr(slots), ptr(tokens), ptr(seen_a),
                                   float(rep_penalty), int(eos_mask), ptr(out), ptr(logits))
        if rc != 0:
            raise RuntimeError("oracle decode rejected")
        return out, logits

    def decode_sampled(self, slots, tokens, noise, seen=None, top_k=15, top_p=1.0, temperature=1.0,
                       rep_penalty=1.0, eos_mask=True):
        slots = np.ascontiguousarray(slots, dtype=np.int32)
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        n, V = slots.size, self.model.vocab
        noise_a = None if noise is None else np.ascontiguousarray(noise, dtype=np.float32).reshape(n, V)
        seen_a = None if seen is None else np.ascontiguousarray(seen, dtype=np.float32).reshape(n, V)
        sampled = np.empty(n, dtype=np.int32)
        greedy = np.empty(n, dtype=np.int32)
        rc = lib().orc_decode_step2(self.h, n, ptr(slots), ptr(tokens), ptr(seen_a), ptr(noise_a), int(top_k),
                                    float(top_p), float(temperature), float(rep_penalty), int(eos_mask),
                                    ptr(sampled), ptr(greedy), None)
        if rc != 0:
            raise RuntimeError("oracle decode rejected")
        return sampled, greedy

    def release(self, slot):
        if lib().orc_slot_release(self.h, slot) != 0:
            raise RuntimeError("oracle release rejected")

    def n_pos(self, slot):
        return lib().orc_slot_n_pos(self.h, slot)

    def read_kv(self, slot, layer, which):
        n = self.n_pos(slot)
        out = np.empty((n, self.model.d), dtype=np.uint16)
        lib().orc_read_kv(self.h, slot, layer, which, ptr(out))
        return out

    def close(self):
        if self.h:
            lib().orc_session_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def set_threads(n: int):
    lib().orc_set_threads(int(n))
