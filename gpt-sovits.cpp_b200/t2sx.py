"""Python binding of libt2sx.so (include/t2sx.h) over ctypes.

Host-side mirror of the reference's T2S model/session interface (include/gpt_sovits/t2s.h):
`Model` ~ t2s_model (t2s_model_load / t2s_model_free), `Session` ~ t2s_session
(t2s_session_init, find_free_slot, slot_release, slot_n_pos, flex-graph prefill, persistent
decode graph).  Errors raise `T2SXError` carrying the library's status code and message; the
reference returns false or aborts in the same places.  There is no CPU fallback: without the
CUDA library (or a GPU) every call fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libt2sx.so")

OK, ERR_INVALID, ERR_IO, ERR_FORMAT, ERR_CUDA, ERR_OOM, ERR_STATE, ERR_BOUNDS, ERR_TIMEOUT = range(9)
F32, F16, Q4_0, Q8_0, Q4_K = 0, 1, 2, 8, 12

# Every symbol include/t2sx.h declares: (restype, argtypes).
_P, _I, _I64, _F, _U32P = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.POINTER(C.c_uint32)
SIGNATURES = {
    "t2sx_last_error": (C.c_char_p, []),
    "t2sx_version": (C.c_int, []),
    "t2sx_device_count": (C.c_int, [_P]),
    "t2sx_model_load": (C.c_int, [C.c_char_p, _I, _P]),
    "t2sx_model_free": (None, [_P]),
    "t2sx_model_hparams": (C.c_int, [_P, _P, _P]),
    "t2sx_model_device_bytes": (C.c_int, [_P, _P]),
    "t2sx_session_create": (C.c_int, [_P, C.c_uint32, C.c_uint32, _P, _P]),
    "t2sx_session_free": (None, [_P]),
    "t2sx_session_find_free_slot": (C.c_int, [_P]),
    "t2sx_session_slot_release": (C.c_int, [_P, _I]),
    "t2sx_session_slot_n_pos": (C.c_int, [_P, _I]),
    "t2sx_session_slot_audio_offset": (C.c_int, [_P, _I]),
    "t2sx_session_device_bytes": (C.c_int, [_P, _P]),
    "t2sx_embed_prefill": (C.c_int, [_P, _P, _P, _I, _P, _I, _P, _I]),
    "t2sx_prefill": (C.c_int, [_P, _I, _P, _P, _P, _P, _I, _P]),
    "t2sx_flex_step": (C.c_int, [_P, _I, _P, _P, _I, _P, _P, _P, _P, _P]),
    "t2sx_decode": (C.c_int, [_P, _I, _P]),
    "t2sx_decode_async": (C.c_int, [_P, _I]),
    "t2sx_synchronize": (C.c_int, [_P]),
    "t2sx_decode_step_host": (C.c_int, [_P, _P, _P]),
    "t2sx_active_slots": (C.c_int, [_P, _P, _P]),
    "t2sx_read_logits": (C.c_int, [_P, _P, _I, _P]),
    "t2sx_read_kv": (C.c_int, [_P, _I, _I, _I, _P]),
    "t2sx_set_seen": (C.c_int, [_P, _I, _P]),
    "t2sx_last_decode_ms": (C.c_int, [_P, _P]),
    "t2sx_set_exp_noise": (C.c_int, [_P, _P, _I]),
    "t2sx_read_greedy": (C.c_int, [_P, _P, _I, _P]),
    "t2sx_decode_graph_kernels": (C.c_int, [_P, _P]),
    "t2sx_profile_step": (C.c_int, [_P, _I, _P]),
    "t2sx_weight_create": (C.c_int, [_I, _I, _P, _I64, _I64, _P]),
    "t2sx_weight_free": (None, [_P]),
    "t2sx_matmul": (C.c_int, [_P, _P, _I64, _P, _P, _P]),
    "t2sx_matmul_noalloc": (C.c_int, [_P, _P, _I64, _P, _P, _P]),
    "t2sx_weight_sync": (C.c_int, [_P, _P]),
    "t2sx_probe_l2_read": (C.c_int, [_I, _I64, _I, _P]),
    "t2sx_probe_i8_mma": (C.c_int, [_I, _I, _I, _P]),
    "t2sx_read_hidden": (C.c_int, [_P, _P, _I, _P]),
    "t2sx_model_tensor_info": (C.c_int, [_P, C.c_char_p, _P, _P, _P]),
    "t2sx_test_set_tc_wait_cycles": (C.c_int, [_I64]),
    "t2sx_kvcache_create": (C.c_int, [_I, _I, _I, _P]),
    "t2sx_kvcache_free": (None, [_P]),
    "t2sx_kvcache_write": (C.c_int, [_P, _I, _I, _I, _P, _P]),
    "t2sx_kvcache_attn_decode": (C.c_int, [_P, _I, _P, _P, _P, _P, _P]),
    "t2sx_kvcache_attn_prefill": (C.c_int, [_P, _I, _P, _P, _P, _P, _P]),
    "t2sx_extract_latent": (C.c_int, [_P, _P, _I, _P]),
}
NOALLOC_MAX_ELEMS = 1 << 21


class T2SXError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[t2sx {code}] {msg}")
        self.code = code


class SamplerConfig(C.Structure):
    _fields_ = [("top_k", C.c_int32), ("top_p", C.c_float), ("temperature", C.c_float),
                ("repetition_penalty", C.c_float), ("eos_mask", C.c_int32)]


_lib = None


def lib(path: str | None = None):
    """Load libt2sx.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise T2SXError(ERR_INVALID, f"{p} is missing: run __graft_entry__.build()")
        L = C.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ck(rc):
    if rc != OK:
        raise T2SXError(rc, lib().t2sx_last_error().decode())
    return rc


def _p(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def test_set_tc_wait_cycles(cycles: int):
    """Test hook: cycles > 0 makes later tensor-core matmul launches wait first on a barrier that
    nothing completes, every wait bounded by `cycles` (their error path runs); 0 = normal."""
    _ck(lib().t2sx_test_set_tc_wait_cycles(int(cycles)))


def probe_l2_read_gbs(device: int = 0, bytes_: int = 32 << 20, iters: int = 200) -> float:
    """Measured L2 read bandwidth (GB/s) of an L2-resident buffer."""
    v = C.c_double(0)
    _ck(lib().t2sx_probe_l2_read(device, bytes_, iters, C.byref(v)))
    return v.value


def probe_i8_mma_tops(device: int = 0, iters: int = 20000, issuers: int = 1) -> float:
    """Measured dense int8 tcgen05 rate (TOP/s)."""
    v = C.c_double(0)
    _ck(lib().t2sx_probe_i8_mma(device, iters, issuers, C.byref(v)))
    return v.value


def device_count() -> int:
    n = C.c_int32(0)
    _ck(lib().t2sx_device_count(C.byref(n)))
    return n.value


class Model:
    """t2s_model: weights of one GGUF on one device."""

    def __init__(self, path: str, device: int = 0):
        h = C.c_void_p()
        _ck(lib().t2sx_model_load(path.encode(), device, C.byref(h)))
        self.h = h
        self.device = device
        hp = np.zeros(9, dtype=np.uint32)
        wt = np.zeros(4, dtype=np.int32)
        _ck(lib().t2sx_model_hparams(self.h, _p(hp), _p(wt)))
        self.hp = hp
        (self.embedding_dim, self.d, self.n_head, self.ff, self.n_layer, self.vocab,
         self.phone_vocab, self.eos, self.inter_channels) = [int(v) for v in hp]
        self.wtypes = wt

    def device_bytes(self) -> int:
        b = C.c_uint64(0)
        _ck(lib().t2sx_model_device_bytes(self.h, C.byref(b)))
        return b.value

    def close(self):
        if self.h:
            lib().t2sx_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """t2s_session: n_slots sequences of up to slot_size positions (paged f16 KV)."""

    def __init__(self, model: Model, n_slots: int, slot_size: int, top_k=15, top_p=1.0, temperature=1.0,
                 repetition_penalty=1.35, eos_mask=False):
        self.model = model
        self.cfg = SamplerConfig(top_k, top_p, temperature, repetition_penalty, int(eos_mask))
        h = C.c_void_p()
        _ck(lib().t2sx_session_create(model.h, n_slots, slot_size, C.byref(self.cfg), C.byref(h)))
        self.h = h
        self.n_slots, self.slot_size = n_slots, slot_size

    # ---- slots -------------------------------------------------------------------------------
    def find_free_slot(self) -> int:
        return lib().t2sx_session_find_free_slot(self.h)

    def slot_release(self, slot: int):
        _ck(lib().t2sx_session_slot_release(self.h, slot))

    def slot_n_pos(self, slot: int) -> int:
        return lib().t2sx_session_slot_n_pos(self.h, slot)

    def slot_audio_offset(self, slot: int) -> int:
        return lib().t2sx_session_slot_audio_offset(self.h, slot)

    def active_slots(self):
        out = np.zeros(self.n_slots, dtype=np.int32)
        n = C.c_int32(0)
        _ck(lib().t2sx_active_slots(self.h, _p(out), C.byref(n)))
        return out[: n.value]

    def device_bytes(self) -> int:
        b = C.c_uint64(0)
        _ck(lib().t2sx_session_device_bytes(self.h, C.byref(b)))
        return b.value

    # ---- prefill -----------------------------------------------------------------------------
    def embed_prefill(self, phones, bert, sem, out_dev_ptr: int | None = None):
        phones = np.ascontiguousarray(phones, dtype=np.int32)
        sem = np.ascontiguousarray(sem, dtype=np.int32)
        bert = np.ascontiguousarray(bert, dtype=np.float32)
        T = phones.size + sem.size
        if out_dev_ptr is not None:
            _ck(lib().t2sx_embed_prefill(self.h, _p(phones), _p(bert), phones.size, _p(sem), sem.size,
                                         C.c_void_p(out_dev_ptr), 1))
            return None
        x = np.empty((T, self.model.d), dtype=np.float32)
        _ck(lib().t2sx_embed_prefill(self.h, _p(phones), _p(bert), phones.size, _p(sem), sem.size, _p(x), 0))
        return x

    def extract_latent(self, hubert: np.ndarray) -> np.ndarray:
        """Prompt semantic codes of HuBERT frames f32 [T][768] (T >= 2): int32 [(T - 2) // 2 + 1]."""
        hubert = np.ascontiguousarray(hubert, dtype=np.float32)
        T = hubert.shape[0]
        out = np.empty((T - 2) // 2 + 1, dtype=np.int32)
        _ck(lib().t2sx_extract_latent(self.h, _p(hubert), T, _p(out)))
        return out

    def prefill(self, slots, n_query, t_prompt, x=None, x_dev_ptr: int | None = None):
        slots = np.ascontiguousarray(np.atleast_1d(slots), dtype=np.int32)
        nq = np.ascontiguousarray(np.atleast_1d(n_query), dtype=np.int32)
        tp = np.ascontiguousarray(np.atleast_1d(t_prompt), dtype=np.int32)
        toks = np.zeros(slots.size, dtype=np.int32)
        if x_dev_ptr is not None:
            _ck(lib().t2sx_prefill(self.h, slots.size, _p(slots), _p(nq), _p(tp), C.c_void_p(x_dev_ptr), 1, _p(toks)))
        else:
            x = np.ascontiguousarray(x, dtype=np.float32)
            assert x.shape == (int(nq.sum()), self.model.d)
            _ck(lib().t2sx_prefill(self.h, slots.size, _p(slots), _p(nq), _p(tp), _p(x), 0, _p(toks)))
        return toks

    def flex_step(self, dec_slots, dec_tokens, pre_slots=(), n_query=(), t_prompt=(), x=None):
        """One pass over a mixed plan: a decode step of dec_slots (input tokens dec_tokens) and the
        prefill of pre_slots (rows x f32 [sum n_query][d]); returns the decode slots' tokens then the
        prefill slots' first tokens."""
        ds = np.ascontiguousarray(np.atleast_1d(dec_slots), dtype=np.int32)
        dt = np.ascontiguousarray(np.atleast_1d(dec_tokens), dtype=np.int32)
        ps = np.ascontiguousarray(np.atleast_1d(pre_slots), dtype=np.int32)
        nq = np.ascontiguousarray(np.atleast_1d(n_query), dtype=np.int32)
        tp = np.ascontiguousarray(np.atleast_1d(t_prompt), dtype=np.int32)
        assert ds.size == dt.size and ps.size == nq.size == tp.size
        xp = None
        if ps.size:
            x = np.ascontiguousarray(x, dtype=np.float32)
            assert x.shape == (int(nq.sum()), self.model.d)
            xp = _p(x)
        toks = np.zeros(ds.size + ps.size, dtype=np.int32)
        _ck(lib().t2sx_flex_step(self.h, ds.size, _p(ds) if ds.size else None, _p(dt) if dt.size else None, ps.size,
                                 _p(ps) if ps.size else None, _p(nq) if ps.size else None,
                                 _p(tp) if ps.size else None, xp, _p(toks)))
        return toks

    # ---- decode ------------------------------------------------------------------------------
    def decode(self, n_steps: int, want_tokens=True):
        n_act = len(self.active_slots())
        out = np.zeros((n_steps, n_act), dtype=np.int32) if want_tokens else None
        _ck(lib().t2sx_decode(self.h, n_steps, _p(out)))
        return out

    def decode_async(self, n_steps: int):
        _ck(lib().t2sx_decode_async(self.h, n_steps))

    def synchronize(self):
        _ck(lib().t2sx_synchronize(self.h))

    def decode_step_host(self, tokens_in=None, want_tokens=True):
        n_act = len(self.active_slots())
        tin = None if tokens_in is None else np.ascontiguousarray(tokens_in, dtype=np.int32)
        out = np.zeros(n_act, dtype=np.int32) if want_tokens else None
        _ck(lib().t2sx_decode_step_host(self.h, _p(tin), _p(out)))
        return out

    def last_decode_ms(self) -> float:
        v = C.c_float(0)
        _ck(lib().t2sx_last_decode_ms(self.h, C.byref(v)))
        return v.value

    def graph_kernels(self) -> int:
        n = C.c_int32(0)
        _ck(lib().t2sx_decode_graph_kernels(self.h, C.byref(n)))
        return n.value

    def profile_step(self, iters: int = 20):
        ms = np.zeros(9, dtype=np.float32)
        _ck(lib().t2sx_profile_step(self.h, iters, _p(ms)))
        return dict(zip(["attention", "mm_qkv", "mm_out", "mm_up", "mm_down", "mm_lm_head", "residual_ln",
                         "quant_2048", "attention_kernel"], ms.tolist()))

    def read_logits(self, max_rows: int | None = None):
        max_rows = max_rows or self.n_slots
        out = np.zeros((max_rows, self.model.vocab), dtype=np.float32)
        rows = C.c_int32(0)
        _ck(lib().t2sx_read_logits(self.h, _p(out), max_rows, C.byref(rows)))
        return out[: rows.value]

    def read_hidden(self, max_rows: int):
        """Final-layer rows f32 [rows][d] of the last pass."""
        out = np.empty((max_rows, self.model.d), dtype=np.float32)
        n = C.c_int32(0)
        _ck(lib().t2sx_read_hidden(self.h, _p(out), max_rows, C.byref(n)))
        return out[:n.value]

    def read_kv(self, slot: int, layer: int, which: int):
        n = self.slot_n_pos(slot)
        out = np.zeros((max(n, 1), self.model.d), dtype=np.uint16)
        _ck(lib().t2sx_read_kv(self.h, slot, layer, which, _p(out)))
        return out[:n]

    def set_exp_noise(self, noise):
        """Exp(1) noise [rows][vocab] for the following passes (None: back to greedy)."""
        if noise is None:
            _ck(lib().t2sx_set_exp_noise(self.h, None, 0))
            return
        noise = np.ascontiguousarray(noise, dtype=np.float32).reshape(-1, self.model.vocab)
        _ck(lib().t2sx_set_exp_noise(self.h, _p(noise), noise.shape[0]))

    def read_greedy(self, max_rows: int | None = None):
        max_rows = max_rows or self.n_slots
        out = np.zeros(max_rows, dtype=np.int32)
        rows = C.c_int32(0)
        _ck(lib().t2sx_read_greedy(self.h, _p(out), max_rows, C.byref(rows)))
        return out[: rows.value]

    def set_seen(self, slot: int, seen):
        seen = np.ascontiguousarray(seen, dtype=np.uint8)
        _ck(lib().t2sx_set_seen(self.h, slot, _p(seen)))

    def close(self):
        if self.h:
            lib().t2sx_session_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Weight:
    """A repacked linear weight for the isolated matmul entry point."""

    def __init__(self, wtype: int, host_bytes: np.ndarray, N: int, K: int, device: int = 0):
        h = C.c_void_p()
        host_bytes = np.ascontiguousarray(host_bytes)
        _ck(lib().t2sx_weight_create(device, wtype, _p(host_bytes), N, K, C.byref(h)))
        self.h, self.N, self.K = h, N, K

    def matmul(self, x_ptr: int, M: int, y_ptr: int, bias_ptr: int | None = None, stream: int = 0):
        _ck(lib().t2sx_matmul(self.h, C.c_void_p(x_ptr), M, None if bias_ptr is None else C.c_void_p(bias_ptr),
                              C.c_void_p(y_ptr), C.c_void_p(stream)))

    def matmul_noalloc(self, x_ptr: int, M: int, y_ptr: int, bias_ptr: int | None = None, stream: int = 0):
        """Same result as matmul(), using the library's fixed scratch instead of allocating."""
        _ck(lib().t2sx_matmul_noalloc(self.h, C.c_void_p(x_ptr), M, None if bias_ptr is None else C.c_void_p(bias_ptr),
                                      C.c_void_p(y_ptr), C.c_void_p(stream)))

    def sync(self, stream: int = 0):
        """Waits for the stream; raises T2SXError(ERR_TIMEOUT) if a matmul on this weight gave up
        a bounded wait since the last check (its outputs are then NaN)."""
        _ck(lib().t2sx_weight_sync(self.h, C.c_void_p(stream)))

    def close(self):
        if self.h:
            lib().t2sx_weight_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KVCache:
    """One-layer paged f16 KV cache for the isolated attention entry points."""

    def __init__(self, n_seqs: int, max_len: int, device: int = 0):
        h = C.c_void_p()
        _ck(lib().t2sx_kvcache_create(device, n_seqs, max_len, C.byref(h)))
        self.h, self.n_seqs, self.max_len = h, n_seqs, max_len

    def write(self, seq: int, pos0: int, k16: np.ndarray, v16: np.ndarray):
        """k16, v16: f16 bits (uint16) [len][16][32]."""
        k16 = np.ascontiguousarray(k16, dtype=np.uint16)
        v16 = np.ascontiguousarray(v16, dtype=np.uint16)
        _ck(lib().t2sx_kvcache_write(self.h, seq, pos0, k16.shape[0], _p(k16), _p(v16)))

    def _attn(self, fn, seqs, lens, q_ptr: int, out_ptr: int, stream: int):
        seqs = np.ascontiguousarray(seqs, dtype=np.int32)
        lens = np.ascontiguousarray(lens, dtype=np.int32)
        _ck(fn(self.h, len(seqs), _p(seqs), _p(lens), C.c_void_p(q_ptr), C.c_void_p(out_ptr), C.c_void_p(stream)))

    def attn_decode(self, seqs, lens, q_ptr: int, out_ptr: int, stream: int = 0):
        self._attn(lib().t2sx_kvcache_attn_decode, seqs, lens, q_ptr, out_ptr, stream)

    def attn_prefill(self, seqs, lens, q_ptr: int, out_ptr: int, stream: int = 0):
        self._attn(lib().t2sx_kvcache_attn_prefill, seqs, lens, q_ptr, out_ptr, stream)

    def close(self):
        if self.h:
            lib().t2sx_kvcache_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
