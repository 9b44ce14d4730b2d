"""Golden fixtures under tests/golden/ (written by tests/golden/make_golden.py).

- converter_<type>_L2.json: the reference's converter (python/convert_t2s_to_gguf.py) run on the
  synthetic weights; synth.py's GGUF files must hold the same tensors, byte for byte, in the same
  order with the same metadata, so the files every test loads are the reference's own format.
- oracle_decode_<type>_L2.npz: greedy streams of a small seeded case; the oracle must reproduce
  them (regression pin of the checker), and the GPU path must reproduce them bit for bit without
  running the oracle.
"""
import json
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
sys.path.insert(0, GOLDEN)


@pytest.mark.parametrize("wtype", ["q8_0", "q4_0", "q5_0", "f16"])
def test_synth_gguf_equals_reference_converter_output(wtype):
    import make_golden
    import synth
    fx = json.load(open(os.path.join(GOLDEN, f"converter_{wtype}_L2.json")))
    mine = make_golden.gguf_index(synth.ensure_gguf(wtype, make_golden.SEED, n_layer=make_golden.N_LAYER))
    assert mine["kv"] == fx["kv"]
    assert [t["name"] for t in mine["tensors"]] == [t["name"] for t in fx["tensors"]]
    for a, b in zip(mine["tensors"], fx["tensors"]):
        assert (a["shape"], a["type"]) == (b["shape"], b["type"]), a["name"]
        assert a["sha256"] == b["sha256"], f"{a['name']}: bytes differ from the reference converter's"


@pytest.mark.parametrize("wtype", ["q8_0", "q4_k"])
def test_oracle_reproduces_golden_decode(orc, wtype):
    import make_golden
    fx = np.load(os.path.join(GOLDEN, f"oracle_decode_{wtype}_L2.npz"))
    toks, lg = make_golden.oracle_decode(wtype)
    assert np.array_equal(toks, fx["tokens"])
    assert np.array_equal(lg.view(np.uint32), fx["logits"].view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("wtype", ["q8_0", "q4_k"])
def test_gpu_reproduces_golden_decode(t2sx_mod, wtype):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import make_golden
    import synth
    fx = np.load(os.path.join(GOLDEN, f"oracle_decode_{wtype}_L2.npz"))
    lengths, steps = make_golden.DECODE_CASE["lengths"], make_golden.DECODE_CASE["steps"]
    m = t2sx_mod.Model(synth.ensure_gguf(wtype, make_golden.SEED, n_layer=make_golden.N_LAYER))
    cap = max(tt + tp for tt, tp, _ in lengths) + steps + 1
    s = t2sx_mod.Session(m, len(lengths), cap, repetition_penalty=1.0, eos_mask=True)
    xs = [s.embed_prefill(*synth.session_inputs(seed, tt, tp)) for tt, tp, seed in lengths]
    first = s.prefill(np.arange(len(lengths)), [tt + tp for tt, tp, _ in lengths], [tp for _, tp, _ in lengths],
                      np.concatenate(xs))
    toks = np.concatenate([np.asarray(first, dtype=np.int32)[None], s.decode(steps)])
    lg = np.asarray(s.read_logits(len(lengths)), dtype=np.float32)
    s.close()
    m.close()
    assert np.array_equal(toks, fx["tokens"])
    assert np.array_equal(lg.view(np.uint32), fx["logits"].view(np.uint32))
