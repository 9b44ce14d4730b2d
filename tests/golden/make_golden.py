"""Golden fixtures (test infrastructure; regenerate, never hand-edit).

1. converter_<type>_L2.json -- the reference's own converter, python/convert_t2s_to_gguf.py, run on
   synthetic checkpoints that hold synth.tensor_values(seed 7, 2 layers): per GGUF tensor its
   name, shape, GGML type and the SHA-256 of the bytes the converter writes, in file order, and
   the KV metadata.  The converter needs the reference checkout; run this where it exists:

       python tests/golden/make_golden.py --reference /root/reference

2. oracle_decode_<type>_L2.npz -- the oracle's greedy streams for a small seeded case (3 sessions
   of the 2-layer model, 12 steps, EOS masked): tokens [13][3] (the prefill token, then one row
   per step) and the last step's logits [3][1025].  It needs only this repository.

tests/test_golden.py checks synth.py's GGUF files against (1), and the oracle (CPU) and the GPU
path (-m gpu) against (2).
"""
import argparse
import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "gpt-sovits.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

# converter --type names -> synth.py type names
CONVERTER_TYPES = {"q8": "q8_0", "q4": "q4_0", "q5": "q5_0", "f16": "f16"}
SEED, N_LAYER = 7, 2
DECODE_CASE = {"lengths": [(24, 16, 901), (9, 30, 902), (40, 5, 903)], "steps": 12}


def gguf_index(path):
    """Tensor list (name, shape, type, sha256 of the data bytes) and KV metadata of a GGUF file."""
    from gguf import GGUFReader
    rd = GGUFReader(path)
    tensors = [{"name": t.name, "shape": [int(v) for v in t.shape], "type": int(t.tensor_type),
                "sha256": hashlib.sha256(np.ascontiguousarray(t.data).tobytes()).hexdigest()} for t in rd.tensors]
    kv = {}
    for f in rd.fields.values():
        if f.name.startswith(("t2s.", "sovits.")):
            kv[f.name] = int(f.parts[f.data[0]][0])
    return {"tensors": tensors, "kv": kv}


def converter_fixture(reference, ctype, out_dir):
    import torch
    import synth
    sys.path.insert(0, os.path.join(reference, "python"))
    import convert_t2s_to_gguf as conv
    to_ckpt = {}
    for gname, cname in conv.T2S_ATTENTION_MAP:
        for i in range(N_LAYER):
            to_ckpt[gname.format(i=i)] = ("t2s", cname.format(i=i))
    for gname, cname in conv.T2S_ENCODER_MAP + conv.T2S_SAMPLER_MAP:
        to_ckpt[gname] = ("t2s", cname)
    for gname, cname in conv.SOVITS_EXTRACT_LATENT_MAP:
        to_ckpt[gname] = ("sovits", cname)
    sd = {"t2s": {}, "sovits": {}}
    for name, arr in synth.tensor_values(SEED, N_LAYER):
        which, cname = to_ckpt[name]
        sd[which][cname] = torch.from_numpy(np.ascontiguousarray(arr))
    with tempfile.TemporaryDirectory() as tmp:
        t2s_path, sovits_path = os.path.join(tmp, "t2s.ckpt"), os.path.join(tmp, "sovits.pth")
        torch.save({"weight": sd["t2s"], "config": {"model": {
            "embedding_dim": 512, "hidden_dim": 512, "head": 16, "linear_units": 2048, "n_layer": N_LAYER,
            "vocab_size": 1025, "phoneme_vocab_size": 732, "EOS": 1024}}}, t2s_path)
        torch.save({"weight": sd["sovits"], "config": {"model": {"inter_channels": 192}}}, sovits_path)
        out = os.path.join(tmp, "ref.gguf")
        conv.convert(t2s_path, sovits_path, out, ctype)
        idx = gguf_index(out)
    idx["source"] = f"python/convert_t2s_to_gguf.py --type {ctype} on synth.tensor_values(seed={SEED}, n_layer={N_LAYER})"
    path = os.path.join(out_dir, f"converter_{CONVERTER_TYPES[ctype]}_L{N_LAYER}.json")
    with open(path, "w") as f:
        json.dump(idx, f, indent=1)
    return path


def oracle_decode(wtype):
    """Greedy streams of the small decode case on the oracle: tokens [steps + 1][n], logits [n][V]."""
    import oracle
    import synth
    m = oracle.Model(synth.ensure_gguf(wtype, SEED, n_layer=N_LAYER))
    lengths, steps = DECODE_CASE["lengths"], DECODE_CASE["steps"]
    cap = max(tt + tp for tt, tp, _ in lengths) + steps + 1
    s = oracle.Session(m, len(lengths), cap)
    first = []
    for i, (tt, tp, seed) in enumerate(lengths):
        ph, bert, sem = synth.session_inputs(seed, tt, tp)
        first.append(s.prefill(i, m.embed_prefill(ph, bert, sem), tp, eos_mask=True)[0])
    toks = [np.array(first, dtype=np.int32)]
    cur = toks[0]
    lg = None
    for k in range(steps):
        cur, lg = s.decode(np.arange(len(lengths)), cur, eos_mask=True, want_logits=(k == steps - 1))
        toks.append(cur.copy())
    return np.stack(toks).astype(np.int32), np.asarray(lg, dtype=np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="checkout of the reference (for the converter fixtures)")
    args = ap.parse_args()
    if args.reference:
        for ctype in CONVERTER_TYPES:
            print("wrote", converter_fixture(args.reference, ctype, HERE))
    for wtype in ("q8_0", "q4_k"):
        toks, lg = oracle_decode(wtype)
        path = os.path.join(HERE, f"oracle_decode_{wtype}_L{N_LAYER}.npz")
        np.savez_compressed(path, tokens=toks, logits=lg)
        print("wrote", path)


if __name__ == "__main__":
    main()
