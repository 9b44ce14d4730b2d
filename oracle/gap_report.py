"""How far the canonical evaluation order (the one the CUDA kernels reproduce bit for bit) lies
from ggml's CPU operator definitions -- TEST INFRASTRUCTURE ONLY.

Three oracle sessions run the same prompts:
  canon  : the canonical order (GPU == canon, bit for bit, checked by the -m gpu tests);
  ggml16 : ggml's CPU operator definitions with an F16 KV cache (the cache type this path keeps);
  ggml32 : the same with an F32 KV cache (the reference's default kv_cache_type).
Teacher-forced: every session is fed canon's greedy tokens, so each step compares logits of the
same inputs: the max abs difference, the largest |a - b| / (1e-2 + 1e-3 |b|) (at most 1 when the
logit tolerance of 1e-2 absolute plus 1e-3 relative holds), argmax agreement with EOS
masked, and at each disagreement the top1 - top2 margin of canon's logits.  Free-running: ggml16
decodes its own greedy tokens; the first step where its stream leaves canon's is reported.
Sensitivity: canon itself is run again on inputs with a one-ulp change in 1% of the prefill
input elements; its logit change is the model's own rounding sensitivity.

  python oracle/gap_report.py [--configs bs1_q8_0,bs32_q4_0,bs2048_q4_k] [--steps N] [--sessions N]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "gpt-sovits.cpp_b200"))


def _masked(lg, eos):
    lg = lg.copy()
    lg[..., eos] = -np.inf
    return lg.argmax(axis=-1), lg


def ulp_sensitivity(path, lengths, seed=1):
    """Largest logit change of the canonical order when 1% of the prefill input elements move by
    one ulp (first prompt of the list)."""
    import oracle
    import synth
    m = oracle.Model(path)
    tt, tp, sd = lengths[0]
    x = m.embed_prefill(*synth.session_inputs(sd, tt, tp))
    rng = np.random.default_rng(seed)
    xp = x.copy()
    idx = rng.random(x.shape) < 0.01
    xp[idx] = np.nextafter(xp[idx], np.float32(np.inf))
    out = []
    for xx in (x, xp):
        s = oracle.Session(m, 1, tt + tp + 2)
        _, lg, _ = s.prefill(0, xx, tp, want_logits=True)
        out.append(lg)
        s.close()
    m.close()
    return float(np.abs(out[1] - out[0]).max())


def measure(path, lengths, steps, free_running=True):
    import oracle
    import synth
    m = oracle.Model(path)
    n = len(lengths)
    cap = max(tt + tp for tt, tp, _ in lengths) + steps + 2
    modes = {"canon": (0, False), "ggml16": (7, False), "ggml32": (7, True)}
    sess = {}
    for name, (go, f32) in modes.items():
        s = oracle.Session(m, n, cap)
        s.set_mode(ggml_order=go, kv_f32=f32)
        sess[name] = s
    first = {k: [] for k in modes}
    lg0 = {k: [] for k in modes}
    for i, (tt, tp, seed) in enumerate(lengths):
        x = m.embed_prefill(*synth.session_inputs(seed, tt, tp))
        for k, s in sess.items():
            tok, lg, _ = s.prefill(i, x, tp, want_logits=True)
            first[k].append(tok)
            lg0[k].append(lg)
    stats = {k: {"max_abs": 0.0, "max_tol_ratio": 0.0, "rows": 0, "argmax_equal": 0, "flip_margins": []}
             for k in ("ggml16", "ggml32")}

    def compare(ref_lg, lgs):
        ref_tok, ref_m = _masked(ref_lg, m.eos)
        srt = np.sort(ref_m, axis=-1)
        margin = srt[..., -1] - srt[..., -2]
        for k, st in stats.items():
            lg = lgs[k]
            d = np.abs(lg - ref_lg)
            st["max_abs"] = max(st["max_abs"], float(d.max()))
            st["max_tol_ratio"] = max(st["max_tol_ratio"], float((d / (1e-2 + 1e-3 * np.abs(ref_lg))).max()))
            tok, _ = _masked(lg, m.eos)
            st["rows"] += int(tok.size)
            st["argmax_equal"] += int((tok == ref_tok).sum())
            st["flip_margins"] += [float(v) for v in margin[tok != ref_tok]]

    compare(np.stack(lg0["canon"]), {k: np.stack(v) for k, v in lg0.items()})
    slots = np.arange(n)
    cur = np.array(first["canon"], dtype=np.int32)
    canon_stream = [cur.copy()]
    for _ in range(steps):
        lgs = {}
        for k, s in sess.items():
            _, lgs[k] = s.decode(slots, cur, want_logits=True)
        compare(lgs["canon"], lgs)
        cur = _masked(lgs["canon"], m.eos)[0].astype(np.int32)
        canon_stream.append(cur.copy())
    for s in sess.values():
        s.close()
    out = {"sessions": n, "steps": steps, "teacher_forced": {}}
    for k, st in stats.items():
        out["teacher_forced"][k] = {"max_abs": st["max_abs"], "max_tol_ratio": st["max_tol_ratio"],
                                    "argmax_agreement": st["argmax_equal"] / max(st["rows"], 1),
                                    "rows": st["rows"], "flips": len(st["flip_margins"]),
                                    "max_flip_margin": max(st["flip_margins"]) if st["flip_margins"] else None}
    if free_running:
        s = oracle.Session(m, n, cap)
        s.set_mode(ggml_order=True)
        cur = []
        for i, (tt, tp, seed) in enumerate(lengths):
            cur.append(s.prefill(i, m.embed_prefill(*synth.session_inputs(seed, tt, tp)), tp)[0])
        cur = np.array(cur, dtype=np.int32)
        stream = [cur.copy()]
        for _ in range(steps):
            cur, _ = s.decode(slots, cur)
            stream.append(cur.copy())
        stream, canon = np.stack(stream), np.stack(canon_stream)
        first_div = []
        for j in range(n):
            dif = np.nonzero(stream[:, j] != canon[:, j])[0]
            first_div.append(int(dif[0]) if dif.size else None)
        out["free_running_ggml16"] = {"sessions_identical": int(sum(v is None for v in first_div)),
                                      "first_divergence_step": first_div,
                                      "tokens_equal_fraction": float((stream == canon).mean())}
        s.close()
    m.close()
    return out


def main():
    import oracle
    import synth
    ap = argparse.ArgumentParser()
    ap.add_argument("--configs", default="bs1_q8_0,bs32_q4_0,bs2048_q4_k")
    ap.add_argument("--steps", type=int, default=None, help="decode steps (default: 500, 100, 100)")
    ap.add_argument("--sessions", type=int, default=None, help="sessions of the multi-session workloads")
    ap.add_argument("--no-free-running", action="store_true")
    args = ap.parse_args()
    oracle.set_threads(os.cpu_count() or 1)
    defaults = {"bs1_q8_0": (500, 1), "bs32_q4_0": (100, 32), "bs2048_q4_k": (100, 8)}
    for name in args.configs.split(","):
        w = synth.WORKLOADS[name]
        steps, n = defaults[name]
        steps = args.steps or steps
        if args.sessions and w["sessions"] > 1:
            n = args.sessions
        path = synth.ensure_gguf(w["wtype"], w["seed"], n_layer=24)
        lengths = synth.workload_lengths(name)[:n]
        t0 = time.time()
        r = measure(path, lengths, steps, free_running=not args.no_free_running)
        r["ulp_sensitivity_max_abs"] = ulp_sensitivity(path, lengths)
        r.update({"workload": name, "weights": w["wtype"], "seconds": round(time.time() - t0, 1)})
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
