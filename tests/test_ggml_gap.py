"""The canonical evaluation order (the one the CUDA kernels reproduce bit for bit) against ggml's
CPU operator definitions (the oracle's ggml-order mode: generic vec_dot folds, sequential
LayerNorm sums, per-query flash attention with an f16 V accumulator, libm expf), on the 24-layer
model with the one-session workload's prompt, teacher-forced (both fed the canonical tokens).

* F16 weights (convert_t2s_to_gguf.py's default output type): logits agree within the stated
  tolerance, |a - b| <= 1e-2 + 1e-3 |b|, with an F16 and with an F32 KV cache, and every greedy
  token agrees.
* Q8_0 weights: activations are quantised to Q8_0 before every matmul, so a one-ulp change of an
  input can move a value by a whole quantisation step.  The gap then equals the model's own
  rounding sensitivity (the logit change from a one-ulp change of 1% of the prefill inputs under
  the same order): it stays within 3x that sensitivity, and a greedy token differs only where the
  top two logits are closer than twice the gap.
"""
import os

import numpy as np
import pytest

STEPS = 24


def _gap(path, steps):
    import oracle
    import synth
    import gap_report
    oracle.set_threads(os.cpu_count() or 1)
    lengths = synth.workload_lengths("bs1_q8_0")
    return gap_report.measure(path, lengths, steps, free_running=False), gap_report.ulp_sensitivity(path, lengths)


def test_f16_weights_within_logit_tolerance(orc):
    import synth
    r, _ = _gap(synth.ensure_gguf("f16", 0, n_layer=24), STEPS)
    for mode in ("ggml16", "ggml32"):
        t = r["teacher_forced"][mode]
        assert t["max_tol_ratio"] <= 1.0, (mode, t)
        assert t["argmax_agreement"] == 1.0, (mode, t)


def test_q8_0_gap_is_the_models_rounding_sensitivity(orc):
    import synth
    r, ulp = _gap(synth.ensure_gguf("q8_0", 0, n_layer=24), STEPS)
    assert ulp > 1e-3   # a one-ulp input change moves the logits by whole quantisation steps
    for mode in ("ggml16", "ggml32"):
        t = r["teacher_forced"][mode]
        assert t["max_abs"] <= 3.0 * ulp, (mode, t, ulp)
        if t["flips"]:
            assert t["max_flip_margin"] <= 2.0 * t["max_abs"], (mode, t)
