"""T2S decode throughput on B200: the box-scale batched-session workload.

Workload (default): 2048 independent sessions, Q4_K weights (synthetic, seed 3), each a
200-phoneme + 150-semantic-token prompt, greedy decode with EOS masked, sharded evenly over
the GPUs (one process per GPU, no collective on the data path).  A step = one decode step of
every session on the GPU; value = tokens/s over all ranks (max device time over ranks).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload bs2048_q4_k|bs32_q4_0|bs1_q8_0]

--impl reference times the reference's CPU arithmetic (the oracle restatement; the reference's
ggml cannot be built here) on the host cores for a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "gpt-sovits.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}

# the arithmetic of each weight format's matmuls (the activation rows are converted to the
# weight's dot type first) and of the KV cache
DTYPES = {
    "q4_k": "int8xint8->int32 per 32-block, f32 fold per 256-block (Q4_K weights x Q8_K rows); f16 KV",
    "q4_0": "int8xint8->int32 per 32-block, f32 fold (Q4_0 weights x Q8_0 rows); f16 KV",
    "q8_0": "int8xint8->int32 per 32-block, f32 fold (Q8_0 weights x Q8_0 rows); f16 KV",
    "q5_0": "int8xint8->int32 per 32-block, f32 fold (Q5_0 weights x Q8_0 rows); f16 KV",
    "f16": "f16xf16->f32 (F16 weights x f16 rows); f16 KV",
    "f32": "f32; f16 KV",
}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return rank, world, local


def session_prompts(workload, sessions):
    import synth
    return synth.workload_lengths(workload, sessions)


# ------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------
def run_ours(args):
    import torch
    import synth
    import t2sx
    import build as t2sx_build

    rank, world, local = dist_setup(args.gpus)
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    t2sx_build.build()
    import shard
    w = synth.WORKLOADS[args.workload]
    total_sessions = w["sessions"] if args.sessions is None else args.sessions * world
    lo, hi = shard.session_shard(total_sessions, world, rank)
    per = hi - lo
    lengths_all = session_prompts(args.workload, total_sessions)
    mine = lengths_all[lo:hi]
    # rank 0 writes the synthetic GGUF (once per cache directory); the others wait for it
    if rank == 0:
        path = synth.ensure_gguf(w["wtype"], w["seed"], n_layer=24)
    if world > 1:
        dist.barrier()
    path = synth.ensure_gguf(w["wtype"], w["seed"], n_layer=24)

    # roofline denominators this run measures itself: L2 read bandwidth and the int8 tensor rate
    probes = measure_probes(local) if (rank == 0 and not args.no_probes) else None

    W, K = args.warmup, args.steps
    max_prompt = max(tt + tp for tt, tp, _ in mine)
    slot_size = max_prompt + W + K + 1

    model = t2sx.Model(path, device=local)
    sess = t2sx.Session(model, per, slot_size, repetition_penalty=1.0, eos_mask=True)

    # ---- prefill (outside the decode timing): GPU embedding of the seeded prompts, then one
    # batched prefill of all sessions.  embed_s counts the embedding calls (host BERT features
    # copied in, rows written on the device), prefill_s the t2sx_prefill call; generating the
    # synthetic inputs on the host is in neither.
    total_rows = sum(tt + tp for tt, tp, _ in mine)
    xdev = torch.empty((total_rows, 512), dtype=torch.float32, device="cuda")
    off = 0
    embed_s = 0.0
    for tt, tp, seed in mine:
        ph, bert, sem = synth.session_inputs(seed, tt, tp)
        t0 = time.perf_counter()
        sess.embed_prefill(ph, bert, sem, out_dev_ptr=xdev[off].data_ptr())
        embed_s += time.perf_counter() - t0
        off += tt + tp
    t0 = time.perf_counter()
    torch.cuda.synchronize()
    embed_s += time.perf_counter() - t0
    t0 = time.perf_counter()
    first = sess.prefill(np.arange(per), [tt + tp for tt, tp, _ in mine], [tp for _, tp, _ in mine],
                         x_dev_ptr=xdev.data_ptr())
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    del xdev

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        return shard.max_over_ranks(v, device="cuda")

    def sum_over_ranks(v: float) -> float:
        return shard.sum_over_ranks(v, device="cuda")

    # ---- warm-up: W host-driven steps (also captures the step graph) ----
    # the token streams of the first n_par sessions (prefill token, then every warm-up and timed
    # step) are kept for the step-by-step comparison with the CPU oracle after the timed region
    n_par = min(args.parity_sessions, per) if rank == 0 else 0
    par_tokens = [first[:n_par].copy()]
    cur = first.copy()
    for _ in range(W):
        cur = sess.decode_step_host(cur, want_tokens=True)
        par_tokens.append(cur[:n_par].copy())
    n_kernels = sess.graph_kernels()
    ctx_before = np.array([sess.slot_n_pos(i) for i in range(per)], dtype=np.int64)
    prof_start = sess.profile_step(iters=10)

    # ---- timed region: K decode steps through the C ABI with host buffers every step ----
    # (e2e = wall clock of the loop incl. the per-step host<->device token copies;
    #  value = the same steps' device time of the step graphs, CUDA events on the session stream)
    barrier()
    torch.cuda.synchronize()
    dev_ms = 0.0
    step_ms = []
    torch.cuda.cudart().cudaProfilerStart()   # profilers started with --profile-from-start off see only this loop
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        for _ in range(K):
            cur = sess.decode_step_host(cur, want_tokens=True)
            par_tokens.append(cur[:n_par].copy())
            ms = sess.last_decode_ms()
            step_ms.append(ms)
            dev_ms += ms
        wall_s = time.perf_counter() - t0
    torch.cuda.cudart().cudaProfilerStop()
    barrier()
    t_max = max_over_ranks(dev_ms / 1e3)
    e2e_max = max_over_ranks(wall_s)
    tokens = sum_over_ranks(float(per * K))
    value = tokens / t_max
    e2e_value = tokens / e2e_max

    # ---- per-kernel device times on the final state, for the roofline ----
    prof = sess.profile_step(iters=10)
    ctx_now = np.array([sess.slot_n_pos(i) for i in range(per)], dtype=np.int64)
    # attention of one layer at the last step: each session reads K and V of its whole prefix
    # (ctx_now positions): 2 (K,V) * 16 heads * 32 dims * 2 B = 2048 B per position, plus q/out
    attn_bytes = float((ctx_now * 2048).sum() + per * (512 * 2 + 512 * 4))
    attn_gbs = attn_bytes / (prof["attention_kernel"] * 1e-3) / 1e9
    # DRAM bytes per algorithmic byte of this kernel, from one ncu capture (dram__bytes_read.sum +
    # dram__bytes_write.sum = 189.98 MB for 186.91 MB algorithmic, 256 sessions at context 353);
    # the full launch is too large to capture, so its traffic is that ratio times its algorithmic
    # bytes (the kernel streams each byte once).
    ATTN_DRAM_PER_ALGO_BYTE = 189.981184 / 186.908672

    # ---- the bs=1 decode step (the other half of the metric), measured in the same run ----
    bs1 = None
    if rank == 0 and args.workload != "bs1_q8_0" and not args.no_bs1:
        bs1 = bs1_step(local, args.bs1_steps)

    # ---- CPU oracle (rank 0): token parity of the first sessions over all W + K steps; at N=1
    # its last steps are also the timed CPU baseline (bounded sample) ----
    cpu = parity = None
    if rank == 0 and not args.no_cpu:
        cpu, ref_tok = oracle_streams(args.workload, path, n_par, W + K,
                                      timed_steps=args.cpu_steps)
        parity = parity_report(np.stack(par_tokens), ref_tok)
        if world > 1:
            cpu = None

    peaks, peak_kind = load_peaks()
    if rank == 0:
        clocks = clk.summary()
        line = {
            "metric": "T2S decode tokens/s (batched sessions)",
            "value": round(value, 2),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": K,
            "warmup": W,
            "ms_per_step": round(t_max * 1e3 / K, 4),
            "p50_step_ms": round(float(np.median(step_ms)), 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": DTYPES[w["wtype"]],
            "data": "synthetic (seeded N(0,0.02) weights, uniform ids, N(0,1) BERT features)",
            "config": {
                "workload": args.workload,
                "model": "T2S GPT-SoVITS v2 shape: 24 post-norm layers, d=512, 16x32 heads, FFN 2048, vocab 1025",
                "weights": w["wtype"],
                "sessions_total": total_sessions,
                "sessions_per_gpu": per,
                "prompt": "200 phonemes + 150 semantic tokens" if args.workload == "bs2048_q4_k" else "see synth.WORKLOADS",
                "context_at_start": int(ctx_before.mean()),
                "context_at_end": int(ctx_now.mean()),
                "global_batch": total_sessions,
                "parallelism": f"session-sharded dp{world}, no collective",
                "l2": "inputs larger than L2: KV cache %.1f GB per GPU" % (sess.device_bytes() / 1e9),
                "prefill_s": round(prefill_s, 3),
                "prefill_rows": int(total_rows),
                "embed_s": round(embed_s, 3),
            },
            "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 4 * per,
                    "d2h_bytes_per_step": 4 * per,
                    "how": "t2sx_decode_step_host per step: host tokens -> device, one step graph, tokens -> host; wall clock"},
            "gpu_launches": int(n_kernels * K),
            "roofline": {
                "kernel": "k_attn_decode (paged f16 KV attention, one layer)",
                "bound": "hbm",
                "achieved": round(attn_gbs, 1),
                "peak": peaks["hbm_gbs"],
                "unit": "GB/s",
                "frac": round(attn_gbs / peaks["hbm_gbs"], 4),
                "traffic": int(attn_bytes * ATTN_DRAM_PER_ALGO_BYTE),
                "traffic_source": "ncu dram bytes at 256 sessions scaled by algorithmic bytes",
                "peak_kind": peak_kind,
                "algorithmic_bytes_per_launch": int(attn_bytes),
                "launch_ms": round(prof["attention_kernel"], 4),
            },
            "kernel_ms": {k: round(v, 4) for k, v in prof.items()},
            "kernel_ms_at_start": {k: round(v, 4) for k, v in prof_start.items()},
            "clocks": clocks,
        }
        if probes is not None:
            line["peaks_probe"] = probes
            # the batched tcgen05 Q4_K matmul (QKV projection, one launch at this run's rows):
            # algorithmic int8 ops 2*M*N*K per launch, the tensor core issues 3x that (three planes)
            ops = 2.0 * per * 1536 * 512
            tops = ops / (prof["mm_qkv"] * 1e-3) / 1e12
            line["roofline_tc_qkv"] = {"kernel": "k_mm_tc_q4k (QKV, 1536 x 512)" if per >= 64 else "QKV matmul",
                                       "bound": "tensor", "achieved": round(tops, 1), "unit": "TOP/s (int8)",
                                       "peak": probes["i8_tensor_tops"], "frac": round(tops / probes["i8_tensor_tops"], 4),
                                       "issued_frac": round(3 * tops / probes["i8_tensor_tops"], 4),
                                       "rows": per, "launch_ms": round(prof["mm_qkv"], 4)}
        if parity is not None:
            line["parity"] = parity
        if bs1 is not None:
            if probes is not None:
                # bs=1 step: the Q8_0 weights (80,773,664 B) from L2 and the K/V prefix from HBM,
                # 49,152 B per position at the steps' mean context
                kv = 49152.0 * (bs1["context"][0] + bs1["context"][1]) / 2
                t_min = 80773664 / (probes["l2_read_gbs"] * 1e9) + kv / (peaks["hbm_gbs"] * 1e9)
                bs1["roofline"] = {"l2_bytes": 80773664, "hbm_bytes": int(kv), "bound_ms": round(t_min * 1e3, 4),
                                   "frac": round(t_min * 1e3 / bs1["p50_step_ms"], 4),
                                   "peaks": "l2_read_gbs of peaks_probe, hbm_gbs of MEASURED_PEAKS.json"}
            line["bs1"] = bs1
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line))
    sess.close()
    model.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def oracle_streams(workload, path, n_sessions, n_steps, timed_steps=None):
    """The oracle (CPU restatement of the reference arithmetic) on all host cores: prefill of the
    first `n_sessions` prompts of the workload (untimed), then `n_steps` greedy decode steps.
    Returns (cpu_baseline dict timed over the last `timed_steps` steps, tokens int32
    [n_steps + 1][n_sessions]: the prefill token, then one row per decode step)."""
    import oracle
    import synth
    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    m = oracle.Model(path)
    lengths = synth.workload_lengths(workload)[:n_sessions]
    cap = max(tt + tp for tt, tp, _ in lengths) + n_steps + 2
    s = oracle.Session(m, len(lengths), cap)
    cur = []
    for i, (tt, tp, seed) in enumerate(lengths):
        ph, bert, sem = synth.session_inputs(seed, tt, tp)
        x = m.embed_prefill(ph, bert, sem)
        cur.append(s.prefill(i, x, tp)[0])
    slots = np.arange(len(lengths))
    cur = np.array(cur, dtype=np.int32)
    toks = [cur.copy()]
    timed = n_steps if timed_steps is None else min(timed_steps, n_steps)
    t0 = None
    for k in range(n_steps):
        if k == n_steps - timed:
            t0 = time.perf_counter()
        cur, _ = s.decode(slots, cur)
        toks.append(cur.copy())
    dt = time.perf_counter() - t0 if t0 is not None else float("nan")
    s.close()
    m.close()
    cpu = {"value": round(len(lengths) * timed / dt, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
           "sample": f"{len(lengths)} sessions of {workload}, {timed} timed greedy decode steps after prefill "
                     f"and {n_steps - timed} untimed ones (oracle restatement; ggml is absent from the "
                     f"reference snapshot)"}
    return cpu, np.stack(toks)


def measure_probes(device):
    """L2 read bandwidth (best of three L2-resident sizes) and the dense int8 tcgen05 rate (best
    of one and two issuing threads per SM), measured by the library's own probe kernels."""
    import t2sx
    l2 = max(t2sx.probe_l2_read_gbs(device, mb << 20, 100) for mb in (8, 16, 32, 48))
    i8 = max(t2sx.probe_i8_mma_tops(device, 20000, k) for k in (1, 2))
    return {"l2_read_gbs": round(l2, 1), "i8_tensor_tops": round(i8, 1),
            "how": "t2sx_probe_l2_read: 8/16/32/48 MiB buffers streamed with ld.global.cg, 100 passes; "
                   "t2sx_probe_i8_mma: tcgen05.mma.kind::i8 M128 N256 K32 from smem on every SM"}


def bs1_step(device, steps, warm=5):
    """The bs=1 decode step of the reference's one-session workload (Q8_0 weights seed 0, 128
    phonemes + 150 prompt tokens, greedy, EOS masked) on this GPU: `warm` untimed steps, then
    `steps` steps through t2sx_decode_step_host, each timed on the device (CUDA events around
    the step graph) and on the host (token in, step, token out).  Returns the p50 of both."""
    import synth
    import t2sx
    w = synth.WORKLOADS["bs1_q8_0"]
    path = synth.ensure_gguf(w["wtype"], w["seed"], n_layer=24)
    (tt, tp, seed), = synth.workload_lengths("bs1_q8_0")
    model = t2sx.Model(path, device=device)
    sess = t2sx.Session(model, 1, tt + tp + warm + steps + 1, repetition_penalty=1.0, eos_mask=True)
    ph, bert, sem = synth.session_inputs(seed, tt, tp)
    x = sess.embed_prefill(ph, bert, sem)
    cur = sess.prefill([0], [tt + tp], [tp], x)
    for _ in range(warm):
        cur = sess.decode_step_host(cur, want_tokens=True)
    ctx0 = sess.slot_n_pos(0)
    dev, host = [], []
    for _ in range(steps):
        t0 = time.perf_counter()
        cur = sess.decode_step_host(cur, want_tokens=True)
        host.append((time.perf_counter() - t0) * 1e3)
        dev.append(sess.last_decode_ms())
    ctx1 = sess.slot_n_pos(0)
    n_kernels = sess.graph_kernels()
    sess.close()
    model.close()
    return {"workload": "bs1_q8_0", "p50_step_ms": round(float(np.median(dev)), 4),
            "p50_e2e_step_ms": round(float(np.median(host)), 4), "steps": steps, "warmup": warm,
            "context": [int(ctx0), int(ctx1)], "kernels_per_step": int(n_kernels),
            "how": "one session; device ms = CUDA events around the step graph; e2e = host wall clock of "
                   "t2sx_decode_step_host (token in, step, token out)"}


def parity_report(gpu_tokens, ref_tokens):
    """Step-by-step comparison of GPU and oracle token streams ([steps + 1][sessions], row 0 the
    prefill token)."""
    n = min(len(gpu_tokens), len(ref_tokens))
    g, r = np.asarray(gpu_tokens[:n]), np.asarray(ref_tokens[:n])
    diff = np.nonzero((g != r).any(axis=1))[0]
    return {"sessions": int(g.shape[1]), "steps": int(n - 1), "tokens_equal": bool(diff.size == 0),
            "first_mismatch_step": None if diff.size == 0 else int(diff[0]),
            "checked": "prefill token and every decode step (warm-up and timed) against the CPU oracle"}


# ------------------------------------------------------------------------------------------------
# reference arm
# ------------------------------------------------------------------------------------------------
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    import synth
    w = synth.WORKLOADS[args.workload]
    path = synth.ensure_gguf(w["wtype"], w["seed"], n_layer=24)
    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    m = oracle.Model(path)
    n_sess = min(args.cpu_sessions, w["sessions"])
    lengths = synth.workload_lengths(args.workload)[:n_sess]
    W, K = args.warmup, args.steps
    cap = max(tt + tp for tt, tp, _ in lengths) + W + K + 2
    s = oracle.Session(m, n_sess, cap)
    cur = []
    for i, (tt, tp, seed) in enumerate(lengths):
        ph, bert, sem = synth.session_inputs(seed, tt, tp)
        cur.append(s.prefill(i, m.embed_prefill(ph, bert, sem), tp)[0])
    slots = np.arange(n_sess)
    cur = np.array(cur, dtype=np.int32)
    for _ in range(W):
        cur, _ = s.decode(slots, cur)
    t0 = time.perf_counter()
    for _ in range(K):
        cur, _ = s.decode(slots, cur)
    dt = time.perf_counter() - t0
    value = n_sess * K / dt
    sample = (f"{n_sess} sessions of {args.workload} per step (bounded sample), oracle restatement of the "
              f"reference CPU arithmetic; ggml is an empty submodule in the reference and cannot be built")
    print(json.dumps({
        "impl": "reference",
        "metric": "T2S decode tokens/s (batched sessions)",
        "value": round(value, 3),
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(dt * 1e3 / K, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": DTYPES[w["wtype"]],
        "data": "synthetic",
        "config": {"workload": args.workload, "sessions_timed": n_sess, "weights": w["wtype"]},
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def run_matmul_sweep(args):
    """Isolated dequant-matmul sweep: weight shapes of the layer (qkv, out, ffn-up, ffn-down,
    lm_head) x formats x activation rows, through t2sx_matmul (activation quantisation + matmul),
    N(0,0.02) weights, N(0,1) activations, seeded per shape.  One JSON line per case."""
    import torch
    import gguf
    import synth
    import t2sx
    import build as t2sx_build
    t2sx_build.build()
    torch.cuda.set_device(0)
    shapes = [(1536, 512), (512, 512), (2048, 512), (512, 2048), (1025, 512)]
    fmts = args.formats.split(",")
    rows = [int(v) for v in args.rows.split(",")]
    tid = {"q8_0": 8, "q4_0": 2, "q4_k": 12, "f16": 1}
    stream = torch.cuda.current_stream()
    for fmt in fmts:
        for (N, K) in shapes:
            rng = np.random.default_rng(hash((N, K, fmt)) % (2 ** 32))
            w = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
            if fmt == "q4_k":
                wb = synth.quantize_q4_k(w)
            elif fmt == "f16":
                wb = w.astype(np.float16).view(np.uint8)
            else:
                wb = gguf.quantize(w, gguf.GGMLQuantizationType.Q8_0 if fmt == "q8_0" else gguf.GGMLQuantizationType.Q4_0)
            W = t2sx.Weight(tid[fmt], wb, N, K)
            wbytes = int(np.asarray(wb).nbytes)
            for M in rows:
                x = torch.randn((M, K), dtype=torch.float32, device="cuda", generator=torch.Generator("cuda").manual_seed(M))
                y = torch.empty((M, N), dtype=torch.float32, device="cuda")
                for _ in range(3):
                    W.matmul(x.data_ptr(), M, y.data_ptr(), stream=stream.cuda_stream)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                iters = args.steps
                e0.record(stream)
                for _ in range(iters):
                    W.matmul(x.data_ptr(), M, y.data_ptr(), stream=stream.cuda_stream)
                e1.record(stream)
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / iters
                flops = 2.0 * M * N * K
                print(json.dumps({"sweep": "matmul", "format": fmt, "N": N, "K": K, "M": M, "us": round(us, 3),
                                  "tops": round(flops / us / 1e6, 2), "weight_bytes": wbytes,
                                  "weight_gbs": round(wbytes / us / 1e3, 1)}))
            W.close()


def run_attention_sweep(args):
    """Isolated batched attention over a paged f16 KV cache (one layer), through the
    t2sx_kvcache_* entry points: decode = 256 sequences with prefixes uniform in [200, 1500] and one
    query each; prefill = the same 256 sequences with 256-token prompts, causal, empty prefix.
    K/V ~ N(0,1)/sqrt(32) and q ~ N(0,1), stored f16, seed 3.  One JSON line per case."""
    import torch
    import t2sx
    import build as t2sx_build
    t2sx_build.build()
    torch.cuda.set_device(0)
    peaks, peak_kind = load_peaks()
    rng = np.random.default_rng(3)
    n, max_len = 256, 1500
    lens = rng.integers(200, 1501, size=n).astype(np.int32)
    cache = t2sx.KVCache(n, max_len)
    scale = np.float32(1.0 / np.sqrt(32.0))
    for s_ in range(n):
        L = int(lens[s_])
        k = (rng.standard_normal((L, 16, 32), dtype=np.float32) * scale).astype(np.float16).view(np.uint16)
        v = (rng.standard_normal((L, 16, 32), dtype=np.float32) * scale).astype(np.float16).view(np.uint16)
        cache.write(s_, 0, k, v)
    stream = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    seqs = np.arange(n, dtype=np.int32)
    q = torch.randn((n, 512), generator=torch.Generator().manual_seed(3)).to(torch.float16).cuda()
    out = torch.empty((n, 512), dtype=torch.float32, device="cuda")
    ms = timed(lambda: cache.attn_decode(seqs, lens, q.data_ptr(), out.data_ptr(), stream=stream.cuda_stream))
    byts = float(lens.astype(np.int64).sum() * 2048 + n * (512 * 2 + 512 * 4))
    gbs = byts / (ms * 1e-3) / 1e9
    print(json.dumps({"sweep": "attention", "case": "decode", "sequences": n, "prefix": "uniform [200,1500]",
                      "sum_prefix": int(lens.sum()), "us": round(ms * 1e3, 2), "bytes": int(byts),
                      "achieved_gbs": round(gbs, 1), "peak_gbs": peaks["hbm_gbs"], "frac": round(gbs / peaks["hbm_gbs"], 4),
                      "peak_kind": peak_kind, "l2": "K/V %.0f MB > L2" % (byts / 1e6)}))
    # causal prefill: 256 sequences x 256 new tokens over an empty prefix (positions 0..255 rewritten)
    T = 256
    for s_ in range(n):
        k = (rng.standard_normal((T, 16, 32), dtype=np.float32) * scale).astype(np.float16).view(np.uint16)
        v = (rng.standard_normal((T, 16, 32), dtype=np.float32) * scale).astype(np.float16).view(np.uint16)
        cache.write(s_, 0, k, v)
    pseqs = np.repeat(np.arange(n, dtype=np.int32), T)
    plens = np.tile(np.arange(1, T + 1, dtype=np.int32), n)
    pq = torch.randn((n * T, 512), generator=torch.Generator().manual_seed(4)).to(torch.float16).cuda()
    pout = torch.empty((n * T, 512), dtype=torch.float32, device="cuda")
    ms = timed(lambda: cache.attn_prefill(pseqs, plens, pq.data_ptr(), pout.data_ptr(), stream=stream.cuda_stream))
    flops = float(n * 16 * 4 * 32 * (T * (T + 1) // 2))
    print(json.dumps({"sweep": "attention", "case": "prefill", "sequences": n, "new_tokens": T, "prefix": 0,
                      "us": round(ms * 1e3, 2), "flops": int(flops), "gflops": round(flops / (ms * 1e-3) / 1e9, 1),
                      "unique_kv_bytes": n * T * 2048,
                      "note": "32 position lanes per (query, head) with the online softmax: CUDA cores, not tensor cores"}))
    cache.close()
    # decode rows of one fixed context each: time against context gives the per-launch cost that
    # does not scale with the prefix (row start-up, merge, output)
    nf = 2048
    ctxs = [int(c) for c in args.attn_ctx.split(",") if c]
    if ctxs:
        cmax = max(ctxs)
        cache = t2sx.KVCache(nf, cmax)
        k = (rng.standard_normal((cmax, 16, 32), dtype=np.float32) * scale).astype(np.float16).view(np.uint16)
        v = (rng.standard_normal((cmax, 16, 32), dtype=np.float32) * scale).astype(np.float16).view(np.uint16)
        for s_ in range(nf):
            cache.write(s_, 0, k, v)
        fseqs = np.arange(nf, dtype=np.int32)
        fq = torch.randn((nf, 512), generator=torch.Generator().manual_seed(5)).to(torch.float16).cuda()
        fout = torch.empty((nf, 512), dtype=torch.float32, device="cuda")
        for c in ctxs:
            flens = np.full(nf, c, dtype=np.int32)
            ms = timed(lambda: cache.attn_decode(fseqs, flens, fq.data_ptr(), fout.data_ptr(), stream=stream.cuda_stream))
            byts = float(nf * c * 2048 + nf * (512 * 2 + 512 * 4))
            gbs = byts / (ms * 1e-3) / 1e9
            print(json.dumps({"sweep": "attention", "case": "decode_fixed", "sequences": nf, "prefix": c,
                              "us": round(ms * 1e3, 2), "bytes": int(byts), "achieved_gbs": round(gbs, 1),
                              "frac": round(gbs / peaks["hbm_gbs"], 4), "peak_kind": peak_kind}))
        if cmax >= 1500:   # the same rows with ragged prefixes (uniform in [200, 1500])
            flens = rng.integers(200, 1501, size=nf).astype(np.int32)
            ms = timed(lambda: cache.attn_decode(fseqs, flens, fq.data_ptr(), fout.data_ptr(), stream=stream.cuda_stream))
            byts = float(flens.astype(np.int64).sum() * 2048 + nf * (512 * 2 + 512 * 4))
            gbs = byts / (ms * 1e-3) / 1e9
            print(json.dumps({"sweep": "attention", "case": "decode_ragged", "sequences": nf, "prefix": "uniform [200,1500]",
                              "us": round(ms * 1e3, 2), "bytes": int(byts), "achieved_gbs": round(gbs, 1),
                              "frac": round(gbs / peaks["hbm_gbs"], 4), "peak_kind": peak_kind}))
        cache.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="bs2048_q4_k")
    ap.add_argument("--sessions", type=int, default=None,
                    help="sessions per GPU (default: the workload's total / GPUs); smaller cases for profiling")
    ap.add_argument("--cpu-sessions", type=int, default=8)
    ap.add_argument("--cpu-steps", type=int, default=20)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--parity-sessions", type=int, default=8,
                    help="sessions whose token streams are compared with the CPU oracle (rank 0)")
    ap.add_argument("--no-bs1", action="store_true", help="skip the bs=1 step measurement")
    ap.add_argument("--no-probes", action="store_true", help="skip the L2 / int8 tensor peak probes")
    ap.add_argument("--bs1-steps", type=int, default=200)
    ap.add_argument("--sweep", choices=["matmul", "attention"], default=None,
                    help="isolated kernel sweep instead of the decode workload (--steps = timed iterations)")
    ap.add_argument("--formats", default="q8_0,q4_0,q4_k,f16")
    ap.add_argument("--rows", default="1,8,16,64,256,2048")
    ap.add_argument("--attn-ctx", default="",
                    help="attention sweep: also time 2048 decode rows at each of these fixed prefixes")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.sweep == "matmul":
        run_matmul_sweep(args)
    elif args.sweep == "attention":
        run_attention_sweep(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
