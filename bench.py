#!/usr/bin/env python
"""Decode throughput of the dense decoder on B200, with its roofline and the CPU baseline.

Workload: Llama-3-8B architecture, random-init bf16
weights (seeded synthetic, ~N(0, 0.02)), a 512-token uniform-random prompt,
then greedy decode at batch 1, one step = one decode token.  At N GPUs the
model is tensor-parallel over the N ranks (strong scaling: the same sequence,
the work of each token split across ranks).  Weights are 15 GB per token,
larger than L2, so no L2 flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl vvli|reference]

Rank 0 prints one JSON line.  --impl reference times the reference's CPU
decoder (the C++ restatement in oracle/, since the Zig reference cannot be
built here) on this host's cores for the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s + HBM-roofline fraction at 1/2/4/8 B200 vs host-CPU ref"
FALLBACK_HBM_GBS = 6650.0
SHORT_CONTEXT_NOTE = ("the CPU decodes at shorter positions than the GPU arm (which decodes after the "
                      "prompt): its per-token KV read is smaller, a few percent of an 8B token's bytes at most")
KERNEL_NAMES = {0: "gemv q|k|v (rmsnorm prologue)", 1: "gemv o_proj (+residual)",
                2: "gemv gate|up (rmsnorm prologue, silu*mul)", 3: "gemv down_proj (+residual)",
                4: "gemv lm_head (final norm, argmax)"}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["vvli", "reference"], default="vvli")
    ap.add_argument("--config", default="llama3-8b")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--kernel-reps", type=int, default=64)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the other BASELINE configs and the op sweep")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (profiling small cases)")
    ap.add_argument("--batch", type=int, default=16, help="rows of the decode-batch measurement (0: skip)")
    ap.add_argument("--long-prompt", type=int, default=4096,
                    help="tokens of the long-prompt prefill on the Llama-3.2-1B architecture (BASELINE config 3; 0: skip)")
    ap.add_argument("--format", choices=["bf16", "q8_0", "q4_0"], default="bf16",
                    help="weight format of the --profile decode case (block-quantised on the device)")
    ap.add_argument("--trace", action="store_true",
                    help="print the decode megakernel's phase timeline (VVLI_TRACE=1, every rank) instead of the "
                         "bench line; the timestamps add stores, so its step time is not a bench figure")
    ap.add_argument("--profile", choices=["none", "prefill", "batch", "decode", "sample"], default="none",
                    help="run one call of that kind inside a CUDA profiler range (for ncu --profile-from-start off) "
                         "on a --layers cut of the model, print nothing, exit")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


def tensor_peak():
    """Dense bf16 TFLOP/s of this pool's B200s (burst: prefill kernels run for milliseconds)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, cuBLAS burst)"
    except Exception:
        return 1590.0, "fallback 1.59 PFLOP/s"


def prefill_roofline(gemm_flops, attn_flops, ms, peak, peak_source):
    """Tensor roofline of a prefill: algorithmic FLOPs (2 per multiply-add of the reference's fp32 math) and the
    MMA FLOPs actually issued (GEMMs: activations as bf16 hi + lo, 2 MMAs per product; attention: hi.hi + hi.lo +
    lo.hi, 3 MMAs), both over the measured dense bf16 peak."""
    s = ms / 1e3
    achieved = (gemm_flops + attn_flops) / s / 1e12
    issued = (2.0 * gemm_flops + 3.0 * attn_flops) / s / 1e12
    return {"bound": "tensor", "achieved": achieved, "issued": issued, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak, "frac_issued": issued / peak, "peak_source": peak_source}


def ncu_traffic(kernel_key):
    """DRAM bytes per launch of a kernel from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "ncu_summary.txt")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch") and kernel_key in line:
                return float(line.split("=")[-1].strip())
    except OSError:
        pass
    return None


class Clocks:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
    REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, local_rank):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [v for v in vis.split(",") if v.strip()]
        self.index = ids[local_rank] if local_rank < len(ids) and ids[local_rank].isdigit() else str(local_rank)
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-i", self.index,
                 "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) == 8:
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = sorted({self.REASONS[i] for r in rows for i in range(4) if r[4 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def time_oracle(cfg, seed, seconds, min_tokens=2, max_tokens=None):
    """Times the CPU oracle's decode forwards (threads = all host cores)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    import numpy as np
    oracle.build()
    max_seq = 512
    t0 = time.perf_counter()
    r = oracle.RefRunner(cfg, synthetic_seed=seed, max_seq=max_seq, threads=0)
    gen_s = time.perf_counter() - t0
    tok = int(np.random.default_rng(1).integers(0, cfg.vocab_size))
    logits = r.forward_token(tok, 0)  # warm-up (first touch)
    pos, n, t_start = 1, 0, time.perf_counter()
    while True:
        tok = oracle.argmax(logits)
        logits = r.forward_token(tok, pos)
        pos += 1
        n += 1
        el = time.perf_counter() - t_start
        if (n >= min_tokens and el >= seconds) or (max_tokens and n >= max_tokens) or pos >= max_seq:
            break
    cores = min(os.cpu_count() or 1, 64)  # linearInto spawns at most 64 workers (src/llm.zig:11)
    sample = (f"{n} greedy decode tokens of the full {cfg.num_hidden_layers}-layer model at positions 1-{n} "
              f"(weights generated in {gen_s:.1f} s, excluded), {os.cpu_count()} host threads visible; "
              f"{SHORT_CONTEXT_NOTE}")
    r.close()
    return n / el, cores, sample


def run_reference(args, rank, out_fd=1):
    if rank != 0:
        return 0
    from vvli_b200.config import PRESETS
    cfg = PRESETS[args.config]()
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    import numpy as np
    oracle.build()
    t0 = time.perf_counter()
    r = oracle.RefRunner(cfg, synthetic_seed=args.seed, max_seq=min(cfg.max_position_embeddings, 1024), threads=0)
    gen_s = time.perf_counter() - t0
    tok = int(np.random.default_rng(1).integers(0, cfg.vocab_size))
    pos = 0
    logits = None
    tw = time.perf_counter()
    for _ in range(max(1, args.warmup)):
        logits = r.forward_token(tok, pos)
        tok = oracle.argmax(logits)
        pos += 1
    per_tok = (time.perf_counter() - tw) / max(1, args.warmup)
    steps = min(args.steps, max(2, int(150.0 / max(per_tok, 1e-6))), r.max_seq - pos)
    t = time.perf_counter()
    for _ in range(steps):
        logits = r.forward_token(tok, pos)
        tok = oracle.argmax(logits)
        pos += 1
    el = time.perf_counter() - t
    value = steps / el
    cores = min(os.cpu_count() or 1, 64)
    sample = (f"{steps} of {args.steps} requested greedy decode steps (bounded to ~150 s), full model, positions "
              f"{pos - steps}-{pos - 1}; weights generated in {gen_s:.1f} s (excluded); {SHORT_CONTEXT_NOTE}")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": 1000.0 * el / steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, cfg, args.gpus),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample,
                             "what": "C++ restatement of the reference CPU path (src/llm.zig, src/generator.zig); "
                                     "the Zig reference cannot be built here"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line, out_fd)
    return 0


def workload_config(args, cfg, n):
    return {"workload": f"{args.config} greedy decode, batch 1, {args.prompt}-token prompt (BASELINE configs[4])",
            "model": args.config, "global_batch": 1, "seq_len": args.prompt, "ctx": cfg.max_position_embeddings,
            "parallelism": f"tp{n}", "weights": "bf16 synthetic ~N(0,0.02), seeded", "activations": "f32",
            "kv_cache": "f32 paged", "l2": "inputs larger than L2 (every step streams all weights, >15 GB)"}


def greedy_stream(runner, prompt, n_tokens):
    """The first n_tokens greedy tokens after `prompt` (prefill, then on-device decode)."""
    runner.reset()
    runner.prefill(prompt, 0, logits=False)
    first = int(runner.last_argmax)
    rest, _ = runner.decode(n_tokens - 1)
    return [first] + list(rest)


def stream_check(args, cfg, runner, prompt, n, rank, local_rank, barrier, vvli_b200, n_tokens=32):
    """Compares this run's greedy stream with a single-GPU stream of the same weights.  Every rank
    takes part in the tensor-parallel stream; rank 0 alone builds the 1-GPU context (the others wait
    at the barrier)."""
    got = greedy_stream(runner, prompt, n_tokens)
    barrier()
    out = None
    if rank == 0:
        saved = os.environ.get("VVLI_MEGAKERNEL")
        if n == 1:
            os.environ["VVLI_MEGAKERNEL"] = "0"  # the per-kernel step (CUDA graph of separate kernels)
        try:
            r1 = vvli_b200.Runner(cfg, max_seq=len(prompt) + n_tokens + 8, device=local_rank)
        finally:
            if saved is None:
                os.environ.pop("VVLI_MEGAKERNEL", None)
            else:
                os.environ["VVLI_MEGAKERNEL"] = saved
        r1.fill_synthetic(args.seed)
        ref_path = "per-kernel step, 1 GPU" if n == 1 else "megakernel, 1 GPU"
        ref = greedy_stream(r1, prompt, n_tokens)
        r1.close()
        first_diff = next((i for i, (a, b) in enumerate(zip(got, ref)) if a != b), None)
        out = {"equal": got == ref, "tokens": n_tokens, "distinct_tokens": len(set(ref)),
               "first_divergence": first_diff,
               "compared": f"{'tensor-parallel decode on ' + str(n) + ' GPUs' if n > 1 else 'megakernel decode'} "
                           f"vs {ref_path}, greedy tokens after the {len(prompt)}-token prompt"}
    barrier()
    return out


def decode_config(vvli_b200, cfg, name, n_prompt, n_new, seed, hbm, local_rank, note):
    """One BASELINE decode config on one GPU: the reference's own run shape (prompt, then n_new
    greedy tokens) through vvli_cuda_generate_greedy (host prompt in, host tokens out: the
    reference's `[N output tokens | X tok/sec | Ys decode]` line, src/main.zig:203-209), and the
    same decode device-timed (CUDA events around the on-device loop) with its roofline."""
    import numpy as np
    from vvli_b200.config import decode_bytes_per_token
    r = vvli_b200.Runner(cfg, max_seq=n_prompt + n_new + 8, device=local_rank)
    r.fill_synthetic(seed)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, size=n_prompt).astype(np.uint32)
    r.generate_greedy(prompt, n_new)  # warm-up (first prefill allocates)
    r.reset()
    toks, stats = r.generate_greedy(prompt, n_new)
    decode_s = stats.decode_nanoseconds / 1e9
    r.reset()
    r.prefill(prompt, 0, logits=False)
    pf_ms = r.last_forward_ms()
    _, ms = r.decode(n_new - 1)
    r.close()
    per_tok = ms / (n_new - 1)
    mean_pos = n_prompt + n_new // 2
    b = decode_bytes_per_token(cfg, mean_pos)
    ach = b / (per_tok / 1e3) / 1e9
    return {"config": name, "prompt": n_prompt, "generated": len(toks), "distinct_tokens": len(set(toks)),
            "e2e_generate": {"tok_per_s": (len(toks) - 1) / decode_s if decode_s > 0 else None,
                             "decode_s": decode_s, "prefill_s": stats.prefill_nanoseconds / 1e9,
                             "api": "vvli_cuda_generate_greedy (the reference's generation line)"},
            "decode_tok_per_s": 1000.0 / per_tok, "prefill_ms": pf_ms,
            "roofline": {"bound": "hbm", "bytes_per_token": b, "achieved": ach, "peak": hbm, "unit": "GB/s",
                         "frac": ach / hbm, "frac_of_8TBs_spec": ach / 8000.0,
                         "bytes_definition": f"weights + norms/biases + fp32 KV at mean position {mean_pos}"},
            "note": note}


def prefill_decode_config(vvli_b200, seed, hbm, tpeak, tpeak_src, local_rank, L=4096, n_new=32, batch=8):
    """Llama-3.2-1B, a 4,096-token prompt, then 32 decode tokens; batch 1 and
    batch 8 independent sequences (prefilled one after another into their slots, then decoded
    together with vvli_cuda_forward_batch)."""
    import numpy as np
    from vvli_b200.config import PRESETS, decode_bytes_per_token
    cfg = PRESETS["llama3.2-1b"]()
    out = {"config": "llama3.2-1b 4096-token prompt + 32 decode tokens (BASELINE configs[3])"}
    r = vvli_b200.Runner(cfg, max_seq=L + n_new + 8, device=local_rank)
    r.fill_synthetic(seed)
    prompt = np.random.default_rng(3).integers(0, cfg.vocab_size, size=L).astype(np.uint32)
    r.prefill(prompt, 0, logits=False)
    r.reset()
    r.prefill(prompt, 0, logits=False)
    pf = r.last_forward_ms()
    _, ms = r.decode(n_new - 1)
    r.close()
    per_tok = ms / (n_new - 1)
    b = decode_bytes_per_token(cfg, L + n_new // 2)
    out["batch1"] = {"prefill_ms": pf, "prefill_tok_per_s": L / (pf / 1e3), "decode_tok_per_s": 1000.0 / per_tok,
                     "decode_roofline": {"bound": "hbm", "achieved": b / (per_tok / 1e3) / 1e9, "peak": hbm,
                                         "unit": "GB/s", "frac": b / (per_tok / 1e3) / 1e9 / hbm}}
    rb = vvli_b200.Runner(cfg, max_seq=L + n_new + 8, device=local_rank, max_batch=batch)
    rb.fill_synthetic(seed)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, cfg.vocab_size, size=L).astype(np.uint32) for _ in range(batch)]
    rb.prefill_batch(prompts[:1], logits=False)  # first call allocates
    _, am = rb.prefill_batch(prompts, logits=False)
    pfb = rb.last_forward_ms()
    toks, pos = list(am), [L] * batch
    bms = []
    for _ in range(n_new - 1):
        _, am = rb.forward_batch(toks, pos, logits=False)
        bms.append(rb.last_forward_ms())
        toks, pos = list(am), [q + 1 for q in pos]
    rb.close()
    step = float(np.mean(bms[2:])) if len(bms) > 4 else float(np.mean(bms))
    wb = decode_bytes_per_token(cfg, 0) - decode_bytes_per_token(cfg, -1)  # one position of KV
    bb = decode_bytes_per_token(cfg, -1) + batch * wb * (L + n_new // 2 + 1)  # weights once + every row's KV
    out[f"batch{batch}"] = {"prefill_ms": pfb, "prefill_tok_per_s": batch * L / (pfb / 1e3),
                            "decode_ms_per_step": step, "decode_tok_per_s": batch / (step / 1e3),
                            "decode_roofline": {"bound": "hbm", "bytes_per_step": bb,
                                                "achieved": bb / (step / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                                                "frac": bb / (step / 1e3) / 1e9 / hbm},
                            "path": "vvli_cuda_prefill_batch (slot b = sequence b), then vvli_cuda_forward_batch"}
    return out


OP_SHAPES = [(896, 896), (4864, 896), (896, 4864), (151936, 896), (2048, 2048), (8192, 2048), (2048, 8192),
             (14336, 4096), (4096, 14336), (128256, 4096)]


def moe_block(hbm, local_rank, reps=20):
    """The OLMoE sparse block (vvli_cuda_moe_ffn) at the OLMoE-1B-7B shape: h 2048, 64 experts of
    I 1024, 8 per token, random bf16 weights on the device.  Per call: device time (CUDA events around
    the call alone) with L2 flushed before it and new token rows each time; algorithmic bytes = the
    router + the routed experts' gate|up and down rows (each routed expert once) + activations."""
    import numpy as np
    import torch
    from vvli_b200.moe import MoeFfn
    dev = torch.device("cuda", local_rank)
    g = torch.Generator(device=dev).manual_seed(7)
    h, inter, E, k = 2048, 1024, 64, 8

    def bf16(*shape, scale, mean=0.0):
        return (torch.randn(*shape, device=dev, generator=g) * scale + mean).to(torch.bfloat16).view(torch.int16)

    block = MoeFfn(bf16(h, scale=0.1, mean=1.0), bf16(E, h, scale=1.5 / h ** 0.5),
                   bf16(E, 2 * inter, h, scale=1 / h ** 0.5), bf16(E, h, inter, scale=1 / inter ** 0.5), k,
                   False, 1e-5, local_rank)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = {"config": "olmoe-1b-7b sparse block (h 2048, 64 experts x I 1024, top-8), random bf16 weights",
           "path": "vvli_cuda_moe_ffn: route, group, grouped expert GEMVs (only routed experts read), combine"}
    for T in (1, 16):
        xs = [torch.randn(T, h, device=dev, generator=g) for _ in range(reps + 3)]
        times, bytes_ = [], []
        for i, x in enumerate(xs):
            flush.fill_(i & 255)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            idx, _ = block(x, routing=True)
            e1.record()
            torch.cuda.synchronize()
            if i >= 3:
                times.append(e0.elapsed_time(e1))
                n_exp = int(torch.unique(idx).numel())
                bytes_.append(E * h * 2 + n_exp * 3 * inter * h * 2 + 2 * T * h * 4)
        ms = float(np.median(times))
        b = float(np.median(bytes_))
        out[f"tokens_{T}"] = {"us_per_call": round(ms * 1e3, 2), "tok_per_s": round(T / (ms * 1e-3), 1),
                              "routed_experts_median": int(round((b - E * h * 2 - 2 * T * h * 4) / (3 * inter * h * 2))),
                              "roofline": {"bound": "hbm", "bytes_per_call": b, "achieved": b / (ms * 1e-3) / 1e9,
                                           "peak": hbm, "unit": "GB/s", "frac": b / (ms * 1e-3) / 1e9 / hbm}}
    return out


def op_sweep(vvli_b200, hbm, tpeak, local_rank, reps=20):
    """y = W.x over (N, K) x M, each through the kernel the decoder uses for M rows,
    weight copies rotated past 2x L2.  GB/s for M <= 64 (HBM-bound), TFLOP/s for M = 512."""
    import ctypes
    from vvli_b200 import _abi
    rows = []
    kinds = {0: "gemv (bulk-copy)", 1: "tcgen05 skinny GEMM", 2: "tcgen05 skinny GEMM x2 (32 rows each)",
             3: "tcgen05 prefill GEMM"}
    for (N, K) in OP_SHAPES:
        for M in (1, 8, 64, 512):
            ms, b, f, kind = ctypes.c_float(), ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
            rc = _abi.lib().vvli_cuda_op_bench(local_rank, M, N, K, reps, ctypes.byref(ms), ctypes.byref(b),
                                               ctypes.byref(f), ctypes.byref(kind))
            if rc != 0:
                rows.append({"N": N, "K": K, "M": M, "error": _abi.lib().vvli_cuda_last_error().decode()})
                continue
            sec = ms.value / 1e3
            gbs = b.value / sec / 1e9
            tfl = f.value / sec / 1e12
            row = {"N": N, "K": K, "M": M, "us": round(ms.value * 1e3, 2), "GB/s": round(gbs, 1),
                   "TFLOP/s": round(tfl, 2), "kernel": kinds[kind.value]}
            row["frac"] = round(tfl / tpeak, 3) if M == 512 else round(gbs / hbm, 3)
            row["frac_of"] = "bf16 peak (TFLOP/s)" if M == 512 else "HBM peak (GB/s)"
            rows.append(row)
    return rows


def quantized_decode(vvli_b200, cfg, prompt, seed, hbm, local_rank, steps=64, warmup=4):
    """8B decode with every matrix block-quantised on the device (GGML Q8_0 and Q4_0, the GGUF
    types the reference names but rejects): the same megakernel streaming the blocks and
    dequantising them in registers.  Roofline bytes = the stored matrix rows (quants + fp16
    scales) + norms + fp32 KV."""
    out = {}
    for fmt in ("q8_0", "q4_0"):
        r = vvli_b200.Runner(cfg, max_seq=len(prompt) + warmup + steps + 8, device=local_rank)
        r.fill_synthetic_quantized(seed, fmt)
        r.prefill(prompt, 0, logits=False)  # token by token: the tensor-core prefill is bf16-only
        r.decode(warmup)
        toks, ms = r.decode(steps)
        wbytes = r.query("weight_stream_bytes")
        r.close()
        per_tok = ms / steps
        mean_pos = len(prompt) + warmup + steps // 2
        kv = cfg.num_hidden_layers * (mean_pos + 1) * cfg.kv_dim() * 2 * 4
        b = wbytes + (2 * cfg.num_hidden_layers + 1) * cfg.hidden_size * 2 + kv
        ach = b / (per_tok / 1e3) / 1e9
        out[fmt] = {"decode_tok_per_s": 1000.0 / per_tok, "ms_per_token": per_tok, "distinct_tokens": len(set(toks)),
                    "roofline": {"bound": "hbm", "bytes_per_token": b, "achieved": ach, "peak": hbm, "unit": "GB/s",
                                 "frac": ach / hbm},
                    "weights": "vvli_cuda_fill_synthetic_quantized: the synthetic bf16 model quantised on the device"}
    return out


def _second_id(dist, vvli_b200, rank):
    """A fresh NCCL unique id shared by all ranks (for a second tensor-parallel context)."""
    obj = [vvli_b200.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


def profile_case(args):
    """One prefill / batch step / decode step inside cudaProfilerStart/Stop, after warm-up calls."""
    import numpy as np
    import torch
    import vvli_b200
    from vvli_b200.config import PRESETS

    cfg = PRESETS[args.config]()
    if args.layers:
        cfg.num_hidden_layers = args.layers
    torch.cuda.init()
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, size=args.prompt).astype(np.uint32)
    if args.profile == "batch":
        B = max(1, args.batch)
        r = vvli_b200.Runner(cfg, max_seq=args.prompt + 64, max_batch=B)
        r.fill_synthetic(args.seed)
        toks = list(range(1, B + 1))
        for w in range(2):
            r.forward_batch(toks, [args.prompt + w] * B, logits=False)
        call = lambda: r.forward_batch(toks, [args.prompt + 2] * B, logits=False)
    elif args.profile == "prefill":
        r = vvli_b200.Runner(cfg, max_seq=args.prompt + 64)
        r.fill_synthetic(args.seed)
        r.prefill(prompt, 0, logits=False)

        def call():
            r.reset()
            r.prefill(prompt, 0, logits=False)
    elif args.profile == "sample":
        # Sampler.next with the reference's default options over the last forward's logits
        r = vvli_b200.Runner(cfg, max_seq=args.prompt + 64)
        r.fill_synthetic(args.seed)
        r.prefill(prompt, 0, logits=False)
        sopt = vvli_b200.Options()
        recent = np.arange(1, 65, dtype=np.uint32)
        state = np.array([1, 2, 3, 4], dtype=np.uint64)
        for _ in range(3):
            r.sample(sopt, recent, state)
        call = lambda: r.sample(sopt, recent, state)
    else:
        r = vvli_b200.Runner(cfg, max_seq=args.prompt + 64)
        if args.format == "bf16":
            r.fill_synthetic(args.seed)
        else:
            r.fill_synthetic_quantized(args.seed, args.format)
        r.prefill(prompt, 0, logits=False)
        r.decode(3)
        call = lambda: r.decode(2)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    call()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    r.close()


def main():
    args = parse_args()
    if args.profile != "none":
        return profile_case(args)
    # Libraries (NCCL, torch.distributed) may print to stdout; the JSON line is the
    # only thing this process writes there: everything else goes to stderr.
    real_stdout = os.dup(1)
    sys.stdout.flush()
    os.dup2(2, 1)
    try:
        return _main(args, real_stdout)
    finally:
        sys.stdout.flush()
        os.dup2(real_stdout, 1)


def emit(line: dict, fd: int) -> None:
    """Writes the result line to the real stdout."""
    os.write(fd, (json.dumps(line) + "\n").encode())


def _main(args, out_fd):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, out_fd)

    import numpy as np
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import vvli_b200
    from vvli_b200.config import PRESETS, decode_bytes_per_token

    n = world
    torch.cuda.set_device(local_rank)
    nccl_id = None
    if n > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank), timeout=timedelta(seconds=300))
        obj = [vvli_b200.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]

    def barrier():
        if n > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def allmax(v):
        if n == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    cfg = PRESETS[args.config]()
    if args.layers:
        cfg.num_hidden_layers = args.layers
    max_seq = min(cfg.max_position_embeddings, args.prompt + args.warmup + args.steps + args.e2e_steps + 16)
    if args.trace:
        os.environ["VVLI_TRACE"] = "1"
    runner = vvli_b200.Runner(cfg, max_seq=max_seq, device=local_rank, tp_rank=rank, tp_size=n, nccl_id=nccl_id)
    runner.fill_synthetic(args.seed)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, size=args.prompt).astype(np.uint32)
    # Prefill: the first call allocates the activation buffers and tensor maps,
    # so two untimed calls come first; the figure is the median of three more
    # (CUDA events around each whole call; every call rewrites positions 0..P-1).
    pf = []
    for i in range(5):
        runner.prefill(prompt, 0, logits=False)
        if i >= 2:
            pf.append(runner.last_forward_ms())
    prefill_ms = allmax(float(np.median(pf)))
    runner.decode(max(3, args.warmup))
    if args.trace:
        from vvli_b200.trace import summarize
        runner.decode(4)
        sms = torch.cuda.get_device_properties(local_rank).multi_processor_count
        mine = summarize(runner.trace(), sms, cfg.num_hidden_layers) if runner.query("megakernel") == 1 else None
        allr = [None] * n
        if n > 1:
            dist.all_gather_object(allr, mine)
        else:
            allr = [mine]
        if rank == 0:
            emit({"trace": {str(r): v for r, v in enumerate(allr)}, "n_gpus": n, "config": args.config,
                  "position": args.prompt + max(3, args.warmup) + 4,
                  "note": "us per phase kind, mean over layers, of one decode step; VVLI_TRACE build"}, out_fd)
        runner.close()
        if n > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    # ---- device-timed decode: K graph replays, inputs resident in HBM
    clocks = Clocks(local_rank)
    barrier()
    clocks.start()
    pos0 = args.prompt + max(3, args.warmup)
    barrier()
    _, ms = runner.decode(args.steps)
    barrier()
    clk = clocks.stop()
    ms = allmax(ms)
    value = args.steps / (ms / 1000.0)
    ms_per_step = ms / args.steps

    # ---- end to end through the C ABI: host token in, logits and argmax out, every step
    tok = runner.last_argmax if runner.last_argmax is not None else 0
    pos = pos0 + args.steps
    tok = int(tok)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        runner.forward_token(tok, pos, logits=True)
        tok = runner.last_argmax
        pos += 1
    e2e_s = allmax(time.perf_counter() - t0)
    e2e = {"value": args.e2e_steps / e2e_s, "unit": "tok/s",
           "h2d_bytes_per_step": 4 + 32, "d2h_bytes_per_step": cfg.vocab_size * 4 + 32,
           "api": "vvli_cuda_forward_token (host token in; host logits + argmax out; synchronous)"}

    # ---- roofline of the dominant kernel
    hbm, peak_src = peaks()
    mean_pos = pos0 + args.steps // 2
    step_bytes = decode_bytes_per_token(cfg, mean_pos) / n
    mega = runner.query("megakernel") == 1
    gemv = {}
    for k in range(5):  # each decode GEMV timed alone, cycling over every layer's weights
        kms, kbytes = runner.time_kernel(k, args.kernel_reps)
        gemv[KERNEL_NAMES[k]] = {"ms": kms, "GB/s": kbytes / (kms / 1000.0) / 1e9,
                                 "per_token_ms": kms * (1 if k == 4 else cfg.num_hidden_layers)}
    if mega:
        # One persistent kernel runs the whole step: its launch is the token.
        achieved = step_bytes / (ms_per_step / 1000.0) / 1e9
        roofline = {"kernel": "decode_megakernel (one launch per token)", "bound": "hbm", "achieved": achieved,
                    "peak": hbm, "unit": "GB/s", "frac": achieved / hbm, "frac_of_8TBs_spec": achieved / 8000.0,
                    "peak_source": peak_src,
                    # the committed capture is of the 1-GPU kernel; ranks of a tensor-parallel run differ
                    "traffic": ncu_traffic("decode_megakernel") if n == 1 else None,
                    "bytes_per_launch": step_bytes, "launch_ms": ms_per_step,
                    "bytes_per_launch_definition": "all weight matrices (bf16) + norms/biases + fp32 KV read "
                                                   "for positions 0..p + KV row written, p = mean position",
                    "standalone_gemv_kernels": gemv}
    else:
        dom = max(gemv, key=lambda k: gemv[k]["per_token_ms"])
        kms = gemv[dom]["ms"]
        achieved = gemv[dom]["GB/s"]
        roofline = {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                    "frac": achieved / hbm, "peak_source": peak_src, "traffic": ncu_traffic(dom),
                    "launch_ms": kms, "all_kernels": gemv}
    step_gbs = step_bytes / (ms_per_step / 1000.0) / 1e9
    step_roofline = {"bytes_per_token_per_gpu": step_bytes, "achieved": step_gbs, "peak": hbm, "unit": "GB/s",
                     "frac": step_gbs / hbm, "frac_of_8TBs_spec": step_gbs / 8000.0}

    # Prefill of the prompt: tensor-core GEMMs (tcgen05) per linear layer.
    h, kv, inter = cfg.hidden_size, cfg.kv_dim(), cfg.intermediate_size
    layer_params = h * h + 2 * kv * h + h * h + 3 * inter * h
    P = args.prompt
    attn_flops = 4 * cfg.num_attention_heads * cfg.head_dim() * cfg.num_hidden_layers * P * (P + 1) / 2
    gemm_flops = 2.0 * P * layer_params * cfg.num_hidden_layers
    tpeak, tpeak_src = tensor_peak()
    prefill = {"tokens": P, "ms": prefill_ms, "tok_per_s": P / (prefill_ms / 1000.0),
               "algorithmic_tflops": (gemm_flops + attn_flops + 2.0 * h * cfg.vocab_size) / (prefill_ms / 1e3) / 1e12,
               "roofline": prefill_roofline(gemm_flops, attn_flops, prefill_ms, tpeak, tpeak_src),
               "tensor_core_gemm": runner.query("tc_prefill") == 1,
               "note": "activations enter the tensor cores as bf16 hi+lo pairs (2 MMAs per product) for fp32-level "
                       "parity; attention on the tensor cores (q, k, v, p as hi+lo pairs, 3 MMAs per product)"}
    launches_per_step = int(runner.query("kernels_per_step"))
    # Sampler.next on the device (generator.Options defaults: T 0.8, top-p 0.95, top-k 40, rp 1.1 over 64)
    # over the last forward's logits, host call to token (includes the synchronising copies).
    from vvli_b200 import sampler as _smp
    sopt = vvli_b200.Options()
    sstate = np.array(_smp.Xoshiro256(1).s, dtype=np.uint64)
    recent = np.arange(1, 65, dtype=np.uint32)  # the prompt + generated tokens, as a caller keeps them
    runner.sample(sopt, recent, sstate)
    t_s = []
    for _ in range(50):
        t0 = time.perf_counter()
        runner.sample(sopt, recent, sstate)
        t_s.append(time.perf_counter() - t0)
    sampler_line = {"us_per_token_median": round(float(np.median(t_s)) * 1e6, 1), "options": "T 0.8, top_p 0.95, "
                    "top_k 40, repeat_penalty 1.1 over 64", "vocab": cfg.vocab_size}
    # ---- decode batch (batch 16): B sequences per step at context ~prompt,
    # each linear layer one tensor-core GEMM over all rows; device time of whole forward_batch calls.
    batch = None
    if args.batch > 0:
        rb = vvli_b200.Runner(cfg, max_seq=args.prompt + 64, device=local_rank, tp_rank=rank, tp_size=n,
                              nccl_id=nccl_id if n == 1 else _second_id(dist, vvli_b200, rank), max_batch=args.batch)
        rb.fill_synthetic(args.seed)
        btoks = np.random.default_rng(2).integers(0, cfg.vocab_size, size=args.batch).astype(np.uint32)
        for w in range(3):
            rb.forward_batch(btoks, [args.prompt + w] * args.batch, logits=False)
        barrier()
        bms = []
        for i in range(16):
            rb.forward_batch(btoks, [args.prompt + 3 + i] * args.batch, logits=False)
            bms.append(rb.last_forward_ms())
        bms_step = allmax(float(np.mean(bms)))
        # weights once per step + every row's fp32 KV over its context (positions prompt + 3 .. + 18)
        kv_pos = cfg.num_hidden_layers * cfg.kv_dim() * 2 * 4
        bbytes = (decode_bytes_per_token(cfg, -1) + args.batch * kv_pos * (args.prompt + 3 + 8 + 1)) / n
        bach = bbytes / (bms_step / 1e3) / 1e9
        batch = {"rows": args.batch, "context": args.prompt, "ms_per_step": bms_step,
                 "tok_per_s": args.batch / (bms_step / 1000.0), "steps": 16,
                 "roofline": {"bound": "hbm", "bytes_per_step_per_gpu": bbytes, "achieved": bach, "peak": hbm,
                              "unit": "GB/s", "frac": bach / hbm,
                              "bytes_definition": "all weight matrices once + each row's fp32 KV read at its mean "
                                                  "position"},
                 "path": "vvli_cuda_forward_batch: tcgen05 GEMMs with weight rows as M and the batch as N, "
                         "paged attention per row; device time of each call (host token ids in, argmax out)"}
        rb.close()

    # ---- long-prompt prefill: Llama-3.2-1B architecture, one uniform-random prompt of
    # --long-prompt tokens (chunks of up to 2,048), tensor-core GEMMs and attention; CUDA events around each call.
    prefill_long = None
    if args.long_prompt > 0 and n == 1:
        lcfg = PRESETS["llama3.2-1b"]()
        L = args.long_prompt
        rl = vvli_b200.Runner(lcfg, max_seq=L + 32, device=local_rank)
        rl.fill_synthetic(args.seed)
        lprompt = np.random.default_rng(3).integers(0, lcfg.vocab_size, size=L).astype(np.uint32)
        lms = []
        for i in range(3):
            rl.prefill(lprompt, 0, logits=False)
            if i > 0:
                lms.append(rl.last_forward_ms())
        lms_med = float(np.median(lms))
        lh, lkv, linter = lcfg.hidden_size, lcfg.kv_dim(), lcfg.intermediate_size
        l_params = lh * lh + 2 * lkv * lh + lh * lh + 3 * linter * lh
        l_gemm = 2.0 * L * l_params * lcfg.num_hidden_layers
        l_attn = 4 * lcfg.num_attention_heads * lcfg.head_dim() * lcfg.num_hidden_layers * L * (L + 1) / 2
        l_flops = l_gemm + l_attn
        tpeak, tpeak_src = tensor_peak()
        prefill_long = {"model": "llama3.2-1b", "tokens": L, "ms": lms_med, "tok_per_s": L / (lms_med / 1000.0),
                        "algorithmic_tflops": l_flops / (lms_med / 1e3) / 1e12,
                        "roofline": prefill_roofline(l_gemm, l_attn, lms_med, tpeak, tpeak_src),
                        "timing": "median of 2 calls after 1 warm-up call"}
        rl.close()

    # ---- stream check: the greedy stream of this run's decode path after the prompt against a
    # single-GPU stream of the same weights (N > 1: the tensor-parallel path against a 1-GPU context
    # on rank 0's GPU; N = 1: the megakernel against the per-kernel step).
    parity = stream_check(args, cfg, runner, prompt, n, rank, local_rank, barrier, vvli_b200)

    # ---- every BASELINE config (one GPU): decode configs 1 and 3, the prefill + decode config 4 at batch
    # 1 and 8, and the op sweep of config 2.
    configs = None
    if n == 1 and not args.no_configs:
        configs = {
            "qwen2.5-0.5b": decode_config(vvli_b200, PRESETS["qwen2.5-0.5b"](), "qwen2.5-0.5b 32-token prompt, "
                                          "64 greedy tokens (BASELINE configs[0])", 32, 64, args.seed, hbm, local_rank,
                                          "tied embeddings, q/k/v bias"),
            "llama3.2-1b": decode_config(vvli_b200, PRESETS["llama3.2-1b"](), "llama3.2-1b 128-token prompt, 256 "
                                         "greedy tokens (BASELINE configs[2])", 128, 256, args.seed, hbm, local_rank,
                                         "llama3 rope scaling"),
            "llama3.2-1b-4096": prefill_decode_config(vvli_b200, args.seed, hbm, tpeak, tpeak_src, local_rank),
            "op_sweep": op_sweep(vvli_b200, hbm, tpeak, local_rank),
            "llama3-8b-quantized": quantized_decode(vvli_b200, cfg, prompt, args.seed, hbm, local_rank),
            "olmoe-moe-block": moe_block(hbm, local_rank),
        }

    cpu = None
    if rank == 0 and n == 1 and not args.no_cpu_baseline:
        v, cores, sample = time_oracle(cfg, args.seed, args.cpu_seconds)
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": n, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_config(args, cfg, n),
                "roofline": roofline, "step_roofline": step_roofline, "cpu_baseline": cpu, "e2e": e2e,
                "tp_parity": parity["equal"] if parity else None, "stream_check": parity,
                "prefill": prefill, "prefill_long": prefill_long, "sampler": sampler_line, "batch": batch,
                "configs": configs,
                "gpu_launches": launches_per_step * args.steps, "clocks": clk}
        emit(line, out_fd)
    runner.close()
    if n > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
