"""Benchmark: fused KL-GEMM distillation loss, forward + backward, loss-rows/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c2]

One step = the full training-path loss over one batch of rows (klg_fwd_bwd):
valid-row count, pass 1 (both views' log-sum-exps over all vocab tiles on CTA
pairs), pass 2 (logit recompute -> dZ chunks with the KL cross term -> dW and
dH GEMMs), loss.
Workload at N=1 is the 16,384-row SmolLM2-135M training shape (H=576,
V=49,152, bf16, block-32 mask with ratio U(0,1)); synthetic seeded inputs.
At N>1 each rank runs its own 16,384 rows (weak scaling, row sharded): the
valid count and loss are all-reduced and dW is all-reduced over NCCL.
``--config c4`` at N>1 shards the 248,320-row lm_head by vocab instead (strong
scaling): every rank holds all 32,768 rows and one W slice, the per-row
(m, S, m, S, A) partial records are all-gathered and merged, and the partial
dH is all-reduced; ``value`` then counts each row once.

``value``  device-timed throughput with inputs resident (CUDA events per step,
           L2 flushed between steps by writing a 256 MiB buffer), max over ranks.
``roofline`` / ``kernels``  per-kernel times from CUDA events recorded around every
           launch on the launching stream, over K more steps run right after the
           timed ones (the per-launch events would serialise the programmatic
           dependent launches of the timed steps).
``e2e``    the same metric through the public autograd API with the step's
           inputs copied host->device (pinned) and the loss read back each step;
           the copies run on a second stream, double-buffered, so step i+1's copy
           overlaps step i's compute; each step's loss lands in pinned host memory
           and the host reads it during the next step (the last one before the
           timed region ends).
``--impl reference`` times the CPU restatement of the reference's loss (its
           own op sequence in fp32 torch, all host threads) on a bounded row
           sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    # name: rows, hidden, vocab, description
    "c2": (16384, 576, 49152, "SmolLM2-135M training shape, [8,2048,576] per view, V=49152, bf16, "
                              "block-32 mask ratio U(0,1)"),
    "c5": (12288, 576, 49152, "ragged/edge: 12288 rows, ~25% valid, teacher x4, T=2, bf16"),
    "c3": (65536, 2048, 49152, "SmolLM2-1.7B shape, [32,2048,2048] per view, V=49152, bf16"),
    "c4": (32768, 1024, 248320, "large-vocab shape, [16,2048,1024] per view, V=248320, bf16 (vocab-sharded at N>1)"),
    "c2n": (16384, 576, 49152, "the 16384-row SmolLM2-135M shape on hidden states before the final RMSNorm: "
                               "norm (both views) + loss + norm backward in the step, bf16"),
}
METRIC = "KL-GEMM fwd+bwd loss-rows/sec"
SAMPLE_METRIC = "lm_head token selections/sec"
# fused lm_head + token selection (inference): rows, hidden, vocab, temperature, description
SAMPLE_CONFIGS = {
    "s1": (32, 576, 49153, 1.0, "decode: one K=32 block of rows (generate.py:149-188), SmolLM2-135M lm_head "
                               "H=576, V=49153 (with the mask token), T=1 sampling"),
    "s2": (16384, 576, 49153, 1.0, "scoring: 16384 rows, H=576, V=49153, T=1 sampling"),
    "s1f": (32, 576, 49153, 0.8, "decode with top-k 50 / top-p 0.9 (generate.py:59-73): one K=32 block of rows, "
                                "H=576, V=49153, T=0.8"),
}
SAMPLE_FILTERS = {"s1f": (50, 0.9)}   # top_k, top_p of the filtered workloads
L2_FLUSH_BYTES = 256 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS) + sorted(SAMPLE_CONFIGS) + sorted(ATTN_CONFIGS), default="c2")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="time budget of the CPU baseline sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-overlap", action="store_true",
                    help="row sharding: one dW all-reduce after the step instead of per-chunk buckets overlapped "
                         "(the default from 8 ranks)")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="nccl",
                    help="row sharding: dW all-reduced by NCCL, overlapped per chunk (nccl), or summed inside "
                         "the step over NVLink peer memory (p2p)")
    ap.add_argument("--sm-reserve", type=int, default=0,
                    help="SMs left out of the persistent kernels' grids (room for NCCL beside them)")
    ap.add_argument("--sustained-seconds", type=float, default=2.5,
                    help="length of the extra back-to-back region reported as 'sustained' (0: skip)")
    return ap.parse_args()


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), "measured"
    return 1590.0, 1400.0, "fallback"


def load_hbm_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()).get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def load_traffic(kernel: str, config: str):
    """Bytes per launch from a committed ncu summary (profiles/traffic.json), else None."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(config, {}).get(kernel)
    except Exception:
        return None


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons of one GPU while running."""

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 7:
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        if not self.rows:
            return None
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[3 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ----------------------------------------------------------------------------- CPU baseline
def cpu_baseline(config: str, seconds: float):
    """Reference loss (its op sequence, fp32 torch on the host cores) on a row sample."""
    import torch
    from oracle import klgemm_oracle as O

    N, H, V, _ = CONFIGS[config]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sample = 256
    p = O.make_problem("c2" if config == "c2n" else config, n_rows=sample, seed=7)
    hs, ht, W, m, T = p["h_s"].float(), p["h_t"].float(), p["W"].float(), p["mask"], p["T"]
    times = []
    t_end = time.perf_counter() + seconds
    while True:
        t0 = time.perf_counter()
        O.aligned_kl_torch_with_grads(hs, ht, W, m, T)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end and len(times) >= 2:
            break
    t = statistics.median(times[1:]) if len(times) > 1 else times[0]
    return {"value": sample / t, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{sample} of {N} rows x full V={V}, H={H}, fp32 torch (reference op sequence, "
                      f"train.py:142-210) fwd+bwd incl. dW; median of {len(times) - 1} runs"}


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    N, H, V, desc = CONFIGS[args.config]
    import torch
    from oracle import klgemm_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sample = 128
    p = O.make_problem("c2" if args.config == "c2n" else args.config, n_rows=sample, seed=7)
    hs, ht, W, m, T = p["h_s"].float(), p["h_t"].float(), p["W"].float(), p["mask"], p["T"]
    for _ in range(max(1, args.warmup)):
        O.aligned_kl_torch_with_grads(hs, ht, W, m, T)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.aligned_kl_torch_with_grads(hs, ht, W, m, T)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = sample * args.steps / total
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded)",
        "impl": "reference",
        "config": {"workload": f"{args.config}: {desc}", "rows": N, "hidden": H, "vocab": V,
                   "rows_per_step_sample": sample, "parallelism": "host CPU"},
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port",
                         "sample": f"{sample} of {N} rows per step, full V, fp32 fwd+bwd incl. dW"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


# stdout carries exactly one line, the JSON result: everything else written to file
# descriptor 1 (NCCL's version banner, library messages) is sent to stderr.
_RESULT_OUT = None


def _claim_stdout():
    global _RESULT_OUT
    if _RESULT_OUT is None:
        sys.stdout.flush()
        _RESULT_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def emit(line: dict) -> None:
    _claim_stdout()
    _RESULT_OUT.write(json.dumps(line) + "\n")
    _RESULT_OUT.flush()


# ----------------------------------------------------------------------------- sampling workload
def _timed(fn, steps, flush):
    import torch
    ms = []
    for _ in range(steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ms.append(a.elapsed_time(b))
    return ms


def run_sample(args):
    """One step = one token per row of ``h`` from ``h @ W^T`` (the lm_head of generate.py:161-188
    followed by sample_token, generate.py:40-78): the fused kernel against the reference's op
    sequence on cuBLAS logits (same GPU) and the float64 oracle on the host."""
    import torch
    import torch.nn.functional as F

    from oracle import klgemm_oracle as O
    from orthrus_training_test_b200 import _lib, sampling

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        if int(os.environ.get("RANK", "0")) == 0:
            emit({"metric": SAMPLE_METRIC, "impl": args.impl, "unavailable": "sampling workloads run on one GPU"})
        return
    N, H, V, T, desc = SAMPLE_CONFIGS[args.config]
    if args.impl == "reference":
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        g = torch.Generator().manual_seed(1)
        sample = min(N, 32)
        h = torch.randn(sample, H, generator=g).to(torch.bfloat16).float()
        W = (torch.randn(V, H, generator=g) * 0.05).to(torch.bfloat16).float()
        for _ in range(max(1, args.warmup)):
            O.sample_token_torch(F.linear(h, W), T)
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            O.sample_token_torch(F.linear(h, W), T)
            times.append(time.perf_counter() - t0)
        value = sample * args.steps / sum(times)
        emit({"metric": SAMPLE_METRIC, "value": value, "unit": "rows/s", "n_gpus": args.gpus, "steps": args.steps,
              "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / args.steps, "higher_is_better": True,
              "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded)",
              "impl": "reference",
              "config": {"workload": f"{args.config}: {desc}", "rows": N, "hidden": H, "vocab": V,
                         "rows_per_step_sample": sample, "parallelism": "host CPU"},
              "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port",
                               "sample": f"{sample} of {N} rows per step: fp32 F.linear + sample_token op sequence"},
              "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        return

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    g = torch.Generator().manual_seed(1)
    h_host = torch.randn(N, H, generator=g).to(torch.bfloat16)
    W = (torch.randn(V, H, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    h = h_host.to(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    ws = torch.empty(sampling.workspace_bytes(N, V), dtype=torch.uint8, device=dev)
    seeds = iter(range(1, 1 << 30))

    top_k, top_p = SAMPLE_FILTERS.get(args.config, (0, 1.0))
    filtered = top_k > 0 or top_p < 1.0

    def ours(temp):
        if filtered and temp >= sampling.GREEDY_TEMPERATURE:
            return sampling.lm_head_sample_filtered(h, W, temp, top_k, top_p, next(seeds))
        return sampling.lm_head_sample(h, W, temp, next(seeds), workspace=ws)

    def torch_ref(temp):
        return O.sample_token_torch(F.linear(h, W).float(), temp, top_k, top_p)

    for _ in range(args.warmup):
        ours(T), ours(0.0), torch_ref(T), torch_ref(0.0)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    sampler = ClockSampler(0)
    sampler.start()
    time.sleep(0.3)
    _timed(lambda: ours(T), 3, flush)          # clocks back up after the sampler's start
    launches0 = _lib.launch_count()
    ms = _timed(lambda: ours(T), args.steps, flush)
    launches = _lib.launch_count() - launches0
    ms_greedy = _timed(lambda: ours(0.0), args.steps, flush)
    clocks = sampler.stop()
    ms_torch = _timed(lambda: torch_ref(T), args.steps, flush)
    ms_torch_greedy = _timed(lambda: torch_ref(0.0), args.steps, flush)
    _lib.trace_begin(4096)
    for _ in range(args.steps):
        flush.zero_()
        ours(T)
    torch.cuda.synchronize()
    trace = _lib.trace_end(4096)
    assert _lib.device_status() == 0
    # the dominant kernel: the lm_head sweep (the filtered path runs two of them per call)
    k_ms = [t for kind, t in trace if kind == "sample"]
    k_ms = sorted(k_ms)[len(k_ms) // 2:] if filtered else k_ms
    k_avg = sum(k_ms) / len(k_ms)
    by_kind = {}
    for kind, t in trace:
        by_kind.setdefault(kind, [0.0, 0])
        by_kind[kind][0] += t
        by_kind[kind][1] += 1
    tot = sum(v[0] for v in by_kind.values())
    kernels = {k: {"launches": n, "total_ms": t, "share": t / tot} for k, (t, n) in by_kind.items()}

    hbm_peak, hbm_src = load_hbm_peak()
    peak_burst, _, peak_src = load_peaks()
    bytes_alg = 2.0 * V * H + 2.0 * N * H + 12.0 * N
    flops = 2.0 * N * H * V
    if bytes_alg / (hbm_peak * 1e9) >= flops / (peak_burst * 1e12):
        ach = bytes_alg / (k_avg / 1e3) / 1e9
        roofline = {"bound": "hbm", "kernel": "sample", "achieved": ach, "peak": hbm_peak, "unit": "GB/s",
                    "frac": ach / hbm_peak, "traffic": load_traffic("sample", args.config),
                    "peak_kind": f"{hbm_src} copy bandwidth", "algorithmic_bytes_per_launch": bytes_alg}
    else:
        ach = flops / (k_avg / 1e3) / 1e12
        roofline = {"bound": "tensor", "kernel": "sample", "achieved": ach, "peak": peak_burst, "unit": "TFLOP/s",
                    "frac": ach / peak_burst, "traffic": load_traffic("sample", args.config),
                    "peak_kind": f"{peak_src} burst bf16", "algorithmic_flops_per_launch": flops}

    # end to end: h from pinned host memory, tokens back to the host every step
    h_pin = h_host.pin_memory()
    tok_host = torch.empty(N, dtype=torch.int64).pin_memory()

    def e2e_step():
        hd = h_pin.to(dev, non_blocking=True)
        if filtered:
            tok, _, _ = sampling.lm_head_sample_filtered(hd, W, T, top_k, top_p, next(seeds))
        else:
            tok, _, _ = sampling.lm_head_sample(hd, W, T, next(seeds), workspace=ws)
        tok_host.copy_(tok, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(3):
        e2e_step()
    e_ms = _timed(e2e_step, args.steps, flush)

    cpu = None
    if not args.no_cpu_baseline:
        sample = min(N, 8)
        hs = h_host[:sample].float().numpy()
        Wn = W.float().cpu().numpy()
        times = []
        t_end = time.perf_counter() + min(args.cpu_seconds, 10.0)
        while True:
            t0 = time.perf_counter()
            O.lm_head_sample_np(hs, Wn, T, seed=1)
            times.append(time.perf_counter() - t0)
            if time.perf_counter() > t_end and len(times) >= 2:
                break
        cpu = {"value": sample / statistics.median(times), "unit": "rows/s", "cores": 1, "kind": "port",
               "sample": f"{sample} rows x V={V}: float64 numpy lm_head + Gumbel-max keys (the oracle)"}

    total = sum(ms)
    emit({
        "metric": SAMPLE_METRIC, "value": N * args.steps / (total / 1e3), "unit": "rows/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) hidden, "
        "N(0,0.05) lm_head)",
        "config": {"workload": f"{args.config}: {desc}", "rows": N, "hidden": H, "vocab": V, "temperature": T,
                   "top_k": top_k, "top_p": top_p,
                   "parallelism": "single GPU", "l2": "flushed between steps (256 MiB write)"},
        "greedy_ms_per_step": sum(ms_greedy) / args.steps,
        "torch_cublas_ms_per_step": {"sampled": sum(ms_torch) / args.steps,
                                     "greedy": sum(ms_torch_greedy) / args.steps,
                                     "what": "F.linear (cuBLAS, bf16) + the reference's sample_token ops, same GPU"},
        "roofline": roofline, "kernels": kernels, "gpu_launches": int(launches),
        "e2e": {"value": N * args.steps / (sum(e_ms) / 1e3), "unit": "rows/s", "h2d_bytes_per_step": 2 * N * H,
                "d2h_bytes_per_step": 8 * N, "ms_per_step": sum(e_ms) / args.steps,
                "api": "sampling.lm_head_sample"},
        "cpu_baseline": cpu, "clocks": clocks,
    })


# ----------------------------------------------------------------------------- block-diffusion attention
ATTN_METRIC = "diffusion-attention query rows/sec"
# batch, heads, kv heads, block K, diffusion length, AR length, description (one layer, SmolLM2-135M heads)
ATTN_CONFIGS = {
    "a1": (1, 9, 3, 32, 32, 2048, "decode: one K=32 block over a 2048-token AR cache (generate.py:149-176), "
                                  "9 heads / 3 KV heads, head_dim 64, per layer"),
    "a2": (4, 9, 3, 32, 2048, 2048, "training diffusion pass: 4 x 64 blocks of 32, each over the AR prefix "
                                    "before its anchor (model.py:400-446), per layer"),
    "a2b": (4, 9, 3, 32, 2048, 2048, "training diffusion pass, forward + backward (dQ and the blocks' own dK / dV; "
                                     "the AR cache is frozen): 4 x 64 blocks of 32 over their AR prefixes, per layer"),
}


def run_attn(args):
    """One step = one layer's diffusion attention (model.py:136-176) over the config's
    queries: the fused kernel against torch SDPA with the same boolean mask on the same GPU,
    and the float64 oracle on the host."""
    import numpy as np
    import torch
    import torch.nn.functional as F

    from oracle import klgemm_oracle as O
    from orthrus_training_test_b200 import _lib
    from orthrus_training_test_b200.attention import block_attention, workspace_bytes

    B, H, Hkv, K, Ld, AL, desc = ATTN_CONFIGS[args.config]
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        if int(os.environ.get("RANK", "0")) == 0:
            emit({"metric": ATTN_METRIC, "impl": args.impl, "unavailable": "attention workloads run on one GPU"})
        return
    if args.impl == "reference":
        # the attention semantics of the reference's flex path (model.py:45-96, 435-446) in the
        # float64 oracle on the host, one block of K positions x H heads per step
        g = torch.Generator().manual_seed(3)
        q = torch.randn(1, H, K, 64, generator=g).numpy()
        ks, vs = torch.randn(1, Hkv, K, 64, generator=g).numpy(), torch.randn(1, Hkv, K, 64, generator=g).numpy()
        ka, va = torch.randn(1, Hkv, AL, 64, generator=g).numpy(), torch.randn(1, Hkv, AL, 64, generator=g).numpy()
        lim = np.full((1, K), AL // 2 if Ld > K else AL - 1)
        do = torch.randn(1, H, K, 64, generator=g).numpy()
        train_ref = args.config.endswith("b")

        def ref_step():
            O.block_attention_np(q, ks, vs, ka, va, lim, K)
            if train_ref:
                O.block_attention_bwd_np(q, ks, vs, ka, va, lim, K, do)

        for _ in range(max(1, args.warmup)):
            ref_step()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            ref_step()
        dt = time.perf_counter() - t0
        value = H * K * args.steps / dt
        emit({"metric": ATTN_METRIC, "value": value, "unit": "rows/s", "n_gpus": args.gpus, "steps": args.steps,
              "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True,
              "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded)", "impl": "reference",
              "config": {"workload": f"{args.config}: {desc}", "rows_per_step_sample": H * K, "parallelism": "host CPU"},
              "cpu_baseline": {"value": value, "unit": "rows/s", "cores": 1, "kind": "port",
                               "sample": f"one block of {K} positions x {H} heads per step: the float64 oracle"},
              "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        return
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    g = torch.Generator().manual_seed(3)
    bf = lambda *sh: torch.randn(*sh, generator=g).to(torch.bfloat16).to(dev)
    q, ks, vs, ka, va = bf(B, H, Ld, 64), bf(B, Hkv, Ld, 64), bf(B, Hkv, Ld, 64), bf(B, Hkv, AL, 64), bf(B, Hkv, AL, 64)
    if Ld == K:
        lim = torch.full((B, Ld), AL - 1, dtype=torch.int32)
    else:
        anchors = torch.randint(1, AL, (B, Ld // K), generator=g).sort(dim=1).values
        lim = (anchors - 1).repeat_interleave(K, dim=1).to(torch.int32)
    lim_d = lim.to(dev)
    ws = torch.empty(workspace_bytes(B, H, Hkv, Ld, K, AL), dtype=torch.uint8, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    # SDPA comparison: keys [AR ; own diffusion keys], boolean mask of the same visibility
    kv_idx = torch.arange(AL + Ld, device=dev)
    q_blk = torch.arange(Ld, device=dev) // K
    vis_ar = kv_idx[None, None, :AL] <= lim_d.long()[:, :, None]
    vis_self = (q_blk[:, None] == (kv_idx[AL:] - AL)[None, :] // K)[None].expand(B, -1, -1)
    mask = torch.cat([vis_ar, vis_self], dim=2)[:, None]               # [B, 1, Ld, AL + Ld]
    k_full, v_full = torch.cat([ka, ks], dim=2), torch.cat([va, vs], dim=2)

    train = args.config.endswith("b")   # forward + backward
    d_out = bf(B, H, Ld, 64)
    qg, ksg, vsg = (t.detach().clone().requires_grad_(True) for t in (q, ks, vs))

    def ours():
        if train:
            qg.grad = ksg.grad = vsg.grad = None
            o = block_attention(qg, ksg, vsg, ka, va, lim_d, K)
            o.backward(d_out)
            return o
        return block_attention(q, ks, vs, ka, va, lim_d, K, workspace=ws)

    def sdpa():
        if train:
            qg.grad = ksg.grad = vsg.grad = None
            kf, vf = torch.cat([ka, ksg], dim=2), torch.cat([va, vsg], dim=2)
            o = F.scaled_dot_product_attention(qg, kf, vf, attn_mask=mask, enable_gqa=True)
            o.backward(d_out)
            return o
        return F.scaled_dot_product_attention(q, k_full, v_full, attn_mask=mask, enable_gqa=True)

    for _ in range(args.warmup):
        ours(), sdpa()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    sampler = ClockSampler(0)
    sampler.start()
    time.sleep(0.3)
    _timed(ours, 3, flush)                     # clocks back up after the sampler's start
    launches0 = _lib.launch_count()
    ms = _timed(ours, args.steps, flush)
    launches = _lib.launch_count() - launches0
    clocks = sampler.stop()
    ms_sdpa = _timed(sdpa, args.steps, flush)
    _lib.trace_begin(4096)
    for _ in range(args.steps):
        flush.zero_()
        ours()
    torch.cuda.synchronize()
    trace = _lib.trace_end(4096)
    assert _lib.device_status() == 0
    by_kind = {}
    for kind, t in trace:
        by_kind.setdefault(kind, [0.0, 0])
        by_kind[kind][0] += t
        by_kind[kind][1] += 1
    tot = sum(v[0] for v in by_kind.values())
    kernels = {k: {"launches": n, "total_ms": t, "share": t / tot} for k, (t, n) in by_kind.items()}
    k_avg = by_kind["attn"][0] / by_kind["attn"][1]
    # algorithmic work: every visible (query, key) pair costs 2 x 64 MACs (Q K and P V) forward;
    # the backward recomputes Q K and adds dO V^T and dS K (3 x 64 MACs; dV / dK of the blocks'
    # own keys add 2 x 64 on those pairs); with the forward and backward launches alternating,
    # k_avg is their mean and the work per launch is half the step's
    visible = float((lim.clamp(-1, AL - 1).long() + 1).sum()) * H + B * H * Ld * K
    flops = 4.0 * 64 * visible
    if train:
        flops = (4.0 * 64 * visible + 6.0 * 64 * visible + 4.0 * 64 * B * H * Ld * K) / 2
    # bytes: Q + O + every K / V row some query sees, once (the AR prefix up to the sequence's
    # largest limit, and the diffusion positions' own keys)
    ar_rows = float((lim.clamp(-1, AL - 1).long().amax(dim=1) + 1).sum()) * Hkv
    kv_rows = ar_rows + B * Hkv * Ld
    bytes_alg = 2.0 * B * H * Ld * 64 * 2 + kv_rows * 64 * 2 * 2
    hbm_peak, hbm_src = load_hbm_peak()
    peak_burst, _, peak_src = load_peaks()
    if bytes_alg / (hbm_peak * 1e9) >= flops / (peak_burst * 1e12):
        ach = bytes_alg / (k_avg / 1e3) / 1e9
        roofline = {"bound": "hbm", "kernel": "attn", "achieved": ach, "peak": hbm_peak, "unit": "GB/s",
                    "frac": ach / hbm_peak, "traffic": load_traffic("attn", args.config),
                    "peak_kind": f"{hbm_src} copy bandwidth", "algorithmic_bytes_per_launch": bytes_alg}
    else:
        ach = flops / (k_avg / 1e3) / 1e12
        roofline = {"bound": "tensor", "kernel": "attn", "achieved": ach, "peak": peak_burst, "unit": "TFLOP/s",
                    "frac": ach / peak_burst, "traffic": load_traffic("attn", args.config),
                    "peak_kind": f"{peak_src} burst bf16", "algorithmic_flops_per_launch": flops}
    # e2e: q and the diffusion keys / values from pinned host memory, the output back to the host
    q_h, ks_h, vs_h = q.cpu().pin_memory(), ks.cpu().pin_memory(), vs.cpu().pin_memory()
    out_h = torch.empty(B, H, Ld, 64, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        if train:
            qd = q_h.to(dev, non_blocking=True).requires_grad_(True)
            ksd = ks_h.to(dev, non_blocking=True).requires_grad_(True)
            vsd = vs_h.to(dev, non_blocking=True).requires_grad_(True)
            o = block_attention(qd, ksd, vsd, ka, va, lim_d, K)
            o.backward(d_out)
            out_h.copy_(qd.grad, non_blocking=True)   # the step's result read back: dQ
        else:
            o = block_attention(q_h.to(dev, non_blocking=True), ks_h.to(dev, non_blocking=True),
                                vs_h.to(dev, non_blocking=True), ka, va, lim_d, K, workspace=ws)
            out_h.copy_(o, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(3):
        e2e_step()
    e_ms = _timed(e2e_step, args.steps, flush)
    cpu = None
    if not args.no_cpu_baseline:
        nb = 1
        sl = slice(0, nb * K)
        qs = q[:1, :, sl].float().cpu().numpy()
        t_end = time.perf_counter() + min(args.cpu_seconds, 10.0)
        times = []
        cargs = (qs, ks[:1, :, sl].float().cpu().numpy(), vs[:1, :, sl].float().cpu().numpy(),
                 ka[:1].float().cpu().numpy(), va[:1].float().cpu().numpy(), lim[:1, sl].numpy(), K)
        dos = d_out[:1, :, sl].float().cpu().numpy()
        while True:
            t0 = time.perf_counter()
            O.block_attention_np(*cargs)
            if train:
                O.block_attention_bwd_np(*cargs, dos)
            times.append(time.perf_counter() - t0)
            if time.perf_counter() > t_end and len(times) >= 2:
                break
        cpu = {"value": H * K / statistics.median(times), "unit": "rows/s", "cores": 1, "kind": "port",
               "sample": f"one block of {K} positions x {H} heads over its AR prefix: the float64 oracle"
                         + (" forward and backward" if train else "")}
    rows = B * H * Ld
    total = sum(ms)
    emit({
        "metric": ATTN_METRIC, "value": rows * args.steps / (total / 1e3), "unit": "rows/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) q, k, v)",
        "config": {"workload": f"{args.config}: {desc}", "batch": B, "heads": H, "kv_heads": Hkv, "block": K,
                   "diff_len": Ld, "ar_len": AL, "parallelism": "single GPU", "l2": "flushed between steps (256 MiB write)"},
        "sdpa_ms_per_step": sum(ms_sdpa) / args.steps,
        "sdpa_what": "torch scaled_dot_product_attention with the same boolean mask and GQA, same GPU"
                     + (" (forward + autograd backward)" if train else ""),
        "roofline": roofline, "kernels": kernels, "gpu_launches": int(launches),
        "e2e": {"value": rows * args.steps / (sum(e_ms) / 1e3), "unit": "rows/s",
                "h2d_bytes_per_step": int((q_h.numel() + ks_h.numel() + vs_h.numel()) * 2),
                "d2h_bytes_per_step": int(out_h.numel() * 2), "ms_per_step": sum(e_ms) / args.steps,
                "api": "attention.block_attention"},
        "cpu_baseline": cpu, "clocks": clocks,
    })


# ----------------------------------------------------------------------------- our arm
def main():
    args = parse()
    _claim_stdout()
    if args.config in SAMPLE_CONFIGS:
        run_sample(args)
        return
    if args.config in ATTN_CONFIGS:
        run_attn(args)
        return
    if args.impl == "reference":
        run_reference_arm(args)
        return

    import torch
    import torch.distributed as dist

    from oracle import klgemm_oracle as O  # input generator only (seeded workload shapes)
    from orthrus_training_test_b200 import _lib, ops
    from orthrus_training_test_b200.parallel import row_sharded_kl_loss, shard_bounds, vocab_sharded_kl_loss

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("--gpus N > 1 must be launched with torch.distributed.run (one process per GPU)")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    _lib.lib()
    if args.sm_reserve:
        ops.set_sm_reserve(args.sm_reserve)

    N, H, V, desc = CONFIGS[args.config]
    vocab_sharded = args.config == "c4" and world > 1
    prenorm = args.config == "c2n"
    pcfg = "c2" if prenorm else args.config
    p = O.make_problem(pcfg, seed=42 if vocab_sharded else 42 + rank)   # this rank's rows
    pw = O.make_problem(pcfg, n_rows=1, seed=42)   # shared lm_head
    T = p["T"]
    hs = p["h_s"].to(dev)
    ht = p["h_t"].to(dev)
    W = pw["W"].to(dev)
    V_work = V                                            # lm_head rows this rank computes over
    if vocab_sharded:
        lo, hi = shard_bounds(V, world, rank)
        W = W[lo:hi].contiguous()
        V_work = hi - lo
    m = ops.mask_u8(p["mask"].to(dev))
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    if prenorm:
        # pre-norm residual-stream rows (scale 3) and a norm weight around 1
        gn = torch.Generator().manual_seed(43 + rank)
        hs = (p["h_s"].float() * 3.0).to(torch.bfloat16).to(dev)
        ht = (p["h_t"].float() * 3.0).to(torch.bfloat16).to(dev)
        gamma = (1.0 + 0.1 * torch.randn(H, generator=gn)).to(torch.bfloat16).float().to(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    fb_ws = int(_lib.lib().klg_fwd_bwd_workspace_bytes(N, H, V_work))
    gathered = torch.empty(world * 2, 2 * N, dtype=torch.float32, device=dev) if vocab_sharded else None
    xbuf = torch.empty(N * H + N, dtype=torch.float32, device=dev) if vocab_sharded else None   # [dH | cross]
    xbuf_dh = xbuf[:N * H].view(N, H) if vocab_sharded else None

    def step_vocab():
        # vocab-sharded training step: pass 1 over the local slice -> all-gather of the (m, S)
        # records -> global log-sum-exps -> pass 2 over the slice (its dW, a partial dH, its part
        # of the KL cross term) -> one all-reduce of [dH | cross] -> loss
        cnt = ops.count_valid(m)                       # the same rows on every rank
        rec = ops.lse_record(hs, ht, W, T)
        dist.all_gather_into_tensor(gathered, rec)
        lse = ops.lse_merge(gathered.view(world, 2, 2 * N))
        dh, dw, cross = ops.pass2(hs, ht, W, m, lse, cnt, temperature=T, workspace_bytes=fb_ws, dh_out=xbuf_dh)
        xbuf[N * H:].copy_(cross)
        dist.all_reduce(xbuf)
        loss, _ = ops.kl_loss(lse, xbuf[N * H:], m, cnt)
        return loss

    def step_prenorm():
        cnt = ops.count_valid(m)
        if world > 1:
            dist.all_reduce(cnt)
        ys, rs = ops.rmsnorm_rows(hs, gamma)
        yt, _ = ops.rmsnorm_rows(ht, gamma, want_rstd=False)
        loss, _, _, _, dh, dw = ops.kl_fwd_bwd(ys, yt, W, m, T, count=cnt, workspace_bytes=fb_ws)
        ops.rmsnorm_rows_backward(hs, gamma, rs, dh)
        if world > 1:
            dist.all_reduce(loss)
            dist.all_reduce(dw)
        return loss

    # row sharding: dW is exchanged in vocab-chunk buckets, each all-reduced on a side stream as
    # soon as its chunk's GEMM is done (overlapping the chunks still computing)
    # row sharding with --exchange p2p: dW summed over the ranks inside the step over NVLink peer
    # memory (the GEMM stores each block of the partial into its owner's buffer)
    xr = None
    os.environ["KLG_XR"] = "1" if args.exchange == "p2p" else "0"   # the e2e leg below takes the same route
    if world > 1 and not vocab_sharded and not prenorm and args.exchange == "p2p":
        from orthrus_training_test_b200.parallel import CudaEngine
        xr = CudaEngine().xr_exchange(None, hs, W)
        if xr is None:
            os.environ["KLG_XR"] = "0"   # the e2e leg below takes the same (NCCL) route
    # per-chunk overlapped buckets up to 4 ranks (as row_sharded_kl_loss): at 8 ranks one
    # all-reduce after the step measured faster
    overlap = 1 < world < 8 and xr is None and not vocab_sharded and not prenorm and not args.no_overlap
    buckets = ops.chunk_bounds(N, H, V_work, fb_ws) if overlap else None
    chunk_evs = ops.new_chunk_events(len(buckets)) if overlap else None
    side = torch.cuda.Stream(device=dev) if overlap else None

    def step():
        if vocab_sharded:
            return step_vocab()
        if prenorm:
            return step_prenorm()
        # the training step: count (all-reduced across ranks) -> loss + dH + dW -> loss and dW all-reduced;
        # on one GPU the step counts the mask itself (inside its pass-1 merge), as the autograd op does
        cnt = None
        if world > 1:
            cnt = ops.count_valid(m)
            dist.all_reduce(cnt)
        if xr is not None:
            loss, dh, dw = ops.kl_fwd_bwd_xr(hs, ht, W, m, T, cnt, True, xr.world, xr.rank, xr.peer_buffers,
                                             xr.next_epoch(), workspace_bytes=fb_ws)
            dist.all_reduce(loss)
            return loss
        loss, _, _, _, dh, dw = ops.kl_fwd_bwd(hs, ht, W, m, T, count=cnt, workspace_bytes=fb_ws,
                                               chunk_events=chunk_evs)
        if world > 1:
            works = []
            if overlap:
                with torch.cuda.stream(side):
                    for (v0, v1), ev in zip(buckets, chunk_evs):
                        side.wait_event(ev)
                        works.append(dist.all_reduce(dw[v0:v1], async_op=True))
            else:
                dist.all_reduce(dw)
            dist.all_reduce(loss)
            for wk in works:
                wk.wait()
        return loss

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0

    # ---------------------------------------------------------------- device-timed steps
    # start the clock sampler first: every rank then leaves the barrier together, so no rank's
    # first timed collective waits for another rank's set-up
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.zero_()                                  # evict inputs from L2 (outside the timed events)
        ev[i][0].record()
        step()
        ev[i][1].record()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches = _lib.launch_count() - launches0
    clocks = sampler.stop() if sampler else None
    # per-kernel breakdown: the same steps again with an event pair around every launch
    _lib.trace_begin(8192)
    for i in range(args.steps):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    trace = _lib.trace_end(8192)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    # sustained: back-to-back steps for a region of >= 2 s (the 1 kW power cap lowers the clocks
    # after ~100 ms of full load), with its own clock record; the step count is sized from the
    # steps above and agreed across ranks so every rank runs the same collectives
    sustained = None
    if args.sustained_seconds > 0:
        per = torch.tensor([statistics.median(step_ms)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(per, op=dist.ReduceOp.MAX)
        n_sus = max(10, int(math.ceil(args.sustained_seconds * 1e3 / float(per.item()))))
        sampler2 = ClockSampler(local) if rank == 0 else None
        if sampler2:
            sampler2.start()
            time.sleep(0.3)
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(n_sus):
            flush.zero_()
            step()
        e1.record()
        torch.cuda.synchronize()
        sus_ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(sus_ms, op=dist.ReduceOp.MAX)
        sus_clocks = sampler2.stop() if sampler2 else None
        sus_ms = float(sus_ms.item())
        sustained = {"steps": n_sus, "seconds": sus_ms / 1e3, "ms_per_step": sus_ms / n_sus,
                     "value": N * (1 if vocab_sharded else world) * n_sus / (sus_ms / 1e3), "unit": "rows/s",
                     "clocks": sus_clocks,
                     "note": "back-to-back steps for >= 2 s, L2 flushed between steps (the flush is inside this "
                             "region): the steady state of a training loop under the 1 kW power cap"}
    total_ms = torch.tensor([sum(step_ms)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
    total_ms = float(total_ms.item())
    assert _lib.device_status() == 0

    rows_total = N * (1 if vocab_sharded else world) * args.steps
    value = rows_total / (total_ms / 1e3)

    # ---------------------------------------------------------------- per-kernel roofline
    peak_burst, peak_sust, peak_src = load_peaks()
    by_kind = {}
    for kind, ms in trace:
        t = by_kind.setdefault(kind, [0.0, 0])
        t[0] += ms
        t[1] += 1
    flops_per_step = {"stats": 4.0 * N * H * V_work, "dz": 4.0 * N * H * V_work, "gemm": 4.0 * N * H * V_work}
    dom = max((k for k in by_kind if k in flops_per_step), key=lambda k: by_kind[k][0])
    dom_ms, dom_n = by_kind[dom]
    dom_flops_per_launch = flops_per_step[dom] * args.steps / dom_n
    dom_avg_ms = dom_ms / dom_n
    achieved = dom_flops_per_launch / (dom_avg_ms / 1e3) / 1e12
    traffic = load_traffic(dom, args.config)
    # The kernels are timed inside a region of well under a second at full clocks, so the
    # denominator is the burst GEMM peak; the sustained figure is shown beside it.
    roofline = {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": peak_burst, "unit": "TFLOP/s",
                "frac": achieved / peak_burst, "traffic": traffic,
                "peak_kind": f"{peak_src} burst bf16 (kernels timed in a sub-second region)",
                "frac_of_sustained_peak": achieved / peak_sust,
                "algorithmic_flops_per_launch": dom_flops_per_launch}
    step_flops = 8.0 * N * H * V_work   # per GPU
    kernels = {k: {"launches": n, "total_ms": t, "share": t / sum(x[0] for x in by_kind.values())}
               for k, (t, n) in sorted(by_kind.items(), key=lambda kv: -kv[1][0])}

    # ---------------------------------------------------------------- end-to-end (public API)
    e2e = None
    if not args.no_e2e:
        hs_h = hs.cpu().pin_memory() if prenorm else p["h_s"].pin_memory()
        ht_h = ht.cpu().pin_memory() if prenorm else p["h_t"].pin_memory()
        m_h = p["mask"].to(torch.uint8).pin_memory()
        Wp = W.clone().requires_grad_(True)
        h2d = hs_h.numel() * hs_h.element_size() + ht_h.numel() * ht_h.element_size() + m_h.numel()

        # Each step copies its own inputs from pinned host memory (double-buffered on a second
        # stream, so step i+1's copy overlaps step i's compute), runs the public API and reads
        # the loss back to the host: copied into pinned memory behind the step and read by the
        # host once that copy has landed, during the next step (the host stays one step ahead
        # instead of idling the GPU while it waits).  The L2 flush runs before each step's
        # compute, inside the timed region.
        copy_stream = torch.cuda.Stream(device=dev)
        slots = [(torch.empty(hs_h.shape, dtype=hs_h.dtype, device=dev), torch.empty(ht_h.shape, dtype=ht_h.dtype, device=dev),
                  torch.empty(m_h.shape, dtype=m_h.dtype, device=dev)) for _ in range(2)]
        landed = [torch.cuda.Event() for _ in range(2)]
        used = [torch.cuda.Event() for _ in range(2)]       # the step reading slot k has finished
        loss_h = torch.zeros(2, dtype=torch.float32).pin_memory()
        read = [torch.cuda.Event() for _ in range(2)]       # loss_h[k] holds that step's loss

        def issue_copy(k, after_use):
            with torch.cuda.stream(copy_stream):
                if after_use:
                    copy_stream.wait_event(used[k])
                for d_, h_ in zip(slots[k], (hs_h, ht_h, m_h)):
                    d_.copy_(h_, non_blocking=True)
                landed[k].record(copy_stream)

        def run_e2e(n):
            issue_copy(0, False)
            out = 0.0
            for i in range(n):
                k = i & 1
                torch.cuda.current_stream().wait_event(landed[k])
                if i + 1 < n:
                    issue_copy(1 - k, i >= 1)   # slot 1-k is refilled once step i-1 has finished with it
                flush.zero_()
                hs_d = slots[k][0].detach().requires_grad_(True)
                ht_d, m_d = slots[k][1], slots[k][2]
                if prenorm and world == 1:
                    loss = ops.prenorm_kl_loss(hs_d, ht_d, gamma, Wp, m_d, T)
                elif vocab_sharded:
                    loss = vocab_sharded_kl_loss(hs_d, ht_d, Wp, m_d, T)
                elif world > 1:
                    loss = row_sharded_kl_loss(hs_d, ht_d, Wp, m_d, T)
                else:
                    loss = ops.kl_gemm_loss(hs_d, ht_d, Wp, m_d, T)
                loss.backward()
                Wp.grad = None
                used[k].record()
                loss_h[k].copy_(loss.detach(), non_blocking=True)   # device -> host copy of the step's result
                read[k].record()
                if i >= 1:
                    read[1 - k].synchronize()
                    out = float(loss_h[1 - k])                        # host read of step i-1's loss
            read[(n - 1) & 1].synchronize()
            return float(loss_h[(n - 1) & 1])

        run_e2e(max(3, args.warmup))
        torch.cuda.synchronize()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        run_e2e(args.steps)
        b.record()
        torch.cuda.synchronize()
        e_ms = [a.elapsed_time(b)]
        et = torch.tensor([sum(e_ms)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e2e = {"value": rows_total / (float(et.item()) / 1e3), "unit": "rows/s", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": 4, "ms_per_step": float(et.item()) / args.steps,
               "copies": "pinned host -> device each step on a second stream, double-buffered (step i+1's copy "
                         "overlaps step i); each step's loss copied to pinned host memory and read by the host "
                         "during the next step; L2 flushed before each step inside the timed region",
               "api": ("vocab_sharded_kl_loss" if vocab_sharded else "row_sharded_kl_loss" if world > 1
                       else "kl_gemm_loss (KLGemmFn autograd)")}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.config, args.cpu_seconds)

    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if vocab_sharded else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) hidden, "
            "N(0,0.02) lm_head)",
            "config": {"workload": f"{args.config}: {desc}", "rows_per_gpu": N, "hidden": H, "vocab": V,
                       "vocab_per_gpu": V_work,
                       "temperature": T, "parallelism": (f"vocab-sharded x{world}" if vocab_sharded else
                                                         f"row-sharded dp{world}" if world > 1 else "single GPU"),
                       "dw_exchange": ("inside the step over NVLink peer memory (klg_fwd_bwd_xr)" if xr is not None
                                       else "per-chunk buckets overlapped on a side stream" if overlap else
                                       "one all-reduce after the step" if world > 1 and not vocab_sharded else None),
                       "sm_reserve": args.sm_reserve,
                       "l2": "flushed between steps (256 MiB write)"},
            "sustained": (dict(sustained, achieved_tflops=step_flops / (sustained["ms_per_step"] / 1e3) / 1e12,
                               frac_of_sustained=step_flops / (sustained["ms_per_step"] / 1e3) / 1e12 / peak_sust,
                               frac_of_burst=step_flops / (sustained["ms_per_step"] / 1e3) / 1e12 / peak_burst)
                          if sustained else None),
            "tensor_peak_frac": {"algorithmic_flops_per_step": step_flops,
                                 "achieved_tflops": step_flops / (total_ms / args.steps / 1e3) / 1e12,
                                 "frac_of_sustained": step_flops / (total_ms / args.steps / 1e3) / 1e12 / peak_sust,
                                 "frac_of_burst": step_flops / (total_ms / args.steps / 1e3) / 1e12 / peak_burst,
                                 "note": "8*N*H*V per fwd+bwd; executed work is 12*N*H*V (logits recomputed)"},
            "roofline": roofline,
            "kernels": kernels,
            "gpu_launches": int(launches),
            "e2e": e2e,
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        emit(line)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
