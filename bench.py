"""Benchmark of the fused MoE MLP hot path on B200.

Workload (default, N=1): the Mixtral-8x7B-shaped MoE layer — T=4096 tokens,
H=4096, I=14336, E=8 experts, top-2, bf16, uniform softmax routing of
N(0,1) logits, activations N(0,1), weights N(0,0.02) (seeded synthetic data).
One step = one call of the top-k fused_moe_mlp (align -> gather -> gate_up
GEMM + SwiGLU -> down GEMM + weighted combine -> bf16) over the resident batch,
replayed from a CUDA graph captured once (the same kernels; --eager calls the
op directly every step).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config NAME]

With N > 1 (torchrun) every rank runs the expert-parallel layer on its own
T tokens (weak scaling): experts are sharded E/N per rank and token rows
travel to their experts and back over NVLink peer memory (mail_b200.ep).

One JSON line (rank 0). Besides the contract keys it carries:
  roofline    the gate_up GEMM's achieved rate against the measured peak; its
              per-launch time comes from the library's device-side kernel
              clocks read over the timed region itself (CUDA-event stage
              times from a separate replay are reported beside it)
  sustained   the same step replayed back to back for >= 1.5 s (power-capped
              clocks), against the sustained bf16 peak
  configs     the other workloads at their own shapes: N=1 — Qwen3-30B-A3B
              decode (T = 1, 8, 32, 128, 256), DeepSeek-V3 w8a8 prefill, the
              load-imbalance stress; N>1 — DeepSeek-V3 w8a8 expert-parallel
              with 8192 tokens per GPU (weak) and 8192 in total (strong);
              each with its own gate_up roofline (HBM for decode, int8 tensor
              against a measured int8 GEMM yardstick for w8a8)
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "mixtral": dict(T=4096, H=4096, I=14336, E=8, k=2, routing="uniform-softmax", dtype="bf16", quant=False,
                    desc="Mixtral-8x7B MoE layer"),
    "tiny": dict(T=64, H=1024, I=512, E=8, k=2, routing="uniform-softmax", dtype="fp32", quant=False,
                 desc="tiny fp32 MoE MLP"),
    "mixtral-prerouted": dict(T=4096, H=4096, I=14336, E=8, k=2, routing="uniform-softmax", dtype="bf16",
                              quant=False, prerouted=True,
                              desc="Mixtral-8x7B MoE layer, reference form: pre-grouped rows + group sizes"),
    "qwen3-decode": dict(T=256, H=2048, I=768, E=128, k=8, routing="zipf1.2", dtype="bf16", quant=False,
                         desc="Qwen3-30B-A3B decode (T=256)"),
    "dsv3-w8a8": dict(T=8192, H=7168, I=2048, E=256, k=8, routing="sigmoid", dtype="bf16", quant=True,
                      desc="DeepSeek-V3 prefill w8a8"),
    "stress-w8a8": dict(T=65536, H=4096, I=1536, E=64, k=6, routing="hot25-zipf1.0", dtype="bf16", quant=True,
                        desc="long-prefill load-imbalance stress w8a8"),
}
STAGES = 7  # MOE_STAGE_* boundaries recorded per step


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return dict(hbm=float(p["hbm_gbs"]), bf16=float(p["bf16_tflops"]),
                    bf16_sus=float(p["bf16_tflops_sustained"]), source="measured")
    except Exception:
        return dict(hbm=6650.0, bf16=1590.0, bf16_sus=1400.0, source="fallback")


def load_traffic(config: str):
    """DRAM bytes (read + write) per launch of the dominant kernel from a
    committed ncu capture of this workload, or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            entry = json.load(f).get(config)
        return None if entry is None else float(entry["bytes"])
    except Exception:
        return None


class ClockSampler:
    """Samples the SM clock and the clock-event (throttle) reasons of one GPU
    every 10 ms through NVML on a background thread (nvidia-smi at 200 ms if
    NVML is unavailable); `stop(t0, t1)` summarises the samples taken between
    two host timestamps, the timed region."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.samples = []  # (host time, sm MHz, max sm MHz, [reasons])
        self.thread = None
        self.proc = None
        self.file = None
        self.stop_flag = False

    def start(self):
        import threading

        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda._get_nvml_device_index(self.dev))
            smax = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            masks = [(n, int(getattr(pynvml, attr))) for n, attr in self.REASONS]

            def run():
                while not self.stop_flag:
                    try:
                        sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                        bits = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
                        self.samples.append((time.time(), sm, smax, [n for n, b in masks if bits & b]))
                    except Exception:
                        pass
                    time.sleep(0.01)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.dev)], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def _smi_rows(self):
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.strip()]
        self.file.close()
        os.unlink(self.file.name)
        out = []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                out.append((None, float(r[1]), float(r[2]),
                            [n for n, v in zip(names, r[6:10]) if v.strip().lower() == "active"]))
            except (ValueError, IndexError):
                continue
        return out

    def stop(self, t0=None, t1=None):
        if self.thread is not None:
            self.stop_flag = True
            self.thread.join(timeout=5)
            rows, source = self.samples, "nvml 10 ms"
            if t0 is not None and t1 is not None:
                inside = [r for r in rows if t0 <= r[0] <= t1]
                rows = inside or [r for r in rows if r[0] >= t0][:1]
        elif self.proc is not None:
            rows, source = self._smi_rows(), "nvidia-smi 200 ms"
        else:
            return None
        if not rows:
            return None
        reasons = sorted({n for r in rows for n in r[3]})
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": max(r[2] for r in rows),
                "reasons": reasons, "samples": len(rows), "sampler": source}


# --------------------------------------------------------------------------- inputs


def make_routing(name: str, T: int, E: int, k: int, seed: int):
    """Seeded synthetic routing of a workload: (topk_ids int32 [T, k],
    topk_weights fp32 [T, k]).
      uniform-softmax / sigmoid: logits ~ N(0, 1), the k largest (ties to the
        lower id), softmax / sigmoid scores renormalised over the k
      zipf1.2: k distinct experts per token drawn from a Zipf(1.2) popularity
        over a seeded permutation of the ids; weights softmax of N(0, 1)
      hot25-zipf1.0: Zipf(1.0), then a quarter of the tokens (seeded) forced
        to also route to one hot expert (it replaces their last choice)
    The CPU-baseline leg builds the same inputs (a test checks they agree)."""
    rng = np.random.default_rng(seed)
    if name in ("uniform-softmax", "sigmoid"):
        lg = rng.standard_normal((T, E), dtype=np.float32)
        ids = np.argsort(-lg, axis=1, kind="stable")[:, :k]
        top = np.take_along_axis(lg, ids, axis=1)
        if name == "uniform-softmax":
            sc = np.exp(top - lg.max(axis=1, keepdims=True)).astype(np.float32)
        else:
            sc = (np.float32(1.0) / (np.float32(1.0) + np.exp(-top))).astype(np.float32)
        return ids.astype(np.int32), (sc / sc.sum(axis=1, keepdims=True)).astype(np.float32)
    if name in ("zipf1.2", "hot25-zipf1.0"):
        s = 1.2 if name == "zipf1.2" else 1.0
        p = np.arange(1, E + 1, dtype=np.float64) ** (-s)
        p /= p.sum()
        perm = rng.permutation(E)
        ids = np.empty((T, k), np.int32)
        for t in range(T):
            ids[t] = perm[rng.choice(E, size=k, replace=False, p=p)]
        if name == "hot25-zipf1.0":
            hot = int(rng.integers(E))
            for t in rng.choice(T, size=T // 4, replace=False):
                if hot not in ids[t]:
                    ids[t, k - 1] = hot
        lg = rng.standard_normal((T, k), dtype=np.float32)
        w = np.exp(lg - lg.max(axis=1, keepdims=True))
        return ids, (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    raise ValueError(name)


def make_inputs(cfg, rank: int, device, variant: int = 0):
    import torch

    T, H, I, E, k = cfg["T"], cfg["H"], cfg["I"], cfg["E"], cfg["k"]
    dt = {"bf16": torch.bfloat16, "fp32": torch.float32, "fp16": torch.float16}[cfg["dtype"]]
    g = torch.Generator(device=device).manual_seed(1234 + rank + 7919 * variant)
    x = torch.randn(T, H, device=device, generator=g).to(dt)
    ids, wts = make_routing(cfg["routing"], T, E, k, seed=rank + 7919 * variant)
    return x, torch.from_numpy(ids).to(device), torch.from_numpy(wts).to(device), dt


def make_weights(cfg, experts, device, dt):
    """Weights of the given experts, logical (E, K, N) views over K-major storage."""
    import torch

    import mail_b200 as mb

    H, I = cfg["H"], cfg["I"]
    g = torch.Generator(device=device).manual_seed(99)
    w13 = torch.empty(len(experts), 2 * I, H, device=device, dtype=dt)
    w2 = torch.empty(len(experts), H, I, device=device, dtype=dt)
    for i, e in enumerate(experts):
        g.manual_seed(1000 + e)
        w13[i] = (torch.randn(2 * I, H, device=device, generator=g) * 0.02).to(dt)
        w2[i] = (torch.randn(H, I, device=device, generator=g) * 0.02).to(dt)
    w13, w2 = w13.transpose(1, 2), w2.transpose(1, 2)
    scales = None
    if cfg["quant"]:
        w13, w2, scales = mb.quantize_weights_int8(w13, w2)
    return w13, w2, scales


# --------------------------------------------------------------------------- reference arm / cpu baseline


def cpu_reference_run(cfg, steps: int, warmup: int, time_limit_s: float = 20.0):
    """Times the oracle port of the reference's torch MoE path (per-expert fp32
    loop, fixed_kernel.py:232-249, extended with the top-k combine) on the
    host cores over a bounded token sample of the workload: the sample size is
    chosen from a quick sgemm calibration so one step takes about
    time_limit_s / steps seconds, and only the experts the sample touches get
    (host-generated) weights."""
    try:
        from threadpoolctl import threadpool_info
        threads = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        threads = os.cpu_count() or 1

    from oracle import moe_oracle as O

    T, H, I, E, k = cfg["T"], cfg["H"], cfg["I"], cfg["E"], cfg["k"]
    rng = np.random.default_rng(0)
    a = rng.standard_normal((256, H), dtype=np.float32)
    b = rng.standard_normal((H, 2048), dtype=np.float32)
    a @ b
    t0 = time.perf_counter()
    for _ in range(3):
        a @ b
    gflops = 3 * 2 * 256 * H * 2048 / (time.perf_counter() - t0) / 1e9
    per_step = max(time_limit_s / max(steps + warmup, 1), 0.25)
    flops_per_token = 6.0 * k * H * I
    n = int(max(1, min(T, per_step * gflops * 1e9 / flops_per_token)))
    ids_all, wts_all = O.synthetic_routing(cfg["routing"], T, E, k, seed=0)
    ids, wts = ids_all[:n], wts_all[:n]
    x = rng.standard_normal((n, H), dtype=np.float32)
    touched = sorted(set(int(e) for e in ids.reshape(-1) if 0 <= e < E))

    class Shared:
        """E experts whose weights alternate between `nw` host arrays: one
        expert's weights (H x 3I floats) exceed any host cache, so the
        per-expert loop still streams every expert's weights from DRAM, while
        the host materialises only nw of them."""

        def __init__(self, arrays, n):
            self.arrays, self.shape = arrays, (n,) + arrays[0].shape

        def __getitem__(self, e):
            return self.arrays[e % len(self.arrays)]

    nw = 2
    w13 = [rng.standard_normal((H, 2 * I), dtype=np.float32) * np.float32(0.02) for _ in range(nw)]
    w2 = [rng.standard_normal((I, H), dtype=np.float32) * np.float32(0.02) for _ in range(nw)]
    ids_l = ids
    if cfg["quant"]:
        q = [O.quantize_weight_per_channel(w.T) for w in w13]
        q2 = [O.quantize_weight_per_channel(w.T) for w in w2]
        q13, s13 = Shared([a for a, _ in q], E), Shared([b for _, b in q], E)
        q2, s2 = Shared([a for a, _ in q2], E), Shared([b for _, b in q2], E)
    w13, w2 = Shared(w13, E), Shared(w2, E)

    def run():
        t1 = time.perf_counter()
        if cfg["quant"]:
            O.moe_mlp_w8a8(x, q13, s13, q2, s2, wts, ids_l)
        else:
            O.moe_mlp_topk(x, w13, w2, wts, ids_l)
        return time.perf_counter() - t1

    for _ in range(warmup):
        run()
    times = [run() for _ in range(steps)]
    t = sum(times) / len(times)
    return dict(value=n / t, unit="tokens/s", cores=int(threads), tokens=n, seconds_per_step=t,
                sample=f"{n} of {T} tokens per step (same H/I/E/k and routing; {len(touched)} experts touched), "
                       f"{'w8a8 ' if cfg['quant'] else ''}fp32 numpy per-expert loop, {threads} BLAS threads")


# --------------------------------------------------------------------------- our arm: measurement helpers

DECODE_TOKENS = (1, 8, 32, 128, 256)
L2_BYTES = 126e6


def n_variants(cfg, T, world, rank):
    """Routings a step cycles through: when one step's active expert weights
    fit in the L2 (decode-sized batches), consecutive steps route to
    different experts so the weights stream from HBM as in serving."""
    wbytes = 1 if cfg["quant"] else (4 if cfg["dtype"] == "fp32" else 2)
    ids0, _ = make_routing(cfg["routing"], T, cfg["E"], cfg["k"], seed=rank)
    active_bytes = len(np.unique(ids0)) * 3 * cfg["H"] * cfg["I"] * wbytes
    if world > 1 or active_bytes >= 2 * L2_BYTES:
        return 1, "active weights of one step (%.2f GB) exceed the 126 MB L2, streamed every step" % (
            active_bytes / 1e9)
    n = int(min(16, -(-3 * L2_BYTES // active_bytes)))
    return n, ("active weights of one step (%.0f MB) fit in the 126 MB L2: steps cycle through %d routings "
               "touching different experts" % (active_bytes / 1e6, n))


class Ctx:
    """Per-process handles the measurement helpers share."""

    def __init__(self, torch, dist, lib, device, local_rank, world, rank):
        self.torch, self.dist, self.lib = torch, dist, lib
        self.device, self.local_rank, self.world, self.rank = device, local_rank, world, rank
        self.stream = torch.cuda.current_stream(device)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier(device_ids=[self.local_rank])

    def max_over_ranks(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], device=self.device, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def kernel_clocks(self, reset=True):
        """(total_ns, launches) per kernel class since the last reset."""
        from mail_b200 import _lib
        tot = (ctypes.c_uint64 * _lib.NUM_CLOCKS)()
        cnt = (ctypes.c_uint64 * _lib.NUM_CLOCKS)()
        _lib.call("moe_kernel_clocks", tot, cnt, _lib.NUM_CLOCKS, int(reset), self.stream.cuda_stream)
        return list(tot), list(cnt)


def run_steps(w, n):
    """Runs steps 0 .. n-1 of a workload: from its chained graph (several
    consecutive steps per replay) where one fits, else one step at a time."""
    chain, G = w.get("chain"), w.get("chain_steps", 1)
    i = 0
    while i < n:
        if chain is not None and n - i >= G:
            chain.replay()
            i += G
        else:
            w["step"](*w["inp"](i))
            i += 1


def timed_region(ctx, w, steps, kernels_per_step=None, sample_clocks=True):
    """Times exactly `steps` steps of workload w on the device (CUDA events
    on the launching stream, barrier + synchronize on both sides, max over
    ranks), with NVML clocks sampled during the region and the library's
    kernel clocks read over it."""
    torch, lib = ctx.torch, ctx.lib
    sampler = ClockSampler(ctx.local_rank) if sample_clocks else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    ctx.barrier()
    torch.cuda.synchronize()
    ctx.kernel_clocks(reset=True)
    launches0 = lib.moe_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    e0.record(ctx.stream)
    run_steps(w, steps)
    e1.record(ctx.stream)
    torch.cuda.synchronize()
    t1 = time.time()
    ctx.barrier()
    clocks = sampler.stop(t0, t1) if sampler else None
    launches = lib.moe_launch_count() - launches0
    if kernels_per_step is not None:  # graph replays bypass the library's launch counter
        launches = kernels_per_step * steps
    tot, cnt = ctx.kernel_clocks(reset=True)
    ms = ctx.max_over_ranks(e0.elapsed_time(e1) / steps)
    kc = {}
    for name, i in (("gate_up", 0), ("down", 1)):
        per = tot[i] / cnt[i] / 1e6 if cnt[i] else float("nan")
        kc[name] = {"ms_per_launch": ctx.max_over_ranks(per), "launches": int(cnt[i])}
    return {"ms": ms, "seconds": t1 - t0, "clocks": clocks, "launches": int(launches), "kernel_clocks": kc}


def int8_yardstick(ctx):
    """Measured int8 tensor-core yardstick: torch._int_mm (cuBLASLt int8 x
    int8 -> int32) on 8192^3, best of 10 launches after 3 warm-ups; None if
    the build lacks it."""
    torch = ctx.torch
    n = 8192
    try:
        a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=ctx.device)
        b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=ctx.device).t().contiguous().t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(ctx.stream)
            torch._int_mm(a, b)
            e1.record(ctx.stream)
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b
        return {"tops": 2.0 * n ** 3 / (best / 1e3) / 1e12, "ms": best,
                "how": "torch._int_mm int8 %d^3 (cuBLASLt, int32 out), best of 10" % n}
    except Exception as exc:  # pragma: no cover - depends on the torch build
        return {"tops": None, "error": str(exc)[:200]}


def one_launch(kernel_clocks):
    """True when the step ran as the one-launch decode kernel: its clock is
    the gate_up class and no down GEMM launched."""
    return kernel_clocks["down"]["launches"] == 0 and kernel_clocks["gate_up"]["launches"] > 0


def gate_up_roofline(cfg, T, world, id_sets, gemm1_ms, peaks, int8, sustained, whole_layer=False):
    """Algorithmic work of one gate_up launch and its achieved rate: FLOPs
    2 * S * H * 2I (S routed slots), bytes = w13 of the experts with slots +
    the padded activation rows read + the h rows written; bound = the larger
    of FLOPs / tensor peak and bytes / HBM peak (the measured peaks).
    whole_layer: the launch is the one-launch decode kernel, whose work is the
    whole layer: w13 + w2 of the active experts, x read, y written."""
    H, I, E, k = cfg["H"], cfg["I"], cfg["E"], cfg["k"]
    wb = 1 if cfg["quant"] else (4 if cfg["dtype"] == "fp32" else 2)
    hb = 4 if cfg["dtype"] == "fp32" else 2
    S = T * k
    if world == 1:
        acts, rows = [], []
        for ids in id_sets:
            counts = np.bincount(ids.reshape(-1), minlength=E)
            acts.append(int((counts > 0).sum()))
            rows.append(int(((counts + 127) // 128 * 128).sum()))
        active, rows_pad = float(np.mean(acts)), float(np.mean(rows))
    else:  # this rank's experts under balanced routing
        active = E // world
        rows_pad = S + active * 64
    flops = 2.0 * S * H * 2 * I
    nbytes = active * 2.0 * I * H * wb + rows_pad * H * wb + rows_pad * I * hb
    if whole_layer:
        flops = 2.0 * S * H * 3 * I
        nbytes = active * 3.0 * I * H * wb + 2.0 * T * H * hb
    if cfg["quant"]:
        if int8 and int8.get("tops"):
            tc_peak, tc_src = int8["tops"], "measured int8 GEMM (%s)" % int8["how"]
        else:
            tc_peak, tc_src = 2.0 * peaks["bf16"], "2 x measured bf16 (no int8 yardstick)"
    else:
        tc_peak = peaks["bf16_sus"] if sustained else peaks["bf16"]
        tc_src = "%s bf16 %s" % (peaks["source"], "sustained" if sustained else "burst")
    s = gemm1_ms / 1e3
    tensor_rate, hbm_rate = flops / s / 1e12, nbytes / s / 1e9
    tensor_bound = flops / (tc_peak * 1e12) >= nbytes / (peaks["hbm"] * 1e9)
    kname = ("moe_decode_kernel (whole layer: routing, gate_up + SwiGLU, down + combine)" if whole_layer
             else "moe_gemm_kernel<SWIGLU> (gate_up GEMM + SwiGLU)")
    r = {"kernel": kname, "bound": "tensor" if tensor_bound else "hbm",
         "flops_per_launch": flops, "bytes_per_launch": nbytes, "active_experts": active,
         "ms_per_launch": gemm1_ms, "frac_tensor": tensor_rate / tc_peak, "frac_hbm": hbm_rate / peaks["hbm"]}
    if tensor_bound:
        r.update(achieved=tensor_rate, peak=tc_peak, unit="TOP/s" if cfg["quant"] else "TFLOP/s",
                 frac=tensor_rate / tc_peak, peak_source=tc_src)
        spec = 4500.0 if cfg["quant"] else 2250.0
    else:
        r.update(achieved=hbm_rate, peak=peaks["hbm"], unit="GB/s", frac=hbm_rate / peaks["hbm"],
                 peak_source=f"{peaks['source']} HBM copy")
        spec = 7700.0
    r.update(spec_peak=spec, frac_of_spec=r["achieved"] / spec)
    return r


def build_single(ctx, cfg, T, n_var, graph, weights=None):
    """One-GPU workload: inputs (n_var routings), weights, and a step that
    replays the op from a CUDA graph (or calls it)."""
    import mail_b200 as mb

    torch, device = ctx.torch, ctx.device
    x, ids, wts, dt = make_inputs(cfg, ctx.rank, device)
    variants = [(x, ids, wts)] + [make_inputs(cfg, ctx.rank, device, v)[:3] for v in range(1, n_var)]
    if weights is None:
        weights = make_weights(cfg, list(range(cfg["E"])), device, dt)
    w13, w2, scales = weights
    kernels = None
    if cfg.get("prerouted"):
        order = torch.argsort(ids.reshape(-1).to(torch.int64), stable=True)
        xg = x[order // cfg["k"]].contiguous()  # T * k rows grouped by expert
        gs = torch.bincount(ids.reshape(-1).to(torch.int64), minlength=cfg["E"])
        variants = [(xg, ids, wts)]

        def step(xx, ii, ww):
            return mb.fused_moe_mlp(xx, w13, w2, gs)
        captured = None
    elif graph:
        # one graph per set of input buffers, bound to them (a replay reads the
        # resident inputs, no copies); the end-to-end pass's buffers get theirs
        # on first use, in its warm-up
        graphs = {}

        def graph_for(xx, ii, ww):
            key = (xx.data_ptr(), ii.data_ptr(), ww.data_ptr())
            if key not in graphs:
                graphs[key] = mb.CapturedMoeMLP(w13, w2, T, cfg["k"], dtype=dt, scales=scales, inputs=(xx, ww, ii))
            return graphs[key]

        for v in variants:
            captured = graph_for(*v)
        kernels = captured.kernels

        def step(xx, ii, ww):
            return graph_for(xx, ii, ww)(xx, ww, ii)

        if T <= 512:
            # decode-sized steps take microseconds, as long as a graph launch:
            # chain several consecutive steps (cycling the routings) in one
            # graph, as a model's decode graph holds consecutive layers
            G = len(variants) * -(-8 // len(variants))
            chain = ctx.torch.cuda.CUDAGraph()
            with ctx.torch.cuda.graph(chain):
                for j in range(G):
                    xx, ii, ww = variants[j % len(variants)]
                    mb.fused_moe_mlp(xx, w13, w2, ww, ii, scales=scales)
            extra = dict(chain=chain, chain_steps=G)
        else:
            extra = {}
    else:
        captured = None

        def step(xx, ii, ww):
            return mb.fused_moe_mlp(xx, w13, w2, ww, ii, scales=scales)
    out = dict(step=step, variants=variants, weights=weights, captured=captured, kernels=kernels, dt=dt,
               inp=lambda i: variants[i % len(variants)])
    if graph and not cfg.get("prerouted"):
        out.update(extra)
    return out


def build_ep(ctx, cfg, T, ep_kind, replicate=False):
    """Expert-parallel workload on this rank: its E / N experts, T tokens.
    replicate: also hold the replicas mail_b200.ep.plan_replicas picks from
    every rank's slot counts of this routing (at most E / N of them)."""
    import mail_b200 as mb
    from mail_b200 import ep as mep

    E, world, rank = cfg["E"], ctx.world, ctx.rank
    assert E % world == 0, "experts must divide evenly over ranks"
    x, ids, wts, dt = make_inputs(cfg, rank, ctx.device)
    local = list(range(rank * E // world, (rank + 1) * E // world))
    w13, w2, scales = make_weights(cfg, local, ctx.device, dt)
    replicas, rep = None, []
    if replicate:
        counts = ctx.torch.empty((world, E), dtype=ctx.torch.int32, device=ctx.device)
        ctx.dist.all_gather_into_tensor(counts, mb.moe_align(ids, E, block_m=1)["group_sizes"])
        rep = mep.plan_replicas(counts, E // world)
        if rep:
            r13, r2, rsc = make_weights(cfg, rep, ctx.device, dt)
            replicas = (rep, r13, r2, rsc)
    if ep_kind == "peer":
        layer = mep.PeerExpertParallelMoE(w13, w2, E, max_tokens=T, top_k=cfg["k"], dtype=dt, scales=scales,
                                          replicas=replicas)
    else:
        layer = mep.ExpertParallelMoE(w13, w2, E, scales=scales, replicas=replicas)

    def step(xx, ii, ww):
        return layer(xx, ww, ii)
    variants = [(x, ids, wts)]
    return dict(step=step, variants=variants, weights=(w13, w2, scales), layer=layer, kernels=None, dt=dt,
                captured=None, inp=lambda i: variants[0], replicas=rep)


def close_workload(ctx, w):
    layer = w.get("layer")
    if layer is not None and hasattr(layer, "close"):
        layer.close()
    w.clear()
    ctx.torch.cuda.synchronize()
    ctx.torch.cuda.empty_cache()


def run_config(ctx, name, T, args, peaks, int8, weights=None, steps=None, warmup=3, ep_kind="peer",
               replicate=False):
    """A sub-configuration of the line: build, warm up, time, roofline."""
    cfg = dict(CONFIGS[name])
    cfg["T"] = T
    steps = steps or args.steps
    if ctx.world > 1:
        w = build_ep(ctx, cfg, T, ep_kind, replicate=replicate)
        n_var, l2 = 1, "expert-parallel, weights streamed every step"
    else:
        n_var, l2 = n_variants(cfg, T, 1, ctx.rank)
        w = build_single(ctx, cfg, T, n_var, graph=True, weights=weights)
    run_steps(w, max(warmup, w.get("chain_steps", 1)))
    ctx.torch.cuda.synchronize()
    r = timed_region(ctx, w, steps, kernels_per_step=w["kernels"])
    ids_sets = [v[1].cpu().numpy() for v in w["variants"]]
    roof = gate_up_roofline(cfg, T, ctx.world, ids_sets, r["kernel_clocks"]["gate_up"]["ms_per_launch"], peaks,
                            int8, sustained=False, whole_layer=one_launch(r["kernel_clocks"]))
    out = {"workload": cfg["desc"].split(" (")[0] + f" T={T}" + ("" if ctx.world == 1 else f" per GPU x {ctx.world}"),
           "tokens_per_gpu": T, "hidden": cfg["H"], "inter": cfg["I"], "experts": cfg["E"], "top_k": cfg["k"],
           "routing": cfg["routing"], "dtype": cfg["dtype"] + ("+w8a8" if cfg["quant"] else ""),
           "value": ctx.world * T / (r["ms"] / 1e3), "unit": "tokens/s", "ms_per_step": r["ms"], "steps": steps,
           "kernel_clocks": r["kernel_clocks"], "roofline": roof, "clocks": r["clocks"], "l2": l2,
           "graph_steps": w.get("chain_steps", 1)}
    if ctx.world > 1:
        out["replicated_experts"] = w.get("replicas", [])
    if ctx.world == 1:
        # the step's own weight-streaming bound: every active expert's three
        # matrices once at the measured copy rate
        wb = 1 if cfg["quant"] else 2
        bound_ms = roof["active_experts"] * 3.0 * cfg["H"] * cfg["I"] * wb / (peaks["hbm"] * 1e9) * 1e3
        out["weight_stream_bound_ms"] = bound_ms
    keep = w.get("weights") if weights is not None else None
    close_workload(ctx, w)
    return out, keep


def decode_from_logits(ctx, weights, T, ids_ms):
    """The Qwen3 decode step called with the router logits
    (fused_moe_mlp_from_logits: routing is phase 0 of the one-launch kernel).
    Each step's logits rank its seeded routing's k experts first, so the
    experts, rows and weight bytes equal the ids-given step's (ids_ms), and
    steps chain in one graph the same way."""
    import mail_b200 as mb

    torch = ctx.torch
    cfg = dict(CONFIGS["qwen3-decode"])
    cfg["T"] = T
    E, k = cfg["E"], cfg["k"]
    w13, w2, _ = weights
    n_var, _ = n_variants(cfg, T, 1, ctx.rank)
    variants = []
    for v in range(n_var):
        x, ids, _, _ = make_inputs(cfg, ctx.rank, ctx.device, v)
        lg = torch.randn(T, E, device=ctx.device) - 20.0
        lg.scatter_(1, ids.long(), (10.0 - torch.arange(k, device=ctx.device, dtype=torch.float32)).expand(T, k))
        variants.append((x, lg, ids))
    same = True
    for x, lg, ids in variants:  # warm-up, and a check that the routing is the seeded one
        _, _, got = mb.fused_moe_mlp_from_logits(x, w13, w2, lg, k)
        same = same and bool(torch.equal(got, ids))
    G = n_var * -(-8 // n_var)
    steps = G * -(-200 // G)

    def chained(fused):
        chain = torch.cuda.CUDAGraph()
        with torch.cuda.graph(chain):
            for j in range(G):
                x, lg, _ = variants[j % n_var]
                if fused:
                    mb.fused_moe_mlp_from_logits(x, w13, w2, lg, k)
                else:  # the router's own launch, then the layer
                    ids, wts = mb.route_topk(lg, k)
                    mb.fused_moe_mlp(x, w13, w2, wts, ids)
        w = dict(chain=chain, chain_steps=G)
        run_steps(w, 3 * G)
        torch.cuda.synchronize()
        r = timed_region(ctx, w, steps, kernels_per_step=1 if fused else 2)
        del w, chain
        return r

    r = chained(True)
    r2 = chained(False)
    out = {"workload": f"Qwen3-30B-A3B decode T={T}, router logits in (routing fused into the one-launch kernel)",
           "value": T / (r["ms"] / 1e3), "unit": "tokens/s", "ms_per_step": r["ms"], "steps": steps,
           "launches_per_step": 1, "router_then_layer_ms_per_step": r2["ms"], "ids_given_ms_per_step": ids_ms,
           "routing_reproduced": same,
           "clocks": r["clocks"], "graph_steps": G}
    del variants
    torch.cuda.synchronize()
    return out


def router_timing(ctx, peaks):
    """The GPU router (route_topk) on the routing inputs of the DeepSeek-V3
    (8192 x 256 fp32 logits, sigmoid top-8) and stress (65536 x 64, softmax
    top-6) workloads: CUDA events around one replay of a graph of 20
    launches; algorithmic bytes = logits read + ids and weights written."""
    import mail_b200 as mb

    torch = ctx.torch
    out = {}
    for name, T, E, k, scoring in (("dsv3", 8192, 256, 8, "sigmoid"), ("stress", 65536, 64, 6, "softmax")):
        # enough logits buffers, cycled, to exceed twice the L2: every launch
        # reads its logits from HBM
        nb = int(math.ceil(2 * L2_BYTES / (T * E * 4)))
        lgs = [torch.randn(T, E, device=ctx.device) for _ in range(nb)]
        for i in range(3):
            mb.route_topk(lgs[i % nb], k, scoring=scoring)
        torch.cuda.synchronize()
        # one graph of 20 launches (one per buffer in turn), so the host's
        # per-call cost is not what is timed
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(20):
                mb.route_topk(lgs[(3 + i) % nb], k, scoring=scoring)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ctx.stream)
        g.replay()
        e1.record(ctx.stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / 20
        del g
        nbytes = T * E * 4 + T * k * 8
        gbs = nbytes / (ms / 1e3) / 1e9
        out[name] = {"tokens": T, "experts": E, "top_k": k, "scoring": scoring, "us_per_launch": ms * 1e3,
                     "bytes": nbytes, "achieved_gbs": gbs, "frac_hbm": gbs / peaks["hbm"],
                     "l2": f"{nb} logits buffers cycled ({nb * T * E * 4 / 1e6:.0f} MB, over twice the L2)"}
        del lgs
    return out


def sub_configs(ctx, args, peaks, int8):
    """The workloads beside the headline, at their own shapes."""
    res = {}
    if ctx.world == 1:
        cfg = dict(CONFIGS["qwen3-decode"])
        weights = None
        for T in DECODE_TOKENS:
            cfg["T"] = T
            steps = max(args.steps, 200)
            if weights is None:
                dt = {"bf16": ctx.torch.bfloat16}[cfg["dtype"]]
                weights = make_weights(cfg, list(range(cfg["E"])), ctx.device, dt)
            res[f"qwen3-decode-T{T}"], _ = run_config(ctx, "qwen3-decode", T, args, peaks, int8, weights=weights,
                                                      steps=steps)
        for T in (1, 8):
            res[f"qwen3-decode-T{T}-from-logits"] = decode_from_logits(ctx, weights, T,
                                                                       res[f"qwen3-decode-T{T}"]["ms_per_step"])
        del weights
        ctx.torch.cuda.empty_cache()
        res["dsv3-w8a8"], _ = run_config(ctx, "dsv3-w8a8", 8192, args, peaks, int8)
        res["stress-w8a8"], _ = run_config(ctx, "stress-w8a8", 65536, args, peaks, int8, steps=max(5, args.steps // 2))
        res["router"] = router_timing(ctx, peaks)
    else:
        res["dsv3-w8a8"], _ = run_config(ctx, "dsv3-w8a8", 8192, args, peaks, int8, ep_kind=args.ep)
        res["dsv3-w8a8"]["scaling"] = "weak"
        Ts = 8192 // ctx.world
        res["dsv3-w8a8-strong"], _ = run_config(ctx, "dsv3-w8a8", Ts, args, peaks, int8, ep_kind=args.ep)
        res["dsv3-w8a8-strong"].update(scaling="strong", tokens_total=8192)
        # load-imbalance stress: expert-parallel as is, then with the replicas
        # plan_replicas picks from the all-gathered slot counts
        st_steps = max(5, args.steps // 2)
        res["stress-w8a8"], _ = run_config(ctx, "stress-w8a8", 65536, args, peaks, int8, steps=st_steps,
                                           ep_kind=args.ep)
        res["stress-w8a8"]["scaling"] = "weak"
        res["stress-w8a8-replicated"], _ = run_config(ctx, "stress-w8a8", 65536, args, peaks, int8, steps=st_steps,
                                                      ep_kind=args.ep, replicate=True)
        res["stress-w8a8-replicated"]["scaling"] = "weak"
    return res


def e2e_pass(ctx, w, steps):
    """End to end through the public API: every step copies its inputs from
    pinned host memory and its result back to pinned host memory, on their
    own streams with two device buffers, so step i+1's upload and step i-1's
    download overlap step i's compute, as a serving loop would run them."""
    torch = ctx.torch
    stream = ctx.stream
    step, variants = w["step"], w["variants"]
    n_var = len(variants)
    host_in = [tuple(t.cpu().pin_memory() for t in v) for v in variants]
    x_h, ids_h, wts_h = host_in[0]
    NB = 2
    x0, ids0, wts0 = variants[0]
    out_shape = tuple(step(x0, ids0, wts0).shape)
    y_h = [torch.empty(out_shape, dtype=w["dt"]).pin_memory() for _ in range(NB)]
    x_d = [torch.empty_like(x0) for _ in range(NB)]
    ids_d = [torch.empty_like(ids0) for _ in range(NB)]
    wts_d = [torch.empty_like(wts0) for _ in range(NB)]
    up, down = torch.cuda.Stream(ctx.device), torch.cuda.Stream(ctx.device)
    h2d_ev = [torch.cuda.Event() for _ in range(NB)]
    comp_ev = [torch.cuda.Event() for _ in range(NB)]
    d2h_buf_ev = [torch.cuda.Event() for _ in range(NB)]  # result of buffer b copied out
    d2h_ev = torch.cuda.Event()

    def e2e_step(i):
        b = i % NB
        with torch.cuda.stream(up):
            if i >= NB:
                up.wait_event(comp_ev[b])  # step i-NB has finished reading buffer b
            xh, ih, wh = host_in[i % n_var]
            x_d[b].copy_(xh, non_blocking=True)
            ids_d[b].copy_(ih, non_blocking=True)
            wts_d[b].copy_(wh, non_blocking=True)
            h2d_ev[b].record(up)
        stream.wait_event(h2d_ev[b])
        if i >= NB:
            stream.wait_event(d2h_buf_ev[b])  # a replay rewrites the output step i-NB's copy reads
        y = step(x_d[b], ids_d[b], wts_d[b])
        comp_ev[b].record(stream)
        with torch.cuda.stream(down):
            down.wait_event(comp_ev[b])
            y.record_stream(down)
            y_h[b].copy_(y, non_blocking=True)
            d2h_buf_ev[b].record(down)
            d2h_ev.record(down)

    for i in range(2 * NB):
        e2e_step(i)
    torch.cuda.synchronize()
    ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up.wait_event(e0)
    for i in range(steps):
        e2e_step(i)
    stream.wait_event(d2h_ev)  # the last result is back in host memory
    e1.record(stream)
    torch.cuda.synchronize()
    ms = ctx.max_over_ranks(e0.elapsed_time(e1) / steps)
    h2d = x_h.numel() * x_h.element_size() + ids_h.numel() * 4 + wts_h.numel() * 4
    d2h = y_h[0].numel() * y_h[0].element_size()
    return ms, int(h2d), int(d2h)


def stage_events_pass(ctx, w, cfg, T, steps):
    """CUDA-event stage times (cross-check of the kernel clocks): a second
    capture of the same op with the library's stage events as graph nodes,
    replayed once per step (these nodes break the launch overlap between
    stages, so the figures are slightly pessimistic)."""
    import mail_b200 as mb

    torch, lib = ctx.torch, ctx.lib
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(STAGES)]
    for e in ev:
        e.record(ctx.stream)
    torch.cuda.synchronize()
    arr = (ctypes.c_void_p * STAGES)(*[e.cuda_event for e in ev])
    w13, w2, scales = w["weights"]
    lib.moe_set_stage_events(arr, STAGES)
    try:
        cap = mb.CapturedMoeMLP(w13, w2, T, cfg["k"], dtype=w["dt"], scales=scales)
    finally:
        lib.moe_set_stage_events(None, 0)
    rows = []
    for i in range(steps):
        xv, iv, wv = w["inp"](i)
        cap(xv, wv, iv)
        torch.cuda.synchronize()
        rows.append([ev[j].elapsed_time(ev[j + 1]) for j in range(STAGES - 1)])
    del cap

    def mean(a, b):
        return statistics.mean(sum(r[a:b]) for r in rows)

    return {"route": mean(0, 1), "gather": mean(1, 2), "gemm1": mean(2, 3), "pre_gemm2": mean(3, 4),
            "gemm2": mean(4, 5), "finalize": mean(5, 6),
            "source": "CUDA events as graph nodes, separate replay after the timed region"}


def cublas_yardsticks(ctx, cfg, S, gemm1_ms, steps):
    """cuBLAS (torch.matmul / torch.bmm) on the gate_up launch's FLOPs, timed
    the same way: one dense GEMM [S, H] x [H, 2I], and a batched GEMM with
    one weight matrix per expert and S / E rows each."""
    torch = ctx.torch
    H, I, E = cfg["H"], cfg["I"], cfg["E"]
    dt = torch.bfloat16
    flops = 2.0 * S * H * 2 * I

    def time_fn(fn):
        for _ in range(3):
            fn()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(3, steps)
        c0.record(ctx.stream)
        for _ in range(reps):
            fn()
        c1.record(ctx.stream)
        torch.cuda.synchronize()
        return c0.elapsed_time(c1) / reps

    out = {}
    a = torch.randn(S, H, device=ctx.device, dtype=dt)
    b = torch.randn(H, 2 * I, device=ctx.device, dtype=dt)
    ms = time_fn(lambda: torch.matmul(a, b))
    out["cublas_dense_same_shape"] = {"ms": ms, "tflops": flops / (ms / 1e3) / 1e12, "ours_vs_cublas": ms / gemm1_ms}
    del a, b
    rows = S // E
    if rows >= 128 and E * H * 2 * I * 2 <= 8 << 30:
        a = torch.randn(E, rows, H, device=ctx.device, dtype=dt)
        b = torch.randn(E, H, 2 * I, device=ctx.device, dtype=dt)
        ms = time_fn(lambda: torch.bmm(a, b))
        bflops = 2.0 * E * rows * H * 2 * I
        out["cublas_batched_per_expert"] = {"shape": f"{E} x [{rows}, {H}] x [{H}, {2 * I}]", "ms": ms,
                                            "tflops": bflops / (ms / 1e3) / 1e12,
                                            "ours_vs_cublas": (flops / gemm1_ms) / (bflops / ms)}
        del a, b
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="mixtral", choices=sorted(CONFIGS))
    ap.add_argument("--tokens", type=int, default=0, help="override tokens per GPU (profiling cases)")
    ap.add_argument("--ep", default="peer", choices=["peer", "nccl"],
                    help="expert-parallel exchange (N > 1): fused into the kernels over NVLink peer memory, "
                         "or NCCL all-to-all")
    ap.add_argument("--gemm", default="auto", choices=["auto", "pair", "single"],
                    help="grouped GEMM variant: CTA pairs (cta_group::2), one CTA per tile, or chosen by size")
    ap.add_argument("--band", type=int, default=0, help="GEMM tile-order band width in M tiles (0: default)")
    ap.add_argument("--band-down", type=int, default=0,
                    help="the down GEMM's band width in M tiles (0: the --band value)")
    ap.add_argument("--pdl", type=int, default=1, choices=[0, 1],
                    help="launch the kernels with programmatic dependent launch (1, default)")
    ap.add_argument("--half-units", type=int, default=1, choices=[0, 1],
                    help="CTA-pair GEMMs: each expert's odd last M tile as an M=128 pair MMA (1, default)")
    ap.add_argument("--swap", default="auto", choices=["auto", "on", "off"],
                    help="grouped GEMM operand roles: weights as the MMA's 128-row operand for few rows per "
                         "expert (auto), always (on), never (off)")
    ap.add_argument("--eager", action="store_true",
                    help="N=1: call the op directly each step instead of replaying it from a captured CUDA graph")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the other workloads (the configs key)")
    ap.add_argument("--sustain-s", type=float, default=1.5,
                    help="seconds of back-to-back steps in the sustained pass (0: skip)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    args.graph = not args.eager
    cfg = dict(CONFIGS[args.config])
    if args.tokens:
        cfg["T"] = args.tokens
        cfg["desc"] += f" (T={args.tokens})"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    T, H, I, E, k = cfg["T"], cfg["H"], cfg["I"], cfg["E"], cfg["k"]
    dtype_name = "int8" if cfg["quant"] else cfg["dtype"]
    config_json = {"workload": cfg["desc"], "tokens_per_gpu": T, "hidden": H, "inter": I, "experts": E,
                   "top_k": k, "routing": cfg["routing"], "dtype": cfg["dtype"] + ("+w8a8" if cfg["quant"] else ""),
                   "parallelism": f"ep{world}" if world > 1 else "single", "gemm": args.gemm,
                   "half_units": bool(args.half_units), "pdl": bool(args.pdl),
                   "ep_exchange": args.ep if world > 1 else None, "cuda_graph": bool(args.graph and world == 1),
                   "swap_ab": args.swap}
    n_var, l2_note = n_variants(cfg, T, world, rank)
    config_json["l2"] = l2_note
    if world == 1 and args.graph and T <= 512 and not cfg.get("prerouted"):
        config_json["graph_steps"] = n_var * -(-8 // n_var)

    if args.impl == "reference":
        if rank != 0:
            return 0
        # the bound lets the Mixtral layer's whole 4096-token batch run every
        # step (about 2 s on 16 host threads), the sample the cpu_baseline leg
        # of the GPU arm times, so both report the same per-token rate
        ref = cpu_reference_run(cfg, args.steps, args.warmup, time_limit_s=100.0)
        line = {"metric": "fused MoE MLP tokens/s", "value": ref["value"], "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ref["seconds_per_step"] * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": config_json, "impl": "reference",
                "cpu_baseline": {"value": ref["value"], "unit": "tokens/s", "cores": ref["cores"], "kind": "port",
                                 "sample": ref["sample"]},
                "e2e": {"value": ref["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    import torch.distributed as dist

    from mail_b200 import _lib

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    lib = _lib.load()
    lib.moe_set_option(_lib.OPT_GEMM_CTA_PAIR, {"pair": 1, "single": 0, "auto": 2}[args.gemm])
    if args.band:
        lib.moe_set_option(_lib.OPT_GEMM_BAND, args.band)
    lib.moe_set_option(_lib.OPT_GEMM_BAND_DOWN, args.band_down)
    lib.moe_set_option(_lib.OPT_GEMM_HALF_UNITS, args.half_units)
    lib.moe_set_option(_lib.OPT_PDL, args.pdl)
    lib.moe_set_option(_lib.OPT_GEMM_SWAP_AB, {"auto": 2, "on": 1, "off": 0}[args.swap])
    lib.moe_set_option(_lib.OPT_KERNEL_CLOCKS, 1)  # before any capture: GEMM launches time themselves
    ctx = Ctx(torch, dist, lib, device, local_rank, world, rank)
    peaks = load_peaks()

    # ---- the headline workload
    if world > 1:
        w = build_ep(ctx, cfg, T, args.ep)
        args.graph = False
    else:
        w = build_single(ctx, cfg, T, n_var, graph=args.graph and not cfg.get("prerouted"))
    run_steps(w, max(args.warmup, w.get("chain_steps", 1)))
    torch.cuda.synchronize()
    reg = timed_region(ctx, w, args.steps, kernels_per_step=w["kernels"])
    ms = reg["ms"]
    gemm1_ms = reg["kernel_clocks"]["gate_up"]["ms_per_launch"]
    gemm2_ms = reg["kernel_clocks"]["down"]["ms_per_launch"]

    # ---- sustained: the same step back to back for >= sustain_s seconds
    sustained = None
    if args.sustain_s > 0:
        n_sus = max(args.steps, int(math.ceil(args.sustain_s * 1e3 / ms)))
        sreg = timed_region(ctx, w, n_sus, kernels_per_step=w["kernels"])
        sroof = gate_up_roofline(cfg, T, world, [v[1].cpu().numpy() for v in w["variants"]],
                                 sreg["kernel_clocks"]["gate_up"]["ms_per_launch"], peaks, None, sustained=True,
                                 whole_layer=one_launch(sreg["kernel_clocks"]))
        sustained = {"value": world * T / (sreg["ms"] / 1e3), "unit": "tokens/s", "ms_per_step": sreg["ms"],
                     "steps": n_sus, "seconds": sreg["seconds"], "clocks": sreg["clocks"],
                     "kernel_clocks": sreg["kernel_clocks"],
                     "roofline": {k2: sroof[k2] for k2 in ("achieved", "peak", "unit", "frac", "peak_source",
                                                           "ms_per_launch", "bound")}}

    # ---- CUDA-event stage times (cross-check), e2e through the public API
    stage = None
    if world == 1 and args.graph and not cfg.get("prerouted"):
        try:
            stage = stage_events_pass(ctx, w, cfg, T, args.steps)
        except Exception as exc:  # the cross-check is optional
            stage = {"error": str(exc)[:200]}
    e2e_ms, h2d, d2h = e2e_pass(ctx, w, args.steps)

    # ---- roofline of the dominant kernel (gate_up GEMM + SwiGLU)
    int8 = int8_yardstick(ctx) if (world == 1 and (cfg["quant"] or not args.no_configs)) else None
    id_sets = [v[1].cpu().numpy() for v in w["variants"]]
    region_s = ms * args.steps / 1e3
    roofline = gate_up_roofline(cfg, T, world, id_sets, gemm1_ms, peaks, int8, sustained=region_s >= 1.0,
                                whole_layer=one_launch(reg["kernel_clocks"]))
    roofline["ms_per_launch_source"] = ("library kernel clocks (device global timer, first CTA past its wait on "
                                        "the previous kernel to last CTA end) over the timed region, "
                                        f"{reg['kernel_clocks']['gate_up']['launches']} launches")
    roofline["down_ms_per_launch"] = gemm2_ms
    if stage and "gemm1" in stage:
        roofline["ms_per_launch_events"] = stage["gemm1"]
    roofline["traffic"] = load_traffic(args.config) if not args.tokens and world == 1 else None
    roofline["traffic_unit"] = "bytes"
    if (world == 1 and not cfg["quant"] and cfg["dtype"] == "bf16" and not cfg.get("prerouted")
            and not one_launch(reg["kernel_clocks"])):
        roofline.update(cublas_yardsticks(ctx, cfg, T * k, gemm1_ms, args.steps))
    flops_step = 6.0 * T * k * H * I
    peak_tc = roofline["peak"] if roofline["bound"] == "tensor" else peaks["bf16"]

    line = {"metric": "fused MoE MLP tokens/s", "value": world * T / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype_name,
            "data": "synthetic", "config": config_json,
            "tflops_per_gpu": flops_step / (ms / 1e3) / 1e12,
            "frac_of_tensor_peak": flops_step / (ms / 1e3) / 1e12 / peak_tc,
            "kernel_clocks": reg["kernel_clocks"], "stage_ms": stage, "roofline": roofline,
            "sustained": sustained,
            "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                    "copies": "pinned host memory, own H2D / D2H streams, double-buffered"},
            "gpu_launches": reg["launches"], "clocks": reg["clocks"]}
    if int8:
        line["int8_yardstick"] = int8
    close_workload(ctx, w)

    # ---- the other workloads
    if not args.no_configs and args.config == "mixtral" and not args.tokens:
        line["configs"] = sub_configs(ctx, args, peaks, int8)

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ref = cpu_reference_run(cfg, steps=3, warmup=1, time_limit_s=20.0)
        line["cpu_baseline"] = {"value": ref["value"], "unit": "tokens/s", "cores": ref["cores"], "kind": "port",
                                "sample": ref["sample"]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
