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
T tokens (weak scaling): experts are sharded E/N per rank and tokens travel
to their experts and back with NCCL all-to-all (mail_b200.ep).
"""
from __future__ import annotations

import argparse
import json
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


# --------------------------------------------------------------------------- our arm


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
    ap.add_argument("--pdl", type=int, default=1, choices=[0, 1],
                    help="launch the kernels with programmatic dependent launch (1, default)")
    ap.add_argument("--half-units", type=int, default=1, choices=[0, 1],
                    help="CTA-pair GEMMs: each expert's odd last M tile as an M=128 pair MMA (1, default)")
    ap.add_argument("--eager", action="store_true",
                    help="N=1: call the op directly each step instead of replaying it from a captured CUDA graph")
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
                   "ep_exchange": args.ep if world > 1 else None, "cuda_graph": bool(args.graph and world == 1)}

    # When one step's active expert weights fit in the L2 (decode-sized
    # batches), consecutive steps cycle through several routings that touch
    # different experts, so the weights stream from HBM as they would in
    # serving instead of being L2 hits of the previous step.
    L2_BYTES = 126e6
    wbytes = 1 if cfg["quant"] else (4 if cfg["dtype"] == "fp32" else 2)
    ids0, _ = make_routing(cfg["routing"], T, E, k, seed=rank)
    active_bytes = len(np.unique(ids0)) * 3 * H * I * wbytes
    n_var = 1 if world > 1 or active_bytes >= 2 * L2_BYTES else int(min(16, -(-3 * L2_BYTES // active_bytes)))
    if n_var > 1:
        config_json["l2"] = ("active weights of one step (%.0f MB) fit in the 126 MB L2: steps cycle through %d "
                             "routings touching different experts" % (active_bytes / 1e6, n_var))
    else:
        config_json["l2"] = "active weights of one step (%.2f GB) exceed the 126 MB L2, streamed every step" % (
            active_bytes / 1e9)

    if args.impl == "reference":
        if rank != 0:
            return 0
        ref = cpu_reference_run(cfg, args.steps, args.warmup)
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

    import mail_b200 as mb
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
    lib.moe_set_option(_lib.OPT_GEMM_HALF_UNITS, args.half_units)
    lib.moe_set_option(_lib.OPT_PDL, args.pdl)

    x, ids, wts, dt = make_inputs(cfg, rank, device)
    variants = [(x, ids, wts)] + [make_inputs(cfg, rank, device, v)[:3] for v in range(1, n_var)]

    def inp(i):
        return variants[i % n_var]

    if world > 1:
        from mail_b200 import ep as mep
        assert E % world == 0, "experts must divide evenly over ranks"
        args.graph = False  # the expert-parallel layer is called directly (host-side plan per call)
        local = list(range(rank * E // world, (rank + 1) * E // world))
        w13, w2, scales = make_weights(cfg, local, device, dt)
        if args.ep == "peer":
            layer = mep.PeerExpertParallelMoE(w13, w2, E, max_tokens=T, top_k=k, dtype=dt, scales=scales)
        else:
            layer = mep.ExpertParallelMoE(w13, w2, E, scales=scales)

        def step(xx, ii, ww):
            return layer(xx, ww, ii)
    elif cfg.get("prerouted"):
        # the reference's call: rows already grouped by expert (T*k of them),
        # group sizes per expert (fused_moe_mlp_triton.py:121, unquant_diff.txt:13-18)
        w13, w2, scales = make_weights(cfg, list(range(E)), device, dt)
        args.graph = False
        order = torch.argsort(ids.reshape(-1).to(torch.int64), stable=True)
        x = x[order // k].contiguous()  # the step's input: T * k grouped rows
        group_sizes = torch.bincount(ids.reshape(-1).to(torch.int64), minlength=E)

        def step(xx, ii, ww):
            return mb.fused_moe_mlp(xx, w13, w2, group_sizes)
    else:
        w13, w2, scales = make_weights(cfg, list(range(E)), device, dt)
        if args.graph:
            captured = mb.CapturedMoeMLP(w13, w2, T, k, dtype=dt, scales=scales)

            def step(xx, ii, ww):
                return captured(xx, ww, ii)
        else:
            def step(xx, ii, ww):
                return mb.fused_moe_mlp(xx, w13, w2, ww, ii, scales=scales)

    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    # ---- warm-up
    for i in range(args.warmup):
        step(*inp(i))
    torch.cuda.synchronize()

    # ---- timed region (device-resident inputs), per-stage events every step
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(STAGES)] for _ in range(args.steps)]
    handles = [(torch.cuda.Event(enable_timing=True)) for _ in range(2)]
    import ctypes
    for row in ev:  # torch creates events lazily: record once so the handles exist
        for e in row:
            e.record(stream)
    torch.cuda.synchronize()
    ev_arrays = [(ctypes.c_void_p * STAGES)(*[e.cuda_event for e in row]) for row in ev]
    assert all(e.cuda_event for row in ev for e in row)
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    launches0 = lib.moe_launch_count()
    t_region0 = time.time()
    handles[0].record(stream)
    for i in range(args.steps):
        if not args.graph:
            lib.moe_set_stage_events(ev_arrays[i], STAGES)
        step(*inp(i))
    lib.moe_set_stage_events(None, 0)
    handles[1].record(stream)
    torch.cuda.synchronize()
    t_region1 = time.time()
    barrier()
    clocks = sampler.stop(t_region0, t_region1)
    launches = lib.moe_launch_count() - launches0
    ms = handles[0].elapsed_time(handles[1]) / args.steps
    stage_rows = None
    stage_source = "eager calls, stage events recorded by the library"
    if args.graph:
        # replays launch the captured kernels without going through the
        # library. Stage times: a second capture of the same op with the
        # library's stage events as graph nodes, replayed once per timed
        # step right after the timed region
        launches = captured.kernels * args.steps
        try:
            lib.moe_set_stage_events(ev_arrays[0], STAGES)
            try:
                cap_ev = mb.CapturedMoeMLP(w13, w2, T, k, dtype=dt, scales=scales)
            finally:
                lib.moe_set_stage_events(None, 0)
            stage_rows = []
            for i in range(args.steps):
                xv, iv, wv = inp(i)
                cap_ev(xv, wv, iv)
                torch.cuda.synchronize()
                stage_rows.append([ev[0][j].elapsed_time(ev[0][j + 1]) for j in range(STAGES - 1)])
            del cap_ev
            stage_source = "graph replay with the stage events as graph nodes"
        except Exception:
            stage_rows = None
        if stage_rows is None:
            for i in range(args.steps):
                lib.moe_set_stage_events(ev_arrays[i], STAGES)
                xv, iv, wv = inp(i)
                mb.fused_moe_mlp(xv, w13, w2, wv, iv, scales=scales)
            lib.moe_set_stage_events(None, 0)
            torch.cuda.synchronize()
    if stage_rows is None:
        stage_rows = [[row[j].elapsed_time(row[j + 1]) for j in range(STAGES - 1)] for row in ev]

    def stage_ms(a, b):
        return statistics.mean(sum(r[a:b]) for r in stage_rows)

    st_ms = {"route": stage_ms(0, 1), "gather": stage_ms(1, 2), "gemm1": stage_ms(2, 3), "pre_gemm2": stage_ms(3, 4),
             "gemm2": stage_ms(4, 5), "finalize": stage_ms(5, 6), "source": stage_source}
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # ---- end to end through the public API: every step copies its inputs
    # from pinned host memory and its result back to pinned host memory. The
    # copies run on their own streams (host->device, device->host) with two
    # device buffers, so step i+1's upload and step i-1's download overlap
    # step i's compute, as a serving loop would run them.
    host_in = [tuple(t.cpu().pin_memory() for t in v) for v in variants]
    x_h, ids_h, wts_h = host_in[0]
    NB = 2
    out_shape = tuple(step(x, ids, wts).shape)
    y_h = [torch.empty(out_shape, dtype=dt).pin_memory() for _ in range(NB)]
    x_d = [torch.empty_like(x) for _ in range(NB)]
    ids_d = [torch.empty_like(ids) for _ in range(NB)]
    wts_d = [torch.empty_like(wts) for _ in range(NB)]
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    h2d_ev = [torch.cuda.Event() for _ in range(NB)]
    comp_ev = [torch.cuda.Event() for _ in range(NB)]
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
        y = step(x_d[b], ids_d[b], wts_d[b])
        comp_ev[b].record(stream)
        with torch.cuda.stream(down):
            down.wait_event(comp_ev[b])
            y.record_stream(down)
            y_h[b].copy_(y, non_blocking=True)
            d2h_ev.record(down)

    for i in range(2 * NB):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up.wait_event(e0)
    for i in range(args.steps):
        e2e_step(i)
    stream.wait_event(d2h_ev)  # the last result is back in host memory
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = x_h.numel() * x_h.element_size() + ids_h.numel() * 4 + wts_h.numel() * 4
    d2h = y_h[0].numel() * y_h[0].element_size()

    # ---- roofline of the dominant kernel (gate_up GEMM + SwiGLU)
    peaks = load_peaks()
    S_local = int(T * k)  # slots per rank (uniform routing keeps the per-rank load ~ T*k)
    flops_gemm1 = 2.0 * S_local * H * 2 * I
    gemm1_s = st_ms["gemm1"] / 1e3
    # algorithmic bytes of one gate_up launch: the weights of the experts that
    # received slots, the padded activation rows read, the h rows written
    wb = 1 if cfg["quant"] else (4 if cfg["dtype"] == "fp32" else 2)
    hb = 4 if cfg["dtype"] == "fp32" else 2
    if world == 1:
        counts = np.bincount(ids.cpu().numpy().reshape(-1), minlength=E)
        active = int((counts > 0).sum())
        rows_pad = int(((counts + 127) // 128 * 128).sum())
    else:  # the rank's local experts, balanced routing
        active = E // world
        rows_pad = S_local + active * 64
    bytes_gemm1 = active * 2.0 * I * H * wb + rows_pad * H * wb + rows_pad * I * hb
    # a timed region shorter than ~1 s runs at boost clocks (burst peak);
    # longer ones settle under the power cap (sustained peak)
    region_s = ms * args.steps / 1e3
    sustained = region_s >= 1.0
    peak_tc = (peaks["bf16_sus"] if sustained else peaks["bf16"]) * (2.0 if cfg["quant"] else 1.0)
    tensor_bound = flops_gemm1 / (peak_tc * 1e12) >= bytes_gemm1 / (peaks["hbm"] * 1e9)
    roofline = {"kernel": "moe_gemm_kernel<SWIGLU> (gate_up GEMM + SwiGLU)",
                "bound": "tensor" if tensor_bound else "hbm",
                "flops_per_launch": flops_gemm1, "bytes_per_launch": bytes_gemm1, "active_experts": active,
                "ms_per_launch": st_ms["gemm1"],
                # the committed capture is of the one-GPU launch at the default size
                "traffic": load_traffic(args.config) if not args.tokens and world == 1 else None,
                "traffic_unit": "bytes"}
    if tensor_bound:
        roofline.update(achieved=flops_gemm1 / gemm1_s / 1e12, peak=peak_tc, unit="TFLOP/s",
                        frac=flops_gemm1 / gemm1_s / 1e12 / peak_tc,
                        peak_source=f"{peaks['source']} bf16 {'sustained' if sustained else 'burst'}"
                                    + (" x2 (int8, spec ratio)" if cfg["quant"] else ""))
    else:
        roofline.update(achieved=bytes_gemm1 / gemm1_s / 1e9, peak=peaks["hbm"], unit="GB/s",
                        frac=bytes_gemm1 / gemm1_s / 1e9 / peaks["hbm"], peak_source=f"{peaks['source']} HBM copy")
    # the same against NVIDIA's dense spec figures (2.25 PFLOP/s bf16, 4.5 POP/s
    # int8, 7.7 TB/s HBM3e), for context
    spec = (4500.0 if cfg["quant"] else 2250.0) if tensor_bound else 7700.0
    roofline.update(spec_peak=spec, frac_of_spec=roofline["achieved"] / spec)
    flops_step = 6.0 * S_local * H * I
    value = world * T / (ms / 1e3)

    # yardsticks: cuBLAS (torch.matmul / torch.bmm) on the gate_up launch's
    # flops, timed the same way right after: one dense GEMM [S, H] x [H, 2I]
    # (no expert boundaries, one weight matrix), and a batched GEMM with one
    # weight matrix per expert and S / E rows each (the MoE launch's weight
    # bytes, no routing imbalance, no padding)
    def time_cublas(fn):
        for _ in range(3):
            fn()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(3, args.steps)
        c0.record(stream)
        for _ in range(reps):
            fn()
        c1.record(stream)
        torch.cuda.synchronize()
        return c0.elapsed_time(c1) / reps

    if world == 1 and not cfg["quant"] and cfg["dtype"] == "bf16":
        a = torch.randn(S_local, H, device=device, dtype=dt)
        b = torch.randn(H, 2 * I, device=device, dtype=dt)
        cub_ms = time_cublas(lambda: torch.matmul(a, b))
        roofline["cublas_dense_same_shape"] = {"ms": cub_ms, "tflops": flops_gemm1 / (cub_ms / 1e3) / 1e12,
                                               "ours_vs_cublas": cub_ms / st_ms["gemm1"]}
        del a, b
        rows = S_local // E
        if rows >= 128 and E * H * 2 * I * 2 <= 8 << 30:
            a = torch.randn(E, rows, H, device=device, dtype=dt)
            b = torch.randn(E, H, 2 * I, device=device, dtype=dt)
            bmm_ms = time_cublas(lambda: torch.bmm(a, b))
            bmm_flops = 2.0 * E * rows * H * 2 * I
            roofline["cublas_batched_per_expert"] = {
                "shape": f"{E} x [{rows}, {H}] x [{H}, {2 * I}]", "ms": bmm_ms,
                "tflops": bmm_flops / (bmm_ms / 1e3) / 1e12,
                "ours_vs_cublas": (flops_gemm1 / st_ms["gemm1"]) / (bmm_flops / bmm_ms)}
            del a, b

    line = {"metric": "fused MoE MLP tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": dtype_name, "data": "synthetic", "config": config_json,
            "tflops_per_gpu": flops_step / (ms / 1e3) / 1e12,
            "frac_of_tensor_peak": flops_step / (ms / 1e3) / 1e12 / peak_tc,
            "stage_ms": st_ms, "roofline": roofline,
            "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_ms,
                    "copies": "pinned host memory, own H2D / D2H streams, double-buffered"},
            "gpu_launches": int(launches), "clocks": clocks}

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ref = cpu_reference_run(cfg, steps=3, warmup=1, time_limit_s=20.0)
        line["cpu_baseline"] = {"value": ref["value"], "unit": "tokens/s", "cores": ref["cores"], "kind": "port",
                                "sample": ref["sample"]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        if hasattr(layer, "close"):
            layer.close()
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
