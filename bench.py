"""MoE-layer benchmark (BASELINE metric: MoE-layer tokens/s on B200).

Workload (N=1 headline): BASELINE config 2, the Qwen3.5-35B-A3B-shaped decode
MoE layer (d=2048, 256 experts, top-8, expert width 512, shared expert, Q8_0),
T=64 tokens per step and per GPU. One step = one MoE-layer forward
(router -> top-k -> dispatch -> expert SwiGLU -> combine) over T tokens. The
steps cycle through L distinct layers (default 8 x 0.86 GB of weights, far
larger than the 126 MB L2), so no step reads weights another step left in L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 (torchrun, one process per GPU) every rank runs its own replica on
its own T tokens (tokens are data-parallel, no collective on the path):
weak scaling; time = max over ranks of the device-timed region.

--impl reference times the reference's CPU path on the host: the C++
restatement in oracle/ (the Rust reference cannot be built in this image),
with the reference's own threading (2 expert threads + the shared expert on
the calling thread), on a bounded token sample per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer tokens/s"
UNIT = "tokens/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--tokens", type=int, default=None, help="tokens per step per GPU (c2: 64, c3: 4096, c5: 8192)")
    p.add_argument("--config", default="c2", choices=["c2", "c3", "c4", "c5"],
                   help="c2: decode Q8_0 (headline); c3: prefill Q4_0 with Zipf-skewed routing; "
                        "c4: hot-neuron sparse FFN (Q4_0, 15%% of 12288 neurons per token); "
                        "c5: one layer of the Q8_0 stack (RMSNorm + residual), prefill-sized")
    p.add_argument("--layers", type=int, default=8, help="distinct layers cycled through")
    p.add_argument("--no-sweep", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


# ---------------------------------------------------------------------------
# algorithmic bytes (per realised routing)
# ---------------------------------------------------------------------------
def q8_bytes(n):
    return n // 32 * 34


def q_bytes(cfg, n):
    return n // 32 * (34 if cfg.qtype == 8 else 18)


def layer_bytes(cfg, U, T):
    """Algorithmic HBM bytes of one C2 layer pass: every routed expert's and the
    shared expert's weights once, the router and shared-gate vector, tokens in/out."""
    per_mat = q_bytes(cfg, cfg.d * cfg.f)
    gu = (U + (1 if cfg.shared else 0)) * 2 * per_mat
    dn = (U + (1 if cfg.shared else 0)) * per_mat
    router = cfg.E * cfg.d * 4 + (cfg.d * 4 if cfg.shared else 0)
    return dict(gateup=gu + T * q8_bytes(cfg.d), down=dn, total=gu + dn + router + T * cfg.d * 4 * 2)


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every 5 ms while active."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, device: int):
        self.device, self.sm, self.mx, self.reasons, self.stop = device, [], 0, set(), threading.Event()

    def _sample(self):
        import pynvml

        self.sm.append(pynvml.nvmlDeviceGetClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        get = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        r = get(self.h)
        for name, bit in self.REASONS.items():
            if r & bit:
                self.reasons.add(name)

    def _run(self):
        while not self.stop.wait(0.005):
            self._sample()

    def __enter__(self):
        self.t = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self.device)
            self.mx = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._sample()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception:
            pass
        return self

    def __exit__(self, *a):
        self.stop.set()
        if self.t is not None:
            self.t.join(timeout=5)
            self._sample()

    def summary(self):
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.mx, "reasons": sorted(self.reasons),
                "samples": len(self.sm)}


# ---------------------------------------------------------------------------
# reference arm / CPU baseline: the oracle's restatement of the reference
# ---------------------------------------------------------------------------
def cpu_layer_tensors(cfg, seed=0, layer=0):
    """Host copies of one layer's tensors (generated on the GPU when one is present)."""
    import torch

    from powerinfer_x64_b200 import synth

    if torch.cuda.is_available():
        t = synth.moe_tensors(cfg, seed, layer)
        h = lambda a: None if a is None else a.cpu().numpy()
        out = dict(router=h(t["router"]), gate_exps=h(t["gate_exps"]), up_exps=h(t["up_exps"]),
                   down_exps=h(t["down_exps"]), shared=tuple(h(a) for a in t["shared"]) if cfg.shared else None)
        del t
        torch.cuda.empty_cache()
        return out
    raise RuntimeError("the CPU baseline uses GPU-generated inputs")


def run_cpu(cfg, tensors, x, reps):
    sys.path.insert(0, str(ROOT / "oracle"))
    import pi_oracle as orc

    orc.set_threads(0)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        orc.moe_layer(x, cfg.d, cfg.f, cfg.E, cfg.k, cfg.qtype, tensors["router"], tensors["gate_exps"],
                      tensors["up_exps"], tensors["down_exps"], shared=tensors["shared"], threads=0)
        times.append(time.perf_counter() - t0)
    return times


def reference_arm(args):
    import numpy as np
    import torch

    from powerinfer_x64_b200 import dist, synth

    rank, local, world = dist.env_rank()
    if rank != 0:
        return 0
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    cfg = synth.C2
    tensors = cpu_layer_tensors(cfg)
    sample = args.tokens or 64  # one step = the same 64-token batch the GPU arm processes
    x = synth.normal_host(synth.stream_seed(0, "x"), sample * cfg.d, 1.0).reshape(sample, cfg.d)
    run_cpu(cfg, tensors, x, args.warmup)
    times = run_cpu(cfg, tensors, x, args.steps)
    tps = sample * len(times) / sum(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": f"{cfg.name} (BASELINE config 2) T={sample}; step = {sample} tokens",
                   "tokens_per_step": sample},
        "cpu_baseline": {"value": tps, "unit": UNIT, "cores": 3, "kind": "port",
                         "sample": f"{sample} tokens of one C2 layer per step (the whole step of the workload)",
                         "host_threads_available": os.cpu_count(),
                         "note": "C++ restatement of the reference CPU path (oracle/); reference threading: "
                                 "2 expert threads + shared expert on the caller"},
        "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# config 4: hot-neuron sparse dense FFN (predictor path), HBM-bound
# ---------------------------------------------------------------------------
def main_c4(args):
    import numpy as np
    import torch

    from powerinfer_x64_b200 import Context, dist, synth
    from powerinfer_x64_b200.predictor import SparseFFN

    rank, local, world = dist.init()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = synth.C4
    T = args.tokens or 8
    ctx = Context.default(local)
    n_layers = max(args.layers, 4)  # 4 x 85 MB of weights > L2
    ffns, xs, csrs, rows = [], [], [], []
    for li in range(n_layers):
        t = synth.sparse_tensors(cfg, seed=rank * 1000 + li)
        ffns.append(SparseFFN(t["gate"], t["up"], t["down"], cfg.qtype, cfg.d, cfg.F))
        del t
        lists = synth.sparse_masks(cfg, T, seed=rank * 1000 + li)
        p_, i_ = SparseFFN.csr(lists)
        csrs.append((torch.from_numpy(p_).to(dev), torch.from_numpy(i_).to(dev)))
        rows.append(len(set(np.concatenate(lists).tolist())))
        xs.append(synth.tokens_dev(cfg.d, T, seed=rank, layer=li))
    out = torch.empty((T, cfg.d), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    step = lambda i: ffns[i % n_layers].forward(xs[i % n_layers], csr=csrs[i % n_layers], out=out)
    for i in range(args.warmup):
        step(i)
    dist.barrier(local)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = dist.max_over_ranks(e0.elapsed_time(e1), device=dev)
    ctx.profile(True)
    for i in range(args.steps):
        step(i)
    torch.cuda.synchronize()
    kern = ctx.profile_read()
    ctx.profile(False)
    row_b = cfg.d // 32 * 18  # one Q4_0 neuron row / column
    byts = sum(rows[i % n_layers] * 3 * row_b + T * cfg.d * 8 for i in range(args.steps))
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    peak = peaks.get("hbm_gbs", 6650.0)
    ach = byts / (ms / 1e3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "sparse-FFN tokens/s", "value": world * T * args.steps / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q4_0 x f32",
            "data": "synthetic (seeded SplitMix64 + Box-Muller; weights N(0,0.02) -> Q4_0; seeded hot-set masks)",
            "config": {"workload": f"{cfg.name} (BASELINE config 4): d=4096 F=12288 Q4_0, 15% active neurons per "
                                   "token (80% from a 20% hot set)", "tokens_per_step_per_gpu": T,
                       "parallelism": f"dp{world} (replicas)",
                       "l2": f"inputs larger than L2: steps cycle through {n_layers} FFNs x 85 MB"},
            "roofline": {"bound": "hbm", "kernel": "sparse FFN step", "achieved": ach, "peak": peak, "unit": "GB/s",
                         "frac": ach / peak, "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                         "algorithmic_bytes_per_step": byts / args.steps, "traffic": None},
            "kernels_ms_per_step": {k: v[0] / args.steps for k, v in kern.items()},
            "kernel_launches_per_step": {k: v[1] / args.steps for k, v in kern.items()},
            "gpu_launches": sum(n for (_, n) in kern.values()),
            "clocks": clk.summary(),
        }), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    if args.config == "c4":
        return main_c4(args)
    import numpy as np
    import torch

    from powerinfer_x64_b200 import Context, dist, synth

    rank, local, world = dist.init()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = {"c2": synth.C2, "c3": synth.C3, "c5": synth.C5}[args.config]
    T = args.tokens or {"c2": 64, "c3": 4096, "c5": 8192}[args.config]
    if args.config != "c2":
        args.no_sweep = True
    fwd_kw = dict(rmsnorm=True, residual=True) if args.config == "c5" else {}
    ctx = Context.default(local)

    # layers + fixed per-layer tokens (each rank its own seed stream). c5: one model
    # (same weights on every rank) sharded by experts over the ranks, tokens per rank
    layers, xs, routing = [], [], []
    for li in range(args.layers):
        x = synth.tokens_dev(cfg.d, T, seed=rank, layer=li)
        if args.config == "c5":
            from powerinfer_x64_b200.ep import EPMoeLayer, local_expert_bytes

            t = synth.moe_tensors(cfg, seed=0, layer=li)
            loc = lambda a: local_expert_bytes(a, cfg.E, rank, world).clone()
            L = EPMoeLayer(t["router"], loc(t["gate_exps"]), loc(t["up_exps"]), loc(t["down_exps"]), cfg.d, cfg.f,
                           cfg.E, cfg.k, rank=rank, world=world, shared=t["shared"])
            del t
            torch.cuda.empty_cache()
            U = cfg.E
        else:
            L = synth.moe_layer(cfg, seed=rank, layer=li)
            r = L.route(x)
            U = int((r["counts"] > 0).sum().item())
        layers.append(L)
        xs.append(x)
        routing.append(U)
    torch.cuda.synchronize()
    out = torch.empty((T, cfg.d), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()

    def step(i):
        layers[i % args.layers].forward(xs[i % args.layers], out=out, **fwd_kw)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    # ---- timed region (device time with CUDA events, no per-kernel events inside) ----
    dist.barrier(local)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
    dist.barrier(local)
    ms = e0.elapsed_time(e1)
    # ---- the same steps again with per-kernel CUDA events (kernel breakdown, roofline) ----
    ctx.profile(True)
    torch.cuda.synchronize()
    for i in range(args.steps):
        step(i)
    torch.cuda.synchronize()
    kern = ctx.profile_read()
    ctx.profile(False)
    ms_max = dist.max_over_ranks(ms, device=dev)
    value = world * T * args.steps / (ms_max / 1e3)

    # per-kernel averages, roofline of the dominant kernel (gate/up GEMV)
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    Us = [routing[i % args.layers] for i in range(args.steps)]
    b_gu = sum(layer_bytes(cfg, U, T)["gateup"] for U in Us)
    b_tot = sum(layer_bytes(cfg, U, T)["total"] for U in Us)
    gu_ms, gu_n = kern.get("k_gateup", (float("nan"), 0))
    achieved = b_gu / (gu_ms / 1e3) / 1e9 if gu_n else float("nan")
    traffic = None
    tf = ROOT / "profiles" / "ncu_traffic.json"
    if tf.exists():
        try:
            traffic = json.loads(tf.read_text()).get("k_gateup_c2_T64_bytes_per_launch")
        except Exception:
            traffic = None
    launches = sum(n for (_, n) in kern.values())
    roofline = {"bound": "hbm", "kernel": "k_gateup", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": peak_src, "traffic": traffic,
                "algorithmic_bytes_per_launch": b_gu / args.steps,
                "avg_launch_us": 1e3 * gu_ms / max(gu_n, 1)}
    if args.config == "c3":
        # prefill: the gate/up GEMM is a dense contraction; FLOPs counted once
        # (the kernel issues 3 f16 MMAs per product for f32-level accuracy)
        tpeak = peaks.get("bf16_tflops", 1590.0)
        slots = T * cfg.k + T
        g_ms, g_n = kern.get("k_gemm_gateup", (float("nan"), 0))
        flops = 2.0 * slots * 2 * cfg.f * cfg.d
        ach_t = flops / (g_ms / max(g_n, 1) / 1e3) / 1e12
        roofline = {"bound": "tensor", "kernel": "k_gemm_gateup", "achieved": ach_t, "peak": tpeak, "unit": "TFLOP/s",
                    "frac": ach_t / tpeak, "peak_source": "measured" if "bf16_tflops" in peaks else "fallback",
                    "traffic": None, "algorithmic_flops_per_launch": flops,
                    "mma_issued_tflops": 3 * ach_t, "avg_launch_us": 1e3 * g_ms / max(g_n, 1)}
    if args.config == "c5":
        # Q8_0 prefill: exact int8 block products (f16 MMAs of the int8 values, one per
        # product), judged against the int8 dense tensor peak (no measured int8 figure
        # exists for this pool: nominal 4.5 POPS)
        slots = T * cfg.k + T
        g_ms, g_n = kern.get("k_gemm_q8_gateup", (float("nan"), 0))
        ops = 2.0 * slots * 2 * cfg.f * cfg.d
        ach_t = ops / (g_ms / args.steps / 1e3) / 1e12  # routed + shared launches of a step
        roofline = {"bound": "tensor", "kernel": "k_gemm_q8_gateup", "achieved": ach_t, "peak": 4500.0,
                    "unit": "TOPS (int8)", "frac": ach_t / 4500.0, "peak_source": "nominal int8 dense (no measured int8 peak)",
                    "frac_of_measured_bf16": ach_t / peaks.get("bf16_tflops", 1590.0), "traffic": None,
                    "algorithmic_ops_per_step": ops, "avg_launch_us": 1e3 * g_ms / max(g_n, 1),
                    "launches_per_step": g_n / args.steps}

    # ---- end to end: host tokens in (pinned), host output back, per step ----
    xh = [x.cpu().pin_memory() for x in xs]
    oh = torch.empty((T, cfg.d), dtype=torch.float32).pin_memory()
    xd = torch.empty((T, cfg.d), dtype=torch.float32, device=dev)

    def e2e_step(i):
        xd.copy_(xh[i % args.layers], non_blocking=True)
        layers[i % args.layers].forward(xd, out=out, **fwd_kw)
        oh.copy_(out, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    dist.barrier(local)
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for i in range(args.steps):
        e2e_step(i)
    f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = dist.max_over_ranks(f0.elapsed_time(f1), device=dev)
    e2e_val = world * T * args.steps / (e2e_ms / 1e3)

    # ---- decode batch sweep (T in 1, 4, 16, 64) ----
    sweep = []
    if not args.no_sweep:
        for Ts in (1, 4, 16, 64):
            xs_s = [synth.tokens_dev(cfg.d, Ts, seed=rank + 100, layer=li) for li in range(args.layers)]
            Us_s = [int((layers[li].route(xs_s[li])["counts"] > 0).sum().item()) for li in range(args.layers)]
            os_ = torch.empty((Ts, cfg.d), dtype=torch.float32, device=dev)
            for i in range(args.warmup):
                layers[i % args.layers].forward(xs_s[i % args.layers], out=os_)
            torch.cuda.synchronize()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record(stream)
            for i in range(args.steps):
                layers[i % args.layers].forward(xs_s[i % args.layers], out=os_)
            g1.record(stream)
            torch.cuda.synchronize()
            sm = g0.elapsed_time(g1)
            byt = sum(layer_bytes(cfg, Us_s[i % args.layers], Ts)["total"] for i in range(args.steps))
            sweep.append({"T": Ts, "tokens_per_s": Ts * args.steps / (sm / 1e3), "us_per_layer": 1e3 * sm / args.steps,
                          "layer_hbm_gbs": byt / (sm / 1e3) / 1e9,
                          "layer_frac_of_peak": byt / (sm / 1e3) / 1e9 / peak})

    # ---- CPU baseline (rank 0, N=1): the oracle, reference threading ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config == "c2":
        tensors = cpu_layer_tensors(cfg, seed=0, layer=0)
        sample = T
        xsmp = xs[0][:sample].cpu().numpy()
        run_cpu(cfg, tensors, xsmp, 1)
        times = run_cpu(cfg, tensors, xsmp, 10)
        med = statistics.median(times)
        cpu = {"value": sample / med, "unit": UNIT, "cores": 3, "kind": "port",
               "sample": f"{sample} tokens of one C2 layer (one full step), median of 10 runs after 1 warm-up",
               "host_threads_available": os.cpu_count()}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16x3->f32" if args.config == "c3" else "int8",
            "data": "synthetic (seeded SplitMix64 + Box-Muller; weights N(0,0.02) -> " + ("Q4_0)" if args.config == "c3" else "Q8_0)"),
            "config": {"workload": f"{cfg.name} (BASELINE config {args.config[1]}): d=2048 "
                                   f"E=256 k=8 f=512 +shared, " + {"c2": "Q8_0 decode", "c3": "Q4_0 prefill, Zipf router bias",
                                                                   "c5": "Q8_0 prefill, one layer of the 40-layer stack, RMSNorm + residual"}[args.config],
                       "tokens_per_step_per_gpu": T, "global_batch": T * world,
                       "parallelism": (f"ep{world} (experts sharded {cfg.E // world} per GPU, tokens data-parallel, "
                                       "NCCL all-to-all-v dispatch/combine)") if args.config == "c5" else f"dp{world} (replicas)",
                       "layers_cycled": args.layers, "l2": "inputs larger than L2: steps cycle through "
                       f"{args.layers} layers x {layer_bytes(cfg, 256, T)['total'] / 1e9:.2f} GB"},
            "roofline": roofline,
            "layer_roofline": {"achieved_gbs": b_tot / (ms_max / 1e3) / 1e9,
                               "frac": b_tot / (ms_max / 1e3) / 1e9 / peak},
            "kernels_ms_per_step": {k: v[0] / args.steps for k, v in kern.items()},
            "kernel_launches_per_step": {k: v[1] / args.steps for k, v in kern.items()},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": T * cfg.d * 4,
                    "d2h_bytes_per_step": T * cfg.d * 4},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "sweep": sweep,
        }
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
