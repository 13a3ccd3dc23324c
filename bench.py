"""MoE-layer benchmark (BASELINE metric: MoE-layer tokens/s on 1/2/4/8 B200).

Default workload (every N): BASELINE config 5, one layer of the 40-layer
Qwen3.5-35B-A3B-shaped Q8_0 stack (d=2048, 256 experts, top-8, expert width
512, shared expert; RMSNorm before the layer, residual after), T=8192 home
tokens per GPU, experts sharded over the N ranks (expert parallelism,
EPMoeLayer; at N=1 one rank holds all 256). One step = one layer forward over
the rank's T tokens. Steps cycle through L distinct layers (default 8 x 0.86 GB
of weights at N=1, far larger than the 126 MB L2).

At N=1 the line also carries the config-2 decode sweep (T = 1, 4, 16, 64) and
its HBM fraction under "decode_c2".

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config c5|c2|c3|c4]

--impl reference times the reference's CPU path on the host: the C++
restatement in oracle/ (the Rust reference cannot be built in this image),
with the reference's own threading (2 expert threads + the shared expert on
the calling thread), on a bounded token sample per step, with inputs built on
the host by the oracle's own generator (no GPU library is loaded).
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
    p.add_argument("--config", default="c5", choices=["c2", "c3", "c4", "c5"],
                   help="c2: decode Q8_0 (headline); c3: prefill Q4_0 with Zipf-skewed routing; "
                        "c4: hot-neuron sparse FFN (Q4_0, 15%% of 12288 neurons per token); "
                        "c5 (default): one layer of the Q8_0 stack (RMSNorm + residual), T=8192 per GPU, expert-parallel")
    p.add_argument("--sample", type=int, default=None, help="reference arm: tokens per step (default 32)")
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
# workload description shared by both arms (the driver compares the configs)
# ---------------------------------------------------------------------------
CFG = {
    "c2": dict(name="c2_decode_q8", d=2048, E=256, k=8, f=512, qtype=8, shared=True, zipf=False, T=64, norm=False),
    "c3": dict(name="c3_prefill_q4", d=2048, E=256, k=8, f=512, qtype=2, shared=True, zipf=True, T=4096, norm=False),
    "c5": dict(name="c5_stack_q8", d=2048, E=256, k=8, f=512, qtype=8, shared=True, zipf=False, T=8192, norm=True),
}


def workload_config(cname, T, world, layers):
    c = CFG[cname]
    kind = {"c2": "Q8_0 decode", "c3": "Q4_0 prefill, Zipf router bias",
            "c5": "Q8_0, one layer of the 40-layer stack, RMSNorm before + residual after"}[cname]
    par = (f"ep{world} (experts sharded {c['E'] // world} per GPU, tokens data-parallel, rows pushed over NVLink "
           "peer memory)" if cname == "c5"
           else f"dp{world} (replicas)")
    return {"workload": f"{c['name']} (BASELINE config {cname[1]}): d=2048 E=256 k=8 f=512 +shared expert, {kind}",
            "tokens_per_step_per_gpu": T, "global_batch": T * world, "parallelism": par, "layers_cycled": layers,
            "l2": f"inputs larger than L2: steps cycle through {layers} layers of "
                  f"{(0.86 if c['qtype'] == 8 else 0.45):.2f} GB of expert weights each"}


# ---------------------------------------------------------------------------
# reference arm / CPU baseline: the oracle's restatement of the reference,
# inputs built on the host by the oracle's generator (no GPU library loaded)
# ---------------------------------------------------------------------------
def _oracle():
    sys.path.insert(0, str(ROOT / "oracle"))
    import pi_oracle as orc

    return orc


def host_layer(cname, seed=0, layer=0):
    c = CFG[cname]
    return _oracle().moe_tensors_host(c["d"], c["E"], c["f"], c["qtype"], c["shared"], zipf=c["zipf"], seed=seed,
                                      layer=layer)


def host_tokens(cname, n, rank=0, layer=0):
    """The first n tokens of the GPU arm's token stream of (rank, layer)."""
    orc = _oracle()
    d = CFG[cname]["d"]
    return orc.synth_normal(orc.stream_seed(rank, "x", layer), n * d, 1.0).reshape(n, d)


def run_cpu(cname, t, x):
    """One timed pass of the oracle over the tokens x, reference threading."""
    orc = _oracle()
    c = CFG[cname]
    orc.set_threads(0)
    t0 = time.perf_counter()
    orc.moe_layer(x, c["d"], c["f"], c["E"], c["k"], c["qtype"], t["router"], t["gate_exps"], t["up_exps"],
                  t["down_exps"], shared=t["shared"], bias=t["router_bias"], threads=0, residual=c["norm"],
                  rmsnorm=c["norm"])
    return time.perf_counter() - t0


def cpu_sample(cname, T, sample, steps, warmup):
    """Times `steps` passes of `sample` tokens each (cycling through the GPU arm's
    first T tokens of layer 0) after `warmup` untimed passes; returns (times, desc)."""
    t = host_layer(cname)
    n = min(T, sample * max(1, steps + warmup))
    xs = host_tokens(cname, n)
    times = []
    for i in range(warmup + steps):
        j = (i * sample) % n
        dt = run_cpu(cname, t, xs[j:j + sample])
        if i >= warmup:
            times.append(dt)
    desc = (f"{sample} tokens per step of layer 0 of the {CFG[cname]['name']} workload (its tokens cycled), "
            f"reference threading: 2 expert threads + the shared expert on the caller; time scales linearly "
            f"with tokens (the reference routes and runs each token on its own)")
    return times, desc


def reference_arm(args):
    from powerinfer_x64_b200 import dist  # pure-Python helpers; loads no GPU library

    rank, local, world = dist.env_rank()
    if rank != 0:
        return 0
    cname = args.config if args.config in CFG else "c5"
    T = args.tokens or CFG[cname]["T"]
    sample = args.sample or {"c2": 64, "c3": 8, "c5": 32}[cname]
    times, desc = cpu_sample(cname, T, sample, args.steps, args.warmup)
    tps = sample * len(times) / sum(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8" if cname != "c3" else "f32",
        "data": "synthetic (seeded SplitMix64 + Box-Muller on the host; weights N(0,0.02) -> "
                + ("Q4_0)" if cname == "c3" else "Q8_0)"),
        "config": workload_config(cname, T, world, args.layers),
        "cpu_baseline": {"value": tps, "unit": UNIT, "cores": 3, "kind": "port", "sample": desc,
                         "host_threads_available": os.cpu_count(),
                         "note": "C++ restatement of the reference CPU path (oracle/); the Rust reference cannot be "
                                 "built here (no Rust toolchain); the reference's MoE path uses at most 3 threads"},
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
def load_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


def time_steps(step, steps, stream):
    import torch

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def decode_sweep(args, ctx, dev, peak):
    """BASELINE config 2 on this GPU: T = 1, 4, 16, 64 tokens per step through
    layers cycled like the headline; the layer's HBM fraction, and the dominant
    kernel's (k_gateup) roofline at T = 64."""
    import torch

    from powerinfer_x64_b200 import synth

    cfg = synth.C2
    nl = max(args.layers, 4)
    layers = [synth.moe_layer(cfg, seed=0, layer=li) for li in range(nl)]
    stream = torch.cuda.current_stream()
    res = {}
    for T in (1, 4, 16, 64):
        xs = [synth.tokens_dev(cfg.d, T, seed=100, layer=li) for li in range(nl)]
        Us = [int((layers[li].route(xs[li])["counts"] > 0).sum().item()) for li in range(nl)]
        out = torch.empty((T, cfg.d), dtype=torch.float32, device=dev)
        step = lambda i: layers[i % nl].forward(xs[i % nl], out=out)
        for i in range(max(args.warmup, 3)):
            step(i)
        torch.cuda.synchronize()
        n = max(args.steps, 50)
        ms = time_steps(step, n, stream)
        byt = sum(layer_bytes(cfg, Us[i % nl], T)["total"] for i in range(n))
        r = {"tokens_per_s": T * n / (ms / 1e3), "us_per_layer": 1e3 * ms / n,
             "layer_hbm_gbs": byt / (ms / 1e3) / 1e9, "layer_frac_of_peak": byt / (ms / 1e3) / 1e9 / peak}
        if T == 64:
            ctx.profile(True)
            for i in range(n):
                step(i)
            torch.cuda.synchronize()
            kern = ctx.profile_read()
            ctx.profile(False)
            gu_ms, gu_n = kern.get("k_gateup", (float("nan"), 0))
            b_gu = sum(layer_bytes(cfg, Us[i % nl], T)["gateup"] for i in range(n))
            ach = b_gu / (gu_ms / 1e3) / 1e9
            r["k_gateup"] = {"achieved_gbs": ach, "frac": ach / peak, "avg_launch_us": 1e3 * gu_ms / max(gu_n, 1),
                             "algorithmic_bytes_per_launch": b_gu / max(gu_n, 1)}
            r["kernels_ms_per_step"] = {k: v[0] / n for k, v in kern.items()}
        res[f"T{T}"] = r
    del layers
    torch.cuda.empty_cache()
    return res


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    if args.config == "c4":
        return main_c4(args)
    import torch

    from powerinfer_x64_b200 import Context, dist, synth
    from powerinfer_x64_b200.pipeline import HostPipeline

    rank, local, world = dist.init()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cname = args.config
    cfg = {"c2": synth.C2, "c3": synth.C3, "c5": synth.C5}[cname]
    T = args.tokens or CFG[cname]["T"]
    fwd_kw = dict(rmsnorm=True, residual=True) if cname == "c5" else {}
    ctx = Context.default(local)
    peaks = load_peaks()
    peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"

    # layers + fixed per-layer tokens (each rank its own token stream). c5: one model
    # (the same weights on every rank) sharded by experts over the ranks
    layers, xs, routing = [], [], []
    comm = None
    if cname == "c5" and world > 1:
        from powerinfer_x64_b200.ep import EPComm

        comm = EPComm(rank, world, T, cfg.d, cfg.k)  # the NVLink data plane shared by every layer
    for li in range(args.layers):
        x = synth.tokens_dev(cfg.d, T, seed=rank, layer=li)
        if cname == "c5":
            from powerinfer_x64_b200.ep import EPMoeLayer, local_expert_bytes

            t = synth.moe_tensors(cfg, seed=0, layer=li)
            loc = lambda a: local_expert_bytes(a, cfg.E, rank, world).clone()
            L = EPMoeLayer(t["router"], loc(t["gate_exps"]), loc(t["up_exps"]), loc(t["down_exps"]), cfg.d, cfg.f,
                           cfg.E, cfg.k, rank=rank, world=world, shared=t["shared"], comm=comm)
            del t
            torch.cuda.empty_cache()
            U = cfg.E
        else:
            L = synth.moe_layer(cfg, seed=rank, layer=li)
            U = int((L.route(x)["counts"] > 0).sum().item())
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

    # ---- timed region: device time with CUDA events, no per-kernel events inside ----
    dist.barrier(local)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ms = time_steps(step, args.steps, stream)
    dist.barrier(local)
    ms_max = dist.max_over_ranks(ms, device=dev)
    value = world * T * args.steps / (ms_max / 1e3)

    # ---- the same steps again with a CUDA-event pair around every launch ----
    ctx.profile(True)
    torch.cuda.synchronize()
    for i in range(args.steps):
        step(i)
    torch.cuda.synchronize()
    kern = ctx.profile_read()
    ctx.profile(False)
    launches = sum(n for (_, n) in kern.values())

    if cname == "c5":
        # Q8_0 prefill: exact int8 block products on the tensor cores; useful int8
        # ops of the gate/up GEMM (routed + shared slots of this rank's tokens, which
        # is also the all-rank average of the slots each rank's experts receive)
        slots = T * cfg.k + T
        g_ms, g_n = kern.get("k_gemm_q8_gateup", (float("nan"), 0))
        ops = 2.0 * slots * 2 * cfg.f * cfg.d
        ach = ops / (g_ms / args.steps / 1e3) / 1e12
        ipeak = peaks.get("int8_tops", 4500.0)
        # The exact method adds sumi * scale product into f32 registers per output and
        # 32-block (one multiply, one add): the CUDA-core floor of that work at the
        # sampled clock, 128 f32 lanes per SM
        sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
        fp32_floor_ms = 2.0 * slots * 2 * cfg.f * (cfg.d // 32) / (128 * sm_count * 1.965e9) * 1e3
        c5_traffic = None
        tf = ROOT / "profiles" / "ncu_traffic.json"
        if tf.exists() and T == 8192:
            try:
                c5_traffic = json.loads(tf.read_text()).get("k_gemm_q8_gateup_c5_T8192_bytes_per_launch")
            except Exception:
                c5_traffic = None
        roofline = {"bound": "tensor", "kernel": "k_gemm_q8_gateup", "achieved": ach, "peak": ipeak,
                    "unit": "TOPS (int8)", "frac": ach / ipeak,
                    "peak_source": "measured" if "int8_tops" in peaks else "nominal int8 dense (no measured int8 peak)",
                    "frac_of_measured_bf16": ach / peaks.get("bf16_tflops", 1590.0), "traffic": c5_traffic,
                    "fp32_epilogue_floor_ms": fp32_floor_ms,
                    "algorithmic_ops_per_step": ops, "avg_launch_us": 1e3 * g_ms / max(g_n, 1),
                    "launches_per_step": g_n / args.steps}
        lops = 2.0 * slots * 3 * cfg.f * cfg.d
        layer_roof = {"useful_int8_tops": lops / (ms_max / args.steps / 1e3) / 1e12,
                      "frac_of_int8_peak": lops / (ms_max / args.steps / 1e3) / 1e12 / ipeak}
    elif cname == "c3":
        tpeak = peaks.get("bf16_tflops", 1590.0)
        slots = T * cfg.k + T
        g_ms, g_n = kern.get("k_gemm_gateup", (float("nan"), 0))
        flops = 2.0 * slots * 2 * cfg.f * cfg.d
        ach = flops / (g_ms / max(g_n, 1) / 1e3) / 1e12
        roofline = {"bound": "tensor", "kernel": "k_gemm_gateup", "achieved": ach, "peak": tpeak, "unit": "TFLOP/s",
                    "frac": ach / tpeak, "peak_source": "measured" if "bf16_tflops" in peaks else "fallback",
                    "traffic": None, "algorithmic_flops_per_launch": flops, "mma_issued_tflops": 3 * ach,
                    "avg_launch_us": 1e3 * g_ms / max(g_n, 1)}
        layer_roof = None
    else:
        Us = [routing[i % args.layers] for i in range(args.steps)]
        b_gu = sum(layer_bytes(cfg, U, T)["gateup"] for U in Us)
        b_tot = sum(layer_bytes(cfg, U, T)["total"] for U in Us)
        gu_ms, gu_n = kern.get("k_gateup", (float("nan"), 0))
        ach = b_gu / (gu_ms / 1e3) / 1e9 if gu_n else float("nan")
        traffic = None
        tf = ROOT / "profiles" / "ncu_traffic.json"
        if tf.exists():
            try:
                traffic = json.loads(tf.read_text()).get("k_gateup_c2_T64_bytes_per_launch")
            except Exception:
                traffic = None
        roofline = {"bound": "hbm", "kernel": "k_gateup", "achieved": ach, "peak": peak, "unit": "GB/s",
                    "frac": ach / peak, "peak_source": peak_src, "traffic": traffic,
                    "algorithmic_bytes_per_launch": b_gu / args.steps, "avg_launch_us": 1e3 * gu_ms / max(gu_n, 1)}
        layer_roof = {"achieved_gbs": b_tot / (ms_max / 1e3) / 1e9, "frac": b_tot / (ms_max / 1e3) / 1e9 / peak}

    # ---- end to end through the public API: pinned host tokens in, host output back,
    # every step; copies of neighbouring steps overlap compute (HostPipeline) ----
    xh = [x.cpu().pin_memory() for x in xs]
    oh = [torch.empty((T, cfg.d), dtype=torch.float32).pin_memory() for _ in range(2)]
    pipe = HostPipeline(layers[0], T, cfg.d, **fwd_kw)

    def e2e_run(i0, n):
        idx = range(i0, i0 + n)
        pipe.run([xh[i % args.layers] for i in idx], [oh[i % 2] for i in idx],
                 layers=[layers[i % args.layers] for i in idx])
        pipe.finish()

    e2e_run(0, args.warmup)
    torch.cuda.synchronize()
    dist.barrier(local)
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    e2e_run(args.warmup, args.steps)
    f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = dist.max_over_ranks(f0.elapsed_time(f1), device=dev)
    e2e_val = world * T * args.steps / (e2e_ms / 1e3)

    extra = {}
    if world == 1 and cname == "c5" and not args.no_sweep:
        extra["decode_c2"] = decode_sweep(args, ctx, dev, peak)

    # ---- CPU baseline (rank 0, N=1): the oracle, reference threading, host inputs ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample = {"c2": 64, "c3": 8, "c5": 64}[cname]
        times, desc = cpu_sample(cname, T, sample, 5, 1)
        med = statistics.median(times)
        cpu = {"value": sample / med, "unit": UNIT, "cores": 3, "kind": "port", "sample": desc + "; median of 5",
               "host_threads_available": os.cpu_count()}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16x3->f32" if cname == "c3" else "int8",
            "data": "synthetic (seeded SplitMix64 + Box-Muller; weights N(0,0.02) -> "
                    + ("Q4_0)" if cname == "c3" else "Q8_0)"),
            "config": workload_config(cname, T, world, args.layers),
            "roofline": roofline,
            "layer_roofline": layer_roof,
            "kernels_ms_per_step": {k: v[0] / args.steps for k, v in kern.items()},
            "kernel_launches_per_step": {k: v[1] / args.steps for k, v in kern.items()},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": T * cfg.d * 4,
                    "d2h_bytes_per_step": T * cfg.d * 4, "ms_per_step": e2e_ms / args.steps,
                    "overlap": "host->device and device->host copies of neighbouring steps overlap compute"},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
