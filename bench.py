#!/usr/bin/env python
"""Benchmark of the SpikeStack Lite hot path on B200.

Default workload (one "step"): the full SpikingTransformer forward at batch
512, seq 1024, input 256, d 512, 8 heads, 6 layers, T = 4 Spire planes, FFN
x4, GSMC on (x ~ N(0, 1), random-init weights from torch.manual_seed(0)),
batch-sharded over the N GPUs: each rank runs its 512/N samples in chunks of
64 (each chunk's forward replayed from one CUDA graph) and one NCCL
all_gather of the logits rebuilds the batch inside the timed region.  Metric:
tokens/s = 512 * 1024 / step time (strong scaling: the batch is fixed).
The line nests the isolated spike-linear measurement under "spike_linear":
S[T=3, M=16384, K=512] ~ Bernoulli(0.10), W[512, 128] fp32, Y fp32, CSR per
plane, in GSOP/s (SOP = one nonzero input spike x one output neuron) with its
HBM roofline (each rank its own instance, weak scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload model_full|spike_linear|sweep|attention|linear|layernorm|model_small]

N > 1: launched by torchrun, one rank per GPU, timing on the device with CUDA
events, max over ranks.  --impl reference: the reference's own CPU
implementation of the path (its PyTorch CPU arithmetic, restated in oracle/)
timed on all host cores, rank 0 only, on a sample of the same workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

# The reference arm times the CPU path with every host core.  torchrun exports
# OMP_NUM_THREADS=1 to each rank; set the pools' sizes before torch starts them.
if "reference" in sys.argv:
    try:
        _n = str(len(os.sched_getaffinity(0)))
    except AttributeError:
        _n = str(os.cpu_count() or 1)
    for _v in ("OMP_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_v] = _n

import numpy as np  # noqa: E402
import torch  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from spikestack_lite_b200.dist import RankGroup, shard_bounds  # noqa: E402

METRIC = "tokens/s full-model fwd & spike-linear GSOP/s (% HBM roofline) at 1/2/4/8 B200"
L2_BYTES = 126 * 1024 * 1024


# ------------------------------------------------------------------ utilities
def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "src": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


def host_threads():
    """Host cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def profile_traffic(name):
    """dram bytes per launch recorded in profiles/<name>.md ('dram_bytes_per_launch: N')."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    try:
        for line in open(path):
            if line.strip().startswith("dram_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        time.sleep(0.2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        mhz, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(mhz)}


# ------------------------------------------------------------- spike-linear
def spike_linear_setup(cfg, dev, nsets, seed):
    T, M, K, N, p = cfg["T"], cfg["M"], cfg["K"], cfg["N"], cfg["p"]
    g = torch.Generator(device=dev).manual_seed(seed)
    wdt = torch.bfloat16 if cfg["w_dtype"] == "bf16" else torch.float32
    W = (torch.randn(K, N, generator=g, device=dev) / K ** 0.5).to(wdt)  # weightT layout [K, N]
    sets = []
    for i in range(nsets):
        S = (torch.rand(T, M, K, generator=g, device=dev) < p).float()
        nnz = int((S > 0).sum().item())
        csr = None
        if cfg["csr"]:
            from spikestack_lite_b200 import ops

            csr = ops.alloc_csr(T, M, K, dev, capacity=int(nnz * 1.02) + 1024)
        sets.append({"S": S, "nnz": nnz, "csr": csr})
    return W, sets


def run_spike_linear(args, dist, cfg):
    from spikestack_lite_b200 import _lib, ops

    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    T, M, K, N = cfg["T"], cfg["M"], cfg["K"], cfg["N"]
    set_bytes = 4 * T * M * K + 4 * T * M * N
    nsets = max(2, int(np.ceil(3 * L2_BYTES / set_bytes)) + 1)
    W, sets = spike_linear_setup(cfg, dev, nsets, seed=1234 + dist.rank)
    branch = args.branch
    stream = torch.cuda.current_stream(dev)

    def step(i):
        s = sets[i % nsets]
        return ops.spike_linear(s["S"], weightT=W, csr=s["csr"], branch=branch)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if args.quick:  # eager steps only (the small case that ncu captures)
        for i in range(args.steps):
            step(i)
        torch.cuda.synchronize()
        return {"workload": cfg["name"], "quick": True, "steps": args.steps}
    launches0 = _lib.launch_count()

    # CUDA graphs (one per input set) keep the host out of the timed region
    graphs = []
    outs = []
    for i in range(nsets):
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph):
            outs.append(step(i))
        graphs.append(gph)
    for i in range(nsets):
        graphs[i].replay()
    torch.cuda.synchronize()

    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        dist.barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for i in range(args.steps):
            graphs[i % nsets].replay()
        stop.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
    ms = start.elapsed_time(stop)
    ms_max = dist.max(ms)
    launches_per_step = (_lib.launch_count() - launches0) / max(1, nsets)  # counted at capture

    sops_step = statistics.mean(s["nnz"] for s in sets) * N
    value = dist.world * sops_step * args.steps / (ms_max / 1e3) / 1e9

    # per-kernel device time with CUDA events on the launch stream (eager steps)
    kernel_ms = {}
    for kname in ("dense", "csr_scan", "w_image", "spmm_csr"):
        _lib.profile_begin(kname)
        for i in range(args.steps):
            step(i)
        tot, n = _lib.profile_end()
        if n:
            kernel_ms[kname] = tot / n
    torch.cuda.synchronize()

    # parity spot check of the timed outputs (one set) against the oracle
    from oracle import spk_oracle as O

    ref = O.spike_linear(sets[0]["S"][:, :2048].cpu().numpy(), W.float().cpu().numpy())
    parity = O.rel_err(outs[0][:, :2048].cpu().numpy(), ref)

    # end to end through the public API from pinned host buffers
    e2e = spike_linear_e2e(args, dist, cfg, W, sets, branch)

    pk = peaks()
    alg_dense = 4 * T * M * K + W.element_size() * K * N + 4 * T * M * N
    alg_step = alg_dense + (4 * T * (M + 1) + 4 * T * M + 4 * statistics.mean(s["nnz"] for s in sets)
                            if cfg["csr"] else 0)
    dom = "dense" if kernel_ms.get("dense") else "spmm_csr"
    dom_ms = kernel_ms.get(dom)
    # bound of the dominant kernel: HBM bytes vs dense tensor FLOPs (counted once,
    # whatever the operand split multiplies them into)
    flops = 2.0 * T * M * K * N
    tensor_bound = dom == "dense" and flops / (pk["bf16_tflops"] * 1e12) > alg_dense / (pk["hbm_gbs"] * 1e9)
    if tensor_bound:
        achieved = flops / (dom_ms / 1e3) / 1e12 if dom_ms else None
        roof = {"bound": "tensor", "achieved": round(achieved, 1) if achieved else None, "peak": pk["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(achieved / pk["bf16_tflops"], 4) if achieved else None,
                "alg_flops_per_launch": flops, "traffic": None}
    else:
        achieved = alg_dense / (dom_ms / 1e3) / 1e9 if dom_ms else None
        roof = {"bound": "hbm", "achieved": round(achieved, 1) if achieved else None, "peak": pk["hbm_gbs"],
                "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4) if achieved else None,
                "alg_bytes_per_launch": int(alg_dense),
                "traffic": profile_traffic(cfg["traffic_profile"]) if cfg.get("traffic_profile") else None}
    step_ms = ms_max / args.steps
    res = {
        "metric": METRIC, "value": round(value, 2), "unit": "GSOP/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32" if cfg["w_dtype"] == "f32" else "bf16", "data": "synthetic",
        "config": {"workload": cfg["name"], "T": T, "M": M, "K": K, "N": N, "p": cfg["p"], "w_dtype": cfg["w_dtype"],
                   "csr_per_plane": cfg["csr"], "branch": branch, "per_rank_rows": T * M,
                   "l2": f"{nsets} rotating input sets ({nsets * set_bytes / 2**20:.0f} MiB > 126 MiB L2)",
                   "timing": "CUDA graph per input set, CUDA events, max over ranks"},
        "step_gbs": round(alg_step / (step_ms / 1e3) / 1e9, 1),
        "step_hbm_frac": round(alg_step / (step_ms / 1e3) / 1e9 / pk["hbm_gbs"], 4),
        "kernel_ms": {k: round(v, 5) for k, v in kernel_ms.items()},
        "roofline": {"kernel": (("spike_linear_wt_kernel" if N > 64 else "spike_linear_tf32_kernel")
                                if cfg["w_dtype"] == "f32" else "spike_linear_tc_kernel")
                     if dom == "dense" else "spmm_csr_kernel", **roof, "peak_src": pk["src"]},
        "gpu_launches": int(round(launches_per_step * args.steps)),
        "parity_rel_err": parity,
        "clocks": clocks.summary(),
        "e2e": e2e,
    }
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_spike_linear(cfg, sets[0]["S"], W)
    return res


def spike_linear_e2e(args, dist, cfg, W, sets, branch):
    """Same metric through ops.spike_linear from pinned host buffers: every step
    copies its S in (H2D) and its Y and CSR out (D2H); copies and compute run on
    separate streams, double-buffered."""
    from spikestack_lite_b200 import ops

    dev = W.device
    T, M, K, N = cfg["T"], cfg["M"], cfg["K"], cfg["N"]
    hosts = [s["S"].cpu().pin_memory() for s in sets[:2]]
    dS = [torch.empty_like(sets[0]["S"]) for _ in range(2)]
    cap = max(s["csr"]["col_idx"].numel() for s in sets) if cfg["csr"] else 0
    csrs = [ops.alloc_csr(T, M, K, dev, capacity=cap) if cfg["csr"] else None for _ in range(2)]
    hY = [torch.empty(T, M, N, dtype=torch.float32).pin_memory() for _ in range(2)]
    hC = [torch.empty(cap, dtype=torch.int32).pin_memory() if cfg["csr"] else None for _ in range(2)]
    hR = [torch.empty(T * (M + 1), dtype=torch.int32).pin_memory() if cfg["csr"] else None for _ in range(2)]
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.current_stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_cmp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    h2d = hosts[0].numel() * 4
    d2h = T * M * N * 4 + ((cap + T * (M + 1)) * 4 if cfg["csr"] else 0)

    def one(i, record=None):
        b = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_cmp[b])  # buffer b free (its previous compute done)
            dS[b].copy_(hosts[b], non_blocking=True)
            ev_in[b].record(s_in)
        s_cmp.wait_event(ev_in[b])
        s_cmp.wait_event(ev_out[b])  # previous readback of buffer b done
        Y = ops.spike_linear(dS[b], weightT=W, csr=csrs[b], branch=branch)
        ev_cmp[b].record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_cmp[b])
            hY[b].copy_(Y, non_blocking=True)
            if csrs[b] is not None:
                hC[b].copy_(csrs[b]["col_idx"][:cap], non_blocking=True)
                hR[b].copy_(csrs[b]["row_ptr"], non_blocking=True)
            Y.record_stream(s_out)
            ev_out[b].record(s_out)

    for i in range(max(2, args.warmup)):
        one(i)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(3, args.steps // 2)
    dist.barrier()
    torch.cuda.synchronize()
    start.record(s_in)
    for i in range(steps):
        one(i)
    stop.record(s_out)
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(start.elapsed_time(stop))
    nnz = statistics.mean(s["nnz"] for s in sets[:2])
    return {"value": round(dist.world * nnz * N * steps / (ms / 1e3) / 1e9, 2), "unit": "GSOP/s",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "ms_per_step": round(ms / steps, 4), "api": "spikestack_lite_b200.ops.spike_linear"}


def cpu_baseline_spike_linear(cfg, S_dev, W, budget_s=10.0):
    """The reference's CPU path (torch.matmul fallback, sparse/__init__.py:104-105,
    restated in oracle/) on a bounded sample, all host threads."""
    from oracle import spk_oracle as O

    torch.set_num_threads(host_threads())
    S = S_dev.cpu()
    Wc = W.float().cpu()
    nnz = float((S > 0).sum().item())
    O.reference_cpu_step(S, Wc)
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        O.reference_cpu_step(S, Wc)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(nnz * cfg["N"] / t / 1e9, 3), "unit": "GSOP/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"full step ({cfg['T']}x{cfg['M']}x{cfg['K']}), median of {len(times)} runs",
            "ms_per_step": round(t * 1e3, 3)}


def run_reference_spike_linear(args, dist, cfg):
    """--impl reference: the reference's CPU implementation, rank 0 only."""
    from oracle import spk_oracle as O

    torch.set_num_threads(host_threads())
    g = torch.Generator().manual_seed(1234)
    T, M, K, N = cfg["T"], cfg["M"], cfg["K"], cfg["N"]
    W = torch.randn(K, N, generator=g) / K ** 0.5
    S = (torch.rand(T, M, K, generator=g) < cfg["p"]).float()
    nnz = float((S > 0).sum().item())
    for _ in range(args.warmup):
        O.reference_cpu_step(S, W)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.reference_cpu_step(S, W)
    dt = time.perf_counter() - t0
    v = round(nnz * N * args.steps / dt / 1e9, 3)
    return {"metric": METRIC, "value": v, "unit": "GSOP/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": cfg["name"], "T": T, "M": M, "K": K, "N": N, "p": cfg["p"],
                       "w_dtype": cfg["w_dtype"]},
            "cpu_baseline": {"value": v, "unit": "GSOP/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": "full step per iteration (reference CPU path: torch.matmul, no CSR)"},
            "e2e": {"value": v, "unit": "GSOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------- attention
def run_attention(args, dist, cfg):
    from spikestack_lite_b200 import _lib, ops

    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    TB, L, H, dh = cfg["T"] * cfg["B"], cfg["L"], cfg["H"], cfg["dh"]
    g = torch.Generator(device=dev).manual_seed(7 + dist.rank)
    q, k, v = ((torch.rand(TB, L, H * dh, generator=g, device=dev) < cfg["p"]).float() for _ in range(3))
    lam = torch.sigmoid(torch.empty(H * dh, device=dev).uniform_(5.0, 8.0, generator=g))
    for _ in range(args.warmup):
        ops.spiking_attention(q, k, v, lam, H)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    start.record()
    for _ in range(args.steps):
        ops.spiking_attention(q, k, v, lam, H)
    stop.record()
    torch.cuda.synchronize()
    ms = dist.max(start.elapsed_time(stop)) / args.steps
    kms = {}
    for kn in ("attn_kv", "attn_out"):
        _lib.profile_begin(kn)
        for _ in range(max(3, args.steps // 4)):
            ops.spiking_attention(q, k, v, lam, H)
        tot, n = _lib.profile_end()
        kms[kn] = tot / max(n, 1)
    bytes_ = 4 * 4 * TB * L * H * dh
    pk = peaks()
    tokens = cfg["B"] * L
    return {"metric": METRIC, "value": round(dist.world * tokens / (ms / 1e3), 1), "unit": "tokens/s",
            "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfg["name"], **{k_: cfg[k_] for k_ in ("T", "B", "L", "H", "dh", "p")}},
            "kernel_ms": {k_: round(v_, 4) for k_, v_ in kms.items()},
            "roofline": {"kernel": "attention (kv + out)", "bound": "hbm",
                         "achieved": round(bytes_ / (ms / 1e3) / 1e9, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(bytes_ / (ms / 1e3) / 1e9 / pk["hbm_gbs"], 4)}}


# ------------------------------------------------------------ linear + activation
# tcgen05 kind::tf32 rate on one SM, measured with back-to-back 128x128x8 MMAs
# (A in TMEM, B in shared memory): 4096 FLOP per clock.
TF32_FLOP_PER_CLK_SM = 4096


def run_linear(args, dist, cfg):
    """The C5 SpikingFFN fc1 with its threshold spike: act = (x W1^T + b - thr > 0)
    over x [T*B*N, d] (ops.linear_act: a tf32 pass and a bf16 correction pass
    over doubled K for fp32 accuracy, the tensor work of two tf32 passes)."""
    from spikestack_lite_b200 import _lib, ops

    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    R, K, N = cfg["R"], cfg["K"], cfg["N"]
    if args.batch is not None:
        R = args.batch * cfg["rows_per_batch"]
    g = torch.Generator(device=dev).manual_seed(11 + dist.rank)
    x = torch.randn(R, K, generator=g, device=dev)
    w = torch.randn(N, K, generator=g, device=dev) / K ** 0.5
    b = torch.randn(N, generator=g, device=dev) * 0.1
    out = torch.empty(R, N, device=dev)

    def step():
        return ops.linear_act(x, w, b, act="heaviside", thr=cfg["thr"])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if args.quick:
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize()
        return {"workload": cfg["name"], "quick": True, "steps": args.steps}
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        dist.barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            out = step()
        stop.record()
        torch.cuda.synchronize()
        dist.barrier()
    ms = dist.max(start.elapsed_time(stop)) / args.steps
    _lib.profile_begin("dense")
    for _ in range(max(3, args.steps // 2)):
        step()
    tot, n = _lib.profile_end()
    kms = tot / max(n, 1)
    # parity spot check: spikes of 256 rows against the fp64 decision away from the threshold
    pre = (x[:256].double() @ w.double().t() + b.double()) - cfg["thr"]
    near = pre.abs() < 1e-5 * pre.abs().max()
    mism = int(((out[:256] > 0) != (pre > 0))[~near].sum().item())
    flops = 2.0 * R * K * N                      # the fp32 GEMM's FLOPs
    tf32_work = 2 * flops                        # tf32 pass + bf16 pass (2K at twice the rate)
    clk = clocks.summary().get("sm_mhz") or 1965.0
    peak_tf32 = TF32_FLOP_PER_CLK_SM * 148 * clk * 1e6 / 1e12
    ach = tf32_work / (kms / 1e3) / 1e12
    return {"metric": METRIC, "value": round(dist.world * flops / (ms / 1e3) / 1e12, 2), "unit": "TFLOP/s (fp32 GEMM)",
            "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfg["name"], "R": R, "K": K, "N": N, "thr": cfg["thr"],
                       "timing": "eager steps (weight image + linear kernel), CUDA events, max over ranks"},
            "kernel_ms": {"linear": round(kms, 4)},
            "roofline": {"kernel": "spike_linear_wt_kernel<heaviside>", "bound": "tensor",
                         "achieved": round(ach, 1), "peak": round(peak_tf32, 1), "unit": "TFLOP/s (tf32)",
                         "frac": round(ach / peak_tf32, 4), "alg_flops_per_launch": tf32_work, "traffic": None,
                         "peak_src": "tcgen05 tf32 probe rate x 148 SMs x median SM clock"},
            "parity_spike_mismatches": mism, "clocks": clocks.summary()}


def run_layernorm(args, dist, cfg):
    """The pre-norm block's residual add + layer norm at the C5 chunk geometry:
    h = x + delta, y = LayerNorm(h) over d (ops.add_layernorm, one pass)."""
    from spikestack_lite_b200 import ops

    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    d = cfg["d"]
    R = (args.batch if args.batch is not None else cfg["batch"]) * cfg["rows_per_batch"]
    g = torch.Generator(device=dev).manual_seed(21 + dist.rank)
    x = torch.randn(R, d, generator=g, device=dev)
    delta = torch.randn(R, d, generator=g, device=dev)
    w = torch.randn(d, generator=g, device=dev)
    b = torch.randn(d, generator=g, device=dev)

    def step():
        return ops.add_layernorm(x, delta, w, b, 1e-5)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if args.quick:
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize()
        return {"workload": cfg["name"], "quick": True, "steps": args.steps}
    # one launch per step, replayed from a CUDA graph (no allocation or host work in the timed region)
    gph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gph):
        h, y = step()
    gph.replay()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        dist.barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            gph.replay()
        stop.record()
        torch.cuda.synchronize()
        dist.barrier()
    ms = dist.max(start.elapsed_time(stop)) / args.steps
    ref = torch.nn.functional.layer_norm(x[:4096] + delta[:4096], (d,), w, b, 1e-5)
    err = float((y[:4096] - ref).abs().max().item())
    alg = 16.0 * R * d                            # x, delta read; h, y written
    pk = peaks()
    gbs = alg / (ms / 1e3) / 1e9
    return {"metric": METRIC, "value": round(dist.world * gbs, 1), "unit": "GB/s", "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfg["name"], "rows": R, "d": d,
                       "l2": f"4 tensors of {R * d * 4 / 2**20:.0f} MiB > 126 MiB L2",
                       "timing": "one launch per step replayed from a CUDA graph, CUDA events, max over ranks"},
            "roofline": {"kernel": "add_layernorm_kernel", "bound": "hbm", "achieved": round(gbs, 1),
                         "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(gbs / pk["hbm_gbs"], 4),
                         "alg_bytes_per_launch": int(alg), "traffic": None, "peak_src": pk["src"]},
            "max_abs_err_vs_torch": err, "clocks": clocks.summary()}


# ------------------------------------------------------------------- model
def model_config(cfg, world):
    """The model line's `config` (identical for both arms)."""
    mc = cfg["model"]
    return {"workload": cfg["name"], "global_batch": cfg["batch"], "seq_len": mc["seq_len"],
            "input_dim": mc["input_dim"], "d_model": mc["d_model"], "layers": mc["num_layers"],
            "heads": mc["num_heads"], "T": mc["n_repeats"], "gsmc": bool(mc.get("use_gsmc", False)),
            "parallelism": f"batch-sharded over {world} GPU(s), NCCL all_gather of the logits",
            "l2": "inputs larger than L2: every chunk's activations are >= 1 GiB (126 MiB L2)"}


def model_inputs(cfg):
    """x ~ N(0, 1) fp32 [batch, seq, input_dim], seeded (host tensor)."""
    mc = cfg["model"]
    g = torch.Generator().manual_seed(1)
    return torch.randn(cfg["batch"], mc["seq_len"], mc["input_dim"], generator=g)


def build_model(cfg, dev):
    """Random-init weights from torch.manual_seed(0), as the reference builds the model."""
    from spikestack_lite_b200.transformer import SpikingTransformer

    torch.manual_seed(0)
    return SpikingTransformer(**cfg["model"]).to(dev).eval()


def model_cpu_sample(cfg, sd, x, n):
    """The reference's CPU forward (restated in oracle/: the reference's own
    PyTorch CPU arithmetic, pinned to its golden models) on the first n samples."""
    from oracle import spk_oracle as O

    mc = cfg["model"]
    return O.transformer_forward(sd, x[:n], mc["num_heads"], mc["num_layers"], use_gsmc=mc.get("use_gsmc", False),
                                 spike_readout=True, threshold=mc.get("spike_threshold", 0.0))


def time_cpu_model(cfg, sd, x, n, budget_s=None, steps=None, warmup=1):
    """Seconds per call of model_cpu_sample over n samples: median within a time
    budget, or the mean of `steps` calls after `warmup`."""
    torch.set_num_threads(host_threads())
    for _ in range(warmup):
        model_cpu_sample(cfg, sd, x, n)
    times = []
    if steps is not None:
        t0 = time.perf_counter()
        for _ in range(steps):
            model_cpu_sample(cfg, sd, x, n)
        return (time.perf_counter() - t0) / steps, steps
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        model_cpu_sample(cfg, sd, x, n)
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times)


def model_kernel_profile(model, xc):
    """One eager chunk forward with the engine's per-class launch timing (CUDA
    events on the launch stream) and the tally of its contractions."""
    from spikestack_lite_b200 import _lib, ops

    prof = {}
    for kname in ("dense", "attn_kv", "attn_out", "gsmc_step", "w_image"):
        _lib.profile_begin(kname)
        with ops.tally() as tl:
            model(xc)
        tot, n = _lib.profile_end()
        prof[kname] = (tot, n)
    torch.cuda.synchronize()
    return prof, tl


def run_model(args, dist, cfg):
    from spikestack_lite_b200 import _lib
    from spikestack_lite_b200.graphs import CapturedForward

    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    model = build_model(cfg, dev)
    mc = cfg["model"]
    B = cfg["batch"]
    lo, hi = shard_bounds(B, dist.rank, dist.world)
    x_all = model_inputs(cfg)
    x = x_all[lo:hi].to(dev)  # this rank's samples, resident before the timed region
    chunk = min(cfg.get("chunk", hi - lo), hi - lo)
    if (hi - lo) % chunk:
        raise SystemExit(f"{hi - lo} samples per rank do not split into chunks of {chunk}")
    n_chunks = (hi - lo) // chunk
    launches0 = _lib.launch_count()
    with torch.no_grad():
        fwd_chunk = CapturedForward(model, x[:chunk])  # one graph per chunk shape, replayed for every chunk
    launches_per_chunk = (_lib.launch_count() - launches0) // 2  # the eager warm-up call, then the capture

    def fwd(xs):
        local = torch.cat([fwd_chunk(xs[i * chunk:(i + 1) * chunk]).clone() for i in range(n_chunks)])
        return dist.gather_rows(local)  # NCCL all_gather of the logits: the only collective

    stream = torch.cuda.current_stream(dev)
    with torch.no_grad():
        for _ in range(args.warmup):
            fwd(x)
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index) as clocks:
            dist.barrier()
            torch.cuda.synchronize()
            start.record(stream)
            for _ in range(args.steps):
                logits = fwd(x)
            stop.record(stream)
            torch.cuda.synchronize()
            dist.barrier()
        ms = dist.max(start.elapsed_time(stop)) / args.steps
        prof, tl = model_kernel_profile(model, x[:chunk])
        e2e = model_e2e(args, dist, fwd_chunk, x_all[lo:hi], chunk, n_chunks, mc["num_classes"])
    tokens = B * mc["seq_len"]
    res = {"metric": METRIC, "value": round(tokens / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": dist.world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic: x ~ N(0,1) seeded, random-init weights from torch.manual_seed(0)",
           "config": model_config(cfg, dist.world),
           "timing": (f"forward of each {chunk}-sample chunk replayed from one CUDA graph "
                      "(spikestack_lite_b200.graphs.CapturedForward), logits all_gather inside the region, "
                      "CUDA events, max over ranks"),
           "gpu_launches": int(launches_per_chunk * n_chunks * args.steps),
           "clocks": clocks.summary(), "e2e": e2e}
    res.update(model_roofline(prof, tl, mc))
    res["logits_checksum"] = float(logits.double().sum().item())
    if dist.rank == 0:
        sd = {k: v.detach().cpu() for k, v in model.state_dict().items()}
        n_par = 2
        with torch.no_grad():
            got = fwd_chunk(x[:chunk])[:n_par].cpu().numpy()
        from oracle import spk_oracle as O

        ref = model_cpu_sample(cfg, sd, x_all, n_par).numpy()
        res["parity"] = {"logits_rel_err": O.rel_err(got, ref), "samples": n_par,
                         "vs": "oracle CPU forward (the reference's arithmetic) on the same weights and inputs"}
        if dist.world == 1 and not args.no_cpu_baseline:
            n_cpu = 2
            t, runs = time_cpu_model(cfg, sd, x_all, n_cpu, budget_s=12.0)
            res["cpu_baseline"] = {"value": round(n_cpu * mc["seq_len"] / t, 1), "unit": "tokens/s",
                                   "cores": torch.get_num_threads(), "kind": "port",
                                   "sample": f"{n_cpu} of {B} samples per forward (samples are independent), "
                                             f"median of {runs} runs",
                                   "ms_per_sample_forward": round(t * 1e3 / n_cpu, 1)}
    return res


def model_e2e(args, dist, fwd_chunk, x_host, chunk, n_chunks, n_classes):
    """The same metric through the public forward (CapturedForward / the
    model's __call__) from pinned host inputs: every step copies each chunk of
    this rank's samples host->device (a copy stream, two buffers, so chunk
    i+1 crosses PCIe while chunk i computes), gathers the logits over NCCL and
    reads them back to the host on rank 0."""
    dev = torch.device("cuda", dist.local)
    pinned = x_host.contiguous().pin_memory()
    dbuf = [torch.empty((chunk,) + tuple(pinned.shape[1:]), device=dev) for _ in range(2)]
    s_copy = torch.cuda.Stream(dev)
    stream = torch.cuda.current_stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    for e in ev_used:
        e.record(stream)
    host_logits = torch.empty((n_chunks * chunk * dist.world, n_classes)).pin_memory()

    def step():
        s_copy.wait_stream(stream)
        outs = []
        for i in range(n_chunks):
            b = i % 2
            with torch.cuda.stream(s_copy):
                s_copy.wait_event(ev_used[b])
                dbuf[b].copy_(pinned[i * chunk:(i + 1) * chunk], non_blocking=True)
                ev_in[b].record(s_copy)
            stream.wait_event(ev_in[b])
            outs.append(fwd_chunk(dbuf[b]).clone())
            ev_used[b].record(stream)
        logits = dist.gather_rows(torch.cat(outs))
        if dist.rank == 0:
            host_logits.copy_(logits, non_blocking=True)

    with torch.no_grad():
        for _ in range(2):
            step()
        torch.cuda.synchronize()
        steps = max(3, args.steps // 2)
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(steps):
            step()
        stop.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
    ms = dist.max(start.elapsed_time(stop)) / steps
    tokens = n_chunks * chunk * dist.world * pinned.shape[1]
    return {"value": round(tokens / (ms / 1e3), 1), "unit": "tokens/s",
            "h2d_bytes_per_step": int(pinned.numel() * 4 * dist.world),
            "d2h_bytes_per_step": int(host_logits.numel() * 4), "ms_per_step": round(ms, 3), "steps": steps,
            "api": "spikestack_lite_b200.graphs.CapturedForward over SpikingTransformer (pinned host x in, "
                   "logits out)", "copies": "all ranks' inputs H2D (whole job), gathered logits D2H on rank 0"}


def model_roofline(prof, tl, mc):
    """Roofline of the dominant kernel class: the tcgen05 contractions
    (spike_linear_wt_kernel instances: the fp32-accurate linear op and the
    spike-linear), tensor-bound at this geometry."""
    pk = peaks()
    tot, n = prof["dense"]
    flops = tl.flops()  # algorithmic: 2*rows*K*N of every contraction in one chunk forward
    # tensor-core work in tf32-pass equivalents: the linear op issues one tf32 pass and one bf16
    # correction pass over twice the K at twice the rate (= one tf32 pass), spike-linear on fp32
    # spikes two tf32 passes, on packed spikes three bf16 passes (the three-way split of W) = 1.5
    passes = sum((1.5 if op == "spike_linear_bits" else 2.0) * 2.0 * r * k * nn for op, r, k, nn in tl.calls)
    peak = pk["bf16_tflops_sustained"] / 2.0
    ach = flops / (tot / 1e3) / 1e12 if tot else None
    other = {k: round(v[0], 3) for k, v in prof.items()}
    return {
        "roofline": {"kernel": "spike_linear_wt_kernel (linear-op and spike-linear instances)", "bound": "tensor",
                     "achieved": round(ach, 1) if ach else None, "peak": round(peak, 1), "unit": "TFLOP/s",
                     "frac": round(ach / peak, 4) if ach else None,
                     "alg_flops_per_launch": round(flops / max(n, 1)), "launches_per_chunk": n,
                     "traffic": None,
                     "peak_src": f"{pk['src']} bf16 sustained {pk['bf16_tflops_sustained']} TFLOP/s / 2 "
                                 "(the tf32 dense rate is half the bf16 rate)",
                     "tf32_pass_frac": round(passes / (tot / 1e3) / 1e12 / peak, 4) if tot else None,
                     "note": "achieved counts each fp32 GEMM's 2*rows*K*N once; for fp32 accuracy the kernel "
                             "issues the work of 2 tf32 passes (linear op: a tf32 pass plus a bf16 correction pass "
                             "over doubled K; spike-linear on fp32 spikes: tf32 hi and lo) or 1.5 (packed spikes: "
                             "three bf16 passes over the split of W), tf32_pass_frac counts them"},
        "kernel_ms_per_chunk": other,
    }


def run_crossover(args, dist, cfg):
    """Density sweep S[4, 65536, 2048], W[2048, 2048] bf16: step time of the
    dense branch, the CSR branch and the automatic choice at each density
    (each step replayed from a CUDA graph over two rotating input sets of
    2.1 GB each, CUDA events)."""
    from spikestack_lite_b200 import _lib, ops

    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    T, M, K, N = cfg["T"], cfg["M"], cfg["K"], cfg["N"]
    g = torch.Generator(device=dev).manual_seed(77 + dist.rank)
    W = (torch.randn(K, N, generator=g, device=dev) / K ** 0.5).to(torch.bfloat16)
    pk = peaks()
    table = []
    for p in cfg["densities"]:
        sets = [(torch.rand(T, M, K, generator=g, device=dev) < p).float() for _ in range(2)]
        nnz = statistics.mean(int((S > 0).sum().item()) for S in sets)
        row = {"p": p, "nnz": int(nnz)}
        for br in ("dense", "csr", "auto"):
            for i in range(2):
                ops.spike_linear(sets[i], weightT=W, branch=br)
            torch.cuda.synchronize()
            graphs = []
            for i in range(2):
                gph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gph):
                    ops.spike_linear(sets[i], weightT=W, branch=br)
                graphs.append(gph)
            steps = args.steps
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            for i in range(2):
                graphs[i].replay()
            torch.cuda.synchronize()
            start.record()
            for i in range(steps):
                graphs[i % 2].replay()
            stop.record()
            torch.cuda.synchronize()
            row[f"{br}_ms"] = round(dist.max(start.elapsed_time(stop)) / steps, 4)
            del graphs
        _lib.profile_begin("dense")
        for i in range(3):
            ops.spike_linear(sets[i % 2], weightT=W, branch="dense")
        tot, n = _lib.profile_end()
        dense_kernel_ms = tot / max(n, 1)
        row["dense_kernel_tflops"] = round(2.0 * T * M * K * N / (dense_kernel_ms / 1e3) / 1e12, 1)
        row["dense_tensor_frac"] = round(row["dense_kernel_tflops"] / pk["bf16_tflops"], 4)
        row["faster"] = "csr" if row["csr_ms"] < row["dense_ms"] else "dense"
        row["auto_took"] = "csr" if abs(row["auto_ms"] - row["csr_ms"]) < abs(row["auto_ms"] - row["dense_ms"]) else "dense"
        row["gsops"] = round(nnz * N / (min(row["auto_ms"], 1e9) / 1e3) / 1e9, 1)
        table.append(row)
        del sets
        torch.cuda.empty_cache()
    return {"metric": METRIC, "value": None, "unit": "ms", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": False, "dtype": "bf16 W, fp32 S / accumulate",
            "data": "synthetic", "config": {"workload": cfg["name"], "T": T, "M": M, "K": K, "N": N,
                                            "timing": "CUDA graph per input set (2 sets of 2.1 GB), CUDA events"},
            "peak_bf16_tflops": pk["bf16_tflops"], "crossover": table}


def run_gsmc(args, dist, cfg):
    """The GSMC recurrence at the model's chunk geometry (M = 64 samples x
    1024 tokens, d = 512, T = 4): the two-kernel form (gr through the
    spike-linear dense branch, then the step kernel) against the fused form
    (one kernel per plane, gates in the epilogue), CUDA events."""
    from spikestack_lite_b200 import ops

    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    T, M, d = cfg["T"], cfg["M"], cfg["d"]
    g = torch.Generator(device=dev).manual_seed(5)
    gi = torch.randn(T, M, 4 * d, generator=g, device=dev) * 2.0
    wd = torch.randn(T, M, d, generator=g, device=dev) * 0.5
    w_rec = torch.randn(4 * d, d, generator=g, device=dev) * (0.5 / d ** 0.5)
    bias = torch.randn(4 * d, generator=g, device=dev)
    res = {}
    outs = {}
    for form in ("two_kernel", "fused"):
        f = form == "fused"
        for _ in range(args.warmup):
            ops.gsmc_forward(gi, wd, w_rec, bias, fused=f)
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            outs[form] = ops.gsmc_forward(gi, wd, w_rec, bias, fused=f)
        stop.record()
        torch.cuda.synchronize()
        res[form + "_ms"] = round(dist.max(start.elapsed_time(stop)) / args.steps, 4)
    same = bool(torch.equal(outs["two_kernel"], outs["fused"]))
    return {"metric": METRIC, "value": res["two_kernel_ms"], "unit": "ms", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": False, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfg["name"], "T": T, "M": M, "d": d}, **res,
            "fused_equals_two_kernel": same,
            "gr_bytes_not_written_per_plane": 2 * 4 * M * 4 * d}


def run_reference_model(args, dist, cfg):
    """--impl reference for the model: the reference's CPU forward (restated in
    oracle/, the reference's own PyTorch CPU arithmetic) on a sample of the
    batch, all host threads, rank 0 only; samples are independent, so tokens/s
    of the sample is the CPU path's throughput on the whole batch."""
    model = build_model(cfg, torch.device("cpu"))
    sd = {k: v.detach() for k, v in model.state_dict().items()}
    x_all = model_inputs(cfg)
    n = 2
    t, _ = time_cpu_model(cfg, sd, x_all, n, steps=args.steps, warmup=args.warmup)
    seq = cfg["model"]["seq_len"]
    v = round(n * seq / t, 1)
    return {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t * 1e3, 1), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: x ~ N(0,1) seeded, random-init weights from torch.manual_seed(0)",
            "impl": "reference", "config": model_config(cfg, dist.world),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"each step one CPU forward of {n} of the {cfg['batch']} samples"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


NESTED_KEYS = ("value", "unit", "ms_per_step", "config", "step_gbs", "step_hbm_frac", "kernel_ms", "roofline",
               "gpu_launches", "parity_rel_err", "clocks", "e2e", "cpu_baseline", "scaling")


WORKLOADS = {
    "spike_linear": {"name": "isolated spike-linear S[3,16384,512] p=0.10, W[512,128] fp32, CSR per plane",
                     "T": 3, "M": 16384, "K": 512, "N": 128, "p": 0.10, "w_dtype": "f32", "csr": True},
    "sweep": {"name": "spike-linear density sweep S[4,65536,2048], W[2048,2048] bf16", "T": 4, "M": 65536,
              "K": 2048, "N": 2048, "p": 0.10, "w_dtype": "bf16", "csr": False},
    "crossover": {"name": "spike-linear density sweep S[4,65536,2048], W[2048,2048] bf16: dense vs CSR vs auto",
                  "T": 4, "M": 65536, "K": 2048, "N": 2048,
                  "densities": [0.01, 0.02, 0.05, 0.1, 0.2, 0.35, 0.5]},
    "gsmc": {"name": "GSMC recurrence at the model's chunk geometry: M = 65536, d = 512, T = 4", "T": 4,
             "M": 65536, "d": 512},
    "linear": {"name": "C5 SpikingFFN fc1 + threshold spike: x[4*512*1024, 512] -> [.., 2048]", "R": 4 * 512 * 1024,
               "rows_per_batch": 4 * 1024, "K": 512, "N": 2048, "thr": 0.0},
    "attention": {"name": "spiking linear attention B=64 H=8 L=4096 dh=64 T=4 p=0.15", "T": 4, "B": 64,
                  "L": 4096, "H": 8, "dh": 64, "p": 0.15},
    "layernorm": {"name": "block residual add + layer norm, C5 chunk: [4*64*1024, 512]", "batch": 64,
                  "rows_per_batch": 4 * 1024, "d": 512},
    "model_small": {"name": "SpikingTransformer fwd, batch 256, seq 64, d 128, 1 layer, T=3", "batch": 256,
                    "model": dict(input_dim=48, d_model=128, seq_len=64, num_classes=10, num_heads=4, num_layers=1,
                                  n_repeats=3, temporal=True, expansion=4, use_spikeskip=True)},
    "model_full": {"name": "SpikingTransformer fwd, batch 512, seq 1024, d 512, 6 layers, T=4, GSMC", "batch": 512,
                   "chunk": 64,
                   "model": dict(input_dim=256, d_model=512, seq_len=1024, num_classes=10, num_heads=8,
                                 num_layers=6, n_repeats=4, temporal=True, expansion=4, use_gsmc=True,
                                 use_exact=True, use_spikeskip=True)},
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="model_full", choices=sorted(WORKLOADS))
    ap.add_argument("--p", type=float, default=None, help="spike density override")
    ap.add_argument("--branch", default="dense", choices=["auto", "dense", "csr"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quick", action="store_true", help="eager steps only, no JSON metrics (profiling case)")
    ap.add_argument("--eager", action="store_true", help="model workloads: eager forward instead of a CUDA graph")
    ap.add_argument("--rows", type=int, default=None, help="override M (rows per plane) of spike-linear workloads")
    ap.add_argument("--batch", type=int, default=None, help="override B of the attention workload")
    ap.add_argument("--no-nested", action="store_true",
                    help="model workload: skip the nested isolated spike-linear measurement")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    cfg = dict(WORKLOADS[args.workload])
    if args.p is not None:
        cfg["p"] = args.p
    if args.rows is not None:
        cfg["M"] = args.rows
        cfg["name"] += f" (M overridden to {args.rows})"
    if args.workload == "spike_linear" and args.rows is None and args.p is None:
        cfg["traffic_profile"] = "spike_linear_dense_c2"  # the ncu capture of this exact configuration
    if args.batch is not None and "B" in cfg:
        cfg["B"] = args.batch
        cfg["name"] += f" (B overridden to {args.batch})"
    dist = RankGroup("nccl")

    if args.impl == "reference":
        if dist.rank != 0:
            return
        if args.workload == "model_full":
            res = run_reference_model(args, dist, cfg)
            if not args.no_nested:
                sub = run_reference_spike_linear(args, dist, dict(WORKLOADS["spike_linear"]))
                res["spike_linear"] = {k: sub[k] for k in ("value", "unit", "ms_per_step", "config", "cpu_baseline")}
            print(json.dumps(res), flush=True)
            return
        if args.workload != "spike_linear":
            print(json.dumps({"impl": "reference", "unavailable": "reference arm implemented for the model and "
                              "the isolated spike-linear workloads only"}))
            return
        print(json.dumps(run_reference_spike_linear(args, dist, cfg)), flush=True)
        return

    dist.init()
    try:
        if args.workload in ("spike_linear", "sweep"):
            res = run_spike_linear(args, dist, cfg)
        elif args.workload == "gsmc":
            res = run_gsmc(args, dist, cfg)
        elif args.workload == "crossover":
            res = run_crossover(args, dist, cfg)
        elif args.workload == "attention":
            res = run_attention(args, dist, cfg)
        elif args.workload == "linear":
            res = run_linear(args, dist, cfg)
        elif args.workload == "layernorm":
            res = run_layernorm(args, dist, cfg)
        else:
            res = run_model(args, dist, cfg)
            if args.workload == "model_full" and not args.no_nested:
                c2 = dict(WORKLOADS["spike_linear"], traffic_profile="spike_linear_dense_c2")
                sub = run_spike_linear(args, dist, c2)
                res["spike_linear"] = {k: sub[k] for k in NESTED_KEYS if k in sub}
                res["gpu_launches"] += sub.get("gpu_launches", 0)
        if dist.rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
