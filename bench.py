"""Benchmark of vllm-exact B200: exact_int8 GEMM throughput against the roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload ("step"): the decode part of the BASELINE configs[1] sweep on one B200 -- for M in {1, 16, 64} and
each (K, N) in {QKV (4096, 6144), O-proj (4096, 4096), gate_up (4096, 24576), down (12288, 4096), lm_head
(4096, 151936)}: bf16 activations -> digitize -> exact two-digit GEMM -> bf16 output (the exactmm::linear op).
value = algorithmic HBM bytes of the 15 GEMMs (weight digits 2NK + weight scales 4N + activation digits 2MK + row
scales 4M + bf16 output 2MN) / device time of the step, in TB/s. Weights of one (K, N) are re-used only after the four
other matrices (>= 1.5 GB) went through the 126 MB L2, so every step streams its weights from HBM.

Also reported (not part of `value`): per-layer chains of the decode shapes beside the reference's own Triton op on the
same inputs with a bitwise comparison (`sweep_decode`), the tensor-bound sweep M in {256, 4096} as executed
digit-product ops (6 M N K) against an INT8 dense peak measured in the run (and the bf16 peak), the paged decode
attention of configs[3], config 5's hot-path share against cuBLAS bf16 (`decode_step`) and through the real vLLM
engine (`engine`), the end-to-end rate through the public op with host copies, and the SM clocks during the run.

After the timed region, rank 0 checks the step's outputs bit for bit against the CPU oracle on a row sample
(`bitwise_ok`) and times the reference's CPU integer path on a bounded sample (`cpu_baseline`).

--gpus N > 1 (under torchrun, one rank per GPU) runs the same step tensor-parallel: qkv, gate_up and lm_head
column-parallel, o_proj and down K-sharded with the exact int64 sum over peer memory or NCCL (the faster of the two),
every rank's outputs checked against the oracle of the unsharded layers; value = the step's bytes / its time, max
over ranks (strong scaling).

--impl reference times the reference's own CPU integer path (digitize_torch + exact_linear_torch from its
kernels.py, installed under baseline/_ref; the numpy restatement in oracle/ only if it is missing) on a bounded
sample of the same workload with all host threads, and prints the same metric.
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
from pathlib import Path

os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep NCCL's version banner off stdout: rank 0 prints one JSON line
ROOT = Path(__file__).resolve().parent
for p in (ROOT, ROOT / "vllm-exact_b200", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

SHAPES = [("qkv", 4096, 6144), ("o_proj", 4096, 4096), ("gate_up", 4096, 24576), ("down", 12288, 4096),
          ("lm_head", 4096, 151936)]
DECODE_M = [1, 16, 64]
TENSOR_M = [256, 4096]
ATTN = [(256, 1024), (64, 8192), (16, 16384)]
METRIC = "exact-GEMM TB/s (exact_int8 linear, decode shapes M<=64 of the configs[1] sweep)"
WORKLOAD = ("configs[1] decode sweep: M in {1,16,64} x (K,N) in {(4096,6144),(4096,4096),(4096,24576),"
            "(12288,4096),(4096,151936)}, F=14 truncated, bf16 out")
# DRAM bytes (read + write) per k_exact_tc_i8 launch, averaged over the 15 launches of one decode step, from the ncu
# capture summarised in profiles/k_exact_tc_i8__decode_sweep.md (1.007 x the algorithmic bytes).
GEMM_TRAFFIC_PER_LAUNCH = 331_005_542


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def gemm_bytes(M, K, N):
    return 2 * N * K + 4 * N + 2 * M * K + 4 * M + 2 * M * N


# ------------------------------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ------------------------------------------------------------------------------------------------------------------
class ClockSampler:
    """SM clock, power and throttle reasons during the timed region. Read-only NVML queries every 2 ms in a thread
    (a decode step is ~1 ms, so nvidia-smi's 200 ms period would see a short timed region once at most); nvidia-smi
    -lms 200 when NVML is not available. The GPU is found by the UUID torch reports, so CUDA_VISIBLE_DEVICES cannot
    make it sample another GPU."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.nvml = None
        self.stop = threading.Event()

    def _nvml_open(self):
        import pynvml as N
        import torch
        N.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.index).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        h = N.nvmlDeviceGetHandleByUUID(uuid)
        return N, h

    def _nvml_loop(self):
        N, h = self.nvml
        mx = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
        bits = [("hw_slowdown", N.nvmlClocksEventReasonHwSlowdown),
                ("hw_thermal_slowdown", N.nvmlClocksEventReasonHwThermalSlowdown),
                ("sw_thermal_slowdown", N.nvmlClocksEventReasonSwThermalSlowdown),
                ("sw_power_cap", N.nvmlClocksEventReasonSwPowerCap)]
        while not self.stop.is_set():
            try:
                sm = N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)
                pw = N.nvmlDeviceGetPowerUsage(h) / 1000.0
                r = N.nvmlDeviceGetCurrentClocksEventReasons(h)
                flags = ["Active" if r & b else "Not Active" for _, b in bits]
                self.lines.append(", ".join([str(sm), str(mx), f"{pw:.1f}", hex(r)] + flags))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        try:
            self.nvml = self._nvml_open()
            self.t = threading.Thread(target=self._nvml_loop, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first_sample(self, timeout=5.0):
        t = time.time()
        while (self.proc is not None or self.nvml is not None) and not self.lines and time.time() - t < timeout:
            time.sleep(0.02)

    def __exit__(self, *a):
        if self.nvml is not None:
            self.stop.set()
            self.t.join(timeout=2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, since=0, until=None):
        """Median SM clock, max clock and throttle reasons seen over the samples [since, until)."""
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[since:until]:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvml every 2 ms" if self.nvml is not None else "nvidia-smi -lms 200"}

    def mark(self):
        """Index of the next sample (for summary(since, until))."""
        return len(self.lines)


# ------------------------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------------------------
def make_activation(M, K, seed, dev):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=dev)
    x[torch.rand(M, K, generator=g, device=dev) < 0.001] *= 50
    return x.bfloat16()


def make_weight_digits(K, N, seed, dev, F=14):
    """Weights ~N(0, 0.02) in bf16, digitized at load time like the plugin (kernels.digitize_weight: generated and
    digitized in row blocks to bound memory, then marked static as digitize_weight marks its result)."""
    import torch
    from vllm_exact import kernels as KK
    g = torch.Generator(device=dev).manual_seed(seed)
    out = KK._alloc_digits(N, K, dev)
    for i in range(0, N, 16384):
        j = min(N, i + 16384)
        w = (torch.randn(j - i, K, generator=g, device=dev) * 0.02).bfloat16()
        KK.digitize(w, F, out=tuple(t[i:j] for t in out))
    KK.mark_static(*out)
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist
    from vllm_exact import kernels as KK, paged_attn as PA
    import vllm_exact.ops  # noqa: F401  (registers exactmm::linear without importing vLLM)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
        return run_tp(args, dev, rank, world, local)
    hbm, bf16_burst, bf16_sust, peak_kind = peaks()

    # ---------------- workload: weights resident in HBM, activations per (M, shape)
    W = {name: make_weight_digits(K, N, 1000 + i, dev) for i, (name, K, N) in enumerate(SHAPES)}
    X = {(M, name): make_activation(M, K, 17 * M + i, dev) for M in DECODE_M for i, (name, K, N) in enumerate(SHAPES)}
    Y = {(M, name): torch.empty(M, N, device=dev, dtype=torch.bfloat16) for M in DECODE_M for name, K, N in SHAPES}
    order = [(M, name, K, N) for M in DECODE_M for name, K, N in SHAPES]
    step_bytes = sum(gemm_bytes(M, K, N) for M, name, K, N in order)
    # the workspace for split tiles, sized for the largest plan, before timing
    KK.reserve_workspace(max(KK.lib().ex_linear_workspace_bytes(M, N, K, 0, 0) for M, _, K, N in order), dev)
    stream = torch.cuda.Stream(dev)
    KK.reserve_workspace(max(KK.lib().ex_linear_workspace_bytes(M, N, K, 0, 0) for M, _, K, N in order), dev,
                         stream=stream)

    def one_step():
        for M, name, K, N in order:
            KK.exact_linear(KK.digitize(X[(M, name)], 14), W[name], 14, True, out=Y[(M, name)])
        return 2 * len(order)

    # the same 15 GEMMs on digits computed once: the GEMM kernel alone, back to back (roofline timing basis)
    XD = {key: KK.digitize(x, 14) for key, x in X.items()}

    def gemm_step():
        for M, name, K, N in order:
            KK.exact_linear(XD[(M, name)], W[name], 14, True, out=Y[(M, name)])

    # CUDA graphs, as vLLM runs decode: graph A = one step; graph G = the step's GEMMs alone. No timing events inside
    # either graph: events between launches break the programmatic-dependent-launch overlap and add microseconds.
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            one_step()
            gemm_step()
    torch.cuda.synchronize()
    gA = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gA, stream=stream):
        launches_per_step = one_step()
    gG = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gG, stream=stream):
        gemm_step()
    for _ in range(args.warmup):
        gG.replay()
        gA.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t2, t3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t2.record()
        for _ in range(args.steps):
            gG.replay()
        t3.record()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        clk.wait_first_sample()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        c0 = clk.mark()
        with torch.cuda.stream(stream):
            t0.record()
            for _ in range(args.steps):
                gA.replay()
            t1.record()
        torch.cuda.synchronize()
        c1 = clk.mark()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1)
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt)
    gemm_ms = t2.elapsed_time(t3) / args.steps
    ms_per_step = ms / args.steps
    value = world * step_bytes / (ms_per_step * 1e-3) / 1e12
    achieved = step_bytes / (gemm_ms * 1e-3) / 1e9  # GB/s of the GEMM launches alone
    launches = {"n": launches_per_step * args.steps}
    del gG

    result = {
        "metric": METRIC, "value": round(value, 4), "unit": "TB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8 digits (exact int32/int64), bf16 in/out", "data": "synthetic",
        "config": {"workload": WORKLOAD,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2: 1.63 GB of weight digits rotated between re-uses of a matrix",
                   "per_step_bytes": step_bytes, "timing": "CUDA graph of one step (15 x digitize + GEMM), "
                   "replayed --steps times between two events",
                   "gemm_ms_per_step": round(gemm_ms, 4)},
        "gpu_launches": launches["n"],
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": GEMM_TRAFFIC_PER_LAUNCH,
                     "algorithmic_bytes_per_launch": step_bytes // len(order), "peak_kind": peak_kind,
                     "kernel": "k_exact_tc_i8: the step's 15 GEMM launches back to back in one CUDA graph on digits "
                               "computed beforehand, replayed --steps times between two events; average launch "
                               "duration = that time / 15, algorithmic bytes per launch = step bytes / 15; traffic "
                               "= ncu average per launch"},
        "clocks": clk.summary(c0, c1),
    }
    e2e = e2e_bench(dev, W, order, args)  # every rank: whole-job end-to-end rate, max time over ranks
    if world > 1:
        tt = torch.tensor([e2e["ms_per_step"]], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e["ms_per_step"] = round(float(tt), 4)
        e2e["value"] = round(world * step_bytes / (float(tt) * 1e-3) / 1e12, 4)
        e2e["h2d_bytes_per_step"] *= world
        e2e["d2h_bytes_per_step"] *= world
    result["e2e"] = e2e
    # every rank runs the per-kernel sections on its own GPU (rank 0 reports them), so all ranks reach the final
    # barrier together instead of waiting inside an NCCL collective for rank 0 alone
    result["sweep_tensor"] = tensor_sweep(dev, W, bf16_burst, args.quick)
    result["attention"] = attention_bench(dev, hbm, args.quick)
    if rank == 0:
        # CPU leg: the oracle checks the timed step's outputs (as the checker), then the CPU baseline is timed
        result["bitwise"] = bitwise_check(W, X, Y, order)
        result["bitwise_ok"] = result["bitwise"]["ok"]
        if world == 1:
            result["sweep_decode"] = decode_layers(dev, W, hbm, with_ref=not args.quick)
        if world == 1 and not args.quick:
            del W, X, Y, XD
            torch.cuda.empty_cache()
            result["decode_step"] = decode_step_bench(dev)
            result["cpu_baseline"] = cpu_baseline()
            torch.cuda.empty_cache()
            result["engine"] = engine_both_arms()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


# ------------------------------------------------------------------------------------------------------------------
# tensor-parallel arm (--gpus N > 1): the same decode sweep, every layer sharded over the N ranks
# ------------------------------------------------------------------------------------------------------------------
ROW_PARALLEL = ("o_proj", "down")  # K-sharded (row-parallel); the others are N-sharded (column-parallel)


def tp_shards(rank, world, dev):
    """This rank's shard of every headline weight matrix, cut from the full digits of the 1-GPU run (same seeds):
    column-parallel layers keep rows [r N/p, (r+1) N/p) of the full-K digits; row-parallel layers keep columns
    [r K/p, (r+1) K/p) of digits made with whole-row scales, which is exactly what digitize_weight_row_sharded
    produces (row maxima all-reduced with MAX before digitizing; F = 14 has no row sums)."""
    from vllm_exact import kernels as KK
    W = {}
    for i, (name, K, N) in enumerate(SHAPES):
        full = make_weight_digits(K, N, 1000 + i, dev)
        if name in ROW_PARALLEL:
            ks = K // world
            c = slice(rank * ks, (rank + 1) * ks)
            shard = (full[0][:, c].contiguous(), full[1][:, c].contiguous(), full[2].clone(), full[3].clone())
        else:
            ns = N // world
            r = slice(rank * ns, (rank + 1) * ns)
            shard = tuple(t[r].contiguous() for t in full)
        KK.mark_static(*shard)
        W[name] = shard
        del full
    return W


def run_tp(args, dev, rank, world, local):
    """--gpus N > 1: the headline decode sweep as an N-way tensor-parallel model would run it. qkv, gate_up and
    lm_head are column-parallel (each rank: full activations, N/p weight rows, its slice of the outputs; no
    collective); o_proj and down are row-parallel, every rank holding the full output, on the faster of two paths
    with bitwise the same results (both step times are reported): parallel.PeerRowParallel (row maxima of the K slice
    exchanged over peer memory and the slice digitized with the whole-row maxima -> int64 partial GEMM ->
    reduce-scatter + epilogue + all-gather over peer memory) or parallel.row_parallel_linear (the same steps with
    NCCL all-reduces for both exchanges). value =
    the algorithmic bytes of the whole 15-GEMM step (the same bytes as on one GPU, now spread over N GPUs) / the
    step's device time, max over ranks: total work is fixed, so scaling is strong. Every output row sample is checked
    against the CPU oracle (row-parallel outputs against the unsharded weights), so the line also shows that N GPUs
    give the 1-GPU bits."""
    import torch
    import torch.distributed as dist
    from vllm_exact import _lib, kernels as KK, parallel as P
    g = dist.group.WORLD
    hbm, _, _, peak_kind = peaks()
    W = tp_shards(rank, world, dev)
    X = {(M, name): make_activation(M, K, 17 * M + i, dev) for M in DECODE_M for i, (name, K, N) in enumerate(SHAPES)}
    XS = {}  # row-parallel inputs: this rank's K slice
    for (M, name), x in X.items():
        if name in ROW_PARALLEL:
            ks = x.shape[1] // world
            XS[(M, name)] = x[:, rank * ks:(rank + 1) * ks].contiguous()
    order = [(M, name, K, N) for M in DECODE_M for name, K, N in SHAPES]
    step_bytes = sum(gemm_bytes(M, K, N) for M, name, K, N in order)
    Y = {(M, name): torch.empty(M, N if name in ROW_PARALLEL else N // world, device=dev, dtype=torch.bfloat16)
         for M, name, K, N in order}
    stream = torch.cuda.Stream(dev)

    def ws_need(M, name, K, N):
        return KK.lib().ex_linear_workspace_bytes(M, N, K // world, 0, 0) if name in ROW_PARALLEL else \
            KK.lib().ex_linear_workspace_bytes(M, N // world, K, 0, 0)
    KK.reserve_workspace(max(ws_need(*o) for o in order), dev, stream=stream)

    peer = P.PeerRowParallel(256, max(N for name, K, N in SHAPES if name in ROW_PARALLEL), group=g)

    def layer(M, name, path="peer"):
        if name not in ROW_PARALLEL:
            KK.exact_linear(KK.digitize(X[(M, name)], 14), W[name], 14, True, out=Y[(M, name)])
        elif path == "peer":
            peer.linear(XS[(M, name)], *W[name], 14, True, out=Y[(M, name)])
        else:
            P.row_parallel_linear(XS[(M, name)], *W[name], 14, True, group=g, out=Y[(M, name)])

    def step(path="peer"):
        for M, name, K, N in order:
            layer(M, name, path)

    def graph_of(fn, warm=2):
        with torch.cuda.stream(stream):
            for _ in range(warm):
                fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            fn()
        return gr

    def timed(gr, reps):
        for _ in range(2):
            gr.replay()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            a.record()
            for _ in range(reps):
                gr.replay()
            b.record()
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / reps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    # the row-parallel exchanges run either as peer-memory kernels or as NCCL all-reduces (bitwise the same results):
    # both steps are timed and the faster one is the step timed below, as autotune_exact picks a GEMM configuration
    ms_path = {path: timed(graph_of(lambda: step(path)), args.steps) for path in ("peer", "nccl")}
    best = min(ms_path, key=ms_path.get)
    gS = graph_of(lambda: step(best), warm=args.warmup)
    for _ in range(args.warmup):
        gS.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        clk.wait_first_sample()
        dist.barrier()
        torch.cuda.synchronize()
        c0 = clk.mark()
        with torch.cuda.stream(stream):
            t0.record()
            for _ in range(args.steps):
                gS.replay()
            t1.record()
        torch.cuda.synchronize()
        c1 = clk.mark()
    dist.barrier()
    tt = torch.tensor([t0.elapsed_time(t1)], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms_per_step = float(tt) / args.steps
    value = step_bytes / (ms_per_step * 1e-3) / 1e12

    # the GEMM kernels alone (digits computed once; row-parallel layers write their int64 partials), this rank
    XD = {key: KK.digitize(x, 14) for key, x in X.items() if key[1] not in ROW_PARALLEL}
    for key, x in XS.items():
        XD[key] = P.CudaOps.digitize_given(x, 14, P.global_row_absmax(x, g))
    PART = {(M, name): torch.empty(M, N, device=dev, dtype=torch.int64) for M, name, K, N in order
            if name in ROW_PARALLEL}

    def gemms():
        for M, name, K, N in order:
            if name in ROW_PARALLEL:
                KK.exact_linear_partial_i64(XD[(M, name)], W[name], 14, True, out=PART[(M, name)])
            else:
                KK.exact_linear(XD[(M, name)], W[name], 14, True, out=Y[(M, name)])
    gemm_ms = timed(graph_of(gemms), args.steps)
    rank_bytes = sum(2 * (N // world if name not in ROW_PARALLEL else N) * (K if name not in ROW_PARALLEL else
                                                                            K // world) for M, name, K, N in order)
    # the step re-run after the GEMM-only graph, so Y holds the step's outputs for the bit check
    gS.replay()
    torch.cuda.synchronize()

    # per layer: 10 calls back to back in one graph (us per call, max over ranks), and the two collectives alone
    per_layer, coll = {}, {}
    for M, name, K, N in order:
        row = {}
        for path in (("peer", "nccl") if name in ROW_PARALLEL else ("peer",)):
            gl = graph_of(lambda: [layer(M, name, path) for _ in range(10)])
            row[path] = round(timed(gl, 5) * 100, 2)
            del gl
        if name in ROW_PARALLEL:
            # the peer path's three launches, each timed alone (10 back to back per graph): maxima exchange +
            # digitize, partial GEMM into the shared buffer, reduce-scatter + epilogue + all-gather
            # every call of the peer object on this rank goes to one stream: two of its kernels overlapping on the GPU
            # would read the same call epoch and leave this rank's epochs out of step with the other ranks'
            with torch.cuda.stream(stream):
                xd = peer.digitize(XS[(M, name)], 14)
            torch.cuda.synchronize()
            part = peer.partial(M, N)
            parts = {}
            for step_name, fn in (("exchange_digitize", lambda: peer.digitize(XS[(M, name)], 14, out=xd)),
                                  ("partial_gemm", lambda: KK.exact_linear_partial_i64(xd, W[name], 14, True,
                                                                                       out=part)),
                                  ("reduce_epilogue", lambda: peer.reduce(M, N, xd[3], W[name][3], Y[(M, name)]))):
                gl = graph_of(lambda: [fn() for _ in range(10)])
                parts[step_name] = round(timed(gl, 5) * 100, 2)
                del gl
            row["peer_launches"] = parts
        per_layer[f"{name}/M{M}"] = row if name in ROW_PARALLEL else row["peer"]
    # the row-parallel layers at M = 256 (the b256 decode batch), both paths, and whether they give the same bits
    for i, (name, K, N) in enumerate(SHAPES):
        if name not in ROW_PARALLEL:
            continue
        ks = K // world
        xs = make_activation(256, K, 9000 + i, dev)[:, rank * ks:(rank + 1) * ks].contiguous()
        ys = {path: torch.empty(256, N, device=dev, dtype=torch.bfloat16) for path in ("peer", "nccl")}
        fns = {"peer": lambda: peer.linear(xs, *W[name], 14, True, out=ys["peer"]),
               "nccl": lambda: P.row_parallel_linear(xs, *W[name], 14, True, group=g, out=ys["nccl"])}
        row = {}
        for path in ("peer", "nccl"):
            gl = graph_of(lambda: [fns[path]() for _ in range(10)])
            row[path] = round(timed(gl, 5) * 100, 2)
            del gl
        torch.cuda.synchronize()
        row["same_bits"] = bool(torch.equal(ys["peer"], ys["nccl"]))
        per_layer[f"{name}/M256"] = row
    for M in DECODE_M:
        amax = torch.ones(M, device=dev)
        tot = torch.zeros(M, 4096, dtype=torch.int64, device=dev)
        gm = graph_of(lambda: [dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=g) for _ in range(10)])
        gsum = graph_of(lambda: [dist.all_reduce(tot, op=dist.ReduceOp.SUM, group=g) for _ in range(10)])
        coll[f"M{M}"] = {"max_f32_us": round(timed(gm, 5) * 100, 2),
                         "sum_i64_M_x_4096_us": round(timed(gsum, 5) * 100, 2)}
        del gm, gsum

    # end to end through the public API with host buffers: inputs copied in from pinned host memory and outputs
    # copied back into pinned host memory inside the timed graph, on every rank
    H = {k: (XS[k] if k[1] in ROW_PARALLEL else X[k]).cpu().pin_memory() for k in X}
    O = {k: torch.empty(Y[k].shape, dtype=torch.bfloat16).pin_memory() for k in Y}
    DX = {k: torch.empty_like(v, device=dev) for k, v in H.items()}

    def e2e_step():
        for M, name, K, N in order:
            k = (M, name)
            DX[k].copy_(H[k], non_blocking=True)
            if name in ROW_PARALLEL and best == "peer":
                peer.linear(DX[k], *W[name], 14, True, out=Y[k])
            elif name in ROW_PARALLEL:
                P.row_parallel_linear(DX[k], *W[name], 14, True, group=g, out=Y[k])
            else:
                KK.exact_linear(KK.digitize(DX[k], 14), W[name], 14, True, out=Y[k])
            O[k].copy_(Y[k], non_blocking=True)
    e2e_ms = timed(graph_of(e2e_step), max(3, args.steps // 4))
    h2d = world * sum(v.numel() * 2 for v in H.values())
    d2h = world * sum(v.numel() * 2 for v in O.values())

    # bit check against the CPU oracle on a row sample (rank by rank; row-parallel layers against the full weights)
    gS.replay()
    torch.cuda.synchronize()
    check = {"ok": True, "elements": 0, "mismatches": 0, "first_mismatch": None}
    if not args.quick:
        Wc, oc = {}, []
        for i, (name, K, N) in enumerate(SHAPES):
            if name in ROW_PARALLEL:
                Wc[name] = make_weight_digits(K, N, 1000 + i, dev)
                oc += [(M, name, K, N) for M in DECODE_M]
            else:
                Wc[name] = W[name]
                oc += [(M, name, K, N // world) for M in DECODE_M]
        r = bitwise_check(Wc, X, Y, oc)
        del Wc
        agg = torch.tensor([r["elements"], r["mismatches"]], dtype=torch.int64, device=dev)
        dist.all_reduce(agg, op=dist.ReduceOp.SUM)
        check = {"ok": int(agg[1]) == 0, "elements": int(agg[0]), "mismatches": int(agg[1]),
                 "first_mismatch": r["first_mismatch"],
                 "sample": "every rank: rows {0, M-1} of each of its 15 layer outputs x all its output columns vs the "
                           "CPU oracle of the unsharded layer (bf16 bits)"}
    # a bounded wait in a peer kernel that ran out anywhere above sets the device error word: reported, max over ranks
    derr = torch.tensor([_lib.device_error()], dtype=torch.int64, device=dev)
    dist.all_reduce(derr, op=dist.ReduceOp.MAX)
    launches = sum((3 if best == "peer" else 4) if name in ROW_PARALLEL else 2 for M, name, K, N in order)
    result = {
        "metric": METRIC, "value": round(value, 4), "unit": "TB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8 digits (exact int32/int64), bf16 in/out", "data": "synthetic",
        "config": {"workload": WORKLOAD, "parallelism": f"tp{world}",
                   "sharding": "qkv, gate_up, lm_head column-parallel (N/p weight rows per rank, outputs stay "
                               "sharded); o_proj, down row-parallel (K/p per rank, full output on every rank)",
                   "row_parallel_path": best,
                   "row_parallel_paths_ms_per_step": {k: round(v, 4) for k, v in ms_path.items()},
                   "row_parallel_paths": {"peer": "row maxima exchanged and the slice digitized in one peer-memory "
                                          "kernel, partial int64 GEMM, reduce-scatter + epilogue + all-gather in one "
                                          "peer-memory kernel (NVLink loads and stores, no NCCL)",
                                          "nccl": "row maxima, MAX all-reduce, digitize, partial int64 GEMM, int64 "
                                          "SUM all-reduce, epilogue (parallel.row_parallel_linear)"},
                   "l2": "inputs larger than L2: each rank rotates its 1.63/p GB of weight digits",
                   "per_step_bytes": step_bytes, "timing": "CUDA graph of one step (NCCL collectives captured), "
                   "replayed --steps times between two events, max over ranks"},
        "gpu_launches": launches * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(rank_bytes / (gemm_ms * 1e-3) / 1e9, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(rank_bytes / (gemm_ms * 1e-3) / 1e9 / hbm, 4), "traffic": None,
                     "peak_kind": peak_kind,
                     "kernel": "k_exact_tc_i8 on one rank: its 15 GEMM launches of the step back to back in one "
                               "CUDA graph (weight-digit bytes of its shards / time, max over ranks)"},
        "clocks": clk.summary(c0, c1),
        "e2e": {"value": round(step_bytes / (e2e_ms * 1e-3) / 1e12, 4), "unit": "TB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                "api": "kernels.exact_linear / the row-parallel path above, per rank, pinned host in and out inside "
                       "one CUDA graph per step, max over ranks"},
        "per_layer_us": per_layer, "collectives_us": coll,
        "bitwise": check, "bitwise_ok": check["ok"], "device_error": int(derr),
    }
    del gS
    torch.cuda.synchronize()
    dist.barrier()
    peer.close()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def _graph_time(fns, reps, stream, warm=2):
    """Capture `fns` (a list of launch callables) into one CUDA graph with external timing events around each, replay
    it `reps` times, and return (ms per replay, [median ms of each fn])."""
    import torch
    with torch.cuda.stream(stream):
        for _ in range(warm):
            for f in fns:
                f()
    torch.cuda.synchronize()
    ev = [[[torch.cuda.Event(enable_timing=True, external=True) for _ in range(2)] for _ in fns]
          for _ in range(reps)]
    graphs = []
    for r in range(reps):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i, f in enumerate(fns):
                ev[r][i][0].record()
                f()
                ev[r][i][1].record()
        graphs.append(g)
    graphs[0].replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record()
        for g in graphs:
            g.replay()
        b.record()
    torch.cuda.synchronize()
    per = [statistics.median(ev[r][i][0].elapsed_time(ev[r][i][1]) for r in range(reps)) for i in range(len(fns))]
    del graphs
    return a.elapsed_time(b) / reps, per


def int8_peak(dev, n=8192, reps=10):
    """Dense INT8 tensor-core peak of this GPU, measured like the bf16 peak of MEASURED_PEAKS.json: torch._int_mm
    (cuBLASLt, int8 x int8 -> int32) at n^3, 2 n^3 integer ops per call, best of `reps` single calls (burst)."""
    import torch
    a = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=dev)
    b = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del a, b
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


def tensor_sweep(dev, W, peak_bf16, quick):
    """M in {256, 4096}, the tensor-bound part of configs[1]: each (shape, M) timed as a chain of GEMMs back to back in
    one CUDA graph (digits computed beforehand; weights rotating over copies worth >= 3 x L2, as in decode_layers).
    Executed digit-product ops (6 M N K) against the INT8 dense peak measured here (the kernel runs INT8 MMAs, which
    B200 executes at twice the bf16 rate, so frac_i8_peak is its roofline) and, for reference, the measured bf16 dense
    peak."""
    import torch
    from vllm_exact import kernels as KK
    stream = torch.cuda.Stream(dev)
    peak_i8 = int8_peak(dev)
    out = {"int8_peak_TOPs": round(peak_i8, 1)}
    for i, (name, K, N) in enumerate(SHAPES):
        C = max(1, -(-3 * L2_BYTES // (2 * N * K)))
        Wc = [W[name]] + [tuple(t.clone() for t in W[name]) for _ in range(C - 1)]
        for w in Wc[1:]:
            KK.mark_static(*w)
        for M in TENSOR_M:
            if quick and M > 256:
                continue
            xd = KK.digitize(make_activation(M, K, 7 * M + i, dev), 14)
            y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            KK.reserve_workspace(KK.lib().ex_linear_workspace_bytes(M, N, K, 0, 0), dev, stream=stream)
            R = C * max(1, -(-(4 if M > 256 else 8) // C))
            us = _chain_time(lambda r: KK.exact_linear(xd, Wc[r % C], 14, True, out=y), R, stream,
                             reps=2 if M > 256 else 5)
            fl = 6.0 * M * N * K
            out[f"{name}/M{M}"] = {"us": round(us, 1), "TOPs_executed": round(fl / us / 1e6, 1),
                                   "frac_i8_peak": round(fl / us / 1e6 / peak_i8, 3),
                                   "frac_bf16_peak": round(fl / us / 1e6 / peak_bf16, 3),
                                   "TOPs_useful": round(fl / 3 / us / 1e6, 1)}
            del xd, y
        del Wc
        torch.cuda.empty_cache()
    return out


def attention_bench(dev, hbm, quick):
    """H=32, KV=8, D=128, page 16, lengths +-25%; one graph with the three batches in sequence."""
    import torch
    import recipes as R
    from vllm_exact import paged_attn as PA
    PA.MAX_LEN = 20480
    stream = torch.cuda.Stream(dev)
    cases, fns = [], []
    for n, ctx in ATTN:
        q, kv, bt, sl = R.paged_case(n, ctx, 16, 32, 8, 128, ctx_jitter=True)
        q, kv, bt, sl = q.to(dev), kv.to(dev), bt.to(dev), sl.to(dev)
        kc, vc = R.kv_views(kv, 128)
        o = torch.empty(n, 32, 128, device=dev, dtype=torch.bfloat16)
        ws = torch.empty(PA.workspace_bytes(n, 32, 128), dtype=torch.uint8, device=dev)
        L = int(sl.sum())
        by = L * 8 * 128 * 2 * 2 + 2 * n * 32 * 128 * 2 + sum((int(l) + 15) // 16 for l in sl.tolist()) * 4 + 4 * n
        cases.append((n, ctx, by, (q, kv, bt, sl, o, ws)))
        fns.append(lambda q=q, kc=kc, vc=vc, bt=bt, sl=sl, o=o, ws=ws, n=n:
                   PA.paged_decode(q, kc, vc, bt, sl, 128 ** -0.5, o, n, workspace=ws))
    _, per = _graph_time(fns, 5 if quick else 20, stream)
    res = {}
    for (n, ctx, by, _), ms in zip(cases, per):
        res[f"b{n}/{ctx // 1024}K"] = {"us": round(ms * 1e3, 1), "GBps": round(by / ms / 1e6, 1),
                                       "frac_hbm": round(by / ms / 1e6 / hbm, 3), "bytes": by}
    return res


def e2e_bench(dev, W, order, args):
    """Same decode sweep through the public op exactmm::linear with host buffers: every step copies each GEMM's
    activations from pinned host memory and reads each bf16 result back into pinned host memory, inside the timed
    region (one CUDA graph per step, as vLLM captures decode). The copies run on two copy streams (host to device,
    device to host) and overlap the GEMM chain on the compute stream, as a serving pipeline overlaps them: GEMM i
    waits for its own input only, and result i is read back while GEMM i+1 runs. The step's GEMMs are independent,
    so they run largest result first, which leaves only small read-backs after the last GEMM. Every tensor of the step
    stays referenced until the step ends, so no memory is reused across streams."""
    import torch
    order = sorted(order, key=lambda t: -t[0] * t[3])  # (M, name, K, N): largest M x N output first
    H = {(M, name): make_activation(M, K, 17 * M + i, dev).cpu().pin_memory()
         for M in DECODE_M for i, (name, K, N) in enumerate(SHAPES)}
    O = {(M, name): torch.empty(M, N, dtype=torch.bfloat16).pin_memory() for M, name, K, N in order}
    h2d = sum(M * K * 2 for M, name, K, N in order)
    d2h = sum(M * N * 2 for M, name, K, N in order)
    by = sum(gemm_bytes(M, K, N) for M, name, K, N in order)
    stream = torch.cuda.Stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def step():
        cur = torch.cuda.current_stream(dev)
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        xs, ready = [], []
        with torch.cuda.stream(s_in):
            for M, name, K, N in order:
                xs.append(H[(M, name)].to(dev, non_blocking=True))
                ev = torch.cuda.Event()
                ev.record(s_in)
                ready.append(ev)
        ys = []
        for i, (M, name, K, N) in enumerate(order):
            cur.wait_event(ready[i])
            y = torch.ops.exactmm.linear(xs[i], W[name][0], W[name][1], W[name][2], W[name][3])
            ys.append(y)
            done = torch.cuda.Event()
            done.record(cur)
            s_out.wait_event(done)
            with torch.cuda.stream(s_out):
                O[(M, name)].copy_(y, non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)
        return xs, ys

    with torch.cuda.stream(stream):
        keep = step()
    torch.cuda.synchronize()
    del keep
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        keep = step()
    reps = max(3, args.steps // 4)
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    return {"value": round(by / (ms * 1e-3) / 1e12, 4), "unit": "TB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 4),
            "api": "torch.ops.exactmm.linear (pinned host in, pinned host out), CUDA graph per step, copies on "
                   "two copy streams overlapping the GEMM chain"}


# Hybrid decoder of BASELINE configs[4]: hidden 4096, 32 layers = 8 full-attention (GQA 32 q / 8 kv heads x 128) +
# 24 Gated-DeltaNet layers, SwiGLU MLP 12288, vocab 151936. GDN projection sizes follow the reference's tuned shapes
# (scripts/tune_table.py:12-13: in_proj_qkvz N=12288, in_proj_ba N=64, out_proj 4096x4096).
HYBRID_ATTN_LAYERS = (3, 7, 11, 15, 19, 23, 27, 31)
STEP_CONFIGS = [(256, 1024), (64, 8192), (16, 16384)]


def hybrid_layer_ops(layer):
    """(kind, K, N) ops of one decoder layer in execution order; kind 'attn' is the paged decode attention."""
    if layer in HYBRID_ATTN_LAYERS:
        ops = [("qkv", 4096, 6144), ("attn", 0, 0), ("o_proj", 4096, 4096)]
    else:
        ops = [("in_proj_qkvz", 4096, 12288), ("in_proj_ba", 4096, 64), ("out_proj", 4096, 4096)]
    return ops + [("gate_up", 4096, 24576), ("down", 12288, 4096)]


def decode_step_bench(dev, quick=False):
    """Hot-path share of one hybrid-model decode step: every linear (exact: digitize + exact GEMM; plain: cuBLAS bf16
    x @ w.T) and the 8 paged-attention calls (the same batch-invariant kernel in both arms: attention reads the
    same KV bytes either way), with distinct random weights per layer (14.8 GB of digits) and a separate paged KV
    cache per attention layer. GDN recurrence, norms, RoPE and sampling are vLLM's and identical in both arms, so
    they are left out: `exact_ms / plain_ms` bounds the step overhead of exactness from above. One CUDA graph per
    step, replayed."""
    import torch
    import recipes as R
    from vllm_exact import kernels as KK, paged_attn as PA
    PA.MAX_LEN = 20480
    stream = torch.cuda.Stream(dev)
    g = torch.Generator(device=dev).manual_seed(5)
    Wd, Wb = [], []
    for layer in range(32):
        d, b = {}, {}
        for kind, K, N in hybrid_layer_ops(layer):
            if kind == "attn":
                continue
            w = (torch.randn(N, K, generator=g, device=dev) * 0.02).bfloat16()
            d[kind], b[kind] = KK.digitize_weight(w, 14), w
        Wd.append(d)
        Wb.append(b)
    w = (torch.randn(151936, 4096, generator=g, device=dev) * 0.02).bfloat16()
    lm_d, lm_b = KK.digitize_weight(w, 14), w
    del w
    res = {}
    for n, ctx in (STEP_CONFIGS[:1] if quick else STEP_CONFIGS):
        xs = {K: make_activation(n, K, K, dev) for K in (4096, 12288)}
        ys = {}
        caches = []
        for i, layer in enumerate(HYBRID_ATTN_LAYERS):
            q, kv, bt, sl = [t.to(dev) for t in R.paged_case(n, ctx, 16, 32, 8, 128, seed=i, ctx_jitter=True)]
            kc, vc = R.kv_views(kv, 128)
            caches.append((q, kv, kc, vc, bt, sl, torch.empty(n, 32, 128, device=dev, dtype=torch.bfloat16),
                           torch.empty(PA.workspace_bytes(n, 32, 128), dtype=torch.uint8, device=dev)))

        def out(kind, N):
            if (kind, N) not in ys:
                ys[(kind, N)] = torch.empty(n, N, device=dev, dtype=torch.bfloat16)
            return ys[(kind, N)]

        def step(exact):
            ai = 0
            for layer in range(32):
                for kind, K, N in hybrid_layer_ops(layer):
                    if kind == "attn":
                        q, kv, kc, vc, bt, sl, o, ws = caches[ai]
                        PA.paged_decode(q, kc, vc, bt, sl, 128 ** -0.5, o, n, workspace=ws)
                        ai += 1
                    elif exact:
                        KK.exact_linear(KK.digitize(xs[K], 14), Wd[layer][kind], 14, True, out=out(kind, N))
                    else:
                        torch.matmul(xs[K], Wb[layer][kind].t(), out=out(kind, N))
            if exact:
                KK.exact_linear(KK.digitize(xs[4096], 14), lm_d, 14, True, out=out("lm_head", 151936))
            else:
                torch.matmul(xs[4096], lm_b.t(), out=out("lm_head", 151936))

        KK.reserve_workspace(max(KK.lib().ex_linear_workspace_bytes(n, N, K, 0, 0)
                                 for layer in range(32) for kind, K, N in hybrid_layer_ops(layer) if kind != "attn"),
                             dev, stream=stream)
        times = {}
        for exact in (True, False):
            with torch.cuda.stream(stream):
                step(exact)
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                step(exact)
            for _ in range(3):
                gr.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = 10
            with torch.cuda.stream(stream):
                a.record()
                for _ in range(reps):
                    gr.replay()
                b.record()
            torch.cuda.synchronize()
            times[exact] = a.elapsed_time(b) / reps
            del gr
        res[f"b{n}/{ctx // 1024}K"] = {"exact_ms": round(times[True], 3), "plain_bf16_ms": round(times[False], 3),
                                       "overhead": round(times[True] / times[False] - 1, 3)}
        del caches, xs, ys
        torch.cuda.empty_cache()
    return res


def _reference_kernels():
    """The reference's own kernels.py (installed, git-ignored, under baseline/_ref), whose CPU functions
    digitize_torch / exact_linear_torch (kernels.py:22-39, :89-100) are its stock CPU integer path; None when the
    reference is not installed."""
    try:
        return _load_reference_module("kernels")
    except SystemExit:
        return None


class CpuSample:
    """The reference's CPU integer path on a bounded sample of the decode sweep. A step is one (M, shape) GEMM of the
    headline order, taken in turn, with its output columns capped at `ncap` (output columns are independent, so a
    capped GEMM is a faithful sample). Weights are digitized once before timing, as the plugin does at load; a timed
    step digitizes its activations, runs the exact integer GEMM and rounds the output to bf16, as the GPU step does.
    backend "reference": the reference's own digitize_torch + exact_linear_torch + .bfloat16() on CPU tensors with all
    host threads; "port": the numpy restatement in oracle/ (used only when the reference is not installed). Inputs
    follow the sweep's distributions. Metric: algorithmic bytes of the sampled GEMMs / time."""

    def __init__(self, ncap, backend="reference"):
        import torch
        self.torch, self.ncap = torch, ncap
        self.RK = _reference_kernels() if backend == "reference" else None
        self.kind = "reference" if self.RK is not None else "port"
        if self.kind == "port":
            from oracle import exact_oracle as O
            self.O = O
        torch.set_num_threads(os.cpu_count())
        self.order = [(M, name, K, N) for M in DECODE_M for name, K, N in SHAPES]
        g = torch.Generator().manual_seed(0)
        self.wd, self.x = {}, {}
        for name, K, N in SHAPES:
            w = (torch.randn(min(N, ncap), K, generator=g) * 0.02).bfloat16().float()
            self.wd[name] = self._digitize(w)
        for M, name, K, N in self.order:
            x = torch.randn(M, K, generator=g)
            x[torch.rand(M, K, generator=g) < 0.001] *= 50
            self.x[(M, name)] = x.bfloat16().float()
        self.i = 0

    def _digitize(self, x):
        if self.kind == "reference":
            return self.RK.digitize_torch(x, 14)
        return self.O.digitize(x.numpy(), 14)

    def _linear_bf16(self, xd, wd):
        if self.kind == "reference":
            return self.RK.exact_linear_torch(xd, wd, 14, True).bfloat16()
        return self.O.f32_to_bf16_bits(self.O.exact_linear(xd, wd, 14, True))

    def step(self):
        """Run the next GEMM of the order; return (algorithmic bytes, seconds)."""
        M, name, K, N = self.order[self.i % len(self.order)]
        self.i += 1
        t = time.perf_counter()
        self._linear_bf16(self._digitize(self.x[(M, name)]), self.wd[name])
        return gemm_bytes(M, K, min(N, self.ncap)), time.perf_counter() - t

    def threads(self):
        if self.kind == "reference":
            return self.torch.get_num_threads()
        return _blas_threads()


def _blas_threads():
    """Threads of the BLAS that numpy uses (torchrun sets OMP_NUM_THREADS=1 for its ranks; the CPU arms raise it)."""
    import numpy  # noqa: F401  (loads the BLAS, so that its thread pool exists and can be set)
    try:
        from threadpoolctl import threadpool_info, threadpool_limits
        threadpool_limits(limits=os.cpu_count())
        return max((d.get("num_threads", 1) for d in threadpool_info() if d.get("user_api") == "blas"), default=1)
    except Exception:
        return int(os.environ.get("OMP_NUM_THREADS", os.cpu_count()))


def cpu_baseline(budget_s=20.0, ncap=1024):
    """CPU baseline beside the GPU arm's line: whole passes over the 15 sampled GEMMs until `budget_s` (at most 3)."""
    smp = CpuSample(ncap)
    threads = smp.threads()
    tot_bytes, tot_s, passes = 0, 0.0, 0
    while tot_s < budget_s and passes < 3:
        for _ in smp.order:
            b, dt = smp.step()
            tot_bytes += b
            tot_s += dt
        passes += 1
    src = ("the reference's digitize_torch + exact_linear_torch + bf16 (its kernels.py, on CPU tensors)"
           if smp.kind == "reference" else "the numpy restatement in oracle/ (reference not installed)")
    return {"value": round(tot_bytes / tot_s / 1e12, 7), "unit": "TB/s", "cores": threads, "kind": smp.kind,
            "sample": f"{passes} pass(es) of the 15 decode GEMMs with N capped at {ncap} output columns (activation "
                      f"digitize + exact integer GEMM + bf16; weights digitized before timing), {src}, {threads} host "
                      f"threads",
            "seconds": round(tot_s, 2)}


def bitwise_check(W, X, Y, order, rows_of=lambda M: sorted({0, M - 1}), chunk=16384):
    """Bit check of the GPU outputs of the timed step against the CPU oracle (the checker; nothing here is timed):
    for every GEMM of `order`, the rows rows_of(M) of the bf16 activations are digitized on the CPU and multiplied
    exactly with the weight digits (all N output columns, in column chunks), and the bf16 results must equal the GPU's
    output rows bit for bit. Rows are independent (the reference's tests/test_reference_cpu.py:37-46), so a row
    sample is a faithful check of the kernels at these exact grid shapes."""
    import numpy as np
    import torch
    from oracle import exact_oracle as O
    _blas_threads()
    checked, bad, first_bad = 0, 0, None
    for M, name, K, N in order:
        rows = rows_of(M)
        x = X[(M, name)][rows].float().cpu().numpy()
        xd = O.digitize(x, 14)
        y = Y[(M, name)][rows].cpu().view(torch.int16).numpy().view(np.uint16)
        wh, wl, cw, sw = W[name]
        for c0 in range(0, N, chunk):
            c1 = min(N, c0 + chunk)
            wd = [t[c0:c1].cpu().numpy() for t in (wh, wl, cw, sw)]
            ref = O.f32_to_bf16_bits(O.exact_linear(xd, wd, 14, True))
            nbad = int((ref != y[:, c0:c1]).sum())
            checked += ref.size
            if nbad and first_bad is None:
                first_bad = f"{name}/M{M} columns {c0}:{c1}"
            bad += nbad
    return {"ok": bad == 0, "elements": checked, "mismatches": bad, "first_mismatch": first_bad,
            "sample": "rows {0, M-1} of each of the 15 GEMMs of the timed step x all N output columns vs the CPU "
                      "oracle (bf16 bits)"}


def run_reference(args):
    """The reference arm: W untimed warm-up steps, then exactly K timed steps of CpuSample (the reference's own CPU
    path from baseline/_ref), on rank 0 only (the other ranks of a torchrun launch exit at once). The output-column
    cap is sized from a probe so that the K + W steps take about two minutes in all (at most 2048 columns, at
    least 16)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    os.environ["OMP_NUM_THREADS"] = os.environ["OPENBLAS_NUM_THREADS"] = str(os.cpu_count())  # before numpy loads
    target = 120.0 / (args.steps + args.warmup)  # seconds per step
    probe = CpuSample(256)
    costs = [probe.step()[1] for _ in probe.order]  # one pass at 256 columns: the slowest GEMM bounds a step
    ncap = int(max(16, min(2048, 256 * target / max(max(costs), 1e-6))) // 16 * 16)
    smp = CpuSample(ncap)
    threads = smp.threads()
    for _ in range(args.warmup):
        smp.step()
    tot_bytes, tot_s = 0, 0.0
    for _ in range(args.steps):
        b, dt = smp.step()
        tot_bytes += b
        tot_s += dt
    v = round(tot_bytes / tot_s / 1e12, 7)
    src = ("the reference's own digitize_torch + exact_linear_torch + .bfloat16() (src/vllm_exact/kernels.py:22-39, "
           ":89-100, installed under baseline/_ref) on CPU tensors" if smp.kind == "reference" else
           "the numpy restatement in oracle/ (the reference is not installed)")
    sample = (f"{args.steps} timed steps after {args.warmup} warm-up steps; a step is one of the 15 decode GEMMs in "
              f"turn with N capped at {ncap} output columns (activation digitize + exact integer GEMM + bf16; weights "
              f"digitized before timing), {src}, {threads} host threads")
    step_bytes = sum(gemm_bytes(M, K, N) for M in DECODE_M for name, K, N in SHAPES)
    print(json.dumps({
        "metric": METRIC, "value": v, "unit": "TB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(tot_s / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int64 (CPU)", "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD + f"; CPU sample: output columns capped at {ncap} per GEMM",
                   "parallelism": "cpu", "sample": sample, "per_step_bytes": tot_bytes // args.steps,
                   "full_step_ms_at_sampled_rate": round(step_bytes / (v * 1e12) * 1e3, 1)},
        "cpu_baseline": {"value": v, "unit": "TB/s", "cores": threads, "kind": smp.kind, "sample": sample,
                         "seconds": round(tot_s, 2)},
        "e2e": {"value": v, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


ENGINE_MAX_LEN = 21504  # prompts up to 1.25 x 16K plus 321 generated tokens


def _engine_model_dir(layers=32):
    """config.json of BASELINE configs[4]'s model: the qwen3_5 text architecture with hidden 4096, 32 layers (24
    Gated-DeltaNet + 8 full attention, GQA 32q/8kv x 128), SwiGLU 12288, vocab 151936; GDN heads give in_proj_qkvz
    N = 12288 and in_proj_ba N = 64 (the reference's tuned shapes). Weights are vLLM's dummy (random) init."""
    import json
    import tempfile
    cfg = {"architectures": ["HybridQwen35ForCausalLM"], "model_type": "qwen3_5_text", "hidden_size": 4096,
           "intermediate_size": 12288, "num_hidden_layers": layers, "num_attention_heads": 32, "num_key_value_heads": 8,
           "head_dim": 128, "vocab_size": 151936, "linear_num_key_heads": 16, "linear_num_value_heads": 32,
           "linear_key_head_dim": 128, "linear_value_head_dim": 128, "linear_conv_kernel_dim": 4,
           "full_attention_interval": 4, "max_position_embeddings": 32768, "rms_norm_eps": 1e-6,
           "rope_parameters": {"rope_type": "default", "rope_theta": 10000000.0, "partial_rotary_factor": 0.25},
           "tie_word_embeddings": False, "torch_dtype": "bfloat16", "hidden_act": "silu", "eos_token_id": 151643}
    d = tempfile.mkdtemp(prefix="exact_engine_")
    with open(f"{d}/config.json", "w") as f:
        json.dump(cfg, f)
    return d


def _register_engine_model():
    """vLLM 0.22 ships the text-only Qwen3.5 model class without the hybrid (GDN state) interface that only its
    vision-language twin declares; give it that interface (the twin's own state-shape hooks) and register it. Runs in
    every vLLM process (tensor-parallel workers too) through vllm_exact.vllm_plugin's extra hooks; idempotent."""
    from vllm import ModelRegistry
    if "HybridQwen35ForCausalLM" in ModelRegistry.get_supported_archs():
        return
    from vllm.model_executor.models.interfaces import IsHybrid
    from vllm.model_executor.models.qwen3_5 import Qwen3_5ForCausalLM, Qwen3_5ForConditionalGeneration as VL

    class HybridQwen35ForCausalLM(Qwen3_5ForCausalLM, IsHybrid):
        get_mamba_state_dtype_from_config = classmethod(VL.get_mamba_state_dtype_from_config.__func__)
        get_mamba_state_shape_from_config = classmethod(VL.get_mamba_state_shape_from_config.__func__)
        get_mamba_state_copy_func = classmethod(VL.get_mamba_state_copy_func.__func__)

    ModelRegistry.register_model("HybridQwen35ForCausalLM", HybridQwen35ForCausalLM)


def engine_both_arms(timeout_s=1200):
    """BASELINE configs[4] through the real vLLM engine, both arms (exact_int8 with the attention patch, and plain
    non-invariant bf16 vLLM), each in a subprocess running `bench.py --case engine:<arm>` (enable() must run before
    vLLM is imported, so one arm per process). Returns the step times, their ratio and the exact arm's invariance
    counts; an arm that fails or runs out of time is reported as such instead of its numbers."""
    out = {"method": "reference scripts/check_invariance.py: step = (t(321 new tokens) - t(65)) / 256, min of two "
                     "runs each; invariance = 16 targets with 1,024-token prompts alone vs interleaved in a batch of "
                     "64 vs alone again, 256 tokens, greedy and T = 1.0; vLLM 0.22, dummy weights, 32 layers"}
    for arm in ("exact", "plain"):
        t0 = time.time()
        try:
            p = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--case", f"engine:{arm}"],
                               capture_output=True, text=True, timeout=timeout_s, cwd=str(ROOT))
            lines = [l for l in p.stdout.splitlines() if l.startswith("ENGINE_JSON ")]
            if p.returncode != 0 or not lines:
                out[arm] = {"error": f"exit {p.returncode}: " + (p.stderr.strip().splitlines() or ["?"])[-1][-300:]}
            else:
                out[arm] = json.loads(lines[-1][len("ENGINE_JSON "):])
        except subprocess.TimeoutExpired:
            out[arm] = {"error": f"timed out after {timeout_s} s"}
        out[arm]["wall_s"] = round(time.time() - t0, 1)
    ex, pl = out["exact"].get("speed", {}), out["plain"].get("speed", {})
    out["overhead"] = {k: round(ex[k]["step_ms"] / pl[k]["step_ms"] - 1, 3) for k in ex if k in pl}
    return out


def engine_case(args):
    """BASELINE configs[4] through the real vLLM engine: `engine:exact` (vllm_exact.enable(), every linear and the
    lm_head exact_int8, decode attention patched) or `engine:plain` (stock non-invariant bf16 vLLM), same model, dummy
    weights, random-token prompts, both arms with vLLM's engine core in-process (enable() requires it; the plain arm
    is given the same setting). Follows the reference's scripts/check_invariance.py: invariance = 16 targets with
    1,024-token prompts, alone (A), interleaved into a batch of 64 (B), alone again (C), 256 generated tokens, greedy
    and temperature 1.0 (top-k 20, top-p 0.95, per-request seeds), tokens and logprobs compared bitwise; speed =
    (t(321 new tokens) - t(65 new tokens)) / 256 with the minimum of two runs each, at (256, 1K), (64, 8K), (16, 16K),
    prompt lengths uniform in [0.75, 1.25] x ctx. Prints one JSON line. One arm per process. Options after the arm:
    `tp=N` (tensor-parallel size), `layers=L` (default 32), `inv` (invariance only, no speed runs), `peer=R` (row-
    parallel calls of up to R rows over peer memory, 0 = NCCL only; default the package's setting)."""
    import random
    import time
    parts = args.case.split(":")
    arm = parts[1] if len(parts) > 1 else "exact"
    opts = dict(o.split("=") if "=" in o else (o, "1") for o in parts[2:])
    tp, layers, inv_only = int(opts.get("tp", 1)), int(opts.get("layers", 32)), opts.get("inv") == "1"
    if "peer" in opts:  # read by vllm_exact.parallel on import, in this process and in the tensor-parallel workers
        os.environ["VLLM_EXACT_B200_PEER_ROWS"] = opts["peer"]
    kw = {}
    if arm == "exact":
        import vllm_exact
        kw = vllm_exact.enable(max_model_len=ENGINE_MAX_LEN)
        # tensor-parallel workers register the model class through the package's vLLM plugin hook
        os.environ[vllm_exact.EXTRA_PLUGINS_ENV] = "bench:_register_engine_model"
    else:
        os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
        kw = {"enable_prefix_caching": False}
    _register_engine_model()
    from vllm import LLM, SamplingParams
    t0 = time.time()
    llm = LLM(model=_engine_model_dir(layers), load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16",
              max_model_len=ENGINE_MAX_LEN, gpu_memory_utilization=0.85, max_num_seqs=256, seed=0,
              tensor_parallel_size=tp, **kw)
    res = {"arm": arm, "tp": tp, "layers": layers, "startup_s": round(time.time() - t0, 1), "invariance": {},
           "speed": {}}
    if arm == "exact" and tp > 1:
        res["peer_rows"] = int(os.environ.get("VLLM_EXACT_B200_PEER_ROWS", "256"))

    def prompts_of(n, lo, hi, seed):
        rng = random.Random(seed)
        return [[rng.randrange(100, 150000) for _ in range(rng.randint(lo, hi))] for _ in range(n)]

    def toks_lps(o):
        c = o.outputs[0]
        return list(c.token_ids), [float(list(d.values())[0].logprob) for d in (c.logprobs or [])]

    if arm == "exact":
        P = prompts_of(64, 1024, 1024, 0)
        tgt, oth = P[:16], P[16:]
        order, tpos = [], []
        for j in range(16):  # t0, o0, o1, o2, t1, o3, ...
            tpos.append(len(order))
            order.append(tgt[j])
            order += oth[3 * j:3 * j + 3]
        for temp in (1.0, 0.0):
            def mk(seed):
                return SamplingParams(temperature=temp, top_k=20 if temp > 0 else -1, top_p=0.95 if temp > 0 else 1.0,
                                      max_tokens=256, seed=seed, logprobs=0, ignore_eos=True, detokenize=False)
            run = lambda ps, sps: [toks_lps(o) for o in llm.generate([{"prompt_token_ids": p} for p in ps], sps,
                                                                     use_tqdm=False)]
            sa = [mk(1000 + j) for j in range(16)]
            A = run(tgt, sa)
            outb = run(order, [mk(1000 + tpos.index(i)) if i in tpos else mk(1100 + i) for i in range(len(order))])
            B = [outb[i] for i in tpos]
            C = run(tgt, sa)
            same = lambda X, Y: (sum(x[0] == y[0] for x, y in zip(X, Y)), sum(x[1] == y[1] for x, y in zip(X, Y)))
            res["invariance"][f"T{temp}"] = {"A_vs_B_tokens_logprobs": "%d/16, %d/16" % same(A, B),
                                             "A_vs_C_tokens_logprobs": "%d/16, %d/16" % same(A, C)}
            print(json.dumps({"partial": res}), file=sys.stderr, flush=True)
    for n, ctx in ([] if inv_only else STEP_CONFIGS[:1] if args.quick else STEP_CONFIGS):
        prompts = [{"prompt_token_ids": p} for p in prompts_of(n, int(0.75 * ctx), int(1.25 * ctx), n * 7 + ctx)]

        def gen(k):
            sps = [SamplingParams(temperature=1.0, top_k=20, top_p=0.95, max_tokens=k, ignore_eos=True, seed=j,
                                  detokenize=False) for j in range(n)]
            t = time.time()
            llm.generate(prompts, sps, use_tqdm=False)
            return time.time() - t
        gen(321)
        step = (min(gen(321), gen(321)) - min(gen(65), gen(65))) / 256
        res["speed"][f"b{n}/{ctx // 1024}K"] = {"step_ms": round(step * 1000, 3), "tok_per_s": round(n / step, 1)}
        print(json.dumps({"partial": res}), file=sys.stderr, flush=True)
    print("ENGINE_JSON " + json.dumps(res), flush=True)


def tp_case(args):
    """Row-parallel (K-sharded) exact layers on the torchrun group: time per layer call of the NCCL path (int64 SUM
    all-reduce + epilogue kernel) and of the peer-memory path (PeerRowParallel: the row-maxima exchange + digitize and
    the reduce-scatter + epilogue + all-gather as kernels over NVLink), both captured in CUDA graphs (20 calls per
    graph), device time, max over ranks. Both paths include the digitizer and the partial GEMM. Prints one JSON line
    on rank 0. Launch: torchrun --nproc-per-node N bench.py --case tp."""
    import datetime
    import torch
    import torch.distributed as dist
    from vllm_exact import kernels as KK, parallel as P
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    peer = P.PeerRowParallel(64, 4096)
    res = {}
    for name, Kd, N in (("o_proj", 4096, 4096), ("down", 12288, 4096)):
        ks = Kd // world
        w = (torch.randn(N, ks, generator=torch.Generator().manual_seed(rank)) * 0.02).bfloat16().to(dev)
        wd = P.digitize_weight_row_sharded(w, 14)
        for M in (1, 16, 64):
            x = torch.randn(M, ks, generator=torch.Generator().manual_seed(M)).bfloat16().to(dev)
            st = torch.cuda.Stream(dev)
            KK.reserve_workspace(KK.lib().ex_linear_workspace_bytes(M, N, ks, 0, 0), dev, stream=st)
            row = {}
            for path in ("nccl", "peer"):
                fn = (lambda: P.row_parallel_linear(x, *wd, 14, True)) if path == "nccl" else \
                    (lambda: peer.linear(x, *wd, 14, True))
                st.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(st):
                    fn()
                torch.cuda.synchronize(dev)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=st):
                    for _ in range(20):
                        fn()
                g.replay()
                torch.cuda.synchronize(dev)
                dist.barrier()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(st):
                    a.record()
                    for _ in range(5):
                        g.replay()
                    b.record()
                torch.cuda.synchronize(dev)
                t = torch.tensor([a.elapsed_time(b) * 1000 / 100], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                row[path] = round(float(t), 2)
                del g
            res[f"{name}/M{M}"] = row
    torch.cuda.synchronize(dev)
    dist.barrier()
    peer.close()
    if rank == 0:
        print(json.dumps({"case": "tp", "world": world, "us_per_layer_call": res}), flush=True)
    dist.destroy_process_group()


def run_case(args):
    """Workloads for ncu captures, run eagerly --reps times (ncu flushes caches before each captured pass):
    `gemm:<shape>:<M>[:<algo>]` one GEMM, `attn:<n>:<ctx>` one attention batch, `sweep` the 15 GEMMs of the headline
    decode step. Timed sections alone: `step` the config-5 hot-path share, `attnbench` the config-4 attention
    batches, `engine:exact|plain` config 5 through the vLLM engine, `tp` the row-parallel layer under torchrun."""
    if args.case.startswith("engine"):
        return engine_case(args)
    if args.case == "tp":
        return tp_case(args)
    import torch
    from vllm_exact import kernels as KK, paged_attn as PA
    import recipes as R
    dev = torch.device("cuda", 0)
    kind, *rest = args.case.split(":")
    if kind == "gemm":
        name, M = rest[0], int(rest[1])
        algo = {"tc_i8": KK.EX_ALGO_TC_I8, "simt": KK.EX_ALGO_SIMT,
                "auto": KK.EX_ALGO_AUTO}[rest[2] if len(rest) > 2 else "auto"]
        (K, N), = [(k, n) for nm, k, n in SHAPES if nm == name]
        W = make_weight_digits(K, N, 1, dev)
        xd = KK.digitize(make_activation(M, K, 2, dev), 14)
        y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        KK.reserve_workspace(KK.lib().ex_linear_workspace_bytes(M, N, K, 0, algo), dev)
        for _ in range(args.reps):
            KK.exact_linear(xd, W, 14, True, out=y, cfg={"algo": algo})
    elif kind == "sweep":
        # one eager pass of the headline decode step: 15 x (digitize + exact GEMM)
        W = {name: make_weight_digits(K, N, 1000 + i, dev) for i, (name, K, N) in enumerate(SHAPES)}
        for _ in range(args.reps):
            for M in DECODE_M:
                for i, (name, K, N) in enumerate(SHAPES):
                    y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                    KK.exact_linear(KK.digitize(make_activation(M, K, 17 * M + i, dev), 14), W[name], 14, True,
                                    out=y)
    elif kind == "step":
        print(json.dumps(decode_step_bench(dev)), flush=True)
    elif kind == "layers":  # the chain-timed per-layer decode section of the default run alone
        W = {name: make_weight_digits(K, N, 1000 + i, dev) for i, (name, K, N) in enumerate(SHAPES)}
        print(json.dumps(decode_layers(dev, W, peaks()[0], with_ref=rest != ["noref"])), flush=True)
    elif kind == "attnbench":  # the attention section of the default run alone (BASELINE config 4 batches)
        print(json.dumps(attention_bench(dev, peaks()[0], False)), flush=True)
    elif kind == "attn":
        n, ctx = int(rest[0]), int(rest[1])
        PA.MAX_LEN = 20480
        q, kv, bt, sl = [t.to(dev) for t in R.paged_case(n, ctx, 16, 32, 8, 128, ctx_jitter=True)]
        kc, vc = R.kv_views(kv, 128)
        o = torch.empty(n, 32, 128, device=dev, dtype=torch.bfloat16)
        for _ in range(args.reps):
            PA.paged_decode(q, kc, vc, bt, sl, 128 ** -0.5, o, n)
    else:
        raise SystemExit(f"unknown case {args.case}")
    torch.cuda.synchronize()
    print(f"case {args.case} done")


REF_TRITON_CFGS = sorted({(16, 64, 256, 4, 3, 8, 1), (16, 64, 256, 4, 3, 8, 4), (16, 128, 128, 4, 4, 8, 1),
                          (16, 128, 128, 4, 4, 8, 2), (16, 128, 128, 4, 4, 8, 4), (64, 64, 128, 4, 3, 8, 1),
                          (64, 64, 128, 4, 3, 8, 2), (64, 64, 128, 4, 3, 8, 4), (128, 128, 128, 8, 3, 8, 1),
                          (64, 128, 128, 4, 4, 8, 1)})


def _load_reference_module(name):
    """Import a module of the reference package installed (git-ignored) under baseline/_ref, under a private name so
    it cannot clash with this repository's vllm_exact package."""
    import importlib.util
    path = ROOT / "baseline" / "_ref" / "vllm_exact" / f"{name}.py"
    if not path.exists():
        raise SystemExit(f"reference not installed at {path.parent}")
    spec = importlib.util.spec_from_file_location(f"reference_vllm_exact_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# Tile configurations of the reference's shipped B300 tuning table (src/vllm_exact/cfg_table_b300_F14.json) for
# M = 1, 16 and 64, and its defaults (src/vllm_exact/plugin.py:_cfg), as (BM, BN, BK, warps, stages, GM, split_k).
REF_DECODE_CFGS = {1: [(16, 64, 256, 4, 3, 8, 4), (16, 128, 128, 4, 4, 8, 4), (16, 128, 128, 4, 4, 8, 2),
                       (16, 128, 128, 4, 4, 8, 1)],
                   16: [(16, 64, 256, 4, 3, 8, 4), (16, 128, 128, 4, 4, 8, 4), (16, 128, 128, 4, 4, 8, 2),
                        (16, 128, 128, 4, 4, 8, 1)],
                   64: [(64, 64, 128, 4, 3, 8, 4), (64, 64, 128, 4, 3, 8, 2), (64, 64, 128, 4, 3, 8, 1),
                        (16, 64, 256, 4, 3, 8, 4), (64, 128, 128, 4, 4, 8, 1)]}


L2_BYTES = 126 * 1024 * 1024


def _chain_time(op, R, stream, reps=5, warm=2):
    """Capture op(0) .. op(R-1) back to back in one CUDA graph (no events between them, so each launch overlaps its
    neighbours exactly as in a captured decode step), replay it `reps` times between two events, and return the
    device time per op in microseconds."""
    import torch
    with torch.cuda.stream(stream):
        for _ in range(warm):
            for r in range(R):
                op(r)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for r in range(R):
            op(r)
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
    torch.cuda.synchronize()
    del g
    return a.elapsed_time(b) * 1e3 / (reps * R)


def decode_layers(dev, W, hbm, with_ref=True, budget_s=150.0):
    """Per-layer decode figures of the headline shapes (M in {1, 16, 64}), every one timed as a chain: R ops back to
    back in one CUDA graph, events only around the replays, time / R. The ops of a chain rotate over C copies of the
    layer's weight digits with C x bytes >= 3 x L2, so every op streams its weights from HBM.

    * op_us:   the exact linear as vLLM calls it (exactmm::linear = activation digitize + exact GEMM)
    * gemm_us: the GEMM alone on pre-computed digits (k_exact_tc_i8 back to back); frac_hbm = its algorithmic bytes
               (2NK + 4N + 2MK + 4M + 2MN) / gemm_us / the measured HBM peak
    * ref_op_us (with_ref): the reference's own Triton op on the same B200 and the same inputs, timed the same way:
      its digitize + exact_linear (kernels.py:74-85, :257-289: _digitize_kernel, _exact_kernel or _exact_bf16_kernel,
      and _exact_fin for split-K), installed under baseline/_ref. It gets the best of the tile configurations of its
      shipped B300 table and defaults for that M, each with INT8 and bf16 MMAs; its output is compared bitwise with
      ours. Candidates stop after `budget_s` seconds of trying (Triton compiles each one).

    A single kernel between two timing events costs several microseconds more than the same kernel in a chain (the
    event pair alone, around an empty kernel, measured ~6 us on B200), which is why no figure here brackets single
    launches with events."""
    import torch
    from vllm_exact import kernels as KK
    RK = None
    if with_ref:
        try:
            RK = _load_reference_module("kernels")
        except SystemExit as e:
            RK = None
            ref_missing = str(e)
    t_start = time.time()
    stream = torch.cuda.Stream(dev)
    res = {}
    for i, (name, K, N) in enumerate(SHAPES):
        by_w = 2 * N * K
        C = max(1, -(-3 * L2_BYTES // by_w))
        Wc = [W[name]] + [tuple(t.clone() for t in W[name]) for _ in range(C - 1)]
        for w in Wc[1:]:
            KK.mark_static(*w)
        R = C * max(1, -(-8 // C))
        for M in DECODE_M:
            x = make_activation(M, K, 17 * M + i, dev)
            xd = KK.digitize(x, 14)
            xb = KK._alloc_digits(M, K, dev)
            y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            KK.reserve_workspace(KK.lib().ex_linear_workspace_bytes(M, N, K, 0, 0), dev, stream=stream)
            op_us = _chain_time(lambda r: KK.exact_linear(KK.digitize(x, 14, out=xb), Wc[r % C], 14, True, out=y),
                                R, stream)
            gemm_us = _chain_time(lambda r: KK.exact_linear(xd, Wc[r % C], 14, True, out=y), R, stream)
            by = gemm_bytes(M, K, N)
            row = {"op_us": round(op_us, 2), "gemm_us": round(gemm_us, 2), "GBps": round(by / gemm_us / 1e3, 1),
                   "frac_hbm": round(by / gemm_us / 1e3 / hbm, 3)}
            if with_ref and RK is None:
                row["ref"] = ref_missing
            elif RK is not None:
                ours_y = y.clone()
                rb = KK._alloc_digits(M, K, dev)
                best = None
                for cfg in REF_DECODE_CFGS[M]:
                    for mma in (0, 1):
                        if best is not None and time.time() - t_start > budget_s:
                            break
                        c = cfg + (mma,)
                        yr = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                        try:
                            us = _chain_time(lambda r: RK.exact_linear(RK.digitize(x, 14, out=rb), Wc[r % C], 14,
                                                                       True, out=yr, cfg=c), R, stream, reps=3)
                        except Exception as e:  # a configuration that does not compile here
                            print(f"reference cfg {c} failed: {type(e).__name__}", file=sys.stderr)
                            continue
                        same = bool(torch.equal(yr, ours_y))
                        if best is None or us < best[0]:
                            best = (us, c, same and (best is None or best[2]))
                        elif not same:
                            best = (best[0], best[1], False)
                if best is not None:
                    row.update({"ref_op_us": round(best[0], 2), "speedup_op": round(best[0] / op_us, 3),
                                "ref_cfg": list(best[1]), "bitwise_equal": best[2]})
            res[f"{name}/M{M}"] = row
            del x, xd, xb, y
        del Wc
        torch.cuda.empty_cache()
    return res


def run_ref_triton(args):
    """Informational comparison on one B200: the reference's own Triton kernels (kernels.py _exact_kernel /
    _exact_bf16_kernel, paged_attn.py _paged_partial/_paged_merge) against ours on identical inputs, both timed with
    CUDA graphs that rotate the five weight matrices (so weights stream from HBM). For each GEMM shape the reference
    runs its best of the tile configurations of its shipped B300 table and defaults, with INT8 and bf16 MMA; every
    reference output is also checked bitwise against ours."""
    import torch
    from vllm_exact import kernels as KK, paged_attn as PA
    import recipes as R
    RK = _load_reference_module("kernels")
    RP = _load_reference_module("paged_attn")
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    hbm = peaks()[0]
    W = {name: make_weight_digits(K, N, 1000 + i, dev) for i, (name, K, N) in enumerate(SHAPES)}
    out = {"gemm": {}, "attention": {}}
    for M in DECODE_M + [256]:
        xs = {name: KK.digitize(make_activation(M, K, 17 * M + i, dev), 14) for i, (name, K, N) in enumerate(SHAPES)}
        ours_y = {name: torch.empty(M, N, device=dev, dtype=torch.bfloat16) for name, K, N in SHAPES}
        KK.reserve_workspace(max(KK.lib().ex_linear_workspace_bytes(M, N, K, 0, 0) for _, K, N in SHAPES), dev,
                             stream=stream)
        fns = [(lambda n=name: KK.exact_linear(xs[n], W[n], 14, True, out=ours_y[n])) for name, K, N in SHAPES]
        _, ours_ms = _graph_time(fns, 10, stream)
        best = {}
        for cfg in REF_TRITON_CFGS:
            for mma in (0, 1):
                c = cfg + (mma,)
                if c[0] > max(16, 1 << max(0, (M - 1).bit_length())):
                    continue
                ys = {name: torch.empty(M, N, device=dev, dtype=torch.bfloat16) for name, K, N in SHAPES}
                rf = [(lambda n=name, c=c: RK.exact_linear(xs[n], W[n], 14, True, out=ys[n], cfg=c))
                      for name, K, N in SHAPES]
                try:
                    _, ref_ms = _graph_time(rf, 5, stream)
                except Exception as e:  # a config that does not compile here
                    print(f"reference cfg {c} failed: {type(e).__name__}", file=sys.stderr)
                    continue
                for (name, K, N), ms in zip(SHAPES, ref_ms):
                    same = bool(torch.equal(ys[name], ours_y[name]))
                    if name not in best or ms < best[name][0]:
                        best[name] = (ms, c, same)
                    elif not same:
                        best[name] = (best[name][0], best[name][1], False)
        for (name, K, N), ms in zip(SHAPES, ours_ms):
            rms, rc, same = best[name]
            by = gemm_bytes(M, K, N)
            out["gemm"][f"{name}/M{M}"] = {"ours_us": round(ms * 1e3, 1), "ref_us": round(rms * 1e3, 1),
                                           "speedup": round(rms / ms, 2), "ours_GBps": round(by / ms / 1e6, 1),
                                           "ref_GBps": round(by / rms / 1e6, 1), "ref_cfg": list(rc),
                                           "bitwise_equal": same}
        print(json.dumps({f"M{M}": {k: v for k, v in out["gemm"].items() if k.endswith(f"/M{M}")}}), file=sys.stderr)
    PA.MAX_LEN = RP.MAX_LEN = 20480
    for n, ctx in ATTN:
        q, kv, bt, sl = [t.to(dev) for t in R.paged_case(n, ctx, 16, 32, 8, 128, ctx_jitter=True)]
        kc, vc = R.kv_views(kv, 128)
        o1 = torch.empty(n, 32, 128, device=dev, dtype=torch.bfloat16)
        o2 = torch.empty_like(o1)
        ws = torch.empty(PA.workspace_bytes(n, 32, 128), dtype=torch.uint8, device=dev)
        _, (ms1,) = _graph_time([lambda: PA.paged_decode(q, kc, vc, bt, sl, 128 ** -0.5, o1, n, workspace=ws)], 10,
                                stream)
        msl = int(sl.max())
        _, (ms2,) = _graph_time([lambda: RP.paged_decode(q, kc, vc, bt, sl, 128 ** -0.5, o2, n, msl)], 10, stream)
        L = int(sl.sum())
        by = L * 8 * 128 * 2 * 2 + 2 * n * 32 * 128 * 2 + sum((int(l) + 15) // 16 for l in sl.tolist()) * 4 + 4 * n
        out["attention"][f"b{n}/{ctx // 1024}K"] = {
            "ours_us": round(ms1 * 1e3, 1), "ref_us": round(ms2 * 1e3, 1), "speedup": round(ms2 / ms1, 2),
            "ours_frac_hbm": round(by / ms1 / 1e6 / hbm, 3), "ref_frac_hbm": round(by / ms2 / 1e6 / hbm, 3),
            "max_abs_diff": float((o1.float() - o2.float()).abs().max())}
        del kv
    print(json.dumps({"ref_triton": out}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--quick", action="store_true", help="skip the slow secondary measurements")
    ap.add_argument("--case", default=None, help="profiling workload or single section, e.g. gemm:o_proj:64, "
                    "attn:64:8192, sweep, step, attnbench, engine:exact, tp")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--ref-triton", action="store_true",
                    help="time the reference's Triton kernels (installed under baseline/_ref) against ours")
    args = ap.parse_args()
    if args.ref_triton:
        run_ref_triton(args)
        return
    if args.case:
        run_case(args)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
