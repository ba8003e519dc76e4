"""Benchmark of the fused FP8 linear hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

A step is one ``fp8_linear`` over one batch of synthetic FLUX-shaped activations:
per-token e4m3 quantization of x (bf16), the tcgen05 FP8 GEMM against a per-channel
e4m3 weight with the dequant + bias epilogue fused in, bf16 out. The default workload
is the FLUX double-block QKV linear (M=4608 tokens, K=3072 -> N=9216).

Multi-GPU (torchrun, one process per GPU): token rows shard with the weight
replicated and no collective; each rank runs its own M-row batch (weak scaling) and
``value`` is the FLOPs of all ranks over the max-over-ranks device time.

Timing: W untimed warm-up steps, then exactly K timed steps between a barrier and a
device synchronize, on the device with two CUDA events on the launching stream. The K
steps run back to back from one CUDA graph (no host gaps between kernels) and cycle
over several independent operand sets (activations, weights, outputs) whose combined
size is a few times the 126 MB L2, so every step reads operands that were evicted
since their last use. ``e2e`` repeats the step through the C ABI with the activations
copied from pinned host memory and the output copied back inside the timed region.
``roofline`` and ``quantizer`` time the GEMM kernel and the quantizer alone the same
way (K launches over the rotating sets; average device time per launch).
``cpu_baseline`` times the CPU restatement of the reference path (the oracle port:
per-token e4m3 quant, fp32 matmul, dequant + bias) on a bounded row sample.

``--impl reference`` times the reference's path on the host CPU instead (the oracle
port, all host threads) and, when the reference's own CUDA ops were compiled into
oracle/_ref, reports their device time on the same workload as ``gpu_reference``.
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
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "FP8 linear TFLOP/s at FLUX shapes vs 4.5 PF peak; quant GB/s vs 8 TB/s"
FLUSH_BYTES = 256 << 20
# idle time before each timed leg of a sweep: a bandwidth-bound kernel timed right after
# tens of milliseconds of full-power GEMM replays reads up to 30 % slow
SWEEP_PAUSE_S = 0.5
# idle time before each config-4 leg (clocks recover after long full-power GEMM graphs)
CFG_PAUSE_S = 1.0
NOMINAL_FP8_TFLOPS = 4500.0
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
L2_FALLBACK = 126 << 20


# ----------------------------------------------------------------------------- plumbing


def _workloads():
    """fp8linear_b200/workloads.py (the seeded input generators) loaded as a module of
    its own, without importing the package: the package's import maps the native
    binding, which the reference arm must not load."""
    import importlib.util

    name = "fp8linear_b200_bench_workloads"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(
            name, ROOT / "fp8linear_b200" / "workloads.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


DATA = "synthetic (seeded FLUX-shaped tensors; FLUX.1-dev weights unavailable offline)"


def bench_config(wl, world: int) -> dict:
    """The ``config`` of the driver's line, identical in both arms."""
    return {"workload": wl.name, "M_per_gpu": wl.M, "K": wl.K, "N": wl.N,
            "global_tokens": wl.M * world, "x": "bf16", "out": "bf16",
            "parallelism": f"M-shard x{world}, weights replicated, no collective",
            "l2": "inputs larger than L2: steps rotate over operand sets (x, weight, "
                  "output) so that 3x the L2 is touched between two uses of a set"}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "measured"}
    return {**FALLBACK, "source": "fallback"}


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of one GPU, polled through
    NVML (the library nvidia-smi reads) every 2 ms on a background thread; falls back
    to ``nvidia-smi -lms 200`` when NVML is unavailable."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index: int, interval_s: float = 0.002):
        self.cuda_index = cuda_index
        self.interval = interval_s
        self.samples: list[tuple[float, float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self._nvml = None
        self._proc = None
        self._rows: list[list[str]] = []

    def start(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            try:
                idx = torch.cuda._get_nvml_device_index(self.cuda_index)
            except Exception:
                idx = self.cuda_index
            h = nv.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            reasons_fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self._nvml = nv

            def poll():
                while not self._stop.is_set():
                    try:
                        self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                             nv.nvmlDeviceGetPowerUsage(h) / 1000.0,
                                             int(reasons_fn(h))))
                    except Exception:
                        pass
                    time.sleep(self.interval)

            self._t = threading.Thread(target=poll, daemon=True)
            self._t.start()
        except Exception:
            self._start_smi()
        return self

    def _start_smi(self):
        fields = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.cuda_index}", f"--query-gpu={fields}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None
            return

        def pump():
            for line in self._proc.stdout:
                self._rows.append([c.strip() for c in line.split(",")])

        self._t = threading.Thread(target=pump, daemon=True)
        self._t.start()

    def stop(self):
        self._stop.set()
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sm, power, reasons = [], [], set()
        if self._nvml is not None:
            for mhz, w, bits in self.samples:
                sm.append(mhz)
                power.append(w)
                for bit, name in self.REASONS.items():
                    if bits & bit:
                        reasons.add(name)
            source = "nvml"
        else:
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for r in self._rows:
                try:
                    sm.append(float(r[0]))
                    self.max_mhz = float(r[1])
                    power.append(float(r[2]))
                except (ValueError, IndexError):
                    continue
                for name, v in zip(names, r[3:7]):
                    if v.lower().startswith("active"):
                        reasons.add(name)
            source = "nvidia-smi"
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "power_w_max": max(power) if power else None, "samples": len(sm),
                "reasons": sorted(reasons), "source": source}


# ----------------------------------------------------------------------------- timing


def l2_bytes(dev) -> int:
    return int(getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 0) or L2_FALLBACK)


def set_count(per_set_bytes: int, dev, lo: int = 3, hi: int = 512) -> int:
    """Operand sets to rotate over so that, between two uses of one set, the others
    touch at least 3x the L2 capacity (its lines are evicted by then)."""
    need = -(-3 * l2_bytes(dev) // max(1, per_set_bytes))
    return max(lo, min(hi, need))


def operand_sets(wl, n_sets: int, x_seed0: int = 0, quantize_x: bool = True, fmt: str = "fp8"):
    """``n_sets`` independent (x, wq, ws, bias[, xq, xs]) sets of workload ``wl`` on
    the current device (weights quantized once, as offline). Set i's weight depends
    only on i, so ranks hold the same weights; activations use ``x_seed0``. ``fmt``
    "fp8": per-token / per-channel scales; "mx": MXFP8 block scales; "nv": NVFP4;
    "modulated": per-channel weights plus the AdaLN shift / scale [2, K] of a 2-image batch."""
    import fp8linear_b200 as f

    W = _workloads()
    make_weight, make_x = W.make_weight, W.make_x
    qw = {"fp8": f.quantize_weight, "mx": f.quantize_weight_mxfp8,
          "nv": f.quantize_weight_nvfp4, "modulated": f.quantize_weight}[fmt]
    qx = {"fp8": f.quantize_fp8, "mx": f.quantize_mxfp8, "nv": f.quantize_nvfp4,
          "modulated": f.quantize_fp8}[fmt]
    sets = []
    for i in range(n_sets):
        x = make_x(wl, seed=x_seed0 + 7919 * i, gen_device="cuda")
        w, b = make_weight(wl, seed=7919 * i, gen_device="cuda")
        wq, ws = qw(w)
        del w
        s = {"x": x, "wq": wq, "ws": ws, "b": b}
        if fmt == "modulated":
            s["shift"], s["scale"] = modulation(wl, 7919 * i + 17)
        if quantize_x:
            s["xq"], s["xs"] = qx(x)
        sets.append(s)
    return sets


def modulation(wl, seed: int):
    """AdaLN shift and scale [2, K] (a 2-image batch; M divisible by 2), bf16."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    shift = (torch.randn(2, wl.K, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    scale = (torch.randn(2, wl.K, device="cuda", generator=g) * 0.2).to(torch.bfloat16)
    return shift, scale


def unfused_modulation(x, shift, scale, eps=1e-6):
    """The chain a FLUX block runs before its linear without the fusion: torch LayerNorm
    (no affine) and the bf16 modulation ops."""
    K = x.shape[-1]
    b = torch.arange(x.shape[0], device=x.device) // (x.shape[0] // shift.shape[0])
    return torch.nn.functional.layer_norm(x, (K,), eps=eps) * (1 + scale)[b] + shift[b]


def per_set_bytes(wl) -> int:
    """HBM bytes one step's operand set occupies: x, codes + scales, weight codes +
    scales + bias, output."""
    return (2 * wl.M * wl.K + wl.M * wl.K + 4 * wl.M + wl.N * wl.K + 4 * wl.N + 2 * wl.N
            + 2 * wl.M * wl.N)


def graph_launches(call, sets, reps: int, keep: int):
    """A CUDA graph of ``reps`` calls cycling over ``sets``. The outputs of the last
    ``keep`` calls stay referenced during capture, so consecutive calls write distinct
    buffers (like consecutive layers) instead of one recycled block."""
    from collections import deque

    for st in sets:  # eager first calls (per-device setup) outside the capture
        call(st)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    live = deque(maxlen=max(1, keep))
    with torch.cuda.graph(g):
        for i in range(reps):
            live.append(call(sets[i % len(sets)]))
    live.clear()
    return g


def time_graph(g, stream, barrier) -> float:
    """Device milliseconds of one replay of ``g``: a barrier and a synchronize on both
    sides, CUDA events on the launching stream."""
    g.replay()  # untimed replay: warm
    barrier()
    a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    g.replay()
    c.record(stream)
    barrier()
    return a.elapsed_time(c)


# ----------------------------------------------------------------------------- CPU path


def cpu_reference_runner(wl, rows: int, threads: int | None = None):
    """The reference path on the CPU (oracle port) for ``rows`` token rows of ``wl``.

    The weight is quantized once (offline, as the reference's quantize_weight) and kept
    decoded to fp32; each call quantizes x per token (the oracle's multi-threaded torch
    twin), decodes the codes, runs the fp32 matmul and applies (acc * xs) * ws + bias in
    place (the same roundings as the expression).
    """
    import numpy as np
    from oracle import oracle as O

    W = _workloads()
    make_weight, make_x = W.make_weight, W.make_x

    if threads:
        torch.set_num_threads(threads)
    x = make_x(wl, M=rows, seed=7)
    w, b = make_weight(wl)
    w16 = w.contiguous().view(torch.int16).numpy().view(np.uint16)
    wq, ws = O.np_quantize_weight(w16, O.BF16)
    lut = torch.from_numpy(O.e4m3_decode_lut())
    wf = lut[torch.from_numpy(wq).long()]
    wsv = torch.from_numpy(ws)
    bias = b.float()
    x = x.contiguous()

    def step():
        xq, xs = O.torch_quantize_rows(x)
        acc = xq.float() @ wf.T
        return acc.mul_(xs[:, None]).mul_(wsv[None, :]).add_(bias[None, :])

    return step


def time_cpu(step, min_seconds: float = 3.0, max_iters: int = 1000):
    step()  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or n >= max_iters:
            return el / n, n


# ----------------------------------------------------------------------------- GPU arm


def run_gpu(args):
    import torch.distributed as dist

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    import fp8linear_b200 as f
    from fp8linear_b200.capi import CApi

    wl = _workloads().WORKLOADS[args.workload]
    M, K, N = wl.M, wl.K, wl.N
    per_set = per_set_bytes(wl)
    n_sets = set_count(per_set, dev)
    # this rank's token rows (its own seeds) and a replicated weight per set
    sets = operand_sets(wl, n_sets, x_seed0=1000 * rank)
    x, wq, ws, b = sets[0]["x"], sets[0]["wq"], sets[0]["ws"], sets[0]["b"]
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(st):
        return f.fp8_linear(st["x"], st["wq"], st["ws"], st["b"])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # ---- warm-up (the clock sampler starts here: the GPU is busy from now on)
    clocks = ClockSampler(local).start()
    for i in range(args.warmup):
        step(sets[i % n_sets])
    barrier()

    # ---- the quantizer alone first (K launches, same rotation): a memory-bound kernel
    # timed right after seconds of full-power GEMM graphs reads slow, the power-capped
    # clocks outlasting the GEMMs
    g_quant = graph_launches(lambda st: f.quantize_fp8(st["x"]), sets, args.steps, keep=n_sets)
    q_ms = time_graph(g_quant, stream, barrier) / args.steps
    del g_quant

    # ---- timed: K fused steps back to back over the rotating operand sets
    g_step = graph_launches(step, sets, args.steps, keep=n_sets)
    total_ms = time_graph(g_step, stream, barrier)
    del g_step
    if world > 1:
        t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    flops_rank = wl.flops
    value = world * flops_rank * args.steps / (total_ms * 1e-3) / 1e12
    ms_per_step = total_ms / args.steps

    # ---- roofline: the GEMM kernel alone, K launches, same rotation
    g_gemm = graph_launches(lambda st: f.fp8_gemm(st["xq"], st["xs"], st["wq"], st["ws"], st["b"]),
                            sets, args.steps, keep=n_sets)
    g_ms = time_graph(g_gemm, stream, barrier) / args.steps
    del g_gemm
    pk = peaks()
    fp8_peak = 2.0 * pk["bf16_tflops"]
    gemm_tflops = flops_rank / (g_ms * 1e-3) / 1e12
    quant_gbs = wl.quant_bytes / (q_ms * 1e-3) / 1e9
    traffic = None
    prof = ROOT / "profiles" / f"traffic_{args.workload}.json"
    if prof.exists():
        traffic = json.loads(prof.read_text()).get("gemm_dram_bytes_per_launch")

    # ---- e2e through the C ABI with host buffers (H2D x, linear, D2H out), timed:
    # fp8lin_fp8_linear_host, whose row chunks overlap upload, kernels and download
    capi = CApi()
    x_host = x.cpu().pin_memory()
    out_host = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    wsz = int(capi.lib.fp8lin_fp8_linear_host_workspace_size(M, N, K))
    work = torch.empty(wsz, dtype=torch.uint8, device=dev)

    def e2e_step():
        capi.fp8_linear_host(x_host, wq, ws, b, out_host=out_host, workspace=work)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier()
    e2e_ev = []
    for i in range(args.steps):
        flush.zero_()
        a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        e2e_step()
        c.record(stream)
        e2e_ev.append((a, c))
    barrier()
    e2e_total = sum(a.elapsed_time(c) for a, c in e2e_ev)
    if world > 1:
        t = torch.tensor([e2e_total], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_total = float(t.item())
    e2e_value = world * flops_rank * args.steps / (e2e_total * 1e-3) / 1e12
    # clocks were sampled from the first warm-up step through the e2e phase: the whole
    # stretch of continuous GPU work that contains the timed region
    clk = clocks.stop()

    status = capi.device_status()

    # ---- CPU baseline (rank 0, N=1 only): oracle port on a bounded row sample
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        rows = args.cpu_rows
        st = cpu_reference_runner(wl, rows)
        per, n = time_cpu(st, min_seconds=args.cpu_seconds)
        cpu = {"value": 2 * rows * N * K / per / 1e12, "unit": "TFLOP/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{rows} of {M} token rows of {wl.name} (K={K}, N={N}), {n} passes, "
                         f"{per * 1e3:.1f} ms/pass; fp32 torch matmul of decoded e4m3 codes",
               "host_cpus": os.cpu_count()}

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "e4m3",
            "data": DATA,
            "config": bench_config(wl, world),
            "timing": f"{args.steps} steps back to back in one CUDA graph over {n_sets} "
                      f"rotating operand sets of {per_set / 1e6:.0f} MB",
            "roofline": {"bound": "tensor", "kernel": "fp8_gemm_kernel",
                         "achieved": round(gemm_tflops, 1), "peak": round(fp8_peak, 1),
                         "unit": "TFLOP/s", "frac": round(gemm_tflops / fp8_peak, 4),
                         "traffic": traffic,
                         "peak_basis": f"2 x {pk['source']} bf16 dense ({pk['bf16_tflops']} TFLOP/s)",
                         "frac_of_nominal_4p5pf": round(gemm_tflops / NOMINAL_FP8_TFLOPS, 4),
                         "gemm_us": round(g_ms * 1e3, 2),
                         # launch time in SM cycles at the median sampled clock: equal
                         # times at different clocks mean a bound outside the SM clock
                         "gemm_sm_kcycles": (round(g_ms * clk["sm_mhz"], 1)
                                             if clk.get("sm_mhz") else None),
                         "sm_mhz_median": clk.get("sm_mhz")},
            "quantizer": {"achieved": round(quant_gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                          "frac": round(quant_gbs / pk["hbm_gbs"], 4),
                          "us": round(q_ms * 1e3, 2), "bytes": wl.quant_bytes},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 3), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                    "d2h_bytes_per_step": out_host.numel() * out_host.element_size(),
                    "ms_per_step": round(e2e_total / args.steps, 4),
                    "path": "C ABI fp8lin_fp8_linear_host with pinned host buffers (512-row "
                            "chunks: upload, kernels and download overlapped)"},
            "gpu_launches": 2 * args.steps,
            "clocks": clk,
            "watchdog_status": status,
        }
    # ---- north-star sharded configurations, measured after the headline (not part of
    # its timed region): config 4 strong-scaled over the ranks, config 5 column-parallel
    if not args.no_extras:
        sets = x = wq = ws = b = work = None  # free the headline's operands
        torch.cuda.empty_cache()
        extra_clocks = ClockSampler(local).start()
        try:
            cfg4 = mshard_cfg4(args, world, rank, dev, barrier)
        except Exception as e:  # the headline line is still printed
            cfg4 = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
        torch.cuda.empty_cache()
        try:
            cfg5 = nshard_cfg5(args, world, rank, dev, barrier)
        except Exception as e:
            cfg5 = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
        torch.cuda.empty_cache()
        eclk = extra_clocks.stop()
        if rank == 0:
            line["mshard_cfg4"] = cfg4
            line["nshard_cfg5"] = cfg5
            line["extras_clocks"] = eclk
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _max_over_ranks(vals, world, dev):
    """Element-wise max over ranks of a list of floats (device times)."""
    if world == 1:
        return list(vals)
    import torch.distributed as dist

    t = torch.tensor(list(vals), device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def _graph_ms(call, sets, steps, stream, barrier) -> float:
    """Device ms of ``steps`` calls back to back in one CUDA graph over ``sets``."""
    g = graph_launches(call, sets, steps, keep=len(sets))
    ms = time_graph(g, stream, barrier)
    del g
    return ms


def mshard_cfg4(args, world, rank, dev, barrier) -> dict:
    """Config 4: the FLUX single-stream block linears at batch 4 (linear1 18432 x 3072 ->
    21504, linear2 18432 x 15360 -> 3072) with the GLOBAL 18432 token rows split over the
    ranks (strong scaling), weights replicated, no collective. Each rank times its row
    block (steps back to back over rotating operand sets, as the headline); the job time
    is the max over ranks. Rank 0 then times all 18432 rows alone on its GPU, the one-GPU
    figure the efficiency is taken against (t1 / (N x tN)). Every timed leg starts after
    CFG_PAUSE_S idle on every rank: right after seconds of full-power GEMM graphs a GPU
    runs the next graph at lower clocks (one B200: the 2304-row linear2 block 102 us per
    step after a pause, 132 right after one 18432-row linear1 graph, 153 at 1500 MHz
    after four), and rank 0 would otherwise time its block right after its linear1
    reference."""
    import dataclasses

    import fp8linear_b200 as f
    from fp8linear_b200.sharding import row_range

    W = _workloads()
    stream = torch.cuda.current_stream(dev)

    def pause():
        barrier()
        time.sleep(CFG_PAUSE_S)
        barrier()

    def step(st):
        return f.fp8_linear(st["x"], st["wq"], st["ws"], st["b"])

    names = ("flux_linear1", "flux_linear2")
    t_n = {}
    for name in names:  # every rank's own row block, all ranks at once
        wl = W.WORKLOADS[name]
        s0, e0 = row_range(wl.M, world, rank)
        wl_r = dataclasses.replace(wl, M=e0 - s0)
        sets = operand_sets(wl_r, set_count(per_set_bytes(wl_r), dev), x_seed0=1000 * rank,
                            quantize_x=False)
        for i in range(args.warmup):
            step(sets[i % len(sets)])
        pause()
        t_n[name] = _max_over_ranks([_graph_ms(step, sets, args.steps, stream, barrier)],
                                    world, dev)[0] / args.steps
        del sets
        torch.cuda.empty_cache()
    t_1 = dict(t_n)
    if world > 1:  # the one-GPU references: all rows on rank 0's GPU
        import torch.distributed as dist

        for name in names:
            wl = W.WORKLOADS[name]
            t1 = torch.zeros(1, device=dev, dtype=torch.float64)
            sets = None
            if rank == 0:
                sets = operand_sets(wl, set_count(per_set_bytes(wl), dev), quantize_x=False)
                for i in range(args.warmup):
                    step(sets[i % len(sets)])
                torch.cuda.synchronize(dev)
            pause()
            if rank == 0:
                t1[0] = _graph_ms(step, sets, args.steps, stream,
                                  lambda: torch.cuda.synchronize(dev)) / args.steps
            del sets
            torch.cuda.empty_cache()
            dist.broadcast(t1, 0)
            t_1[name] = float(t1.item())
    out = {}
    for name in names:
        wl = W.WORKLOADS[name]
        tf_n = wl.flops / (t_n[name] * 1e-3) / 1e12
        tf_1 = wl.flops / (t_1[name] * 1e-3) / 1e12
        out[name.replace("flux_", "")] = {
            "global_M": wl.M, "K": wl.K, "N": wl.N, "rows_per_gpu_max": -(-wl.M // world),
            "value": round(tf_n, 1), "unit": "TFLOP/s", "ms_per_step": round(t_n[name], 4),
            "one_gpu_tflops": round(tf_1, 1), "one_gpu_ms": round(t_1[name], 4),
            "speedup": round(t_1[name] / t_n[name], 3),
            "efficiency": round(t_1[name] / (world * t_n[name]), 4)}
    out["scaling"] = "strong"
    out["how"] = ("fp8_linear (quantizer + GEMM) on each rank's block of the global 18432 "
                  f"rows, {args.steps} steps back to back in one CUDA graph over rotating "
                  f"operand sets, max over ranks; one_gpu: all rows on rank 0's GPU alone, "
                  f"timed after both row-block legs; {CFG_PAUSE_S} s idle before every leg")
    return out


def nshard_cfg5(args, world, rank, dev, barrier) -> dict:
    """Config 5 at M = 65536, K = N = 3072: column-parallel over the ranks (each rank
    holds N/world output channels and quantizes the full, replicated x), the output
    gathered to every rank as row-major [M, N] two ways: (a) the rank's fused linear, then
    NCCL all_gather_into_tensor + one interleave copy; (b) the all-gather fused into the
    GEMM epilogue (16-byte P2P stores into every rank's peer buffer over NVLink, then a
    one-element all-reduce). Both results are compared bit for bit with the unsharded
    one-GPU result computed on every rank. Steps run eagerly (x and the output are
    403 MB each, beyond L2), each bracketed by CUDA events; max over ranks."""
    import fp8linear_b200 as f
    from fp8linear_b200 import sharding as S
    from fp8linear_b200.capi import CApi

    W = _workloads()
    wl = W.WORKLOADS["sweep_M65536"]
    stream = torch.cuda.current_stream(dev)
    x = W.make_x(wl, gen_device="cuda")
    w, b = W.make_weight(wl, gen_device="cuda")
    wq, ws = f.quantize_weight(w)
    del w
    full = f.fp8_linear(x, wq, ws, b)

    def timed(fn, n):
        """Per-step device ms (total, to the mid event) of ``n`` eager steps."""
        for _ in range(args.warmup):
            fn(None)
        barrier()
        ev = []
        for _ in range(n):
            a, m, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            a.record(stream)
            fn(m)
            c.record(stream)
            ev.append((a, m, c))
        barrier()
        tot = sum(a.elapsed_time(c) for a, m, c in ev) / n
        mid = sum(a.elapsed_time(m) for a, m, c in ev) / n
        return tot, mid

    def unsharded(mark):
        o = f.fp8_linear(x, wq, ws, b)
        if mark is not None:
            mark.record(stream)
        return o

    t_full, _ = timed(unsharded, args.steps)
    t_full = _max_over_ranks([t_full], world, dev)[0]
    res = {"M": wl.M, "K": wl.K, "N": wl.N, "one_gpu_ms": round(t_full, 4),
           "one_gpu_tflops": round(wl.flops / (t_full * 1e-3) / 1e12, 1)}
    if world == 1:
        res["note"] = "one GPU: the unsharded linear only"
        return res
    wqs, wss, bs = S.shard_columns(wq, ws, b, world, rank)
    n_loc = wl.N // world
    peer_bytes = (world - 1) * wl.M * n_loc * 2  # bytes each rank sends (and receives)
    holder = {}

    def nccl_step(mark):
        loc = f.fp8_linear(x, wqs, wss, bs)
        if mark is not None:
            mark.record(stream)
        holder["nccl"] = S.gather_columns(loc, world)

    t_nccl, t_comp = timed(nccl_step, args.steps)
    ok_nccl = bool(torch.equal(holder.pop("nccl"), full))
    capi = CApi()
    work = torch.empty(capi.workspace_size(wl.M, wl.K), dtype=torch.uint8, device=dev)
    fused = S.FusedColumnParallel(wl.M, wl.N, torch.bfloat16, dev, peer=capi)
    try:
        def fused_step(mark):
            holder["fused"] = fused(x, wqs, wss, bs, capi, workspace=work)
            if mark is not None:
                mark.record(stream)

        t_fused, _ = timed(fused_step, args.steps)
        ok_fused = bool(torch.equal(holder.pop("fused"), full))
        torch.cuda.synchronize(dev)
    finally:
        fused.close()
    t_nccl, t_comp, t_fused = _max_over_ranks([t_nccl, t_comp, t_fused], world, dev)
    ok = _max_over_ranks([0.0 if ok_nccl else 1.0, 0.0 if ok_fused else 1.0], world, dev)
    link = 770.0  # measured peer copy GB/s per direction on this pool's B200s
    res.update({
        "parallelism": f"N-shard x{world} (column parallel, x replicated)",
        "scaling": "strong",
        "peer_bytes_per_rank": peer_bytes,
        "nccl": {"ms_per_step": round(t_nccl, 4),
                 "value": round(wl.flops / (t_nccl * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                 "compute_ms": round(t_comp, 4), "allgather_ms": round(t_nccl - t_comp, 4),
                 "allgather_gbs": round(peer_bytes / ((t_nccl - t_comp) * 1e-3) / 1e9, 1),
                 "bitexact_vs_unsharded": ok[0] == 0.0},
        "fused": {"ms_per_step": round(t_fused, 4),
                  "value": round(wl.flops / (t_fused * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                  "peer_store_gbs": round(peer_bytes / (t_fused * 1e-3) / 1e9, 1),
                  "bitexact_vs_unsharded": ok[1] == 0.0,
                  "roofline": {"bound": "nvlink", "peak_gbs_per_direction": link,
                               "target_ms": round(max(peer_bytes / (link * 1e9) * 1e3,
                                                      t_comp), 4),
                               "frac": round(max(peer_bytes / (link * 1e9) * 1e3, t_comp)
                                             / t_fused, 4)}},
        "how": f"{args.steps} eager steps each, CUDA events per step, max over ranks; "
               "compute_ms: the rank's column-block linear alone; fused roofline: the "
               "slower of the rank's compute and its peer bytes at 770 GB/s per direction",
    })
    return res


def measure_workload(name: str, steps: int, warmup: int, fmt: str = "fp8") -> dict:
    """Per-workload device times of the fused op, the GEMM alone and the quantizer
    alone: each is ``max(steps, sets)`` launches back to back in one CUDA graph over
    rotating operand sets (inputs larger than L2), averaged per launch. ``fmt`` "mx" / "nv":
    the MXFP8 / NVFP4 ops (mxfp8_linear, mxfp8_gemm, quantize_mxfp8 / the nvfp4 ones)."""
    import fp8linear_b200 as f

    wl = _workloads().WORKLOADS[name]
    dev = torch.device("cuda", torch.cuda.current_device())
    n_sets = set_count(per_set_bytes(wl), dev)
    sets = operand_sets(wl, n_sets, fmt=fmt)
    stream = torch.cuda.current_stream(dev)
    reps = max(steps, n_sets)

    def timed(call):
        time.sleep(SWEEP_PAUSE_S)  # let the power state settle after the previous replays
        for i in range(warmup):
            call(sets[i % n_sets])
        g = graph_launches(call, sets, reps, keep=n_sets)
        ms = time_graph(g, stream, lambda: torch.cuda.synchronize(dev)) / reps
        del g
        return ms

    # the bandwidth-bound quantizer first: timed after seconds of full-power GEMM replays,
    # a memory-bound kernel reads slow (the power-capped clocks outlast the GEMMs)
    extra = {}
    if fmt == "modulated":
        quant = timed(lambda st: f.layernorm_modulate_quantize_fp8(st["x"], st["shift"],
                                                                   st["scale"]))
        unq = timed(lambda st: f.quantize_fp8(unfused_modulation(st["x"], st["shift"],
                                                                 st["scale"])))
        gemm = timed(lambda st: f.fp8_gemm(st["xq"], st["xs"], st["wq"], st["ws"], st["b"]))
        fused = timed(lambda st: f.fp8_linear_modulated(st["x"], st["shift"], st["scale"], st["wq"],
                                                        st["ws"], st["b"]))
        unf = timed(lambda st: f.fp8_linear(unfused_modulation(st["x"], st["shift"], st["scale"]),
                                            st["wq"], st["ws"], st["b"]))
        extra = {"unfused_us": round(unf * 1e3, 2), "unfused_quant_us": round(unq * 1e3, 2)}
    else:
        lin_op, gemm_op, quant_op = {
            "fp8": (f.fp8_linear, f.fp8_gemm, f.quantize_fp8),
            "mx": (f.mxfp8_linear, f.mxfp8_gemm, f.quantize_mxfp8),
            "nv": (f.nvfp4_linear, f.nvfp4_gemm, f.quantize_nvfp4)}[fmt]
        quant = timed(lambda st: quant_op(st["x"]))
        gemm = timed(lambda st: gemm_op(st["xq"], st["xs"], st["wq"], st["ws"], st["b"]))
        fused = timed(lambda st: lin_op(st["x"], st["wq"], st["ws"], st["b"]))
    # quantizer bytes: read 2MK, write the codes (MK, NV MK/2) and the scales (4M fp32,
    # MK/32 e8m0, MK/16 ue4m3)
    mk = wl.M * wl.K
    qbytes = {"fp8": 3 * mk + 4 * wl.M, "mx": 3 * mk + mk // 32,
              "nv": 2 * mk + mk // 2 + mk // 16, "modulated": 3 * mk + 4 * wl.M}[fmt]
    pk = peaks()
    # bandwidth-aware roofline for the GEMM: min(tensor peak, AI x HBM); the e4m3 forms run
    # at 2x and e2m1 at 4x the measured bf16 rate (the nominal dense ratios), and the NVFP4
    # operands are half the bytes (+ one scale byte per 16 elements)
    if fmt == "nv":
        gbytes = (wl.M + wl.N) * wl.K * 9 // 16 + 2 * wl.N + 2 * wl.M * wl.N
        rate = 4.0
    else:
        gbytes, rate = wl.gemm_bytes, 2.0
    ai = wl.flops / gbytes
    roof = min(rate * pk["bf16_tflops"], ai * pk["hbm_gbs"] / 1e3)
    g_tf = wl.flops / (gemm * 1e-3) / 1e12
    return {"workload": name, "format": fmt, "M": wl.M, "K": wl.K, "N": wl.N, "sets": n_sets,
            "fused_us": round(fused * 1e3, 2),
            "fused_tflops": round(wl.flops / (fused * 1e-3) / 1e12, 1),
            "gemm_us": round(gemm * 1e3, 2), "gemm_tflops": round(g_tf, 1),
            "gemm_roofline_tflops": round(roof, 1), "gemm_frac": round(g_tf / roof, 4),
            "quant_us": round(quant * 1e3, 2),
            "quant_gbs": round(qbytes / (quant * 1e-3) / 1e9, 1),
            "quant_frac": round(qbytes / (quant * 1e-3) / 1e9 / pk["hbm_gbs"], 4), **extra}


def reference_workload(name: str, steps: int, warmup: int, fmt: str = "fp8") -> dict:
    """Device time of the reference's own compiled ops on one workload."""
    wl = _workloads().WORKLOADS[name]

    class A:  # the knobs reference_gpu_timing reads
        pass

    a = A()
    a.steps, a.warmup = steps, warmup
    r = reference_gpu_timing(wl, a, fmt)
    if r and "ms_per_step" in r:
        r = {"workload": name, "format": fmt, "ref_fused_us": round(r["ms_per_step"] * 1e3, 2),
             "ref_fused_tflops": r["value"]}
    else:
        r = {"workload": name, "format": fmt, **(r or {})}
    return r


def run_launch_list(args):
    """Eager launches for a per-kernel launch list: for each workload of ``--sweep``, a
    marker kernel (torch.cuda._sleep), ``--steps`` calls of the fused linear over rotating
    operand sets (ours: fp8_linear; ``--impl reference``: the reference's fp8_linear and
    the .to(bf16) its Fp8Linear.forward applies), then another marker. Run under
    ``ncu --metrics gpu__time_duration.sum``, the kernels between two markers are one
    workload's calls, which splits the reference op into its quantizer, cuBLASLt GEMM,
    dequant and cast kernels. One JSON line per workload names the order."""
    W = _workloads()
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    names = args.sweep.split(",") if args.sweep != "all" else list(W.WORKLOADS)
    if args.impl == "reference":
        from oracle import build_ref

        ref = build_ref.load()
        if ref is None:
            print(json.dumps({"unavailable": "oracle/_ref not built"}))
            return
        qw = ref.quantize_weight

        def lin(st):
            return ref.fp8_linear(st["x"], st["wq"], st["ws"], st["b"]).to(st["x"].dtype)
    else:
        import fp8linear_b200 as f

        qw = f.quantize_weight

        def lin(st):
            return f.fp8_linear(st["x"], st["wq"], st["ws"], st["b"])
    for n in names:
        wl = W.WORKLOADS[n]
        extra = 4 * wl.M * wl.N if args.impl == "reference" else 0  # its fp32 [M, N]
        n_sets = set_count(per_set_bytes(wl) + extra, dev)
        sets = []
        for i in range(n_sets):
            x = W.make_x(wl, seed=7919 * i, gen_device="cuda")
            w, b = W.make_weight(wl, seed=7919 * i, gen_device="cuda")
            wq, ws = qw(w)
            sets.append({"x": x, "wq": wq, "ws": ws, "b": b})
            del w
        for i in range(args.warmup):
            lin(sets[i % n_sets])
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(1000)
        outs = [lin(sets[i % n_sets]) for i in range(args.steps)]
        torch.cuda._sleep(1000)
        torch.cuda.synchronize(dev)
        print(json.dumps({"workload": n, "impl": args.impl, "calls": args.steps,
                          "sets": n_sets}), flush=True)
        del sets, outs
        torch.cuda.empty_cache()


def run_sweep(args):
    WORKLOADS = _workloads().WORKLOADS

    torch.cuda.set_device(0)
    names = args.sweep.split(",") if args.sweep != "all" else list(WORKLOADS)
    for n in names:
        r = reference_workload(n, args.steps, args.warmup, args.format) \
            if args.impl == "reference" else measure_workload(n, args.steps, args.warmup, args.format)
        print(json.dumps(r), flush=True)
        torch.cuda.empty_cache()


def run_nshard(args):
    """Column-parallel (N-shard) FP8 linear: every rank quantizes the full x, runs the
    fused op on its block of output channels, and the blocks are all-gathered over NCCL
    into row-major [M, N] (strong scaling: the total work is fixed)."""
    import torch.distributed as dist

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    import fp8linear_b200 as f
    from fp8linear_b200 import sharding as S

    W = _workloads()
    make_weight, make_x = W.make_weight, W.make_x
    wl = W.WORKLOADS[args.workload]
    x = make_x(wl, gen_device="cuda")                 # replicated activations
    w, b = make_weight(wl, gen_device="cuda")
    wq, ws = f.quantize_weight(w)
    del w
    wqs, wss, bs = S.shard_columns(wq, ws, b, world, rank)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    fused = None
    if args.fused:
        from fp8linear_b200.capi import CApi

        capi = CApi()
        fused = S.FusedColumnParallel(wl.M, wl.N, torch.bfloat16, dev) if world > 1 else None
        work = torch.empty(capi.workspace_size(wl.M, wl.K), dtype=torch.uint8, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def step(timing=None):
        if fused is not None:
            # one kernel pair: the epilogue writes every rank's buffer; the GEMM and the
            # NVLink transfer are one, so there is no separate compute/gather split
            out = fused(x, wqs, wss, bs, capi, workspace=work)
            if timing is not None:
                timing.record(stream)
            return out
        local = f.fp8_linear(x, wqs, wss, bs)
        if timing is not None:
            timing.record(stream)
        return S.gather_columns(local, world) if world > 1 else local

    clocks = ClockSampler(local).start()
    for _ in range(args.warmup):
        flush.zero_()
        step()
    barrier()
    ev = []
    for _ in range(args.steps):
        flush.zero_()
        a, m, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record(stream)
        step(m)
        c.record(stream)
        ev.append((a, m, c))
    barrier()
    clk = clocks.stop()
    total = sum(a.elapsed_time(c) for a, m, c in ev)
    comp = sum(a.elapsed_time(m) for a, m, c in ev)
    if world > 1:
        t = torch.tensor([total, comp], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total, comp = (float(v) for v in t.tolist())
    value = wl.flops * args.steps / (total * 1e-3) / 1e12
    if rank == 0:
        gather_bytes = (world - 1) * wl.M * (wl.N // world) * 2
        print(json.dumps({
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total / args.steps, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "e4m3",
            "data": "synthetic (seeded FLUX-shaped tensors)",
            "config": {"workload": wl.name, "M": wl.M, "K": wl.K, "N": wl.N,
                       "parallelism": f"N-shard x{world} (column parallel) + " + (
                           "all-gather fused into the GEMM epilogue (NVLink P2P stores)"
                           if args.fused else "NCCL all-gather"),
                       "l2": "flushed between steps (256 MiB write)"},
            "compute_ms_per_step": None if args.fused else round(comp / args.steps, 5),
            "allgather_ms_per_step": None if args.fused else round((total - comp) / args.steps, 5),
            "allgather_bytes_per_rank": gather_bytes,
            "gpu_launches": 2 * args.steps, "clocks": clk}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- reference arm


def run_reference(args):
    """The reference arm: the reference's path on the host CPU (the oracle port, all host
    threads), on this arm's workload, metric and config. Under torchrun rank 0 alone runs
    it; each step is one rank's share of the job (all ``M_per_gpu`` token rows), so the
    rate is what the host's cores sustain on the job. Nothing of this package is
    imported: only the oracle's libraries (and, for ``gpu_reference``, the reference's
    own compiled ops) are loaded."""
    world, rank, local = dist_env()
    if rank != 0:
        return
    wl = _workloads().WORKLOADS[args.workload]
    rows = args.ref_rows if args.ref_rows > 0 else wl.M
    threads = os.cpu_count() or 1
    st = cpu_reference_runner(wl, rows, threads=threads)
    for _ in range(args.warmup):
        st()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        st()
        times.append(time.perf_counter() - t0)
    per = sum(times) / len(times)
    value = 2 * rows * wl.N * wl.K / per / 1e12
    sample = (f"{rows} of {wl.M} token rows per step of {wl.name} (one rank's share"
              f"{'' if world == 1 else f' of {world}'}); the reference has no CPU kernels, so "
              "its path on a CPU is the CPU restatement (oracle port): per-token e4m3 quant, "
              "fp32 matmul of decoded codes, dequant + bias")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 5),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(per * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3",
        "data": DATA,
        "config": bench_config(wl, world),
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    gpu_ref = reference_gpu_timing(wl, args) if torch.cuda.is_available() else None
    if gpu_ref is not None:
        line["gpu_reference"] = gpu_ref
    print(json.dumps(line), flush=True)


def reference_gpu_timing(wl, args, fmt: str = "fp8"):
    """Device time of the reference's own compiled CUDA ops (cuBLASLt FP8 GEMM + dequant
    kernel, fp16 out, then the .to(bf16) cast Fp8Linear.forward applies), if built,
    timed like our op: launches back to back over rotating operand sets. ``fmt`` "mx":
    its mxfp8_linear (quantize_mxfp8 + cuBLASLt VEC32_UE8M0 GEMM with bias, fp16 out);
    "nv": its nvfp4_linear (quantize_nvfp4 + cuBLASLt VEC16_UE4M3 e2m1 GEMM)."""
    try:
        from oracle import build_ref
        ref = build_ref.load()
    except Exception as e:  # pragma: no cover
        return {"unavailable": f"reference ops failed to load: {e}"}
    if ref is None:
        return {"unavailable": "oracle/_ref not built"}
    W = _workloads()
    make_weight, make_x = W.make_weight, W.make_x

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n_sets = set_count(per_set_bytes(wl) + 4 * wl.M * wl.N, dev)  # + its fp32 [M, N] buffer
    sets = []
    for i in range(n_sets):
        x = make_x(wl, seed=7919 * i, gen_device="cuda")
        w, b = make_weight(wl, seed=7919 * i, gen_device="cuda")
        qw = {"fp8": ref.quantize_weight, "mx": ref.quantize_mxfp8, "nv": ref.quantize_nvfp4,
              "modulated": ref.quantize_weight}[fmt]
        wq, ws = qw(w)
        st = {"x": x, "wq": wq, "ws": ws, "b": b}
        if fmt == "modulated":
            st["shift"], st["scale"] = modulation(wl, 7919 * i + 17)
        sets.append(st)
        del w
    stream = torch.cuda.current_stream(dev)
    lin = {"fp8": ref.fp8_linear, "mx": ref.mxfp8_linear, "nv": ref.nvfp4_linear,
           "modulated": ref.fp8_linear}[fmt]

    def call(st):
        x = st["x"]
        if fmt == "modulated":  # the FLUX block's LayerNorm + modulation before the linear
            x = unfused_modulation(x, st["shift"], st["scale"])
        return lin(x, st["wq"], st["ws"], st["b"]).to(st["x"].dtype)

    try:
        call(sets[0])
    except RuntimeError as e:  # e.g. cuBLASLt offers no MXFP8 algorithm for a few tokens
        return {"unavailable": f"the reference op raised: {str(e).splitlines()[0][:160]}"}
    for i in range(max(3, args.warmup)):
        call(sets[i % n_sets])
    reps = max(args.steps, n_sets)
    how = "one CUDA graph"
    try:
        g = graph_launches(call, sets, reps, keep=n_sets)
        ms = time_graph(g, stream, lambda: torch.cuda.synchronize(dev)) / reps
        del g
    except Exception:  # pragma: no cover - capture not supported by the library path
        how = "eager launches (graph capture failed)"
        torch.cuda.synchronize(dev)
        a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(reps):
            call(sets[i % n_sets])
        c.record(stream)
        torch.cuda.synchronize(dev)
        ms = a.elapsed_time(c) / reps
    return {"value": round(wl.flops / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
            "ms_per_step": round(ms, 4),
            "timing": f"{reps} steps back to back ({how}) over {n_sets} rotating operand sets",
            "what": "reference fp8_linear (quantize_fp8 + cuBLASLt FP8 GEMM into fp32 + "
                    "dequant_bias_kernel, fp16 out) + .to(bf16), compiled from the "
                    "reference sources for sm_100a"}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default="flux_qkv")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-rows", type=int, default=128,
                    help="token rows of the cpu_baseline sample in this arm's line")
    ap.add_argument("--ref-rows", type=int, default=0,
                    help="token rows per step of the reference arm (0: all M_per_gpu rows)")
    ap.add_argument("--cpu-seconds", type=float, default=5.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the config-4 (strong M-shard) and config-5 (N-shard) legs")
    ap.add_argument("--mode", choices=["mshard", "nshard"], default="mshard",
                    help="multi-GPU split: token rows (default, no collective) or output "
                         "channels with an NCCL all-gather")
    ap.add_argument("--fused", action="store_true",
                    help="with --mode nshard: fuse the all-gather into the GEMM epilogue")
    ap.add_argument("--format", choices=["fp8", "mx", "nv", "modulated"], default="fp8",
                    help="with --sweep: per-channel FP8 ops (default), the MXFP8 or the "
                         "NVFP4 ops, or the LayerNorm + modulation fused into the quantizer "
                         "against the unfused FLUX chain")
    ap.add_argument("--sweep", default="",
                    help="'all' or comma-separated workloads: one JSON line of per-kernel "
                         "device times per workload (not the driver's line)")
    ap.add_argument("--launch-list", action="store_true",
                    help="with --sweep: eager calls between marker kernels, for an ncu "
                         "per-kernel launch list (no timing printed)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)  # the timing rules ask for at least 3 warm-up steps
    if args.sweep and args.launch_list:
        run_launch_list(args)
    elif args.sweep:
        run_sweep(args)
    elif args.mode == "nshard" and args.impl != "reference":
        run_nshard(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
