#!/usr/bin/env python
"""Decoded windows/sec of the Cortex decoder forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config cfg1] [--no-graph]

One process per GPU (torchrun for N > 1). Each rank decodes its own batch of
windows (weak scaling: the BASELINE workload, Cortex-S bf16, 32 windows x 512
events, per GPU); no collective touches the data path -- the only collectives
are the timing barriers and the max-over-ranks reduction. A step is one forward
over one batch. Rank 0 prints one JSON line.

Timing: W untimed warm-up steps; then K steps, each preceded by an L2 flush
(a 256 MiB memset, then a 256 MiB read of another buffer that writes the
memset's dirty lines back, both outside the timed interval) and bracketed by CUDA events on
the launching stream; the run total is the sum of the K step times, max over
ranks. ``value`` uses inputs resident in HBM and a CUDA-graph replay of the
forward; ``e2e`` calls the public API (CortexModel.forward) with host index
tensors every step, so the host work (the native staging of the four int64
arrays into one int32 batch in pinned memory), the host->device copy of that
batch, the Python/ctypes call path, the graph replay of the batch's bucket and
the device->host read of the result are inside its timed interval.

``--impl reference`` times the reference algorithm on the host CPU (the CPU
oracle port in oracle/, all host threads) on the same workload.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "cortex-engine_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "decoded windows/sec (Cortex-S, 512 ev/sample) at 1/2/4/8 B200; p99 batch latency"
# DRAM traffic of the mlp.0 + GELU GEMM launch (8192 x 512 x 2048, bf16 weights)
# from one ncu capture on B200 (10.56 MB read + 45 KB written; the 32 MB
# output is still in L2 when the kernel ends).
GELU_GEMM_TRAFFIC_BYTES = 10_603_008
UNIT = "windows/s"


def percentile(vals, p):
    """Linear-interpolation percentile (scripts/load_test.py:67-76 of the reference)."""
    if not vals:
        return 0.0
    sv = sorted(vals)
    idx = (len(sv) - 1) * p / 100
    lo, hi = math.floor(idx), math.ceil(idx)
    if lo == hi:
        return sv[lo]
    return sv[lo] + (sv[hi] - sv[lo]) * (idx - lo)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p.get("bf16_tflops_sustained"), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """SM clock and throttle reasons sampled every few milliseconds through NVML
    while the timed region runs (nvidia-smi's 200 ms loop would see at most one
    sample of a sub-second timed region); nvidia-smi is the fallback."""

    # NVML clocks-event-reason bits
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index: int, interval_s: float = 0.005):
        self.dev = device_index
        self.interval = interval_s
        self.samples = []
        self.max_mhz = None
        self.err = None
        self._stop = None
        self._thread = None

    def _handle(self):
        import pynvml
        import torch

        try:
            pr = torch.cuda.get_device_properties(self.dev)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = self.dev
            if vis:
                try:
                    idx = int(vis.split(",")[self.dev])
                except (ValueError, IndexError):
                    pass
            return pynvml.nvmlDeviceGetHandleByIndex(idx)

    def start(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            h = self._handle()
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # no NVML: report it instead of guessing
            self.err = f"nvml unavailable: {type(e).__name__}"
            return
        self._stop = threading.Event()
        first = threading.Event()

        def loop():
            while not self._stop.is_set():
                try:
                    mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((mhz, rs))
                except Exception as e:
                    self.err = f"nvml sample failed: {type(e).__name__}"
                first.set()
                time.sleep(self.interval)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        first.wait(timeout=2.0)  # sampling is live before the timed region starts

    def stop(self):
        if self._thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "unavailable"]}
        self._stop.set()
        self._thread.join(timeout=2.0)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz,
                    "reasons": [self.err or "no samples"]}
        mhz = sorted(m for m, _ in self.samples)
        reasons = set()
        for _, rs in self.samples:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(mhz), "source": "nvml"}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ── CPU (reference algorithm) timing ─────────────────────────────────────────


def cpu_forward_timer(wl, seed: int, batch: int, threads: int):
    """Returns a closure running the oracle forward once on `batch` windows."""
    import torch

    from cortex.workloads import build_model, make_inputs
    from oracle import cortex_oracle as O

    torch.set_num_threads(threads)
    model = build_model(wl, "cpu")
    p = {k: v for k, v in model.state_dict().items()}
    inp, _ = make_inputs(wl, seed=seed, batch=batch)
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")

    def run():
        return O.forward(p, wl.config, *(inp[k] for k in cols))

    return run


def cpu_baseline(wl, seconds: float):
    import torch

    threads = os.cpu_count() or 1
    batch = wl.batch if wl.events_per_sample is not None else 32
    run = cpu_forward_timer(wl, seed=1000, batch=batch, threads=threads)
    run()  # warm-up
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    tot = sum(times)
    try:
        cpu_model = open("/proc/cpuinfo").read().split("model name")[1].split("\n")[0].strip(" :\t")
    except Exception:
        cpu_model = "unknown"
    return {"value": round(batch * len(times) / tot, 2), "unit": UNIT, "cores": threads,
            "kind": "port",
            "sample": f"{len(times)} CPU forwards of {batch} windows ({wl.name}, "
                      f"{wl.dtype}) via oracle/cortex_oracle.py, torch {torch.__version__}, "
                      f"{threads} threads on {cpu_model}",
            "p99_batch_latency_ms": round(1e3 * percentile(times, 99), 2)}


def run_reference(args, wl):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    batch = wl.batch if wl.events_per_sample is not None else 32
    run = cpu_forward_timer(wl, seed=1000, batch=batch, threads=threads)
    for _ in range(args.warmup):
        run()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    tot = sum(times)
    value = batch * len(times) / tot
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * tot / len(times), 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if wl.dtype == "bfloat16" else "f32",
        "data": "synthetic",
        "config": {"workload": f"{wl.name}: {wl.description}; CPU sample of {batch} windows "
                               "per step", "global_batch": batch,
                   "parallelism": "host CPU, all threads"},
        "p99_batch_latency_ms": round(1e3 * percentile(times, 99), 3),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{batch} windows per step, oracle/cortex_oracle.py "
                                   "(the reference's eager PyTorch algorithm restated)"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ── GPU (this framework) ─────────────────────────────────────────────────────


class L2Flush:
    """Evicts L2 between timed steps: a 256 MiB memset (the flush), then a read
    of another 256 MiB buffer, so that the dirty lines the memset leaves in L2
    are written back here and not inside the next timed interval."""

    def __init__(self, dev):
        import torch

        self.buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        self.scrub = torch.zeros(32 << 20, dtype=torch.int64, device=dev)
        self.sink = torch.empty((), dtype=torch.int64, device=dev)

    def __call__(self):
        import torch

        self.buf.zero_()
        torch.sum(self.scrub, dim=0, dtype=torch.int64, out=self.sink)


def gemm_roofline(model, wl, dev, iters: int):
    """Time the forward's largest tcgen05 GEMM launch (MLP up-projection with the
    fused GELU epilogue, M = B*L rows) alone, with CUDA events, L2 flushed."""
    import torch

    from cortex import _lib as L
    from cortex.kernels import _ops

    cfg = wl.config
    M = wl.batch * cfg.num_latents
    K = cfg.latent_dim
    blk = model.encoder.self_attn_blocks[0]
    lin = blk.mlp[0]
    w = getattr(lin, "weight_int8", None)
    sc = getattr(lin, "weight_scale", None)
    if w is None:
        w = lin.weight
    N = w.shape[0]
    x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    flush = L2Flush(dev)
    for _ in range(3):
        _ops.linear(x, w, w_scale=sc, epi=L.CK_EPI_GELU, out=out)
    # one launch per graph replay: the host call path stays out of the interval
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _ops.linear(x, w, w_scale=sc, epi=L.CK_EPI_GELU, out=out)
    graph.replay()
    times = []
    st = torch.cuda.current_stream(dev)
    for _ in range(iters):
        flush()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        graph.replay()
        e1.record(st)
        e1.synchronize()
        times.append(e0.elapsed_time(e1) * 1e-3)
    del graph
    avg = sum(times) / len(times)
    flops = 2.0 * M * N * K
    return avg, flops, (M, K, N), ("int8" if sc is not None else "bf16")


def run_ours(args, wl):
    import torch
    import torch.distributed as dist

    from cortex import _lib
    from cortex.workloads import build_model, make_inputs

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    model = build_model(wl, dev)
    B = wl.batch if wl.events_per_sample is not None else wl.batch
    inp, counts = make_inputs(wl, seed=1000 + rank, batch=B)
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")
    E = int(inp["neuron_ids"].shape[0])
    dinp = [inp[k].to(dev) for k in cols]
    st = torch.cuda.current_stream(dev)
    flush = L2Flush(dev)

    with torch.no_grad():
        # launches per forward (the library counts every kernel it launches)
        c0 = _lib.load().ck_launch_count()
        out = model(*dinp, batch_size=B)["behavior"]
        torch.cuda.synchronize()
        launches_per_fwd = _lib.load().ck_launch_count() - c0
        _lib.check_device_status("bench warm-up")

        for _ in range(max(args.warmup, 3)):
            out = model(*dinp, batch_size=B)["behavior"]
        graph = None
        if not args.no_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = model(*dinp, batch_size=B)["behavior"]
            for _ in range(2):
                graph.replay()
        torch.cuda.synchronize()

        def step():
            if graph is not None:
                graph.replay()
            else:
                model(*dinp, batch_size=B)

        sampler = ClockSampler(local)
        sampler.start()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        barrier()
        torch.cuda.synchronize()
        for k in range(args.steps):
            flush()
            ev[k][0].record(st)
            step()
            ev[k][1].record(st)
        torch.cuda.synchronize()
        barrier()
        clocks = sampler.stop()
        step_s = [a.elapsed_time(b) * 1e-3 for a, b in ev]
        total = max_over_ranks(sum(step_s))
        p99 = max_over_ranks(percentile(step_s, 99))
        p50 = max_over_ranks(percentile(step_s, 50))
        _lib.check_device_status("bench timed region")
        if args.only_forward:  # profiling runs: just the timed forwards
            if world > 1:
                dist.destroy_process_group()
            if rank == 0:
                print(json.dumps({"metric": METRIC, "value": round(world * B * args.steps / total, 2),
                                  "unit": UNIT, "n_gpus": world, "steps": args.steps,
                                  "warmup": args.warmup,
                                  "ms_per_step": round(1e3 * total / args.steps, 4),
                                  "mode": "forward only (profiling run)"}), flush=True)
            return

        # end-to-end through the public API: host index tensors in, host result out
        host_idx = [inp[k] for k in cols]  # the caller's int64 host tensors
        host_out = torch.empty(B, wl.config.behavior_dim, dtype=out.dtype).pin_memory()
        for _ in range(max(args.warmup, 3)):
            r = model(*host_idx)["behavior"]
            host_out.copy_(r, non_blocking=True)
        torch.cuda.synchronize()
        eev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        barrier()
        torch.cuda.synchronize()
        for k in range(args.steps):
            flush()
            # idle GPU: the interval starts when the host call starts, so the
            # host-side staging and call path are inside it
            torch.cuda.synchronize()
            eev[k][0].record(st)
            r = model(*host_idx)["behavior"]  # staging, one H2D copy, graph replay
            host_out.copy_(r, non_blocking=True)
            eev[k][1].record(st)
            eev[k][1].synchronize()  # the caller reads the result
        barrier()
        e2e_s = [a.elapsed_time(b) * 1e-3 for a, b in eev]
        e2e_total = max_over_ranks(sum(e2e_s))
        # the one host->device copy per step: the packed int32 batch of the bucket
        from cortex.batching import capacity_for

        h2d = 4 * _lib.batch_words(capacity_for(E))
        d2h = host_out.numel() * host_out.element_size()

        gemm = None
        if rank == 0:
            gemm = gemm_roofline(model, wl, dev, iters=max(10, min(args.steps, 50)))

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    hbm, tf_burst, tf_sust, peak_kind = peaks()
    avg_s, flops, shape, wkind = gemm
    achieved = flops / avg_s / 1e12
    value = world * B * args.steps / total
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if wl.dtype == "bfloat16" else "f32", "data": "synthetic",
        "config": {"workload": f"{wl.name}: {wl.description} per GPU", "global_batch": world * B,
                   "events_per_window": wl.events_per_sample, "events_per_gpu": E,
                   "parallelism": f"{world} independent replicas, batch-sharded, no collectives",
                   "l2": "flushed before every step, outside the timed interval: a 256 MiB "
                         "memset, then a 256 MiB read of another buffer so that the memset's "
                         "dirty lines are written back before the interval",
                   "cuda_graph": graph is not None},
        "p50_batch_latency_ms": round(1e3 * p50, 4),
        "p99_batch_latency_ms": round(1e3 * p99, 4),
        "e2e": {"value": round(world * B * args.steps / e2e_total, 2), "unit": UNIT,
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "p99_batch_latency_ms": round(1e3 * percentile(e2e_s, 99), 4)},
        "roofline": {"kernel": f"gemm_tc_kernel (MLP up-projection + GELU, M,K,N={shape}, "
                               f"{wkind} weights)",
                     "bound": "tensor", "achieved": round(achieved, 1), "peak": tf_burst,
                     "unit": "TFLOP/s", "frac": round(achieved / tf_burst, 4),
                     "peak_kind": f"{peak_kind} bf16 burst",
                     "traffic": GELU_GEMM_TRAFFIC_BYTES if wl.name == "cfg1" else None,
                     "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + "
                                     "dram__bytes_write.sum, one capture of this launch)",
                     "algorithmic_bytes": int(2 * (shape[0] * shape[1] + shape[1] * shape[2]
                                                   + shape[0] * shape[2])),
                     "avg_launch_us": round(avg_s * 1e6, 2)},
        "clocks": clocks,
        "gpu_launches": int(launches_per_fwd) * args.steps,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wl, args.cpu_seconds)
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=25)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="cfg1")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only-forward", action="store_true",
                    help="time the forwards only (no e2e / roofline / CPU legs); for ncu runs")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    args = ap.parse_args()
    from cortex.workloads import WORKLOADS

    wl = WORKLOADS[args.config]
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
