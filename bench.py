#!/usr/bin/env python
"""Decoded windows/sec of the Cortex decoder forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config cfg1] [--global-batch G] [--micro-batch M]
                    [--no-graph] [--no-configs] [--no-cpu-baseline]

One process per GPU (torchrun for N > 1). A step is one decode of a batch of
windows. The global batch is generated once from a fixed seed and split across
the ranks into contiguous window ranges balanced by event count
(``cortex.sharding.shard_bounds`` / ``slice_events``); no collective touches the
data path -- the only collectives are the timing barriers and the
max-over-ranks reductions. By default every rank gets the workload's batch
(32 windows for cfg1), so the global batch grows with N (weak scaling); with
``--global-batch G`` the G windows are split across the N ranks (strong
scaling). A rank's shard runs in micro-batches of ``--micro-batch`` windows
(default: the whole shard, or 256 windows for cfg4), one CUDA graph each.

Timing: W untimed warm-up steps; then K steps, each preceded by an L2 flush
(a 256 MiB memset, then a 256 MiB read of another buffer that writes the
memset's dirty lines back, both outside the timed interval) and bracketed by
CUDA events on the launching stream; the run total is the sum of the K step
times, max over ranks. ``value`` uses inputs resident in HBM; ``e2e`` calls the
public API (CortexModel.forward) with host index tensors every step, so the
host staging, the host->device copy, the Python/ctypes call path, the graph
replay and the device->host read of the result are inside its interval.

After the timed steps (all outside ``value``):
* a latency pass of 200 batches after 25 warm-up, for p50/p99 batch latency;
* a traced eager forward (the library's launch trace: two CUDA events around
  every kernel on its own stream) that gives each kernel class's device time,
  and from it the roofline fraction of every class against the measured peaks;
* at N = 1, a ``configs`` block with the same figures for the other named
  configurations (cfg2 INT8, cfg3 ragged, cfg4 Cortex-M INT8), and the CPU
  baseline: the reference package's own eager forward, timed in a child
  process on the host cores, and the CPU port in oracle/ beside it.

``--impl reference`` times the reference's own CPU forward (the installed
reference package in baseline/_ref, ``use_kernels=False``, all host threads)
on the same seeded windows; without that install it times the CPU port in
oracle/ and says so.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import re
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "cortex-engine_b200")
REF_PKG = os.path.join(ROOT, "baseline", "_ref")

METRIC = "decoded windows/sec (Cortex-S, 512 ev/sample) at 1/2/4/8 B200; p99 batch latency"
UNIT = "windows/s"

# DRAM bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum) of
# the kernel classes captured on B200, keyed by (config, class); see profiles/.
NCU_TRAFFIC = {
    ("cfg1", "gemm_resid"): {"bytes": 28_900_000, "note": "mean over the forward's 14 launches "
                             "with the fused LayerNorm, the cross out_proj counted like an "
                             "out_proj: out_proj 17.4 MB, mlp.2 44.1 MB "
                             "(profiles/gemm_tc_resid_ln_cfg1.md)"},
    ("cfg1", "gemm_gelu"): {"bytes": 10_580_000, "note": "layer 0's mlp.0 "
                            "(profiles/gemm_tc_mlp0_gelu_cfg1.md)"},
    ("cfg1", "attention"): {"bytes": 25_240_000, "note": "layer 0's self-attention "
                            "(profiles/attn_ws_self_cfg1.md)"},
    ("cfg1", "tokenizer"): {"bytes": 1_310_000, "note": "the tokenizer launch: tables and "
                            "indices; the 16 MB of tokens stay in L2 (profiles/tokenize_cfg1.md)"},
}


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


def cpu_model_name() -> str:
    try:
        return open("/proc/cpuinfo").read().split("model name")[1].split("\n")[0].strip(" :\t")
    except Exception:
        return "unknown"


class ClockSampler:
    """SM clock and throttle reasons sampled every few milliseconds through NVML
    while the timed region runs. Without NVML the line says so in ``reasons``
    instead of reporting a clock."""

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


def default_micro_batch(name: str) -> int | None:
    return 256 if name == "cfg4" else None


def cpu_sample_windows(name: str) -> int:
    """Windows per CPU step: the workload's batch, or a fixed subset of the big
    batches (windows are independent, so the rate is well defined)."""
    return {"cfg3": 32, "cfg4": 8}.get(name, 32 if name != "cfg0" else 8)


# ── CPU: the reference's own eager forward (child process or --impl reference) ──


def _load_workloads_module():
    """The workload generator (cortex-engine_b200/cortex/workloads.py) loaded by
    path, so that ``cortex`` can be the reference package in this process."""
    import importlib.util

    spec = importlib.util.spec_from_file_location(
        "ck_bench_workloads", os.path.join(PKG, "cortex", "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # (dataclasses look their module up)
    spec.loader.exec_module(mod)
    return mod


def reference_cpu_runner(name: str, seed: int, batch: int, threads: int):
    """(run, kind, description): one CPU forward over ``batch`` seeded windows of
    workload ``name`` through the reference package's CortexModel
    (baseline/_ref), or the CPU port in oracle/ when that install is absent."""
    import torch

    have_ref = os.path.isdir(os.path.join(REF_PKG, "cortex"))
    if have_ref:
        sys.path.insert(0, REF_PKG)
    else:
        sys.path.insert(0, PKG)
    W = _load_workloads_module()
    wl = W.WORKLOADS[name]
    torch.set_num_threads(threads)
    counts = W.events_per_sample(wl, seed=seed, batch=max(batch, wl.batch))[:batch]
    ev = W.make_events(counts, seed=seed)
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")
    inp = [torch.from_numpy(ev[k]) for k in cols]
    if have_ref:
        import cortex

        from cortex.models.cortex import CortexModel
        from cortex.quantization.calibrate import LayerScales, convert_model

        assert os.path.abspath(cortex.__file__).startswith(os.path.abspath(REF_PKG))
        cfg = wl.config.model_copy(update={"use_kernels": False})
        torch.manual_seed(0)
        model = CortexModel(cfg).eval()
        if wl.dtype == "bfloat16":
            model = model.to(torch.bfloat16)
        if wl.int8:
            scales = {}
            for n in W.int8_layer_names(cfg):
                w = model.get_submodule(n).weight.detach().float()
                scales[n] = LayerScales(weight_scale=w.abs().amax(dim=1).clamp(min=1e-8) / 127.0,
                                        act_scale=1.0)
            convert_model(model, scales)

        def run():
            with torch.no_grad():
                return model(*inp)["behavior"]

        desc = ("the reference package's CortexModel.forward (baseline/_ref, installed from "
                "the reference source; use_kernels=False, eager torch on the CPU)")
        return run, "reference", desc, model, wl, inp
    from cortex.workloads import build_model  # this package (no reference install)

    sys.path.insert(0, ROOT)
    from oracle import cortex_oracle as O

    model = build_model(wl, "cpu")
    p = dict(model.state_dict())

    def run():
        return O.forward(p, wl.config, *inp)

    return run, "port", "the CPU port oracle/cortex_oracle.py (no reference install)", model, wl, inp


def port_runner(model, wl, inp):
    """The CPU port in oracle/ over the same weights and windows."""
    sys.path.insert(0, ROOT)
    from oracle import cortex_oracle as O

    p = dict(model.state_dict())

    def run():
        return O.forward(p, wl.config, *inp)

    return run


def time_cpu(run, seconds: float, min_runs: int = 2):
    run()  # warm-up
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < min_runs:
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    return times


def cpu_sample_main(args):
    """Child process of the GPU arm: the CPU baseline as one JSON line."""
    threads = os.cpu_count() or 1
    batch = cpu_sample_windows(args.config)
    run, kind, desc, model, wl, inp = reference_cpu_runner(args.config, 1000, batch, threads)
    times = time_cpu(run, args.cpu_seconds)
    out = {"value": round(batch * len(times) / sum(times), 2), "unit": UNIT, "cores": threads,
           "kind": kind,
           "sample": f"{len(times)} CPU forwards of {batch} windows ({wl.name}, {wl.dtype}) "
                     f"through {desc}; torch threads {threads} on {cpu_model_name()}",
           "p99_batch_latency_ms": round(1e3 * percentile(times, 99), 2)}
    if kind == "reference" and args.cpu_seconds > 0:
        prun = port_runner(model, wl, inp)
        pt = time_cpu(prun, max(args.cpu_seconds / 2, 1.0))
        out["port"] = {"value": round(batch * len(pt) / sum(pt), 2), "unit": UNIT,
                       "sample": f"{len(pt)} forwards of the same {batch} windows through "
                                 "oracle/cortex_oracle.py"}
    print(json.dumps(out), flush=True)


def cpu_baseline(args, name: str):
    """Runs cpu_sample_main in a child process (its ``cortex`` is the reference)."""
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT")}
    env["CUDA_VISIBLE_DEVICES"] = ""
    cmd = [sys.executable, os.path.abspath(__file__), "--cpu-sample", "--config", name,
           "--cpu-seconds", str(args.cpu_seconds)]
    try:
        r = subprocess.run(cmd, env=env, capture_output=True, text=True,
                           timeout=120 + 4 * args.cpu_seconds)
        line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
        if r.returncode != 0 or not line:
            return {"value": None, "unit": UNIT, "error": (r.stderr or r.stdout)[-400:]}
        return json.loads(line[-1])
    except Exception as e:  # the CPU leg never sinks the GPU line
        return {"value": None, "unit": UNIT, "error": f"{type(e).__name__}: {e}"}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    batch = cpu_sample_windows(args.config)
    run, kind, desc, _, wl, _ = reference_cpu_runner(args.config, 1000, batch, threads)
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
        "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if wl.dtype == "bfloat16" else "f32", "data": "synthetic",
        "config": {"workload": f"{wl.name}: {wl.description}; CPU sample of {batch} windows "
                               "per step", "global_batch": batch,
                   "parallelism": "host CPU, all threads"},
        "p99_batch_latency_ms": round(1e3 * percentile(times, 99), 3),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"{batch} seeded windows per step through {desc}, "
                                   f"{threads} threads on {cpu_model_name()}"},
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


# Kernel classes of the forward, from the launch trace's kernel names.
# gemm_tc_kernel<BN, WMODE, EPI, FUSE, PAIR>: WMODE 2 = int8 weights; EPI 0
# store, 1 GELU, 2 residual, 3 bias; FUSE 3 = the LayerNorm second output.
_GEMM_RE = re.compile(r"gemm_tc_kernel<(\d+), (\d+), (\d+), (\d+), (\w+)>")


def kernel_class(name: str) -> str:
    m = _GEMM_RE.match(name)
    if m:
        epi = int(m.group(3))
        return {0: "gemm_store", 1: "gemm_gelu", 2: "gemm_resid", 3: "gemm_bias"}[epi]
    if name.startswith("attn_"):
        return "attention"
    if name.startswith("tokenize_kernel") or name.startswith("tok_fixup_kernel"):
        return "tokenizer"
    if name.startswith("dequant_kernel"):
        return "dequant"
    if name.startswith("pack_"):
        return "pack"
    if name.startswith("head_"):
        return "head"
    if "norm" in name:
        return "norm"
    if name.startswith("gemm_simt") or name.startswith("gemv"):
        return "gemm_simt"
    return "other"


def forward_work(wl, B: int, E: int, idx_bytes: int, launches: dict) -> dict:
    """Algorithmic work of one forward over B windows and E events, per kernel
    class: FLOPs for the tensor-core classes, DRAM bytes for the others."""
    c = wl.config
    D, Din, L, layers = c.latent_dim, c.hidden_dim, c.num_latents, c.num_layers
    Hm = int(c.latent_dim * c.mlp_ratio)
    es = 2 if wl.dtype == "bfloat16" else 4
    BL = B * L
    store = 2 * L * D * D + 2 * E * Din * 2 * D + layers * 2 * BL * D * 3 * D
    gelu = layers * 2 * BL * D * Hm
    resid = 2 * BL * D * D + layers * (2 * BL * D * D + 2 * BL * Hm * D)
    attn = 4 * L * E * D + layers * B * 4 * L * L * D
    vocab = c.max_neurons + c.max_time_bins + c.spike_value_buckets
    tok = 3 * E * idx_bytes + vocab * Din * es + E * Din * es
    pack = E * idx_bytes + E * 4
    if "pack" not in launches:  # packed inside the tokenizer: batch indices and offsets
        tok += E * idx_bytes + (B + 1) * 4
    head = BL * D * es
    n_norm = launches.get("norm", 0)
    norm = (2 * L * D * es + max(n_norm - 1, 0) * 2 * BL * D * es) if n_norm else 0
    int8 = layers * 2 * BL * (D * 3 * D + D * D + D * Hm + Hm * D) if wl.int8 else 0
    # INT8 weights dequantised to bf16 once per forward: int8 read, bf16 written, scales
    n8 = layers * (D * 3 * D + D * D + D * Hm + Hm * D) if wl.int8 else 0
    deq = 3 * n8 + 4 * layers * (3 * D + D + Hm + D)
    return {
        "gemm_store": ("tensor", store), "gemm_gelu": ("tensor", gelu),
        "gemm_resid": ("tensor", resid), "attention": ("tensor", attn),
        "tokenizer": ("hbm", tok), "pack": ("hbm", pack), "head": ("hbm", head),
        "norm": ("hbm", norm), "dequant": ("hbm", deq), "_int8_flops": int8,
    }


CLASS_DESC = {
    "gemm_resid": "residual GEMMs (cross out_proj, out_proj, mlp.2; LayerNorm of the output "
                  "fused as a second output where N = 512)",
    "gemm_gelu": "MLP up-projection GEMMs with the GELU epilogue",
    "gemm_store": "store GEMMs (q_proj, kv_proj, qkv_proj)",
    "attention": "cross- and self-attention (tcgen05, online softmax)",
    "tokenizer": "spike tokenizer gather-sum + norm_kv (with the packing of sorted batch "
                 "indices and the repack check launch, up to 2^20 events and 4096 windows)",
    "pack": "event packing (counts, offsets, dest)",
    "head": "behaviour head (head_prep + fused head)",
    "norm": "separate LayerNorm launches",
    "dequant": "INT8 block weights dequantised to bf16 once per forward (QuantizedLinear's "
               "expression; the GEMM classes then run on them)",
}


def trace_forwards(fwd, flush, n: int):
    """Per-kernel device times of ``n`` eager forwards from the library's
    launch trace. Each forward starts behind an L2 flush and a ~1 ms spin
    kernel, so that the host has queued the whole forward before the device
    reaches it; the figures are then device time only."""
    import ctypes

    import torch

    from cortex import _lib

    lib = _lib.load()
    per = {}
    for _ in range(n):
        flush()
        torch.cuda.synchronize()
        _lib.check(lib.ck_trace_begin(4096), "ck_trace_begin")
        torch.cuda._sleep(2_000_000)
        fwd()
        torch.cuda.synchronize()
        recs = (_lib.TraceRecord * 4096)()
        cnt = ctypes.c_int32(0)
        _lib.check(lib.ck_trace_end(recs, 4096, ctypes.byref(cnt)), "ck_trace_end")
        for i in range(min(cnt.value, 4096)):
            nm = recs[i].name.decode()
            d = per.setdefault(nm, [0, 0.0])
            d[0] += 1
            d[1] += recs[i].ms
    return {k: (v[0] / n, v[1] / n) for k, v in per.items()}  # launches, ms per forward


def rooflines(wl, B, E, idx_bytes, per_kernel, name_for_traffic):
    """Roofline entries per kernel class, dominant first."""
    hbm, tf_burst, tf_sust, peak_kind = peaks()
    cls_t, cls_n, cls_k = {}, {}, {}
    for k, (n, ms) in per_kernel.items():
        c = kernel_class(k)
        cls_t[c] = cls_t.get(c, 0.0) + ms
        cls_n[c] = cls_n.get(c, 0) + n
        cls_k.setdefault(c, []).append(k)
    work = forward_work(wl, B, E, idx_bytes, cls_n)
    total = sum(cls_t.values())
    out = []
    for c, ms in sorted(cls_t.items(), key=lambda kv: -kv[1]):
        bound, w = work.get(c, (None, None))
        e = {"class": c, "kernels": sorted(cls_k[c]), "launches": round(cls_n[c], 2),
             "ms_per_forward": round(ms, 4), "share": round(ms / total, 4) if total else None}
        if c in CLASS_DESC:
            e["what"] = CLASS_DESC[c]
        if bound == "tensor" and ms > 0:
            ach = w / (ms * 1e-3) / 1e12
            e.update({"bound": "tensor", "achieved": round(ach, 1), "peak": tf_burst,
                      "unit": "TFLOP/s", "frac": round(ach / tf_burst, 4),
                      "peak_kind": f"{peak_kind} bf16 burst", "algorithmic_flops": int(w)})
        elif bound == "hbm" and ms > 0 and w:
            ach = w / (ms * 1e-3) / 1e9
            e.update({"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                      "frac": round(ach / hbm, 4), "peak_kind": f"{peak_kind} HBM copy",
                      "algorithmic_bytes": int(w)})
        tr = NCU_TRAFFIC.get((name_for_traffic, c))
        e["traffic"] = tr["bytes"] if tr else None
        if tr:
            e["traffic_note"] = tr["note"]
        out.append(e)
    int8 = None
    dq = next((e for e in out if e["class"] == "dequant"), None)
    if work["_int8_flops"] and dq is not None:
        int8 = {"what": "the INT8 linears (qkv, out_proj, mlp.0, mlp.2 of every block) run as "
                        "bf16 GEMMs (counted in the GEMM classes) on weights dequantised once "
                        "per forward by the dequant class",
                "dequant_ms_per_forward": dq["ms_per_forward"],
                "dequant_frac_of_hbm": dq.get("frac"),
                "int8_linear_flops": int(work["_int8_flops"])}
    elif work["_int8_flops"]:
        t8 = sum(ms for k, (n, ms) in per_kernel.items()
                 if _GEMM_RE.match(k) and _GEMM_RE.match(k).group(2) == "2")
        if t8 > 0:
            a8 = work["_int8_flops"] / (t8 * 1e-3) / 1e12
            int8 = {"what": "the INT8-weight GEMMs (qkv, out_proj, mlp.0, mlp.2 of every block)",
                    "ms_per_forward": round(t8, 4), "achieved": round(a8, 1), "unit": "TFLOP/s",
                    "frac": round(a8 / tf_burst, 4), "peak": tf_burst,
                    "peak_kind": f"{peak_kind} bf16 burst (activations stay bf16)",
                    "algorithmic_flops": int(work["_int8_flops"])}
    return out, int8


class Decoder:
    """One rank's shard of a workload on the device: the model, the shard's
    micro-batches (device index tensors, batch indices rebased) and one CUDA
    graph per micro-batch."""

    def __init__(self, wl, dev, global_batch: int, world: int, rank: int, micro: int | None,
                 use_graph: bool, seed: int = 1000):
        import numpy as np
        import torch

        from cortex.sharding import shard_bounds, slice_events
        from cortex.workloads import build_model, events_per_sample, make_events

        self.wl, self.dev = wl, dev
        counts = events_per_sample(wl, seed=seed, batch=max(global_batch, wl.batch))
        counts = counts[:global_batch]
        ev = make_events(counts, seed=seed)
        b0, b1 = shard_bounds(counts, world)[rank]
        shard = slice_events(ev, counts, b0, b1)
        self.B = b1 - b0
        self.E = int(counts[b0:b1].sum())
        self.global_batch = global_batch
        self.model = build_model(wl, dev)
        mb = micro or self.B
        self.micro = []  # (B_i, E_i, host int64 tensors, device tensors)
        cols = ("neuron_ids", "time_bins", "values", "batch_indices")
        sc = counts[b0:b1]
        off = np.concatenate([[0], np.cumsum(sc)])
        for lo in range(0, self.B, mb):
            hi = min(lo + mb, self.B)
            e0, e1 = int(off[lo]), int(off[hi])
            host = [torch.from_numpy(np.ascontiguousarray(shard[k][e0:e1])) for k in cols]
            host[3] = host[3] - lo
            self.micro.append((hi - lo, e1 - e0, host, [h.to(dev) for h in host]))
        self.graphs = None
        self.use_graph = use_graph

    def eager(self, i):
        Bi, _, _, d = self.micro[i]
        return self.model(*d, batch_size=Bi)["behavior"]

    def capture(self):
        import torch

        if not self.use_graph:
            return
        self.graphs = []
        for i in range(len(self.micro)):
            for _ in range(2):
                self.eager(i)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.eager(i)
            g.replay()
            self.graphs.append(g)
        torch.cuda.synchronize()

    def step(self):
        if self.graphs is not None:
            for g in self.graphs:
                g.replay()
        else:
            for i in range(len(self.micro)):
                self.eager(i)

    def replay_one(self, i):
        if self.graphs is not None:
            self.graphs[i].replay()
        else:
            self.eager(i)

    def release(self):
        self.graphs = None


# The reference's own benchmark of its fused RMSNorm + linear (Triton), bf16 on
# an NVIDIA A10 (benchmarks/kernels/fused_rmsnorm.json): (M, K, N) -> ms.
REF_RMS_A10_MS = {(256, 512, 1536): 0.0926, (256, 512, 2048): 0.0932,
                  (8192, 512, 1536): 0.6976, (8192, 512, 2048): 0.8796,
                  (8192, 256, 768): 0.1982, (8192, 512, 512): 0.2438}


def norm_linear_block(dev, st, flush, reps: int = 50):
    """rms_norm_linear at the reference benchmark's shapes: the one-launch
    kernel (ck_norm_linear, RMS, bf16, W (K, N) as the reference passes it, and
    the INT8-weight variant), the two-launch path beside it (ck_row_norm, then
    ck_linear), each launch alone in a graph replay after an L2 flush."""
    import torch

    from cortex import _lib as L

    lib = L.load()
    hbm, tf_burst, _, kind = peaks()
    out = []
    for (M, K, N), ref_ms in REF_RMS_A10_MS.items():
        torch.manual_seed(0)
        x = torch.randn(M, K, dtype=torch.bfloat16, device=dev)
        g = (torch.rand(K, device=dev) + 0.5).to(torch.bfloat16)
        w = torch.randn(K, N, dtype=torch.bfloat16, device=dev)
        w8 = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
        sc = torch.rand(N, device=dev) * 1e-2
        y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        xn = torch.empty(M, K, dtype=torch.bfloat16, device=dev)

        def fused():
            L.check(lib.ck_norm_linear(x.data_ptr(), L.CK_BF16, M, K, K, g.data_ptr(), None, 1e-6,
                                       L.CK_NORM_RMS, w.data_ptr(), L.CK_BF16, L.CK_W_KN, N, N,
                                       None, L.CK_EPI_STORE, None, 0, 0, y.data_ptr(), N, None, 0,
                                       L.stream_of(dev)), "ck_norm_linear")

        def fused_int8():
            L.check(lib.ck_norm_linear(x.data_ptr(), L.CK_BF16, M, K, K, g.data_ptr(), None, 1e-6,
                                       L.CK_NORM_RMS, w8.data_ptr(), L.CK_I8, L.CK_W_NK, N, K,
                                       sc.data_ptr(), L.CK_EPI_STORE, None, 0, 0, y.data_ptr(), N,
                                       None, 0, L.stream_of(dev)), "ck_norm_linear int8")

        def two_launch():
            s_ = L.stream_of(dev)
            L.check(lib.ck_row_norm(x.data_ptr(), L.CK_BF16, M, K, K, g.data_ptr(), None, 1e-6,
                                    L.CK_NORM_RMS, xn.data_ptr(), K, s_), "ck_row_norm")
            L.check(lib.ck_linear(xn.data_ptr(), L.CK_BF16, M, K, K, w.data_ptr(), L.CK_BF16,
                                  L.CK_W_KN, N, N, None, L.CK_EPI_STORE, None, 0, 0, y.data_ptr(),
                                  N, s_), "ck_linear")

        def timed(fn):
            for _ in range(3):
                fn()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                fn()
            ts = time_steps(st, flush, gr.replay, reps)
            del gr
            return sum(ts) / len(ts)

        t1, t8, t2 = timed(fused), timed(fused_int8), timed(two_launch)
        fl = 2.0 * M * N * K
        out.append({"M": M, "K": K, "N": N, "one_launch_us": round(t1 * 1e6, 2),
                    "one_launch_tflops": round(fl / t1 / 1e12, 1),
                    "frac": round(fl / t1 / 1e12 / tf_burst, 4),
                    "int8_weights_us": round(t8 * 1e6, 2),
                    "two_launch_us": round(t2 * 1e6, 2),
                    "reference_a10_triton_ms": ref_ms,
                    "vs_reference_a10": round(ref_ms * 1e-3 / t1, 1)})
    return {"what": "rms_norm_linear (RMSNorm in the tcgen05 GEMM's A prologue, 1/rms in its "
                    "epilogue) at the shapes of the reference's kernel benchmark, bf16, W (K, N); "
                    "mean of " + str(reps) + " launches, each alone in a graph replay after an "
                    "L2 flush, CUDA events on the stream",
            "peak_kind": f"{kind} bf16 burst {tf_burst} TFLOP/s",
            "reference": "benchmarks/kernels/fused_rmsnorm.json (NVIDIA A10, Triton)",
            "shapes": out}


def only_kernel(args):
    """A few launches of one kernel (for ncu): the fused RMSNorm + linear at
    8192 x 512 x 1536 (bf16 W (K, N), or int8 W with --only-kernel rms_int8)."""
    import torch

    sys.path.insert(0, PKG)
    from cortex import _lib as L

    lib = L.load()
    dev = torch.device("cuda", 0)
    M, K, N = 8192, 512, 1536
    torch.manual_seed(0)
    x = torch.randn(M, K, dtype=torch.bfloat16, device=dev)
    g = (torch.rand(K, device=dev) + 0.5).to(torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    if args.only_kernel == "rms_int8":
        w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
        sc = torch.rand(N, device=dev) * 1e-2
        wa = (w.data_ptr(), L.CK_I8, L.CK_W_NK, N, K, sc.data_ptr())
    else:
        w = torch.randn(K, N, dtype=torch.bfloat16, device=dev)
        wa = (w.data_ptr(), L.CK_BF16, L.CK_W_KN, N, N, None)
    for _ in range(3):
        L.check(lib.ck_norm_linear(x.data_ptr(), L.CK_BF16, M, K, K, g.data_ptr(), None, 1e-6,
                                   L.CK_NORM_RMS, *wa, L.CK_EPI_STORE, None, 0, 0, y.data_ptr(),
                                   N, None, 0, L.stream_of(dev)), "ck_norm_linear")
    torch.cuda.synchronize()
    L.check_device_status("only-kernel")
    print(json.dumps({"only_kernel": args.only_kernel, "M": M, "K": K, "N": N, "launches": 3}))


def time_steps(st, flush, fn, steps):
    import torch

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for k in range(steps):
        flush()
        ev[k][0].record(st)
        fn()
        ev[k][1].record(st)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) * 1e-3 for a, b in ev]


def measure_config(name, args, dev, st, flush, steps, warmup):
    """The configs-block entry of workload ``name`` on this GPU alone."""
    import torch

    from cortex import _lib
    from cortex.workloads import WORKLOADS

    wl = WORKLOADS[name]
    dec = Decoder(wl, dev, wl.batch, 1, 0, default_micro_batch(name), not args.no_graph)
    with torch.no_grad():
        for i in range(len(dec.micro)):
            dec.eager(i)
        torch.cuda.synchronize()
        _lib.check_device_status(f"{name} warm-up")
        dec.capture()
        for _ in range(warmup):
            dec.step()
        torch.cuda.synchronize()
        times = time_steps(st, flush, dec.step, steps)
        lat = time_steps(st, flush, lambda: dec.replay_one(0), max(steps, 10))
        per_kernel = trace_forwards(lambda: dec.eager(0), flush, 3)
        _lib.check_device_status(f"{name} timed region")
    B0, E0 = dec.micro[0][0], dec.micro[0][1]
    roof, int8 = rooflines(wl, B0, E0, 8, per_kernel, name)
    tot = sum(times)
    entry = {
        "workload": f"{wl.name}: {wl.description}",
        "windows_per_step": dec.B, "events_per_step": dec.E,
        "micro_batch": B0, "micro_batches": len(dec.micro),
        "value": round(dec.B * len(times) / tot, 2), "unit": UNIT,
        "ms_per_step": round(1e3 * tot / len(times), 4), "steps": len(times), "warmup": warmup,
        "p50_batch_latency_ms": round(1e3 * percentile(lat, 50), 4),
        "p99_batch_latency_ms": round(1e3 * percentile(lat, 99), 4),
        "latency_batch": f"one micro-batch of {B0} windows, {len(lat)} replays after the timed "
                         "steps, L2 flushed before each",
        "roofline": roof[0], "roofline_by_kernel": roof[1:],
        "traced_forward": f"one micro-batch of {B0} windows ({E0} events), eager, device int64 "
                          "indices, mean of 3",
    }
    if int8:
        entry["int8_gemm"] = int8
    dec.release()
    del dec
    torch.cuda.empty_cache()
    return entry


def run_ours(args):
    import torch
    import torch.distributed as dist

    sys.path.insert(0, PKG)
    from cortex import _lib
    from cortex.workloads import WORKLOADS

    wl = WORKLOADS[args.config]
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

    strong = args.global_batch is not None
    G = args.global_batch if strong else world * wl.batch
    micro = args.micro_batch or default_micro_batch(wl.name)
    dec = Decoder(wl, dev, G, world, rank, micro, not args.no_graph)
    st = torch.cuda.current_stream(dev)
    flush = L2Flush(dev)

    with torch.no_grad():
        # launches per step (the library counts every kernel it launches)
        c0 = _lib.load().ck_launch_count()
        for i in range(len(dec.micro)):
            dec.eager(i)
        torch.cuda.synchronize()
        launches_per_step = _lib.load().ck_launch_count() - c0
        _lib.check_device_status("bench warm-up")
        for _ in range(max(args.warmup, 3)):
            for i in range(len(dec.micro)):
                dec.eager(i)
        dec.capture()
        for _ in range(2):
            dec.step()
        torch.cuda.synchronize()

        sampler = ClockSampler(local)
        sampler.start()
        barrier()
        torch.cuda.synchronize()
        step_s = time_steps(st, flush, dec.step, args.steps)
        barrier()
        clocks = sampler.stop()
        total = max_over_ranks(sum(step_s))
        _lib.check_device_status("bench timed region")
        windows_per_step = G
        if args.only_forward:  # profiling runs: just the timed forwards
            dec.release()
            if world > 1:
                dist.destroy_process_group()
            if rank == 0:
                print(json.dumps({"metric": METRIC,
                                  "value": round(windows_per_step * args.steps / total, 2),
                                  "unit": UNIT, "n_gpus": world, "steps": args.steps,
                                  "warmup": args.warmup,
                                  "ms_per_step": round(1e3 * total / args.steps, 4),
                                  "mode": "forward only (profiling run)"}), flush=True)
            return

        # latency pass: 200 batches after 25 warm-up, whatever --steps is
        for _ in range(25):
            dec.replay_one(0)
        lat = time_steps(st, flush, lambda: dec.replay_one(0), 200)
        p50 = max_over_ranks(percentile(lat, 50))
        p99 = max_over_ranks(percentile(lat, 99))

        # end-to-end through the public API: host index tensors in, host result out
        host_out = [torch.empty(Bi, wl.config.behavior_dim, dtype=torch.bfloat16
                                if wl.dtype == "bfloat16" else torch.float32).pin_memory()
                    for Bi, _, _, _ in dec.micro]

        def e2e_step():
            for i, (Bi, _, host, _) in enumerate(dec.micro):
                r = dec.model(*host)["behavior"]  # staging, one H2D copy, graph replay
                host_out[i].copy_(r, non_blocking=True)

        for _ in range(max(args.warmup, 3)):
            e2e_step()
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
            e2e_step()
            eev[k][1].record(st)
            eev[k][1].synchronize()  # the caller reads the result
        barrier()
        e2e_s = [a.elapsed_time(b) * 1e-3 for a, b in eev]
        e2e_total = max_over_ranks(sum(e2e_s))
        from cortex.batching import capacity_for

        h2d = sum(4 * _lib.batch_words(capacity_for(Ei)) for _, Ei, _, _ in dec.micro)
        d2h = sum(o.numel() * o.element_size() for o in host_out)

        # per-kernel device times of one traced forward (micro-batch 0)
        per_kernel = trace_forwards(lambda: dec.eager(0), flush, 5) if rank == 0 else None
        dec.release()

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    B0, E0 = dec.micro[0][0], dec.micro[0][1]
    roof, int8 = rooflines(wl, B0, E0, 8, per_kernel, wl.name)
    value = windows_per_step * args.steps / total
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 4), "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None,
        "dtype": "bf16" if wl.dtype == "bfloat16" else "f32", "data": "synthetic",
        "config": {"workload": f"{wl.name}: {wl.description}"
                               + ("" if strong else " per GPU"),
                   "global_batch": G, "windows_per_gpu": dec.B,
                   "events_per_window": wl.events_per_sample, "events_rank0": dec.E,
                   "micro_batch": B0, "micro_batches_per_step": len(dec.micro),
                   "parallelism": f"{world} rank(s), the global batch split into contiguous "
                                  "window ranges balanced by events (shard_bounds), "
                                  "no collectives on the data path",
                   "l2": "flushed before every step, outside the timed interval: a 256 MiB "
                         "memset, then a 256 MiB read of another buffer so that the memset's "
                         "dirty lines are written back before the interval",
                   "cuda_graph": dec.use_graph},
        "p50_batch_latency_ms": round(1e3 * p50, 4),
        "p99_batch_latency_ms": round(1e3 * p99, 4),
        "latency_pass": {"batches": 200, "warmup": 25,
                         "batch": f"one micro-batch of {B0} windows per rank, graph replay, "
                                  "L2 flushed before each; max over ranks"},
        "e2e": {"value": round(windows_per_step * args.steps / e2e_total, 2), "unit": UNIT,
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "p99_batch_latency_ms": round(1e3 * percentile(e2e_s, 99), 4)},
        "roofline": roof[0],
        "roofline_by_kernel": roof[1:],
        "roofline_source": f"library launch trace of 5 eager forwards of micro-batch 0 ({B0} "
                           f"windows, {E0} events, int64 indices): two CUDA events around "
                           "every kernel on its own stream, so no kernel overlaps its "
                           "predecessor; achieved = algorithmic work per forward / traced "
                           "device time per forward",
        "clocks": clocks,
        "gpu_launches": int(launches_per_step) * args.steps,
    }
    if int8:
        line["int8_gemm"] = int8
    if world == 1 and not args.no_configs:
        cfgs = {}
        for name in ("cfg1", "cfg2", "cfg3", "cfg4"):
            if name == wl.name:
                continue
            try:
                cfgs[name] = measure_config(name, args, dev, st, flush, steps=5 if name == "cfg4"
                                            else 20, warmup=3)
            except Exception as e:  # report, do not sink the headline line
                cfgs[name] = {"error": f"{type(e).__name__}: {e}"}
        line["configs"] = cfgs
        try:
            line["norm_linear"] = norm_linear_block(dev, st, flush)
        except Exception as e:
            line["norm_linear"] = {"error": f"{type(e).__name__}: {e}"}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args, wl.name)
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=25)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="cfg1")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="strong scaling: split this many windows across the ranks")
    ap.add_argument("--micro-batch", type=int, default=None,
                    help="windows per device forward (default: the shard; cfg4: 256)")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true")
    ap.add_argument("--only-forward", action="store_true",
                    help="time the forwards only (no e2e / roofline / CPU legs); for ncu runs")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--cpu-sample", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--only-kernel", choices=["rms", "rms_int8"], default=None,
                    help="launch one kernel a few times and exit (for ncu)")
    args = ap.parse_args()
    if args.only_kernel:
        only_kernel(args)
    elif args.cpu_sample:
        cpu_sample_main(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
