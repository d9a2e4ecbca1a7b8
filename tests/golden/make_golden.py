"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in the build container, where the reference is importable:

    PYTHONPATH=/path/to/cortex-engine python tests/golden/make_golden.py

It imports the UNMODIFIED reference package (peterajhgraham/cortex-engine) and
records, for seeded inputs, what the reference's own functions return:

* golden_kernels.pt  -- ``_pack_events`` on sorted / unsorted / gapped batch
  indices, ``fused_tokenizer_reference`` (the reference tests' seeds 42/99),
  ``sparse_cross_attention_reference`` (seed 123) with dense and checkerboard
  masks, ``build_temporal_block_mask``, ``rms_norm_linear_reference`` (seed 17),
  and ``QuantizedLinear.from_linear`` storage.
* golden_models.pt   -- for each benchmark configuration: per-parameter
  checksums of ``torch.manual_seed(0); CortexModel(cfg)`` (so a re-implementation
  can prove it reproduces the same random init), the input checksum, and the
  reference's ``behavior`` output on a CPU-sized sample of the workload.

Nothing here runs on the GPU box; the tests only read the .pt files.
"""

from __future__ import annotations

import importlib.util
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

import cortex  # noqa: E402  (the reference package, from PYTHONPATH)

assert "cortex-engine_b200" not in os.path.abspath(cortex.__file__), \
    "run with the reference on PYTHONPATH, not this repository's package"

from cortex.kernels.fused_rmsnorm import rms_norm_linear_reference  # noqa: E402
from cortex.kernels.sparse_xattn import (  # noqa: E402
    build_temporal_block_mask, sparse_cross_attention_reference)
from cortex.kernels.tokenizer import fused_tokenizer_reference  # noqa: E402
from cortex.models.cortex import CortexModel, _pack_events  # noqa: E402
from cortex.quantization.calibrate import (  # noqa: E402
    LayerScales, QuantizedLinear, convert_model)

# The workload generator is shared with the tests and bench; load it by path.
_spec = importlib.util.spec_from_file_location(
    "ck_workloads", os.path.join(REPO, "cortex-engine_b200", "cortex", "workloads.py"))
W = importlib.util.module_from_spec(_spec)
sys.modules["ck_workloads"] = W
_spec.loader.exec_module(W)

# Samples per configuration that the CPU reference runs for the golden output.
MODEL_SAMPLES = {"cfg0": 8, "cfg1": 32, "cfg2": 32, "cfg3": 8, "cfg4": 2}


def pack_cases():
    g = torch.Generator().manual_seed(5)
    cases = {
        "sorted": torch.tensor([0, 0, 0, 1, 1, 2, 2, 2, 2, 3]),
        "unsorted": torch.randint(0, 5, (97,), generator=g),
        "gap": torch.tensor([0, 0, 2, 2, 2, 5]),
        "single": torch.zeros(7, dtype=torch.int64),
        "one_event": torch.tensor([0]),
        "conftest_small_batch": torch.randint(0, 4, (256,), generator=g).sort().values,
        "reverse": torch.arange(40, dtype=torch.int64).flip(0) // 3,
    }
    out = {}
    for name, bidx in cases.items():
        bidx = bidx.to(torch.int64)
        flat = torch.arange(bidx.shape[0], dtype=torch.float64)[:, None] + 1.0
        tokens, mask = _pack_events(flat, bidx)
        out[name] = {"batch_indices": bidx, "tokens": tokens[..., 0], "mask": mask}
    return out


def tokenizer_cases():
    out = {}
    for dtype in (torch.float32, torch.bfloat16):
        torch.manual_seed(42)
        N, T, V, D, E = 32, 64, 8, 64, 128
        n = torch.randn(N, D, dtype=dtype)
        t = torch.randn(T, D, dtype=dtype)
        v = torch.randn(V, D, dtype=dtype)
        torch.manual_seed(99)
        nid = torch.randint(0, N, (E,))
        tb = torch.randint(0, T, (E,))
        val = torch.randint(0, V, (E,))
        out[str(dtype)] = {"n": n, "t": t, "v": v, "nid": nid, "tb": tb, "val": val,
                           "out": fused_tokenizer_reference(n, t, v, nid, tb, val)}
    return out


def xattn_cases():
    torch.manual_seed(123)
    B, H, L, E, Dh = 1, 2, 64, 128, 16
    q = torch.randn(B, H, L, Dh)
    k = torch.randn(B, H, E, Dh)
    v = torch.randn(B, H, E, Dh)
    n_q, n_k = math.ceil(L / 32), math.ceil(E / 32)
    dense = torch.ones(n_q, n_k, dtype=torch.bool)
    checker = torch.tensor([[(i + j) % 2 == 0 for j in range(n_k)] for i in range(n_q)])
    out = {"q": q, "k": k, "v": v, "dense_mask": dense, "checker_mask": checker,
           "dense": sparse_cross_attention_reference(q, k, v, dense, 32, 32),
           "checker": sparse_cross_attention_reference(q, k, v, checker, 32, 32),
           "none": sparse_cross_attention_reference(q, k, v, None)}
    g = torch.Generator().manual_seed(11)
    tm = {}
    for i, (E_, L_, T_, w, bl, be) in enumerate([(128, 64, 120, 20, 32, 32), (64, 32, 120, 120, 32, 32),
                                                 (128, 64, 120, 0, 32, 32), (500, 256, 600, 30, 64, 64),
                                                 (77, 100, 1024, 5, 16, 8)]):
        et = torch.randint(0, T_, (E_,), generator=g).sort().values if i != 2 else \
            torch.zeros(E_, dtype=torch.long)
        tm[i] = {"event_times": et, "args": (L_, T_, w, bl, be),
                 "mask": build_temporal_block_mask(et, L_, T_, w, bl, be)}
    out["temporal"] = tm
    return out


def rmsnorm_cases():
    torch.manual_seed(17)
    M, K, N = 16, 64, 32
    x = torch.randn(M, K)
    gamma = torch.ones(K)
    w = torch.randn(K, N)
    bias = torch.randn(N)
    g2 = torch.rand(K) + 0.5
    return {"x": x, "gamma": gamma, "w": w, "bias": bias, "gamma2": g2,
            "out": rms_norm_linear_reference(x, gamma, w, None),
            "out_bias": rms_norm_linear_reference(x, gamma, w, bias),
            "out_gamma2": rms_norm_linear_reference(x, g2, w, None)}


def quant_cases():
    torch.manual_seed(0)
    lin = torch.nn.Linear(64, 32, bias=False)
    torch.nn.init.normal_(lin.weight, std=1.0)
    sc = LayerScales(weight_scale=lin.weight.detach().float().abs().amax(1).clamp(min=1e-8) / 127.0,
                     act_scale=0.01)
    ql = QuantizedLinear.from_linear(lin, sc)
    x = torch.randn(16, 64)
    return {"weight": lin.weight.detach().clone(), "w_int8": ql.weight_int8,
            "weight_scale": ql.weight_scale, "x": x, "y": ql(x)}


def build_model(name: str):
    wl = W.WORKLOADS[name]
    torch.manual_seed(0)
    model = CortexModel(wl.config).eval()
    checks = {k: (float(v.double().sum()), float(v.double().pow(2).sum()))
              for k, v in model.state_dict().items()}
    if wl.dtype == "bfloat16":
        model = model.to(torch.bfloat16)
    if wl.int8:
        scales = {}
        for n in W.int8_layer_names(wl.config):
            mod = model.get_submodule(n)
            scales[n] = LayerScales(
                weight_scale=mod.weight.detach().float().abs().amax(1).clamp(min=1e-8) / 127.0,
                act_scale=1.0)
        convert_model(model, scales)
    return model, checks


def model_cases():
    out = {}
    for name, n_samples in MODEL_SAMPLES.items():
        wl = W.WORKLOADS[name]
        counts = W.events_per_sample(wl, seed=0)[:n_samples]
        ev = W.make_events(counts, seed=0)
        model, checks = build_model(name)
        inp = {k: torch.from_numpy(v) for k, v in ev.items()}
        with torch.no_grad():
            y = model(inp["neuron_ids"], inp["time_bins"], inp["values"], inp["batch_indices"])
        q8 = {}
        if wl.int8:
            for n in W.int8_layer_names(wl.config)[:4]:
                mod = model.get_submodule(n)
                q8[n] = {"int8_sum": int(mod.weight_int8.long().sum()),
                         "int8_abs_sum": int(mod.weight_int8.long().abs().sum()),
                         "scale_sum": float(mod.weight_scale.double().sum())}
        out[name] = {
            "param_checksums": checks,
            "counts": torch.from_numpy(counts),
            "input_checksum": {k: int(v.sum()) for k, v in ev.items()},
            "behavior": y["behavior"].float(),
            "int8": q8,
        }
        print(name, tuple(y["behavior"].shape), float(y["behavior"].float().abs().mean()),
              file=sys.stderr)
    return out


if __name__ == "__main__":
    torch.set_num_threads(os.cpu_count() or 1)
    kern = {"pack": pack_cases(), "tokenizer": tokenizer_cases(), "xattn": xattn_cases(),
            "rmsnorm": rmsnorm_cases(), "quant": quant_cases(),
            "torch_version": torch.__version__}
    torch.save(kern, os.path.join(HERE, "golden_kernels.pt"))
    models = model_cases()
    models["torch_version"] = torch.__version__
    torch.save(models, os.path.join(HERE, "golden_models.pt"))
    print("wrote", os.listdir(HERE), file=sys.stderr)
