"""Host-side logic that needs no GPU: the C ABI library, argument checks, the
workload generator, sharding, the reference-compatible module surface."""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT


def _header_functions() -> list[str]:
    txt = open(os.path.join(ROOT, "include", "cortex_b200.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(ck_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_header_symbol():
    from cortex import _lib

    lib = _lib.load()
    names = _header_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.EXPORTED_SYMBOLS)


def test_status_strings_without_gpu():
    from cortex import _lib

    assert _lib.status_string(0) == "ok"
    assert "index" in _lib.status_string(_lib.CK_ERR_INDEX)
    assert "timed out" in _lib.status_string(_lib.CK_ERR_TIMEOUT)


def test_ctypes_structs_match_header_layout(tmp_path):
    """The ctypes mirrors must have the C layout of the header: compile a probe
    with gcc that prints offsetof() of every field and compare."""
    import shutil
    import subprocess

    from cortex import _lib

    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    structs = {"ck_attention_args": _lib.AttentionArgs, "ck_linear_weight": _lib.LinearWeight,
               "ck_block_weights": _lib.BlockWeights, "ck_trace_record": _lib.TraceRecord,
               "ck_model": _lib.Model}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "cortex_b200.h"',
             'int main(void) {']
    for cname, py in structs.items():
        lines.append(f'printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    for line in out.splitlines():
        cname, field, val = line.split()
        py = structs[cname]
        got = ctypes.sizeof(py) if field == "sizeof" else getattr(py, field).offset
        assert got == int(val), (cname, field, got, val)


def test_no_cpu_fallback():
    from cortex.kernels.fused_rmsnorm import rms_norm_linear
    from cortex.kernels.sparse_xattn import sparse_cross_attention
    from cortex.kernels.tokenizer import fused_tokenizer

    t = torch.randn(8, 16)
    i = torch.zeros(4, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        fused_tokenizer(t, t, t, i, i, i)
    q = torch.randn(1, 1, 4, 16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        sparse_cross_attention(q, q, q)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        rms_norm_linear(torch.randn(4, 16), torch.ones(16), torch.randn(16, 8))


def test_model_forward_without_gpu_raises():
    from cortex.models import CORTEX_XS, CortexModel

    model = CortexModel(CORTEX_XS)
    i = torch.zeros(4, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        model(i, i, i, i)


def test_shape_validation_matches_reference():
    from cortex.kernels.tokenizer import fused_tokenizer
    from cortex.models import CORTEX_XS, CortexConfig, SpikeTokenizer

    tok = SpikeTokenizer(CORTEX_XS)
    with pytest.raises(ValueError, match="shape mismatch"):
        tok(torch.zeros(10, dtype=torch.int64), torch.zeros(11, dtype=torch.int64),
            torch.zeros(10, dtype=torch.int64))
    t = torch.randn(8, 16)
    with pytest.raises(ValueError, match="contiguous"):
        fused_tokenizer(t.t().contiguous().t(), t, t, *(torch.zeros(2, dtype=torch.int64),) * 3)
    with pytest.raises(ValueError, match="must equal hidden_dim"):
        CortexConfig(hidden_dim=128, num_layers=2, num_heads=2, head_dim=32, num_latents=32,
                     latent_dim=128, cross_attn_heads=2, max_neurons=256, max_time_bins=512,
                     behavior_dim=2)


def test_block_mask_shape_assertion():
    from cortex.kernels.sparse_xattn import sparse_cross_attention

    q = torch.randn(1, 1, 64, 16)
    with pytest.raises(AssertionError, match="block_mask shape"):
        sparse_cross_attention(q, q, q, torch.ones(3, 3, dtype=torch.bool), 32, 32)


def test_workload_generator_is_deterministic_and_in_range():
    from cortex.workloads import WORKLOADS, events_per_sample, make_events

    for name, wl in WORKLOADS.items():
        counts = events_per_sample(wl, seed=0)[:16]
        a = make_events(counts, seed=0)
        b = make_events(counts, seed=0)
        for k in a:
            assert np.array_equal(a[k], b[k]), (name, k)
        assert a["neuron_ids"].min() >= 0 and a["neuron_ids"].max() < 137
        assert a["time_bins"].min() >= 0 and a["time_bins"].max() < 600
        assert a["values"].min() >= 0 and a["values"].max() <= 7
        assert np.all(np.diff(a["batch_indices"]) >= 0)
        off = np.concatenate([[0], np.cumsum(counts)])
        for w in range(len(counts)):  # time bins sorted within each sample
            assert np.all(np.diff(a["time_bins"][off[w]:off[w + 1]]) >= 0)
    ragged = events_per_sample(WORKLOADS["cfg3"], seed=0)
    assert ragged.shape == (256,) and ragged.min() >= 32 and ragged.max() <= 4096
    assert 500 < ragged.mean() < 1200


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_bounds_cover_and_balance(world):
    from cortex.sharding import shard_bounds
    from cortex.workloads import WORKLOADS, events_per_sample

    counts = events_per_sample(WORKLOADS["cfg3"], seed=0)
    b = shard_bounds(counts, world)
    assert b[0][0] == 0 and b[-1][1] == len(counts)
    assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
    assert all(hi > lo for lo, hi in b)
    ev = [int(counts[lo:hi].sum()) for lo, hi in b]
    assert max(ev) - min(ev) <= 2 * int(counts.max())


def test_quantized_linear_storage_and_conversion():
    from cortex.quantization.calibrate import (LayerScales, QuantizedLinear, convert_model,
                                               weight_scales)
    from oracle import cortex_oracle as O

    torch.manual_seed(0)
    lin = torch.nn.Linear(64, 32, bias=False)
    torch.nn.init.normal_(lin.weight, std=0.5)
    ql = QuantizedLinear.from_linear(lin, LayerScales(weight_scales(lin.weight), 0.01))
    w8, sc = O.quantize_weight(lin.weight)
    assert torch.equal(ql.weight_int8, w8) and torch.equal(ql.weight_scale, sc)
    assert "INT8" in ql.extra_repr() and ql.weight_scale.shape == (32,)
    model = torch.nn.Sequential(torch.nn.Linear(512, 512, bias=False))
    w = model[0].weight.detach().clone()
    convert_model(model, {"0": LayerScales(weight_scales(model[0].weight), 1.0)})
    q = model[0]
    assert isinstance(q, QuantizedLinear) and q.weight_int8.dtype == torch.int8
    assert q.weight_int8.shape == (512, 512) and q.weight_scale.dtype == torch.float32
    # dequantised weight within half a quantisation step of the original
    err = (q.weight_int8.float() * q.weight_scale[:, None] - w).abs()
    assert bool((err <= 0.5 * q.weight_scale[:, None] + 1e-7).all())


def test_int8_workload_converts_exactly_the_self_attention_linears():
    from cortex.quantization.calibrate import QuantizedLinear
    from cortex.workloads import WORKLOADS, build_model, int8_layer_names

    wl = WORKLOADS["cfg2"]
    model = build_model(wl, "cpu")
    q = {n for n, m in model.named_modules() if isinstance(m, QuantizedLinear)}
    assert q == set(int8_layer_names(wl.config)) and len(q) == 28
    assert model.tokenizer.neuron_emb.weight.dtype == torch.bfloat16


def test_int8_to_bf16_bit_trick_is_exact_for_every_byte():
    """The GEMM widens int8 weight tiles to bf16 with integer logic and one
    bf16x2 subtraction (i8x4_to_bf16x4 in csrc/common.cuh): the bf16 with bits
    0x4300 | (v & 0x7F) minus the bf16 0x4300 | (v & 0x80) is v. Restated in
    numpy for all 256 byte values (the byte order of the packed words too)
    against torch's own int8 -> bf16 conversion."""
    v = np.arange(-128, 128, dtype=np.int8)
    u = v.view(np.uint8).astype(np.uint32)
    x = (0x4300 | (u & 0x7F)).astype(np.uint32) << 16  # bf16 bits as the top of an fp32
    s_ = (0x4300 | (u & 0x80)).astype(np.uint32) << 16
    diff = x.view(np.float32) - s_.view(np.float32)  # exact: integers of magnitude <= 256
    assert np.array_equal(diff, v.astype(np.float32))
    got = (diff.view(np.uint32) >> 16).astype(np.uint16)
    ref = torch.from_numpy(v.copy()).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, ref)
    # the byte permute (b0, b2, b1, b3): even 16-bit lanes then hold (b0, b1),
    # odd ones (b2, b3), the order of the bf16 pairs written out
    w = np.uint32(0x44332211)
    b = [(int(w) >> (8 * i)) & 0xFF for i in range(4)]
    r = b[0] | (b[2] << 8) | (b[1] << 16) | (b[3] << 24)
    assert (r & 0xFF, (r >> 16) & 0xFF) == (b[0], b[1])
    assert ((r >> 8) & 0xFF, (r >> 24) & 0xFF) == (b[2], b[3])


def _rn_bf16(x: np.ndarray) -> np.ndarray:
    """Round float64 values (normal range) to the nearest bf16, ties to even:
    8 significant bits, the rounding done once on the exact value."""
    m, e = np.frexp(x)  # x = m * 2**e, 0.5 <= |m| < 1
    return np.ldexp(np.round(m * 256.0) / 256.0, e)  # np.round: half to even


def test_bf16x2_add_equals_fp32_add_then_round():
    """The GEMM's residual and bias epilogues add bf16 pairs with one
    add.rn.bf16x2 (gemm_common.cuh): the exact sum of two bf16 values rounded
    once to bf16. torch's bf16 add rounds the fp32 sum to bf16 instead. The two
    agree because fp32 keeps 24 >= 2 * 8 + 2 significand bits. Checked on
    random bf16 pairs whose exponents differ by up to 40 (their float64 sum is
    then exact), with cancellations and ties to even among them."""
    rng = np.random.default_rng(11)
    n = 1 << 20
    a = torch.from_numpy(rng.standard_normal(n) * np.exp2(rng.integers(-20, 21, n))).to(torch.bfloat16)
    b = torch.from_numpy(rng.standard_normal(n) * np.exp2(rng.integers(-20, 21, n))).to(torch.bfloat16)
    b[: n // 8] = -a[: n // 8] * (1 + torch.from_numpy(rng.integers(-3, 4, n // 8) / 256.0)).to(torch.bfloat16)
    torch_sum = (a.float() + b.float()).to(torch.bfloat16).double().numpy()
    exact = a.double().numpy() + b.double().numpy()
    nz = exact != 0
    ref = np.where(nz, _rn_bf16(np.where(nz, exact, 1.0)), 0.0)
    assert np.array_equal(torch_sum, ref)


def test_bench_flop_accounting_matches_the_per_window_figures():
    """bench.py's algorithmic FLOPs per kernel class (the roofline numerators)
    for cfg1: per window kv_proj 0.537 G, cross-attention QK^T + PV 0.268 G,
    cross out_proj 0.134 G and 7 self-attention blocks of 1.745 G (qkv 0.403,
    attention 0.134, out_proj 0.134, MLP 1.074), plus q_proj 0.134 G once per
    batch (it acts on the batch-invariant latent parameter). The behaviour
    head's kv_proj is not counted: the fused head never computes it."""
    import importlib.util

    from cortex.workloads import WORKLOADS

    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    wl = WORKLOADS["cfg1"]
    B, E = 32, 32 * 512
    w = bench.forward_work(wl, B, E, 8, {})
    D, L, Hm, layers = 512, 256, 2048, 7
    per_window = (2 * 512 * D * 2 * D + 4 * L * 512 * D + 2 * L * D * D
                  + layers * (2 * L * D * 3 * D + 4 * L * L * D + 2 * L * D * D + 4 * L * D * Hm))
    q_proj = 2 * L * D * D
    assert abs(per_window / 1e9 - (0.537 + 0.268 + 0.134 + 7 * 1.745)) < 0.01
    tensor = sum(v[1] for k, v in w.items() if not k.startswith("_") and v[0] == "tensor")
    assert tensor == B * per_window + q_proj
    assert w["gemm_resid"][1] == B * (2 * L * D * D + layers * (2 * L * D * D + 2 * L * Hm * D))
    assert w["attention"][1] == B * (4 * L * 512 * D + layers * 4 * L * L * D)
    # bench.py's class names for the forward's kernels
    assert bench.kernel_class("gemm_tc_kernel<256, 0, 2, 3, 0>") == "gemm_resid"
    assert bench.kernel_class("gemm_tc_kernel<256, 0, 1, 0, 0>") == "gemm_gelu"
    assert bench.kernel_class("gemm_tc_kernel<256, 0, 0, 0, 1>") == "gemm_store"
    assert bench.kernel_class("attn_ws_kernel") == "attention"
    assert bench.kernel_class("tokenize_kernel<__nv_bfloat16, 8, 4, 1, 16>") == "tokenizer"
