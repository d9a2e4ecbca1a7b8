"""Pin the CPU oracle (oracle/cortex_oracle.py) to the reference's own outputs.

The golden vectors were produced by tests/golden/make_golden.py, which imports
and runs the unmodified reference. Integer work must match bit for bit; the
floating-point restatements must match the reference's eager ops.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import cortex_oracle as O


def test_pack_events_matches_reference(golden_kernels):
    for name, case in golden_kernels["pack"].items():
        bidx = case["batch_indices"]
        flat = torch.arange(bidx.shape[0], dtype=torch.float64)[:, None] + 1.0
        tokens, mask = O.pack_events(flat, bidx)
        assert torch.equal(tokens[..., 0], case["tokens"]), name
        assert torch.equal(mask, case["mask"]), name
        info = O.pack_events_index(bidx.numpy())
        # dest is the flat packed row of every event: recover it from the golden
        B, e_max = case["tokens"].shape
        assert info["B"] == B and info["E_max"] == e_max, name
        for e in range(bidx.shape[0]):
            b = int(bidx[e])
            pos = info["dest"][e] - info["offsets"][b]
            assert case["tokens"][b, pos] == e + 1.0, (name, e)
        assert np.array_equal(info["counts"], case["mask"].sum(1).numpy()), name


def test_tile_mask_is_mask_any(golden_kernels):
    for name, case in golden_kernels["pack"].items():
        counts = case["mask"].sum(1).numpy()
        e_max = case["mask"].shape[1]
        for be in (1, 4, 32):
            n_k = (e_max + be - 1) // be
            padded = torch.zeros(counts.shape[0], n_k * be, dtype=torch.bool)
            padded[:, :e_max] = case["mask"]
            expect = padded.view(counts.shape[0], n_k, be).any(-1).numpy()
            assert np.array_equal(O.tile_mask(counts, e_max, be), expect), (name, be)


@pytest.mark.parametrize("dtype", ["torch.float32", "torch.bfloat16"])
def test_tokenizer_matches_reference(golden_kernels, dtype):
    c = golden_kernels["tokenizer"][dtype]
    out = O.tokenize(c["n"], c["t"], c["v"], c["nid"], c["tb"], c["val"])
    assert torch.equal(out, c["out"])


def test_tokenizer_known_answers(golden_kernels):
    c = golden_kernels["tokenizer"]["torch.float32"]
    n, t, v = c["n"], c["t"], c["v"]
    out = O.tokenize(n, t, v, torch.tensor([3]), torch.tensor([7]), torch.tensor([1]))
    assert torch.equal(out[0], n[3] + t[7] + v[1])
    z = torch.zeros(100, dtype=torch.int64)
    same = O.tokenize(n, t, v, z, z, z)
    assert torch.equal(same, same[0:1].expand_as(same))
    empty = torch.zeros(0, dtype=torch.int64)
    assert O.tokenize(n, t, v, empty, empty, empty).shape == (0, n.shape[1])


def test_sparse_attention_matches_reference(golden_kernels):
    c = golden_kernels["xattn"]
    for key, mask in (("dense", c["dense_mask"]), ("checker", c["checker_mask"])):
        out = O.sparse_cross_attention(c["q"], c["k"], c["v"], mask, 32, 32)
        torch.testing.assert_close(out, c[key], rtol=2e-5, atol=2e-5)
    # fp32 SDPA on the host: reduction order may follow the thread count
    out = O.sparse_cross_attention(c["q"], c["k"], c["v"], None)
    torch.testing.assert_close(out, c["none"], rtol=2e-5, atol=2e-5)


def test_all_masked_rows_are_zero():
    torch.manual_seed(123)
    q, k, v = torch.randn(1, 1, 16, 8), torch.randn(1, 1, 32, 8), torch.randn(1, 1, 32, 8)
    out = O.sparse_cross_attention(q, k, v, torch.zeros(1, 1, dtype=torch.bool), 16, 32)
    assert torch.equal(out, torch.zeros_like(out))


def test_temporal_block_mask_matches_reference(golden_kernels):
    from cortex.kernels.sparse_xattn import build_temporal_block_mask

    for i, c in golden_kernels["xattn"]["temporal"].items():
        L, T, w, bl, be = c["args"]
        assert torch.equal(O.build_temporal_block_mask(c["event_times"], L, T, w, bl, be),
                           c["mask"]), i
        # the package's host-side builder (vectorised) must agree as well
        assert torch.equal(build_temporal_block_mask(c["event_times"], L, T, w, bl, be),
                           c["mask"]), i


def test_rms_norm_linear_matches_reference(golden_kernels):
    c = golden_kernels["rmsnorm"]
    torch.testing.assert_close(O.rms_norm_linear(c["x"], c["gamma"], c["w"], None), c["out"],
                               rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(O.rms_norm_linear(c["x"], c["gamma"], c["w"], c["bias"]),
                               c["out_bias"], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(O.rms_norm_linear(c["x"], c["gamma2"], c["w"], None),
                               c["out_gamma2"], rtol=1e-6, atol=1e-6)


def test_quantization_storage_matches_reference(golden_kernels):
    c = golden_kernels["quant"]
    w8, sc = O.quantize_weight(c["weight"])
    assert torch.equal(w8, c["w_int8"])
    assert torch.equal(sc, c["weight_scale"])
    p = {"l.weight_int8": w8, "l.weight_scale": sc}
    torch.testing.assert_close(O.linear(c["x"], p, "l"), c["y"], rtol=0, atol=0)


@pytest.mark.parametrize("name", ["cfg0", "cfg1", "cfg2", "cfg3", "cfg4"])
def test_model_init_reproduces_reference_weights(golden_models, name):
    """torch.manual_seed(0); CortexModel(cfg) here gives the reference's weights."""
    from cortex.models.cortex import CortexModel
    from cortex.workloads import WORKLOADS

    torch.manual_seed(0)
    model = CortexModel(WORKLOADS[name].config)
    ref = golden_models[name]["param_checksums"]
    sd = model.state_dict()
    assert set(sd) == set(ref)
    for k, v in sd.items():
        s, q = float(v.double().sum()), float(v.double().pow(2).sum())
        assert (s, q) == ref[k], k


@pytest.mark.parametrize("name", ["cfg0", "cfg1", "cfg2", "cfg3", "cfg4"])
def test_oracle_forward_matches_reference(golden_models, name):
    from cortex.workloads import WORKLOADS, build_model, make_inputs

    g = golden_models[name]
    wl = WORKLOADS[name]
    n = g["behavior"].shape[0]
    inp, counts = make_inputs(wl, seed=0, batch=n)
    assert np.array_equal(counts, g["counts"].numpy())
    assert {k: int(v.sum()) for k, v in inp.items()} == g["input_checksum"]
    model = build_model(wl, "cpu")
    if wl.int8:
        for qn, ref in g["int8"].items():
            mod = model.get_submodule(qn)
            assert int(mod.weight_int8.long().sum()) == ref["int8_sum"]
            assert int(mod.weight_int8.long().abs().sum()) == ref["int8_abs_sum"]
            assert float(mod.weight_scale.double().sum()) == ref["scale_sum"]
    p = {k: v for k, v in model.state_dict().items()}
    y = O.forward(p, wl.config, inp["neuron_ids"], inp["time_bins"], inp["values"],
                  inp["batch_indices"]).float()
    ref = g["behavior"]
    rel = float((y - ref).norm() / ref.norm())
    # Same torch CPU operators in the same order: essentially exact.
    assert rel <= (1e-6 if wl.dtype == "float32" else 1e-3), rel
