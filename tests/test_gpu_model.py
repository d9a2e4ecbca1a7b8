"""End-to-end kinematics parity of CortexModel.forward on the GPU.

Against the reference's own outputs (golden vectors) and the CPU oracle, with
the north-star tolerances written here: norm-wise relative error
||y - y_ref|| / ||y_ref|| <= 1e-4 for fp32 and <= 2e-2 for bf16 / INT8. Full-size
batches are additionally checked through size-independent properties: every
window's result is independent of the rest of the batch (bit-exact), and the
packing is invariant to how the events of different windows are interleaved.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import cortex_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {"float32": 1e-4, "bfloat16": 2e-2}


def _rel(y, ref):
    y, ref = y.float().cpu(), ref.float().cpu()
    return float((y - ref).norm() / ref.norm())


def _launches(fn):
    """fn()'s result and the number of kernels the library launched for it."""
    from cortex import _lib

    c0 = _lib.load().ck_launch_count()
    out = fn()
    torch.cuda.synchronize()
    return out, _lib.load().ck_launch_count() - c0


def _model(name):
    from cortex.workloads import WORKLOADS, build_model

    wl = WORKLOADS[name]
    return wl, build_model(wl, DEV)


@pytest.mark.parametrize("name", ["cfg0", "cfg1", "cfg2", "cfg3", "cfg4"])
def test_forward_matches_reference_golden(golden_models, name):
    from cortex import _lib
    from cortex.workloads import make_inputs

    wl, model = _model(name)
    g = golden_models[name]
    n = g["behavior"].shape[0]
    inp, _ = make_inputs(wl, seed=0, batch=n)
    with torch.no_grad():
        y = model(*(inp[k].to(DEV) for k in ("neuron_ids", "time_bins", "values",
                                            "batch_indices")))["behavior"]
    assert y.shape == (n, wl.config.behavior_dim)
    assert torch.isfinite(y).all()
    rel = _rel(y, g["behavior"])
    tol = TOL[wl.dtype]
    if wl.dtype == "bfloat16":
        # The bf16 reference itself carries rounding noise. Where that noise is
        # larger than the 2e-2 bound (Cortex-M variant: small random-init outputs
        # after 10 bf16 layers, ~5% from exact math), this implementation must be
        # within the reference's own distance from the fp32 evaluation of the
        # same weights (25% margin: a different bf16 rounding sequence lands at
        # that distance only on average). Its distance from the bf16 reference
        # is then the difference of two independent rounding errors of that
        # size, so that bound is sqrt(2) times larger; the golden holds only
        # 2 windows x 2 outputs, which cannot resolve anything finer (the
        # 256-window micro-batch test below carries cfg4's parity).
        p32 = {k: (v.float() if v.is_floating_point() else v).cpu()
               for k, v in model.state_dict().items()}
        y32 = O.forward(p32, wl.config, *(inp[k] for k in ("neuron_ids", "time_bins", "values",
                                                         "batch_indices"))).float()
        ref_noise = _rel(g["behavior"], y32)
        if ref_noise > tol:
            assert _rel(y, y32) <= 1.25 * ref_noise, (_rel(y, y32), ref_noise)
            tol = 1.25 * math.sqrt(2.0) * ref_noise
    assert rel <= tol, (rel, tol)
    assert _lib.device_status()[0] == 0


def test_cfg3_full_batch_matches_oracle():
    """Ragged B=256 (32..4096 events per window), full size, vs the CPU oracle."""
    from cortex.workloads import make_inputs

    wl, model = _model("cfg3")
    inp, counts = make_inputs(wl, seed=0)
    assert counts.shape == (256,)
    with torch.no_grad():
        y = model(*(inp[k] for k in ("neuron_ids", "time_bins", "values", "batch_indices")))
    p = {k: v.cpu() for k, v in model.state_dict().items()}
    torch.set_num_threads(max(torch.get_num_threads(), 8))
    ref = O.forward(p, wl.config, inp["neuron_ids"], inp["time_bins"], inp["values"],
                    inp["batch_indices"])
    assert _rel(y["behavior"], ref) <= TOL["bfloat16"]


def _pick_windows(inp, counts, picks):
    """The events of windows ``picks`` (in that order), batch indices rebased."""
    off = np.concatenate([[0], np.cumsum(counts)])
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")
    out = {k: [] for k in cols}
    for j, b in enumerate(picks):
        e0, e1 = int(off[b]), int(off[b + 1])
        for k in cols[:3]:
            out[k].append(inp[k][e0:e1])
        out["batch_indices"].append(torch.full((e1 - e0,), j, dtype=torch.int64))
    return [torch.cat(out[k]) for k in cols]


def test_cfg4_micro_batch_matches_oracle():
    """Cortex-M variant with INT8 weights (cfg4) at the bench's micro-batch of
    256 windows x 1024 events: six windows spread over the batch match the
    oracle evaluated in bf16 and in fp32 within the cfg4 bound, max(2e-2, 1.25 x
    the bf16 oracle's own distance from fp32); the first and the last window
    are bit-identical when decoded alone."""
    from cortex.workloads import make_inputs

    wl, model = _model("cfg4")
    inp, counts = make_inputs(wl, seed=3, batch=256)
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")
    with torch.no_grad():
        y = model(*(inp[k].to(DEV) for k in cols))["behavior"]
        picks = [0, 51, 102, 153, 204, 255]
        alone = [model(*(t.to(DEV) for t in _pick_windows(inp, counts, [b])))["behavior"]
                 for b in (0, 255)]
    assert y.shape == (256, 2) and torch.isfinite(y).all()
    assert torch.equal(alone[0][0], y[0]) and torch.equal(alone[1][0], y[255])
    sub = _pick_windows(inp, counts, picks)
    torch.set_num_threads(max(torch.get_num_threads(), 8))
    p16 = {k: v.cpu() for k, v in model.state_dict().items()}
    p32 = {k: (v.float() if v.is_floating_point() else v) for k, v in p16.items()}
    ref16 = O.forward(p16, wl.config, *sub).float()
    ref32 = O.forward(p32, wl.config, *sub).float()
    tol = max(TOL["bfloat16"], 1.25 * _rel(ref16, ref32))
    got = y[picks]
    assert _rel(got, ref16) <= tol, (_rel(got, ref16), tol)
    assert _rel(got, ref32) <= tol, (_rel(got, ref32), tol)


@pytest.mark.parametrize("name", ["cfg1", "cfg3"])
def test_windows_are_independent(name):
    """Result of window b is bit-identical whether it runs alone or in the batch."""
    from cortex.sharding import slice_events
    from cortex.workloads import make_inputs

    wl, model = _model(name)
    inp, counts = make_inputs(wl, seed=1)
    ev = {k: v.numpy() for k, v in inp.items()}
    with torch.no_grad():
        full = model(*(inp[k] for k in ("neuron_ids", "time_bins", "values",
                                         "batch_indices")))["behavior"]
        for b in (0, 5, len(counts) - 1):
            one = slice_events(ev, counts, b, b + 1)
            y = model(*(torch.from_numpy(one[k]) for k in ("neuron_ids", "time_bins", "values",
                                                           "batch_indices")))["behavior"]
            assert torch.equal(y[0], full[b]), b


@pytest.mark.parametrize("name,batch", [("cfg3", 64), ("cfg4", 12)])
def test_sharded_decode_is_the_full_batch_decode(name, batch):
    """The N > 1 path of bench.py and of a multi-GPU deployment, on the product:
    the batch split by shard_bounds (ranges balanced by events) and
    slice_events (batch indices rebased), each shard decoded on its own, gives
    bit-for-bit the full-batch decode for 2, 3 and 8 shards."""
    from cortex.sharding import shard_bounds, slice_events
    from cortex.workloads import make_inputs

    wl, model = _model(name)
    inp, counts = make_inputs(wl, seed=11, batch=batch)
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")
    ev = {k: v.numpy() for k, v in inp.items()}
    with torch.no_grad():
        full = model(*(inp[k].to(DEV) for k in cols))["behavior"]
        for world in (2, 3, 8):
            parts = []
            for b0, b1 in shard_bounds(counts, world):
                one = slice_events(ev, counts, b0, b1)
                parts.append(model(*(torch.from_numpy(one[k]).to(DEV) for k in cols),
                                   batch_size=b1 - b0)["behavior"])
            assert torch.equal(torch.cat(parts), full), world


@pytest.mark.parametrize("name", ["cfg2", "cfg4"])
def test_int8_forward_is_the_bf16_forward_on_dequantised_weights(name):
    """QuantizedLinear.forward dequantises per call: (w_int8.float() * s).to(bf16)
    then a bf16 linear. The INT8 model's forward must equal, bit for bit, the
    forward of a bf16 model whose block linears hold exactly those weights
    (dequantised here by torch)."""
    from cortex.quantization.calibrate import QuantizedLinear
    from cortex.workloads import make_inputs

    wl, model = _model(name)
    _, ref_model = _model(name)  # the same seeded weights and INT8 conversion
    n = 0
    for mod_name, mod in list(ref_model.named_modules()):
        for child_name, child in list(mod.named_children()):
            if isinstance(child, QuantizedLinear):
                lin = torch.nn.Linear(child.in_features, child.out_features, bias=False,
                                      device=DEV, dtype=torch.bfloat16)
                with torch.no_grad():
                    lin.weight.copy_((child.weight_int8.float()
                                      * child.weight_scale.float()[:, None]).to(torch.bfloat16))
                setattr(mod, child_name, lin)
                n += 1
    assert n == 4 * wl.config.num_layers
    inp, _ = make_inputs(wl, seed=21, batch=8)
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")
    with torch.no_grad():
        y8 = model(*(inp[k].to(DEV) for k in cols))["behavior"]
        y16 = ref_model(*(inp[k].to(DEV) for k in cols))["behavior"]
    assert torch.equal(y8, y16)


def test_interleaved_events_and_int32_indices():
    from cortex.workloads import make_inputs

    wl, model = _model("cfg1")
    inp, counts = make_inputs(wl, seed=2, batch=8)
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")
    with torch.no_grad():
        base = model(*(inp[k] for k in cols))["behavior"]
        # interleave windows while keeping each window's own event order
        perm = torch.from_numpy(np.argsort(
            np.concatenate([np.arange(c) * 8 + w for w, c in enumerate(counts)]), kind="stable"))
        shuffled = model(*(inp[k][perm] for k in cols))["behavior"]
        as32 = model(*(inp[k].int() for k in cols))["behavior"]
    assert torch.equal(shuffled, base)
    assert torch.equal(as32, base)


def test_unsorted_device_indices_repack_bit_identical():
    """Batch indices in random order (device tensors): the tokenizer's own
    packing sees them out of order and the repacking launch redoes it as a
    stable counting sort. The result equals the forward over the same events
    stably sorted by window (the packed rows are the same), including an empty
    window and windows after the last event."""
    from cortex import _lib

    wl, model = _model("cfg1")
    g = torch.Generator().manual_seed(5)
    counts = [37, 0, 300, 1, 129, 64, 700, 5]
    E = sum(counts)
    bidx = torch.cat([torch.full((c,), w) for w, c in enumerate(counts)]).long()
    nid = torch.randint(0, 137, (E,), generator=g)
    tb = torch.randint(0, 600, (E,), generator=g)
    val = torch.randint(0, 8, (E,), generator=g)
    perm = torch.randperm(E, generator=g)
    ev = [t[perm].to(DEV) for t in (nid, tb, val, bidx)]
    order = torch.sort(bidx[perm], stable=True).indices
    srt = [t[order] for t in ev]
    with torch.no_grad():
        y = model(*ev, batch_size=10)["behavior"]
        ys = model(*srt, batch_size=10)["behavior"]
    assert torch.equal(y, ys)
    assert torch.equal(y[1], y[8]) and torch.equal(y[8], y[9])  # no events
    assert _lib.device_status()[0] == 0


def test_out_of_range_device_batch_index_sets_status():
    from cortex import _lib

    wl, model = _model("cfg1")
    nid = torch.tensor([1, 2, 3, 4], device=DEV)
    tb = torch.tensor([1, 2, 3, 4], device=DEV)
    val = torch.tensor([1, 2, 3, 4], device=DEV)
    with torch.no_grad():
        model(nid, tb, val, torch.tensor([0, 0, 1, 1], device=DEV), batch_size=2)
        torch.cuda.synchronize()
        assert _lib.device_status()[0] == 0
        model(nid, tb, val, torch.tensor([0, 5, 1, 1], device=DEV), batch_size=2)
        torch.cuda.synchronize()
    assert _lib.device_status()[0] == _lib.CK_ERR_INDEX


def test_module_path_matches_fused_path():
    """return_aux=True runs the composed module forwards (padded tokens + mask)."""
    from cortex.workloads import make_inputs

    wl, model = _model("cfg1")
    inp, _ = make_inputs(wl, seed=3, batch=4)
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")
    with torch.no_grad():
        fused = model(*(inp[k] for k in cols))["behavior"]
        mod = model(*(inp[k] for k in cols), return_aux=True)
    assert mod["masked_spike_logits"].shape == (4, wl.config.spike_value_buckets)
    assert _rel(mod["behavior"], fused) <= 1e-2


def test_empty_window_inside_batch():
    """A window with no events keeps its latents (attention over no keys is 0)."""
    wl, model = _model("cfg1")
    p = {k: v.cpu() for k, v in model.state_dict().items()}
    g = torch.Generator().manual_seed(0)
    E = 300
    bidx = torch.cat([torch.zeros(100), torch.full((200,), 2)]).long()
    nid = torch.randint(0, 137, (E,), generator=g)
    tb = torch.randint(0, 600, (E,), generator=g)
    val = torch.randint(0, 8, (E,), generator=g)
    with torch.no_grad():
        y = model(nid, tb, val, bidx)["behavior"]
    ref = O.forward(p, wl.config, nid, tb, val, bidx)
    assert y.shape == (3, 2) and torch.isfinite(y).all()
    assert _rel(y, ref) <= TOL["bfloat16"]


@pytest.mark.parametrize("name,latents,layers", [("cfg1", None, 1), ("cfg4", None, 1),
                                                  ("cfg1", 200, 1), ("cfg1", 64, 1),
                                                  ("cfg1", 1000, 1)])
def test_fused_head_matches_composed_head(monkeypatch, name, latents, layers):
    """The behaviour head in algebraic form (one clustered tcgen05 kernel on the
    weight-only matrix W_k^T q / W_v^T w_out) against the composed head (both
    LayerNorms, head kv_proj, 2-query attention, out_proj D->1) and the oracle.
    Covers partial 128-latent tiles (L=200, L=64), an 8-CTA cluster (L=1000)
    and the D768/H12 geometry (cfg4: 24 score pairs, 3 vectors per lane)."""
    import dataclasses

    from cortex.workloads import WORKLOADS, build_model, make_inputs

    wl = WORKLOADS[name]
    upd = {"num_layers": layers}
    if latents is not None:
        upd["num_latents"] = latents
    wl = dataclasses.replace(wl, config=wl.config.model_copy(update=upd))
    model = build_model(wl, DEV)
    inp, _ = make_inputs(wl, seed=4, batch=6)
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")
    with torch.no_grad():  # device indices: the eager path reads the switch every call
        monkeypatch.setenv("CK_HEAD_FUSED", "1")
        fused, n_fused = _launches(lambda: model(*(inp[k].to(DEV) for k in cols))["behavior"])
        monkeypatch.setenv("CK_HEAD_FUSED", "0")
        composed, n_comp = _launches(lambda: model(*(inp[k].to(DEV) for k in cols))["behavior"])
    assert n_fused < n_comp  # two different code paths ran
    p32 = {k: (v.float() if v.is_floating_point() else v).cpu()
           for k, v in model.state_dict().items()}
    ref = O.forward(p32, wl.config, *(inp[k] for k in cols)).float()
    assert torch.isfinite(fused).all()
    assert _rel(fused, composed) <= 1e-2, _rel(fused, composed)
    assert _rel(fused, ref) <= TOL["bfloat16"], _rel(fused, ref)
    assert _rel(fused, ref) <= max(1.5 * _rel(composed, ref), 5e-3)


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3"])
def test_layernorm_fused_into_residual_gemm(monkeypatch, name):
    """Each LayerNorm after a residual GEMM with D = 512 is the GEMM's second
    output (a CTA pair per row block exchanging row statistics through
    distributed shared memory), against separate LayerNorm kernels and the
    oracle, with non-trivial gamma / beta. cfg2 runs it on INT8 weights; cfg3
    (B=256, ragged) gives every CTA pair several row blocks."""
    from cortex.workloads import make_inputs

    wl, model = _model(name)
    with torch.no_grad():
        g = torch.Generator(device="cpu").manual_seed(8)
        for blk in model.encoder.self_attn_blocks:
            for nrm in (blk.norm_attn, blk.norm_mlp):
                nrm.weight.copy_(1 + 0.2 * torch.randn(nrm.weight.shape, generator=g))
                nrm.bias.copy_(0.1 * torch.randn(nrm.bias.shape, generator=g))
    inp, _ = make_inputs(wl, seed=9, batch=None if name == "cfg3" else 8)
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")

    with torch.no_grad():
        monkeypatch.setenv("CK_LN_FUSE", "1")
        fused, n_fused = _launches(lambda: model(*(inp[k].to(DEV) for k in cols))["behavior"])
        again = model(*(inp[k].to(DEV) for k in cols))["behavior"]
        monkeypatch.setenv("CK_LN_FUSE", "0")
        separate, n_sep = _launches(lambda: model(*(inp[k].to(DEV) for k in cols))["behavior"])
    assert torch.isfinite(fused).all()
    assert torch.equal(fused, again)  # deterministic
    assert n_sep - n_fused == 2 * wl.config.num_layers  # every block LayerNorm fused
    assert _rel(fused, separate) <= 1e-2, _rel(fused, separate)
    n = 16 if name == "cfg3" else fused.shape[0]  # oracle on a subset (windows are independent)
    from cortex.sharding import slice_events

    sub = slice_events({k: inp[k].numpy() for k in cols},
                       np.bincount(inp["batch_indices"].numpy()), 0, n)
    p32 = {k: (v.float() if v.is_floating_point() else v).cpu()
           for k, v in model.state_dict().items()}
    ref = O.forward(p32, wl.config, *(torch.from_numpy(sub[k]) for k in cols)).float()
    assert _rel(fused[:n], ref) <= TOL["bfloat16"], _rel(fused[:n], ref)


def test_side_stream_prologue_is_bit_identical_and_per_thread(monkeypatch):
    """The weight-only prologue (norm_q, q_proj, the head matrix) runs on a
    side stream forked from the caller's stream; that changes the schedule
    only. The result equals the single-stream forward bit for bit, also from
    short-lived host threads, each of which creates its own side stream and
    releases it when the thread exits."""
    import threading

    from cortex.workloads import make_inputs

    wl, model = _model("cfg1")
    inp, _ = make_inputs(wl, seed=15, batch=8)
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")
    dev_inp = [inp[k].to(DEV) for k in cols]
    with torch.no_grad():  # device indices: the eager path reads the switch every call
        monkeypatch.setenv("CK_SIDE", "0")
        single = model(*dev_inp)["behavior"]
        monkeypatch.setenv("CK_SIDE", "1")
        forked = model(*dev_inp)["behavior"]
        results = []

        def run():
            with torch.no_grad():
                y = model(*dev_inp)["behavior"]
                torch.cuda.current_stream().synchronize()
                results.append(y)

        for _ in range(3):
            t = threading.Thread(target=run)
            t.start()
            t.join()
    torch.cuda.synchronize()
    assert torch.equal(forked, single)
    assert len(results) == 3 and all(torch.equal(y, single) for y in results)

