"""Packed event batches on the GPU: ck_forward_batch and the graph replays of
cortex.batching, and the inference worker built on them.

The padded batch runs the same kernels as ck_forward over the real events
(padding rows are skipped by the packing and written as zeros by the
tokenizer; every row of the forward is computed independently of the rows
after it), so the results must be bit-identical to the eager forward over
device-resident indices.
"""

from __future__ import annotations

import asyncio

import numpy as np
import pytest
import torch

from oracle import cortex_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
COLS = ("neuron_ids", "time_bins", "values", "batch_indices")


def _model(name="cfg1"):
    from cortex.workloads import WORKLOADS, build_model

    wl = WORKLOADS[name]
    return wl, build_model(wl, DEV)


def _device_forward(model, inp, batch_size=None):
    return model(*(inp[k].to(DEV) for k in COLS), batch_size=batch_size)["behavior"]


@pytest.mark.parametrize("name", ["cfg0", "cfg1", "cfg2"])
def test_host_batch_path_is_bit_identical_to_device_path(name):
    from cortex.workloads import make_inputs

    wl, model = _model(name)
    inp, _ = make_inputs(wl, seed=11, batch=min(wl.batch, 8))
    runner = model.batch_runner()
    with torch.no_grad():
        ref = _device_forward(model, inp)
        first = model(*(inp[k] for k in COLS))["behavior"]   # eager launch + capture
        again = model(*(inp[k] for k in COLS))["behavior"]   # graph replay
    assert runner.captures >= 1 and runner.replays >= 1
    assert torch.equal(first, ref)
    assert torch.equal(again, ref)


def test_one_graph_serves_every_batch_of_a_bucket():
    """Event counts that share a capacity bucket replay one graph; each result
    equals the eager forward over exactly its own events."""
    from cortex.batching import capacity_for
    from cortex.workloads import make_events

    wl, model = _model("cfg1")
    runner = model.batch_runner()
    rng = np.random.default_rng(5)
    base = np.array([500, 512, 480, 530, 470, 505, 490, 520], dtype=np.int64)
    caps = set()
    with torch.no_grad():
        for trial in range(4):
            counts = base + rng.integers(-8, 9, size=base.size)
            ev = {k: torch.from_numpy(v) for k, v in make_events(counts, seed=trial).items()}
            caps.add(capacity_for(int(counts.sum())))
            y = model(*(ev[k] for k in COLS))["behavior"]
            assert torch.equal(y, _device_forward(model, ev)), trial
    assert len(caps) == 1
    assert runner.captures == 1 and runner.replays == 3


def test_padding_and_unsorted_and_int32_host_indices():
    from cortex.workloads import make_inputs

    wl, model = _model("cfg1")
    inp, counts = make_inputs(wl, seed=4, batch=6)
    perm = torch.randperm(int(counts.sum()), generator=torch.Generator().manual_seed(0))
    shuffled = {k: inp[k][perm] for k in COLS}
    as32 = {k: inp[k].int() for k in COLS}
    with torch.no_grad():
        for ev in (shuffled, as32):
            ref = _device_forward(model, ev)  # same events, same order, indices on the device
            for _ in range(2):
                assert torch.equal(model(*(ev[k] for k in COLS))["behavior"], ref)


def test_trailing_and_inner_empty_windows_and_explicit_batch_size():
    wl, model = _model("cfg1")
    p = {k: v.cpu() for k, v in model.state_dict().items()}
    g = torch.Generator().manual_seed(1)
    E = 300
    bidx = torch.cat([torch.zeros(100), torch.full((200,), 2)]).long()
    nid = torch.randint(0, 137, (E,), generator=g)
    tb = torch.randint(0, 600, (E,), generator=g)
    val = torch.randint(0, 8, (E,), generator=g)
    with torch.no_grad():
        y = model(nid, tb, val, bidx)["behavior"]              # B = max + 1 = 3
        y5 = model(nid, tb, val, bidx, batch_size=5)["behavior"]
        y0 = model(nid[:0], tb[:0], val[:0], bidx[:0])["behavior"]
    assert y.shape == (3, 2) and y5.shape == (5, 2) and y0.shape == (1, 2)
    ref = O.forward(p, wl.config, nid, tb, val, bidx)
    assert float((y.float().cpu() - ref).norm() / ref.norm()) <= 2e-2
    assert torch.equal(y5[:3], y)
    assert torch.equal(y5[3], y5[4]) and torch.equal(y5[3], y[1])  # windows with no events


def test_host_batch_errors_match_the_eager_path():
    from cortex import _lib

    wl, model = _model("cfg1")
    nid = torch.tensor([1, 2, 3])
    tb = torch.tensor([1, 2, 3])
    val = torch.tensor([1, 2, 3])
    with pytest.raises(IndexError):
        model(nid, tb, val, torch.tensor([0, -1, 1]))
    bad = torch.tensor([1, 2, 10_000])
    model(bad, tb, val, torch.tensor([0, 0, 1]))
    code, _ = _lib.device_status()
    assert code == _lib.CK_ERR_INDEX


def test_graphs_follow_weight_updates():
    from cortex.workloads import make_inputs

    wl, model = _model("cfg1")
    inp, _ = make_inputs(wl, seed=6, batch=4)
    with torch.no_grad():
        a = model(*(inp[k] for k in COLS))["behavior"]
        model(*(inp[k] for k in COLS))
        # in place: the captured graph reads the same parameter storage
        model.behavior_head.out_proj.weight.mul_(2.0)
        b = model(*(inp[k] for k in COLS))["behavior"]
        assert torch.equal(b, _device_forward(model, inp))
        assert not torch.equal(a, b)
        # replaced storage: the graphs are dropped and captured again
        sd = {k: v.clone() for k, v in model.state_dict().items()}
        sd["behavior_head.out_proj.weight"] = sd["behavior_head.out_proj.weight"] * 0.5
        model.load_state_dict(sd)
        c = model(*(inp[k] for k in COLS))["behavior"]
        assert torch.equal(c, _device_forward(model, inp))


def _payloads(counts, seed):
    rng = np.random.default_rng(seed)
    out = []
    for i, c in enumerate(counts):
        ev = [{"neuron_id": int(a), "time_bin": int(b), "value": int(v)}
              for a, b, v in zip(rng.integers(0, 137, c), np.sort(rng.integers(0, 600, c)),
                                 rng.integers(0, 8, c))]
        out.append({"request_id": f"r{i}", "events": ev})
    return out


def test_inference_worker_matches_model_per_request():
    from cortex.serve.worker import InferenceWorker, assemble_events

    wl, model = _model("cfg1")
    worker = InferenceWorker(model, wl.config, torch.device(DEV), max_batch_size=32)
    worker.warmup()
    assert worker.ready
    payloads = _payloads([40, 0, 75, 12, 0, 0], seed=3)  # inner and trailing empty requests
    res = asyncio.run(worker.run_batch(payloads))
    assert [r["request_id"] for r in res] == [p["request_id"] for p in payloads]
    nid, tb, val, bidx = assemble_events(payloads)
    with torch.no_grad():
        ref = model(*(torch.from_numpy(x).to(DEV) for x in (nid, tb, val, bidx)))["behavior"]
    ref = ref.float().cpu().tolist()
    for i in range(4):
        assert res[i]["behavior"] == ref[i]
    for i in (4, 5):
        assert res[i]["behavior"] == [0.0] * wl.config.behavior_dim
    empty = worker._run_batch_sync([{"request_id": "e", "events": []}])
    assert empty[0]["behavior"] == [0.0] * wl.config.behavior_dim
    worker.shutdown()
