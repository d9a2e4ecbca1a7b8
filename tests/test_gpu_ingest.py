"""Device event ingest (ck_collate_bins) against the reference's golden vectors
and the numpy oracle, bit-exact, and the forward over a device-collated batch."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ingest_oracle as IO

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(DEV)


def test_events_from_bin_matrix_matches_reference(golden_ingest):
    from cortex.data import events_from_bin_matrix

    for case in golden_ingest["events"]:
        nid, tb, val = events_from_bin_matrix(_dev(case["counts"]), case["n_buckets"])
        assert np.array_equal(nid.cpu().numpy(), case["neuron_ids"])
        assert np.array_equal(tb.cpu().numpy(), case["time_bins"])
        assert np.array_equal(val.cpu().numpy(), case["values"])


def test_collate_windows_matches_reference_collate(golden_ingest):
    from cortex.data import collate_windows

    g = golden_ingest["collate"]
    sess = _dev(g["counts"])
    pb = collate_windows([(sess, int(s), g["neuron_offset"]) for s in g["starts"]],
                         g["window_bins"], g["n_buckets"], max_neurons=1 << 20)
    got = [t.cpu().numpy() for t in pb.events()]
    for k, name in enumerate(("neuron_ids", "time_bins", "values", "batch_indices")):
        assert np.array_equal(got[k], g[name]), name
    assert pb.n_events == len(g["neuron_ids"]) and pb.batch_size == len(g["starts"])
    assert int(pb.batch[0]) == pb.n_events


def test_collate_windows_cortex_s_batch_matches_oracle():
    """A Cortex-S sized batch: 32 windows of 600 bins over two sessions with
    different unit counts and neuron offsets, against the numpy oracle."""
    from cortex.data import collate_windows

    rng = np.random.default_rng(7)
    s0 = rng.poisson(0.0062, size=(5000, 137)).astype(np.int32)  # ~512 events / window
    s1 = rng.poisson(0.02, size=(3000, 60)).astype(np.int32)
    s1[100:700] = 0  # an all-silent window
    d0, d1 = _dev(s0), _dev(s1)
    wins, items = [], []
    for b in range(32):
        if b % 4 == 3:
            st = 100 if b == 3 else int(rng.integers(0, 3000 - 600))
            wins.append((d1, st, 137))
            items.append(IO.window_events(s1, st, 600, 137, 8, 512))
        else:
            st = int(rng.integers(0, 5000 - 600))
            wins.append((d0, st, 0))
            items.append(IO.window_events(s0, st, 600, 0, 8, 512))
    pb = collate_windows(wins, 600, 8, max_neurons=512)
    want = IO.collate(items)
    got = [t.cpu().numpy() for t in pb.events()]
    for k in range(4):
        assert np.array_equal(got[k], want[k]), k
    assert len(items[3][0]) == 0


def test_collate_windows_errors():
    from cortex.data import collate_windows

    c = _dev(np.ones((50, 10)))
    with pytest.raises(ValueError):  # neuron id past the vocabulary (NLBDataset raises)
        collate_windows([(c, 0, 5)], 20, 8, max_neurons=12)
    with pytest.raises(ValueError):  # window outside its matrix
        collate_windows([(c, 40, 0)], 20, 8, max_neurons=12)
    with pytest.raises(ValueError):  # capacity short of the events
        collate_windows([(c, 0, 0)], 20, 8, max_neurons=12, capacity=64)
    ok = collate_windows([(c, 0, 0)], 20, 8, max_neurons=12)
    assert ok.n_events == 200


def test_forward_packed_equals_forward_on_the_same_events():
    from cortex.data import collate_windows
    from cortex.workloads import WORKLOADS, build_model

    wl = WORKLOADS["cfg1"]
    model = build_model(wl, DEV)
    rng = np.random.default_rng(9)
    sess = rng.poisson(0.0062, size=(4000, 137)).astype(np.int32)
    sess[:, 3] += 9  # counts past the top bucket
    d = _dev(sess)
    starts = [int(s) for s in rng.integers(0, 4000 - 600, 12)]
    pb = collate_windows([(d, s, 0) for s in starts], 600, 8, max_neurons=512)
    with torch.no_grad():
        y = model.forward_packed(pb)["behavior"]
        y2 = model.forward_packed(pb)["behavior"]  # graph replay
        nid, tb, val, bidx = (t.long() for t in pb.events())
        ref = model(nid, tb, val, bidx)["behavior"]
    assert y.shape == (12, 2)
    assert torch.equal(y, ref) and torch.equal(y2, ref)
