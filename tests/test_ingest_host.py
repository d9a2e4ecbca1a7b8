"""Event ingest and batch assembly without a GPU: the oracle against the
reference's golden vectors, the native host staging (ck_batch_stage, a host
function of the C ABI), the worker's payload assembly and the bucket policy."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import ingest_oracle as IO


def test_bucket_values_matches_reference(golden_ingest):
    g = golden_ingest["bucket"]
    assert np.array_equal(IO.bucket_values(g["counts"], g["n_buckets"]), g["out"])
    with pytest.raises(ValueError):
        IO.bucket_values(g["counts"], 0)


def test_events_from_bin_matrix_matches_reference(golden_ingest):
    for case in golden_ingest["events"]:
        nid, tb, val = IO.events_from_bin_matrix(case["counts"], case["n_buckets"])
        assert np.array_equal(nid, case["neuron_ids"])
        assert np.array_equal(tb, case["time_bins"])
        assert np.array_equal(val, case["values"])
        assert nid.dtype == tb.dtype == val.dtype == np.int64


def test_collate_of_windows_matches_reference(golden_ingest):
    g = golden_ingest["collate"]
    items = [IO.window_events(g["counts"], int(s), g["window_bins"], g["neuron_offset"],
                              g["n_buckets"], max_neurons=1 << 20) for s in g["starts"]]
    got = IO.collate(items)
    for k, name in enumerate(("neuron_ids", "time_bins", "values", "batch_indices")):
        assert np.array_equal(got[k], g[name]), name
    with pytest.raises(ValueError):
        IO.window_events(g["counts"], 0, g["window_bins"], g["neuron_offset"], 8, max_neurons=50)


def test_product_collate_events_matches_reference(golden_ingest):
    from cortex.data import collate_events

    g = golden_ingest["collate"]
    items = []
    for s in g["starts"]:
        nid, tb, val = IO.window_events(g["counts"], int(s), g["window_bins"],
                                        g["neuron_offset"], g["n_buckets"], 1 << 20)
        items.append({"neuron_ids": torch.from_numpy(nid), "time_bins": torch.from_numpy(tb),
                      "values": torch.from_numpy(val), "behavior": torch.zeros(2)})
    out = collate_events(items)
    for k in ("neuron_ids", "time_bins", "values", "batch_indices"):
        assert np.array_equal(out[k].numpy(), g[k]), k
    assert out["behavior"].shape == (len(g["starts"]), 2)


def test_worker_assembly_matches_reference(golden_ingest):
    from cortex.serve.worker import assemble_events

    g = golden_ingest["worker"]
    want = [g[k] for k in ("neuron_ids", "time_bins", "values", "batch_indices")]
    for got in (IO.worker_lists(g["payloads"]), assemble_events(g["payloads"])):
        for a, b in zip(got, want):
            assert np.array_equal(a, b) and a.dtype == np.int64
    # requests past max(batch_index) get zeros in the reference worker
    B = IO.batch_size(want[3])
    assert g["request_ids"] == [p["request_id"] for p in g["payloads"]]
    for i, beh in enumerate(g["behavior"]):
        if i >= B:
            assert beh == [0.0] * len(beh)


def _stage(arrays, capacity, dt):
    from cortex import _lib

    lib = _lib.load()
    ts = [torch.as_tensor(a, dtype=dt).contiguous() for a in arrays]
    buf = np.full(_lib.batch_words(capacity), -7, dtype=np.int32)
    B = ctypes.c_int32(-1)
    rc = lib.ck_batch_stage(*(t.data_ptr() for t in ts), _lib.dtype_code(dt), ts[0].numel(),
                            buf.ctypes.data, capacity, ctypes.byref(B))
    return rc, buf, B.value


@pytest.mark.parametrize("dt", [torch.int64, torch.int32])
def test_batch_stage_layout_matches_oracle(golden_ingest, dt):
    from cortex import _lib
    from cortex.batching import capacity_for

    g = golden_ingest["worker"]
    arrays = [g[k] for k in ("neuron_ids", "time_bins", "values", "batch_indices")]
    E = len(arrays[0])
    cap = capacity_for(E)
    rc, buf, B = _stage(arrays, cap, dt)
    assert rc == _lib.CK_OK
    want = IO.packed_batch(*arrays, capacity=cap)
    h = IO.BATCH_HEADER_WORDS
    assert buf[0] == E and list(buf[1:h]) == [0, 0, 0]
    for k in range(4):
        seg = slice(h + k * cap, h + k * cap + E)
        assert np.array_equal(buf[seg], want[seg]), k
        assert (buf[h + k * cap + E:h + (k + 1) * cap] == -7).all()  # padding untouched
    assert B == IO.batch_size(arrays[3])


def test_batch_stage_edge_cases():
    from cortex import _lib

    z = np.zeros(0, dtype=np.int64)
    rc, buf, B = _stage([z, z, z, z], 256, torch.int64)
    assert rc == _lib.CK_OK and buf[0] == 0 and B == 1
    # ids outside int32 saturate (and stay out of every table)
    big = np.array([2**40, -2**40, 5], dtype=np.int64)
    rc, buf, B = _stage([big, big, big, np.array([0, 0, 2])], 256, torch.int64)
    assert rc == _lib.CK_OK and B == 3
    assert list(buf[4:7]) == [2**31 - 1, -2**31, 5]
    # a negative batch index is rejected on the host, as bincount rejects it
    rc, _, _ = _stage([big, big, big, np.array([0, -1, 2])], 256, torch.int64)
    assert rc == _lib.CK_ERR_INDEX
    rc, _, _ = _stage([big, big, big, np.array([0, 2**40, 2])], 256, torch.int64)
    assert rc == _lib.CK_ERR_INDEX
    # capacity too small or not a multiple of 4
    one = np.array([1, 2, 3, 4, 5], dtype=np.int64)
    assert _stage([one] * 4, 4, torch.int64)[0] == _lib.CK_ERR_INVALID_ARG
    assert _stage([one] * 4, 6, torch.int64)[0] == _lib.CK_ERR_INVALID_ARG


def test_capacity_buckets():
    from cortex.batching import capacity_for

    prev = 0
    for n in list(range(0, 3000, 7)) + [16384, 16385, 214_000, 1 << 22]:
        c = capacity_for(n)
        assert c >= n and c % 256 == 0 and c >= prev
        assert c <= max(256, n + n // 16 + 256)  # at most 1/16 padding past the first bucket
        prev = c
    assert capacity_for(16384) == 16384
    # bucket count stays small over a wide range of batch sizes
    assert len({capacity_for(n) for n in range(1, 1 << 16)}) < 200
