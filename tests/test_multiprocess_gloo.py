"""The N > 1 path on CPU: two gloo ranks each decode their own contiguous window
range (balanced by event count, batch indices rebased) and the gathered results
equal decoding the whole batch at once. This is the host logic bench.py and a
multi-GPU deployment use; the data path itself has no collective."""

from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG, ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    import sys

    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    torch.set_num_threads(1)
    from cortex.sharding import shard_bounds, slice_events
    from cortex.workloads import WORKLOADS, build_model, make_events
    from oracle import cortex_oracle as O

    wl = WORKLOADS["cfg0"]
    counts = np.array([40, 7, 120, 33, 1, 64, 90, 15], dtype=np.int64)
    ev = make_events(counts, seed=4)
    b0, b1 = shard_bounds(counts, world)[rank]
    part = slice_events(ev, counts, b0, b1)
    model = build_model(wl, "cpu")
    p = dict(model.state_dict())
    cols = ("neuron_ids", "time_bins", "values", "batch_indices")
    y = O.forward(p, wl.config, *(torch.from_numpy(part[k]) for k in cols))
    sizes = [None] * world
    dist.all_gather_object(sizes, (b0, b1, y))
    if rank == 0:
        full = O.forward(p, wl.config, *(torch.from_numpy(ev[k]) for k in cols))
        got = torch.cat([t for (_, _, t) in sorted(sizes, key=lambda s: s[0])])
        ok = got.shape == full.shape and torch.allclose(got, full, rtol=1e-5, atol=1e-6)
        with open(os.path.join(out_dir, "ok"), "w") as f:
            f.write("1" if ok else f"0 {float((got - full).abs().max())}")
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_sharded_decode_equals_full_batch(tmp_path):
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    assert (tmp_path / "ok").read_text() == "1"
