"""StreamingKVCache on the device: the reference's observable behaviour (golden
trace of the reference cache) and the forward that reuses cached kv_proj rows."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def golden_cache():
    import os

    from conftest import GOLDEN

    return torch.load(os.path.join(GOLDEN, "golden_cache.pt"), weights_only=False)


def test_cache_replays_reference_trace(golden_cache):
    from cortex.cache import StreamingKVCache

    g = golden_cache
    cache = StreamingKVCache(g["num_pages"], g["page_size"], g["hidden_dim"], torch.float32, DEV)
    for i, ((op, sid, start, emb), want) in enumerate(zip(g["ops"], g["results"])):
        if op == "write":
            cache.write(sid, start, emb.to(DEV))
            out = None
        elif op == "read":
            got = cache.read(sid, start)
            out = None if got is None else got.cpu()
        else:
            out = cache.evict_session(sid)
        if isinstance(want["out"], torch.Tensor):
            assert out is not None and torch.equal(out, want["out"]), i
        else:
            assert out == want["out"], i
        assert cache.hit_rate == want["hit_rate"], i
        assert cache.pages_used == want["pages_used"], i


def _windows(rng, n, sessions=("s0", "s1"), starts=range(0, 200, 10)):
    from cortex.workloads import make_events

    counts = rng.integers(300, 700, size=n)
    ev = make_events(counts, seed=int(rng.integers(1 << 30)))
    off = np.concatenate([[0], np.cumsum(counts)])
    out = []
    for b in range(n):
        sl = slice(off[b], off[b + 1])
        out.append({"session_id": sessions[b % len(sessions)],
                    "bin_start": int(list(starts)[b % len(list(starts))]),
                    "neuron_ids": ev["neuron_ids"][sl], "time_bins": ev["time_bins"][sl],
                    "values": ev["values"][sl]})
    return out


def _plain(model, wins):
    cols = [np.concatenate([w[k] for w in wins]) for k in ("neuron_ids", "time_bins", "values")]
    bidx = np.repeat(np.arange(len(wins)), [len(w["neuron_ids"]) for w in wins])
    with torch.no_grad():
        return model(*(torch.from_numpy(c).to(DEV) for c in cols + [bidx]))["behavior"]


def test_forward_streaming_cold_warm_and_mixed_match_forward():
    from cortex.cache import StreamingKVCache
    from cortex.workloads import WORKLOADS, build_model

    wl = WORKLOADS["cfg1"]
    model = build_model(wl, DEV)
    D2 = 2 * wl.config.latent_dim
    cache = StreamingKVCache(num_pages=512, page_size=64, hidden_dim=D2, dtype=torch.bfloat16,
                             device=DEV)
    rng = np.random.default_rng(3)
    wins = _windows(rng, 16)
    with torch.no_grad():
        ref = _plain(model, wins)
        cold = model.forward_streaming(wins, cache)["behavior"]
        assert cache.hit_rate == 0.0 and cache.pages_used > 0
        warm = model.forward_streaming(wins, cache)["behavior"]
        assert cache.hit_rate == 0.5
        # half new windows (new keys), half cached, interleaved
        new = _windows(rng, 16, sessions=("s2",), starts=range(1000, 1160, 10))
        mixed_w = [new[i // 2] if i % 2 else wins[i // 2] for i in range(16)]
        mixed = model.forward_streaming(mixed_w, cache)["behavior"]
        ref_mixed = _plain(model, mixed_w)
    assert torch.equal(cold, ref)
    assert torch.equal(warm, ref)
    assert torch.equal(mixed, ref_mixed)


def test_forward_streaming_with_evictions_and_stale_counts():
    from cortex.cache import StreamingKVCache
    from cortex.workloads import WORKLOADS, build_model

    wl = WORKLOADS["cfg1"]
    model = build_model(wl, DEV)
    cache = StreamingKVCache(num_pages=24, page_size=64, hidden_dim=2 * wl.config.latent_dim,
                             dtype=torch.bfloat16, device=DEV)  # room for ~2-3 windows
    rng = np.random.default_rng(4)
    wins = _windows(rng, 8, sessions=("a", "b", "c", "d"))
    with torch.no_grad():
        for _ in range(3):
            assert torch.equal(model.forward_streaming(wins, cache)["behavior"],
                               _plain(model, wins))
        # a window re-sent under the same key with a different event count is recomputed
        w2 = [dict(w) for w in wins]
        for k in ("neuron_ids", "time_bins", "values"):
            w2[0][k] = w2[0][k][:-5]
        assert torch.equal(model.forward_streaming(w2, cache)["behavior"], _plain(model, w2))
    assert cache.evict_session("a") >= 0
    assert cache.pages_used <= 24
