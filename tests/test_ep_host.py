"""Expert-parallel host logic on the CPU: contiguous expert shards, the IPC
handle swap over a 2-rank gloo group, argument checks that run before any
device work, and the decomposition the device exchange computes (per-rank
partial outputs summed in rank order equal the single-GPU layer), checked
with the oracle."""

from __future__ import annotations

import importlib
import multiprocessing as mp
import os

import numpy as np
import pytest

from conftest import cosine, rel_err


def _store_path() -> str:
    """A fresh file-store path for one group's rendezvous (no TCP port)."""
    import tempfile
    d = tempfile.mkdtemp(prefix="sbb200_pg_")
    return os.path.join(d, "store")


@pytest.fixture(scope="module")
def ep(sbb):
    return importlib.import_module(sbb.__name__ + ".ep")


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_expert_shards_contiguous(ep, world):
    E = 170
    shards = [ep.expert_shard(E, world, r) for r in range(world)]
    assert shards[0][0] == 0
    for (b0, c0), (b1, _) in zip(shards, shards[1:]):
        assert b0 + c0 == b1
    assert sum(c for _, c in shards) == E
    counts = [c for _, c in shards]
    assert max(counts) - min(counts) <= 1 and counts == sorted(counts, reverse=True)
    if world == 8:
        assert counts == [22, 22, 21, 21, 21, 21, 21, 21]


def test_shard_and_create_reject_bad_arguments(sbb, ep):
    with pytest.raises(sbb.Sbb200Error):
        ep.expert_shard(170, 0, 0)
    with pytest.raises(sbb.Sbb200Error):
        ep.expert_shard(4, 8, 0)  # fewer experts than ranks
    L = sbb.lib()
    assert not L.sbb200_ep_create(0, 2, 2, 64, 8, 170, 4096, 1280, 2, 0)  # rank >= world
    assert "rank" in sbb.last_error()
    assert not L.sbb200_ep_create(0, 0, 2, 64, 8, 170, 4096 + 32, 1280, 2, 0)  # K % 256
    assert "256" in sbb.last_error()
    assert not L.sbb200_ep_create(0, 0, 2, 0, 8, 170, 4096, 1280, 2, 0)
    assert "max_tokens" in sbb.last_error()
    assert L.sbb200_ep_launches(None) == -1


def test_handle_exchange_gloo_world2():
    import ep_worker
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    store = _store_path()
    procs = [ctx.Process(target=ep_worker.handles_worker, args=(r, 2, store, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            r, v = q.get(timeout=120)
            got[r] = v
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    want = bytes([1]) * 64 + bytes([2]) * 64
    for r in range(2):
        assert got[r] == want, got[r]


@pytest.mark.parametrize("world", [2, 3])
def test_rank_partials_sum_to_the_layer(oracle, ep, world):
    """What each destination computes (its shard, routes to other ranks as
    -1) and what the source sums (partials of the owning ranks, ascending)."""
    E, K, I, T, top_k = 12, 256, 256, 20, 4
    L = oracle.make_layer(E, K, I, seed=77)
    hidden = oracle.make_hidden(T, K, seed=78)
    ids, w = oracle.route_logits(T, E, top_k, seed=79)
    ids[0, 1] = -1
    full = oracle.moe_forward(hidden, ids, w, L)
    total = np.zeros_like(full)
    for r in range(world):
        b, c = ep.expert_shard(E, world, r)
        shard = oracle.Layer(c, K, I, L.w13[b:b + c], L.s13[b:b + c], L.g13[b:b + c],
                             L.w2[b:b + c], L.s2[b:b + c], L.g2[b:b + c])
        local = np.where((ids >= b) & (ids < b + c), ids - b, -1).astype(np.int32)
        total = total + oracle.moe_forward(hidden, local, w, shard)
    assert rel_err(total, full) <= 1e-5
    assert cosine(total, full) >= 0.999999
