"""Expert parallelism over NVLink on two GPUs: each rank's tokens through the
sharded layer vs the oracle's single-layer result (tolerance of the
north_star bar: normwise relative error <= 1e-2, cosine >= 0.9999), over
several steps with ragged token counts (one rank with none) so the exchange
buffers are reused. Child processes, one per GPU, gloo for the handle swap
only; skipped with fewer than two GPUs."""

from __future__ import annotations

import multiprocessing as mp
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

REL_TOL = 1e-2
COS_TOL = 0.9999


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, shape, steps):
    import ep_worker
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=ep_worker.ep_forward_worker, args=(r, world, port, shape, steps, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            r, v = q.get(timeout=300)
            got[r] = v
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return got


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("shape", [(16, 512, 256, 4, 24), (34, 1024, 512, 8, 64)])
def test_ep_two_ranks_match_oracle(cuda, shape):
    steps = [(shape[4], shape[4] // 2), (5, 0), (1, shape[4])]
    got = _run(2, shape, steps)
    for r in range(2):
        v = got[r]
        assert isinstance(v, dict), v
        assert v["errors"] == 0
        for T, err, cos in v["results"]:
            if T:
                assert err <= REL_TOL, (r, T, err)
                assert cos >= COS_TOL, (r, T, cos)
