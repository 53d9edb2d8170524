"""Device route permutation vs the oracle: bit-exact counts, offsets, sorted
routes and inverse map, including dropped and out-of-range ids."""

from __future__ import annotations

import numpy as np
import pytest

from gpu_util import dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,top_k,E", [
    (1, 8, 170), (8, 8, 170), (64, 8, 170), (511, 8, 170), (512, 8, 170),
    (3000, 8, 170), (8192, 8, 170), (100, 4, 8), (7, 1, 1), (33, 64, 512), (1, 2, 16),
])
def test_route_plan_matches_oracle(sbb, oracle, cuda, M, top_k, E):
    rng = np.random.default_rng(M + top_k + E)
    ids = rng.integers(0, E, size=(M, top_k)).astype(np.int32)
    drop = rng.random((M, top_k)) < 0.05
    ids[drop] = -1
    if M * top_k > 4:
        ids.flat[3] = E + 1   # out of range
        ids.flat[4] = -9      # out of range
    want = oracle.route_plan(ids, E)
    got = sbb.route_plan(dev(ids, cuda), E)
    n = int(want["offsets"][-1])
    assert np.array_equal(got["counts"].cpu().numpy(), want["counts"])
    assert np.array_equal(got["offsets"].cpu().numpy(), want["offsets"])
    assert np.array_equal(got["sorted"].cpu().numpy()[:n], want["sorted"])
    assert np.array_equal(got["slot_of"].cpu().numpy(), want["slot_of"])
    assert int(got["bad_ids"].item()) == want["bad_ids"]


def test_route_plan_skewed_single_expert(sbb, oracle, cuda):
    ids = np.full((4096, 8), 5, np.int32)
    ids[::7, 3] = 2
    want = oracle.route_plan(ids, 170)
    got = sbb.route_plan(dev(ids, cuda), 170)
    assert np.array_equal(got["sorted"].cpu().numpy()[:int(want["offsets"][-1])], want["sorted"])


def test_route_plan_all_dropped(sbb, oracle, cuda):
    ids = np.full((16, 4), -1, np.int32)
    got = sbb.route_plan(dev(ids, cuda), 8)
    assert int(got["offsets"].cpu().numpy()[-1]) == 0
    assert np.all(got["slot_of"].cpu().numpy() == -1)
