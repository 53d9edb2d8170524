"""The scratch-free route plan, sbb200_route_plan_static.

It exists for callers that cannot hand the library device memory: serving
engines whose device memory belongs to a pooling allocator sized up front, and
FFI bindings that hold only the tensors they were given and have no device
allocator. Its scratch is a fixed array inside the library, shared by every
call, so calls in a row must each agree with the workspace entry point,
sbb200_route_plan, whatever the previous call left in that array. Integer
outputs: compared exactly.

The file name sorts last so that a stop-at-first-failure run has already run
every other test when it gets here."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

P = ctypes.c_void_p
S = ctypes.c_size_t


def static_entry(lib):
    f = lib.sbb200_route_plan_static
    f.restype = ctypes.c_int
    f.argtypes = [P, P, S, S, S, P, P, P, P, P]
    return f


def run_static(sbb, ids: torch.Tensor, E: int, with_counter: bool):
    M, top_k = ids.shape
    R = M * top_k
    dev = ids.device
    counts = torch.full((E,), -7, dtype=torch.int32, device=dev)
    offsets = torch.full((E + 1,), -7, dtype=torch.int32, device=dev)
    sorted_routes = torch.full((max(R, 1),), -7, dtype=torch.int32, device=dev)
    slot_of = torch.full((max(R, 1),), -7, dtype=torch.int32, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = static_entry(sbb.lib())(stream, ids.data_ptr(), M, top_k, E, counts.data_ptr(),
                                 offsets.data_ptr(), sorted_routes.data_ptr(),
                                 slot_of.data_ptr(), bad.data_ptr() if with_counter else None)
    assert rc == 0, sbb.last_error()
    return counts, offsets, sorted_routes, slot_of[:R], bad


def test_static_route_plan_matches_workspace_entry_point(sbb, cuda):
    # Two calls in a row with different shapes, both spanning several
    # 4096-route chunks, so the second reads scratch the first one wrote.
    cases = [(3000, 8, 170, 11, True), (5000, 4, 64, 12, False)]
    for M, top_k, E, seed, with_counter in cases:
        rng = np.random.default_rng(seed)
        ids = rng.integers(0, E, size=(M, top_k)).astype(np.int32)
        ids[rng.random((M, top_k)) < 0.05] = -1
        ids[0, 0] = E + 5  # out of range: dropped and counted
        t = torch.from_numpy(ids).to(cuda)
        want = sbb.route_plan(t, E)
        counts, offsets, sorted_routes, slot_of, bad = run_static(sbb, t, E, with_counter)
        torch.cuda.synchronize()
        n = int(want["offsets"][-1].item())
        assert torch.equal(counts, want["counts"])
        assert torch.equal(offsets, want["offsets"])
        assert torch.equal(sorted_routes[:n], want["sorted"][:n])
        assert torch.equal(slot_of, want["slot_of"])
        if with_counter:
            assert int(bad.item()) == int(want["bad_ids"].item()) == 1


def test_static_route_plan_single_chunk_and_empty(sbb, cuda):
    # One 4096-route chunk (no per-chunk counts in the shared array), then a
    # call with no routes (counts and offsets cleared, nothing else touched),
    # then the single-chunk call again after a multi-chunk one.
    rng = np.random.default_rng(21)
    small = rng.integers(-1, 170, size=(100, 8)).astype(np.int32)
    big = rng.integers(0, 96, size=(1500, 8)).astype(np.int32)
    for ids, E in ((small, 170), (np.zeros((0, 8), np.int32), 170), (big, 96), (small, 170)):
        t = torch.from_numpy(ids).to(cuda)
        counts, offsets, sorted_routes, slot_of, bad = run_static(sbb, t, E, False)
        torch.cuda.synchronize()
        if ids.shape[0] == 0:
            assert torch.equal(counts, torch.zeros_like(counts))
            assert torch.equal(offsets, torch.zeros_like(offsets))
            continue
        want = sbb.route_plan(t, E)
        n = int(want["offsets"][-1].item())
        assert torch.equal(counts, want["counts"])
        assert torch.equal(offsets, want["offsets"])
        assert torch.equal(sorted_routes[:n], want["sorted"][:n])
        assert torch.equal(slot_of, want["slot_of"])


def test_static_route_plan_rejects_oversize(sbb):
    lib = sbb.lib()
    dummy = P(1)
    rc = static_entry(lib)(None, dummy, 65537, 4, 170, dummy, dummy, dummy, dummy, None)
    assert rc == -4
    assert "262144" in sbb.last_error()
    # a route count that would wrap around size_t is rejected, not wrapped
    rc = static_entry(lib)(None, dummy, (1 << 63) + 1, 2, 170, dummy, dummy, dummy, dummy, None)
    assert rc == -4
