"""Routing extremes on the B200 against the oracle: every route on one expert
(one expert's token tiles carry the whole call, through the route plan inside
the activation split and through the separate plan kernels, in both term
layouts, W4A16 and W4A4), a call whose routes are all invalid, and top_k = E.

Tolerance as in the other parity tests: max|got - want| / max|want| <= 1e-2
and cosine >= 0.9999 against the fp32-accumulated oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cosine, rel_err
from gpu_util import dev, layer_to, run_moe

pytestmark = pytest.mark.gpu

REL_TOL = 1e-2
COS_TOL = 0.9999


def check(got, want):
    assert rel_err(got, want) <= REL_TOL, rel_err(got, want)
    assert cosine(got, want) >= COS_TOL, cosine(got, want)


# (E, T, top_k): 512 routes (plan inside the split, interleaved terms);
# 2,048 routes over E=16 (separate plan kernels, terms as planes along K:
# 16 full 128-token gate/up tiles of one expert); 2,600 routes over E=170
# (separate plan, interleaved terms, one expert far above the mean)
@pytest.mark.parametrize("E,T,top_k", [(16, 128, 4), (16, 512, 4), (170, 325, 8)])
def test_every_route_on_one_expert(sbb, oracle, cuda, E, T, top_k):
    K, I = 1024, 512
    L = oracle.make_layer(E, K, I, seed=71 + E)
    hidden = oracle.make_hidden(T, K, seed=72 + T)
    ids = np.full((T, top_k), 5, np.int32)
    rng = np.random.default_rng(73)
    w = rng.random((T, top_k), dtype=np.float32) / top_k
    got = run_moe(sbb, hidden, ids, w, L, cuda)
    check(got, oracle.moe_forward(hidden, ids, w, L))
    assert sbb.nvfp4_moe_bad_ids(cuda) == 0
    assert sbb.nvfp4_moe_device_errors(cuda) == 0


@pytest.mark.parametrize("T", [64, 300])
def test_no_valid_route(sbb, oracle, cuda, T):
    E, K, I, top_k = 16, 1024, 512, 4
    L = oracle.make_layer(E, K, I, seed=81)
    hidden = oracle.make_hidden(T, K, seed=82)
    ids = np.full((T, top_k), -1, np.int32)
    w = np.full((T, top_k), 0.25, np.float32)
    out = sbb.nvfp4_moe(dev(hidden, cuda, torch.bfloat16), dev(ids, cuda), dev(w, cuda),
                        *layer_to(L, cuda), out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert out.shape == (T, K) and out.dtype == torch.bfloat16
    assert torch.count_nonzero(out).item() == 0
    assert sbb.nvfp4_moe_bad_ids(cuda) == 0
    assert sbb.nvfp4_moe_device_errors(cuda) == 0


def test_top_k_equals_experts(sbb, oracle, cuda):
    E, K, I, T = 8, 512, 256, 40
    L = oracle.make_layer(E, K, I, seed=91)
    hidden = oracle.make_hidden(T, K, seed=92)
    ids = np.tile(np.arange(E, dtype=np.int32), (T, 1))
    for t in range(T):  # every expert once per token, in a per-token order
        np.random.default_rng(t).shuffle(ids[t])
    w = np.full((T, E), 1.0 / E, np.float32)
    got = run_moe(sbb, hidden, ids, w, L, cuda)
    check(got, oracle.moe_forward(hidden, ids, w, L))


@pytest.mark.parametrize("mode", ["static", "dynamic"])
@pytest.mark.parametrize("T", [128, 512])
def test_w4a4_every_route_on_one_expert(sbb, oracle, cuda, mode, T):
    from test_w4a4 import _static_scales
    E, K, I, top_k = 16, 1024, 512, 4
    L = oracle.make_layer(E, K, I, seed=101 + T)
    hidden = oracle.make_hidden(T, K, seed=102 + T)
    ids = np.full((T, top_k), 11, np.int32)
    w = np.random.default_rng(103).random((T, top_k), dtype=np.float32) / top_k
    scales = _static_scales(oracle, L, hidden, E) if mode == "static" else (None,) * 4
    want = oracle.moe_forward_w4a4(hidden, ids, w, L, *scales)
    ts = [None if s is None else torch.from_numpy(s).to(cuda) for s in scales]
    got = sbb.nvfp4_moe_w4a4(dev(hidden, cuda, torch.bfloat16), dev(ids, cuda), dev(w, cuda),
                             *layer_to(L, cuda), *ts)
    torch.cuda.synchronize()
    check(got.cpu().numpy(), want)
