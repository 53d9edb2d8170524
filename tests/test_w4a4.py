"""W4A4 (activations quantised once to NVFP4 and fed to the block-scaled
MMA): vLLM's static per-expert a1/a2_gscale + g1/g2_alphas convention, and
dynamic per-row quantisation (benchmark config 4), against the oracle's W4A4
path built on the vLLM-pinned quantiser. Bar: normwise relative error <= 1e-2
and cosine >= 0.9999 against the oracle's W4A4 result."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import cosine, rel_err

REL_TOL = 1e-2
COS_TOL = 0.9999


def _static_scales(oracle, L, hidden, E):
    """vLLM-style calibration: one activation global per expert from the
    inputs' amax (a = 448*6/amax), alpha = 1 / (a * G_weight), G_weight =
    1 / g (the stored dequant multiplier)."""
    x = oracle.bf16_bits_to_f32(hidden)
    amax = np.float32(np.abs(x).max())
    a13 = np.full(E, np.float32(2688.0) / amax, np.float32)
    # the SwiGLU rows are much smaller than the inputs; calibrate them at 1/8
    a2 = np.full(E, np.float32(2688.0) / (amax / np.float32(8.0)), np.float32)
    alpha13 = (np.float32(1.0) / a13 * L.g13).astype(np.float32)
    alpha2 = (np.float32(1.0) / a2 * L.g2).astype(np.float32)
    return a13, a2, alpha13, alpha2


def test_w4a4_oracle_close_to_w4a16(oracle):
    """Sanity of the restatement: W4A4 stays near the W4A16 result."""
    E, K, I, T, k = 8, 256, 256, 12, 2
    L = oracle.make_layer(E, K, I, seed=5)
    hidden = oracle.make_hidden(T, K, seed=6)
    ids, w = oracle.route_logits(T, E, k, seed=7)
    a16 = oracle.moe_forward(hidden, ids, w, L)
    a4 = oracle.moe_forward_w4a4(hidden, ids, w, L)
    assert cosine(a4, a16) > 0.98


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["static", "dynamic"])
@pytest.mark.parametrize("E,K,I,T,k", [(16, 512, 256, 40, 4), (34, 1024, 512, 96, 8),
                                       (16, 1024, 512, 2, 4)])
def test_w4a4_matches_oracle(sbb, oracle, cuda, mode, E, K, I, T, k):
    import torch
    from gpu_util import dev, layer_to
    L = oracle.make_layer(E, K, I, seed=T + E)
    hidden = oracle.make_hidden(T, K, seed=T + 1)
    ids, w = oracle.route_logits(T, E, k, seed=T + 2)
    ids[0, 0] = -1
    scales = _static_scales(oracle, L, hidden, E) if mode == "static" else (None,) * 4
    want = oracle.moe_forward_w4a4(hidden, ids, w, L, *scales)
    ts = [None if s is None else torch.from_numpy(s).to(cuda) for s in scales]
    got = sbb.nvfp4_moe_w4a4(dev(hidden, cuda, torch.bfloat16), dev(ids, cuda), dev(w, cuda),
                             *layer_to(L, cuda), *ts)
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    assert rel_err(got, want) <= REL_TOL, rel_err(got, want)
    assert cosine(got, want) >= COS_TOL, cosine(got, want)


@pytest.mark.gpu
def test_w4a4_zipf_prefill_shape(sbb, oracle, cuda):
    """Config-4 shape class: skewed Zipf(1.2) routing, enough tokens for the
    192/96-row prefill tiles on the hot experts; sampled tokens checked."""
    import torch
    from gpu_util import dev, layer_to
    E, K, I, T, k = 64, 1024, 512, 2048, 8
    L = oracle.make_layer(E, K, I, seed=99)
    hidden = oracle.make_hidden(T, K, seed=100)
    ids, w = oracle.route_zipf(T, E, k, seed=101)
    got = sbb.nvfp4_moe_w4a4(dev(hidden, cuda, torch.bfloat16), dev(ids, cuda), dev(w, cuda),
                             *layer_to(L, cuda))
    torch.cuda.synchronize()
    pick = np.random.default_rng(3).choice(T, 48, replace=False)
    want = oracle.moe_forward_w4a4(hidden[pick], ids[pick], w[pick], L)
    g = got.cpu().numpy()[pick]
    assert rel_err(g, want) <= REL_TOL and cosine(g, want) >= COS_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("w4a4", [False, True])
def test_sparse_routes_after_dense_call(sbb, oracle, cuda, w4a4):
    """The shape an expert-parallel shard sees: many rows, few of them routed
    here (the rest -1), right after a call whose routes filled the
    workspace. Both calls against the oracle."""
    import torch
    from gpu_util import dev, layer_to
    E, K, I, M, k = 5, 1024, 512, 256, 4
    L = oracle.make_layer(E, K, I, seed=61)
    ws = layer_to(L, cuda)
    hidden = oracle.make_hidden(M, K, seed=62)
    ids, w = oracle.route_logits(M, E, k, seed=63)
    sparse = ids.copy()
    sparse[5:] = -1
    for case in (ids, sparse):
        fn = sbb.nvfp4_moe_w4a4 if w4a4 else sbb.nvfp4_moe
        got = fn(dev(hidden, cuda, torch.bfloat16), dev(case, cuda), dev(w, cuda), *ws)
        torch.cuda.synchronize()
        want = (oracle.moe_forward_w4a4(hidden[:8], case[:8], w[:8], L) if w4a4
                else oracle.moe_forward(hidden[:8], case[:8], w[:8], L))
        g = got.cpu().numpy()[:8]
        assert rel_err(g, want) <= REL_TOL, (case is sparse, rel_err(g, want))
        assert cosine(g, want) >= COS_TOL
