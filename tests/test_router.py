"""Top-k router (the reference's moe_route_topk): the oracle against the
reference test's own check loop on its fixture (xpu_ops_smoke.cpp:2999-3000:
f32 512x64 k=2, bf16 512x128 k=4, logits sample(i) * 3), then the B200 kernel
against the oracle: ids bit-exact, weights within the reference test's 1e-5
(xpu_ops_smoke.cpp:452); and the fused routing + MoE call against the two
calls it replaces."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import cosine, rel_err


def _fixture(oracle, M, E, dt):
    x = oracle.kat_sample(np.arange(M * E)).reshape(M, E) * np.float32(3.0)
    if dt == "bf16":
        x = oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(x)).reshape(M, E)
    return x.astype(np.float32)


@pytest.mark.parametrize("M,E,k,dt", [(512, 64, 2, "f32"), (512, 128, 4, "bf16")])
def test_oracle_matches_reference_router_test(oracle, M, E, k, dt):
    x = _fixture(oracle, M, E, dt)
    ids, w = oracle.router_topk(x, k)
    rids, rw = oracle.kat_router_reference(x, k)
    assert (ids == rids).all()
    assert np.abs(w - rw).max() < 1e-5


def test_oracle_ties_and_infinities(oracle):
    x = np.array([[1.0, 3.0, 3.0, 2.0], [-np.inf, -np.inf, -np.inf, -np.inf],
                  [np.nan, 0.5, np.nan, 0.25]], np.float32)
    ids, w = oracle.router_topk(x, 2)
    assert ids.tolist()[0] == [1, 2]   # equal logits: lowest index first
    assert ids.tolist()[2] == [1, 3]   # NaN is never chosen


# ---------------------------------------------------------------- GPU

@pytest.mark.gpu
@pytest.mark.parametrize("M,E,k,dt", [(512, 64, 2, "f32"), (512, 128, 4, "bf16")])
def test_router_kernel_reference_fixture(sbb, oracle, cuda, M, E, k, dt):
    import torch
    x = _fixture(oracle, M, E, dt)
    t = torch.from_numpy(x).to(cuda)
    if dt == "bf16":
        t = t.to(torch.bfloat16)
    ids, w = sbb.router_topk(t, k)
    rids, rw = oracle.kat_router_reference(x, k)
    assert (ids.cpu().numpy() == rids).all()
    assert np.abs(w.cpu().numpy() - rw).max() < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("dt", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("M,E,k", [(1, 8, 1), (77, 170, 8), (300, 512, 64), (40, 33, 33)])
def test_router_kernel_vs_oracle(sbb, oracle, cuda, M, E, k, dt):
    import torch
    rng = np.random.default_rng(M * 31 + E + k)
    x = rng.standard_normal((M, E)).astype(np.float32)
    x[:, ::7] = np.round(x[:, ::7], 1)  # plenty of equal logits
    t = torch.from_numpy(x).to(cuda).to(getattr(torch, dt))
    xr = t.float().cpu().numpy()
    ids, w = sbb.router_topk(t, k)
    oids, ow = oracle.router_topk(xr, k)
    assert (ids.cpu().numpy() == oids).all()
    assert np.abs(w.cpu().numpy() - ow).max() < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("T", [64, 1024])  # one route-plan chunk (fused routing) and several
def test_moe_from_logits_equals_router_then_moe(sbb, oracle, cuda, T):
    import torch
    from gpu_util import dev, layer_to
    E, K, I, k = 48, 512, 256, 8
    L = oracle.make_layer(E, K, I, seed=T)
    hidden = dev(oracle.make_hidden(T, K, seed=T + 1), cuda, torch.bfloat16)
    logits = torch.from_numpy(np.random.default_rng(T).standard_normal((T, E)).astype(np.float32)).to(cuda)
    ws = layer_to(L, cuda)
    out, ids, w = sbb.nvfp4_moe_from_logits(hidden, logits, k, *ws)
    rids, rw = sbb.router_topk(logits, k)
    ref = sbb.nvfp4_moe(hidden, rids, rw, *ws)
    torch.cuda.synchronize()
    assert torch.equal(ids, rids) and torch.equal(w, rw)
    assert torch.equal(out, ref)
    want = oracle.moe_forward(hidden.view(torch.int16).cpu().numpy().view(np.uint16),
                              ids.cpu().numpy(), w.cpu().numpy(), L)
    got = out.cpu().numpy()
    assert rel_err(got, want) <= 1e-2 and cosine(got, want) >= 0.9999
