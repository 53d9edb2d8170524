"""The vLLM hook adapter (shooting_brake_b200.plugin): host-side behaviour on
the CPU, forward parity on the B200.

The adapter mirrors HybridRoutedExperts.forward_modular
(src/phase4/src/shooting_brake_vllm/routed_experts.py:2312-2397 of the
reference): x bf16 [M, d], topk_weights fp32 [M, top_k], topk_ids [M, top_k]
in, x-dtype [M, d] out, plus the shared experts' output when given."""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from conftest import cosine, rel_err

REL_TOL = 1e-2
COS_TOL = 0.9999


@pytest.fixture(scope="module")
def plugin(sbb):
    return importlib.import_module(sbb.__name__ + ".plugin")


def _layer_tensors(oracle, device, E=8, K=256, I=256, seed=3):
    L = oracle.make_layer(E, K, I, seed=seed)
    ts = [torch.from_numpy(np.ascontiguousarray(x)).to(device)
          for x in (L.w13, L.s13, L.g13, L.w2, L.s2, L.g2)]
    return L, ts


def test_up_gate_layout_is_reordered_once(plugin, oracle):
    L, ts = _layer_tensors(oracle, "cpu")
    I = L.I
    swapped = [torch.cat([ts[0][:, I:], ts[0][:, :I]], 1), torch.cat([ts[1][:, I:], ts[1][:, :I]], 1)]
    ex = plugin.RoutedExpertsB200(swapped[0], swapped[1], ts[2], ts[3], ts[4], ts[5],
                                  w13_is_up_gate=True)
    assert torch.equal(ex.w13, ts[0]) and torch.equal(ex.w13_scale, ts[1])


def test_from_layer_reads_vllm_attribute_names(plugin, oracle):
    L, ts = _layer_tensors(oracle, "cpu")

    class FakeLayer:
        pass

    layer = FakeLayer()
    for name, t in zip(("w13_weight", "w13_weight_scale", "w13_weight_scale_2", "w2_weight",
                        "w2_weight_scale", "w2_weight_scale_2"), ts):
        setattr(layer, name, torch.nn.Parameter(t, requires_grad=False))
    layer._w13_is_reordered = lambda: False
    ex = plugin.RoutedExpertsB200.from_layer(layer, scale_layout="linear")
    assert ex.num_experts == L.E and torch.equal(ex.w2, ts[3])


def _vllm_swizzle(monkeypatch, sf_u8: torch.Tensor) -> torch.Tensor:
    """vLLM's own swizzle_blockscale on a CPU tensor (the helper ends in
    .cuda(); that move is made a no-op here so it runs without a GPU)."""
    nu = pytest.importorskip("vllm.model_executor.layers.quantization.utils.nvfp4_utils")
    with monkeypatch.context() as m:
        m.setattr(torch.Tensor, "cuda", lambda self, *a, **k: self)
        return nu.swizzle_blockscale(sf_u8.view(torch.float8_e4m3fn)).view(torch.uint8)


def _fake_vllm_layer(ts, monkeypatch, E, scale2_shape="E"):
    class FakeLayer:
        pass

    layer = FakeLayer()
    w13, s13, g13, w2, s2, g2 = ts
    layer.w13_weight = torch.nn.Parameter(w13, requires_grad=False)
    layer.w2_weight = torch.nn.Parameter(w2, requires_grad=False)
    layer.w13_weight_scale = torch.nn.Parameter(_vllm_swizzle(monkeypatch, s13),
                                                requires_grad=False)
    layer.w2_weight_scale = torch.nn.Parameter(_vllm_swizzle(monkeypatch, s2),
                                               requires_grad=False)
    if scale2_shape == "E2":
        g13 = torch.stack([g13, g13], dim=1)
        g2 = torch.stack([g2, g2], dim=1)
    layer.w13_weight_scale_2 = torch.nn.Parameter(g13, requires_grad=False)
    layer.w2_weight_scale_2 = torch.nn.Parameter(g2, requires_grad=False)
    return layer


@pytest.mark.parametrize("K,I", [(256, 256), (512, 96)])
def test_from_layer_unswizzles_vllm_block_scales(plugin, oracle, monkeypatch, K, I):
    """Scales swizzled by vLLM's swizzle_blockscale (rows padded to 128,
    columns to 4 when I/16 is not a multiple of 4) come back byte-exact in
    the linear bank layout, and agree with vLLM's convert_swizzled_to_linear."""
    emu = pytest.importorskip(
        "vllm.model_executor.layers.quantization.utils.nvfp4_emulation_utils")
    E = 3
    L, ts = _layer_tensors(oracle, "cpu", E, K, I, seed=5)
    layer = _fake_vllm_layer(ts, monkeypatch, E, scale2_shape="E2")
    assert layer.w2_weight_scale.shape[-1] % 4 == 0
    ex = plugin.RoutedExpertsB200.from_layer(layer)
    assert torch.equal(ex.w13_scale, ts[1]) and torch.equal(ex.w2_scale, ts[4])
    assert torch.equal(ex.w13_global, ts[2]) and torch.equal(ex.w2_global, ts[5])
    for e in range(E):
        # that helper slices its result to k columns, not k/16, so padding
        # columns may remain on its side
        lin = emu.convert_swizzled_to_linear(layer.w2_weight_scale.data[e], K, I, 16)
        assert torch.equal(lin[:, :I // 16].contiguous().view(torch.uint8), ts[4][e])


def test_from_layer_globals_from_quant_config(plugin, oracle):
    """vLLM's alphas are the weight global over the activation global
    (expert_bank.py:270-295 of the reference): g = alpha * a_gscale."""
    E, K, I = 4, 256, 256
    L, ts = _layer_tensors(oracle, "cpu", E, K, I, seed=7)

    class Desc:
        def __init__(self, v):
            self.alpha_or_gscale = v

    class QC:
        pass

    a1, a2 = torch.tensor([54.75]), torch.full((E,), 154.0)
    qc = QC()
    qc._w1, qc._w2 = Desc(ts[2] / a1), Desc(ts[5] / a2)
    qc._a1, qc._a2 = Desc(a1), Desc(a2)
    g13, g2 = plugin.layer_globals(type("L", (), {"quant_method": type(
        "Q", (), {"moe_quant_config": qc})()})(), E)
    assert torch.allclose(g13, ts[2], rtol=1e-6) and torch.allclose(g2, ts[5], rtol=1e-6)


def test_from_layer_rejects_unpadded_swizzled_scales(plugin, oracle):
    E, K, I = 2, 256, 96
    L, ts = _layer_tensors(oracle, "cpu", E, K, I, seed=9)
    with pytest.raises(ValueError, match="swizzled block scales"):
        plugin.unswizzle_block_scales(ts[4], K, I // 16)  # [E, 256, 6]: not padded to 8


def test_forward_on_cpu_tensors_raises(plugin, oracle):
    """No CPU fallback: host tensors are rejected by the op."""
    L, ts = _layer_tensors(oracle, "cpu")
    ex = plugin.RoutedExpertsB200(*ts)
    x = torch.zeros((2, L.K), dtype=torch.bfloat16)
    ids = torch.zeros((2, 2), dtype=torch.int32)
    w = torch.ones((2, 2), dtype=torch.float32)
    with pytest.raises(Exception):
        ex.forward_modular(x, w, ids)


def test_register_without_modular_routed_experts(plugin):
    """vLLM releases whose RoutedExperts has no forward_modular leave the
    registry untouched."""
    try:
        from vllm.model_executor.layers.fused_moe import RoutedExperts
    except Exception:
        pytest.skip("vLLM not importable")
    if hasattr(RoutedExperts, "forward_modular"):
        pytest.skip("this vLLM has the modular hook")
    assert plugin.register() is False


# ---------------------------------------------------------------- GPU parity

def _check(got, want):
    assert rel_err(got, want) <= REL_TOL, rel_err(got, want)
    assert cosine(got, want) >= COS_TOL, cosine(got, want)


@pytest.mark.gpu
def test_forward_modular_matches_oracle(plugin, oracle, cuda):
    E, K, I, T, top_k = 16, 512, 256, 24, 4
    L, ts = _layer_tensors(oracle, cuda, E, K, I, seed=11)
    hidden = oracle.make_hidden(T, K, seed=12)
    ids, w = oracle.route_logits(T, E, top_k, seed=13)
    ex = plugin.RoutedExpertsB200(*ts)
    x = torch.from_numpy(hidden).to(cuda).view(torch.bfloat16)
    y = ex.forward_modular(x, torch.from_numpy(w).to(cuda), torch.from_numpy(ids).long().to(cuda))
    assert y.dtype == torch.bfloat16 and y.shape == (T, K)
    _check(y.float().cpu().numpy(), oracle.moe_forward(hidden, ids, w, L))


@pytest.mark.gpu
def test_expert_map_shard_and_shared_experts(plugin, oracle, cuda):
    """A shard holding global experts [4, 12) of 16: routes to other experts
    contribute nothing; the shared-expert output is added."""
    E_glob, K, I, T, top_k = 16, 256, 256, 20, 4
    L, _ = _layer_tensors(oracle, "cpu", E_glob, K, I, seed=21)
    lo, hi = 4, 12
    shard = oracle.Layer(hi - lo, K, I, L.w13[lo:hi], L.s13[lo:hi], L.g13[lo:hi],
                         L.w2[lo:hi], L.s2[lo:hi], L.g2[lo:hi])
    ts = [torch.from_numpy(np.ascontiguousarray(x)).to(cuda)
          for x in (shard.w13, shard.s13, shard.g13, shard.w2, shard.s2, shard.g2)]
    emap = torch.full((E_glob,), -1, dtype=torch.int32)
    emap[lo:hi] = torch.arange(hi - lo, dtype=torch.int32)
    hidden = oracle.make_hidden(T, K, seed=22)
    ids, w = oracle.route_logits(T, E_glob, top_k, seed=23)
    ex = plugin.RoutedExpertsB200(*ts, expert_map=emap)
    x = torch.from_numpy(hidden).to(cuda).view(torch.bfloat16)
    shared = lambda inp: torch.full_like(inp, 0.25)  # noqa: E731
    y = ex.forward_modular(x, torch.from_numpy(w).to(cuda), torch.from_numpy(ids).to(cuda),
                           shared_experts=shared)
    local = np.where((ids >= lo) & (ids < hi), ids - lo, -1).astype(np.int32)
    want = oracle.moe_forward(hidden, local, w, shard) + 0.25
    _check(y.float().cpu().numpy(), want)


def _shared_layer(oracle, K, Is, seed):
    S = oracle.make_layer(1, K, Is, seed=seed)
    return S


def test_shared_expert_split_is_exact(plugin, oracle):
    """The n chunk experts of a fused shared expert dequantise to exactly the
    shared expert's gate/up row blocks and down column blocks."""
    import torch
    E, K, I = 4, 256, 128
    L, ts = _layer_tensors(oracle, "cpu", E, K, I, seed=31)
    S = _shared_layer(oracle, K, 3 * I, seed=32)
    sh = [torch.from_numpy(np.ascontiguousarray(x[0] if x.ndim == 3 else x)) for x in
          (S.w13, S.s13, S.g13, S.w2, S.s2, S.g2)]
    ex = plugin.RoutedExpertsB200(*ts, shared=tuple(sh))
    assert ex.shared_chunks == 3 and ex.num_experts == E and ex.w13.size(0) == E + 3
    full13 = oracle.dequant(S.w13[0], S.s13[0], float(S.g13[0]))
    full2 = oracle.dequant(S.w2[0], S.s2[0], float(S.g2[0]))
    Is = 3 * I
    for c in range(3):
        w13 = oracle.dequant(ex.w13[E + c].numpy(), ex.w13_scale[E + c].numpy(), float(ex.w13_global[E + c]))
        assert np.array_equal(w13[:I], full13[c * I:(c + 1) * I])
        assert np.array_equal(w13[I:], full13[Is + c * I:Is + (c + 1) * I])
        w2 = oracle.dequant(ex.w2[E + c].numpy(), ex.w2_scale[E + c].numpy(), float(ex.w2_global[E + c]))
        assert np.array_equal(w2, full2[:, c * I:(c + 1) * I])


@pytest.mark.gpu
def test_fused_shared_expert_matches_oracle(plugin, oracle, cuda):
    """Routed experts plus a shared expert of twice the intermediate size in
    one grouped call, gated per token, against the oracle's two results."""
    import torch
    E, K, I, T, top_k = 12, 512, 256, 30, 4
    L, ts = _layer_tensors(oracle, cuda, E, K, I, seed=41)
    S = _shared_layer(oracle, K, 2 * I, seed=42)
    sh = tuple(torch.from_numpy(np.ascontiguousarray(x[0] if x.ndim == 3 else x)).to(cuda)
               for x in (S.w13, S.s13, S.g13, S.w2, S.s2, S.g2))
    hidden = oracle.make_hidden(T, K, seed=43)
    ids, w = oracle.route_logits(T, E, top_k, seed=44)
    gate = np.random.default_rng(45).uniform(0.2, 1.0, T).astype(np.float32)
    ex = plugin.RoutedExpertsB200(*ts, shared=sh)
    x = torch.from_numpy(hidden).to(cuda).view(torch.bfloat16)
    y = ex.forward_modular(x, torch.from_numpy(w).to(cuda), torch.from_numpy(ids).to(cuda),
                           shared_gate=torch.from_numpy(gate).to(cuda))
    routed = oracle.moe_forward(hidden, ids, w, L)
    shared = oracle.moe_forward(hidden, np.zeros((T, 1), np.int32), np.ones((T, 1), np.float32), S)
    want = routed + gate[:, None] * shared
    _check(y.float().cpu().numpy(), want)


@pytest.mark.gpu
def test_from_layer_swizzled_vllm_layer_matches_oracle(plugin, oracle, cuda):
    """A vLLM-style layer with scales from vLLM's swizzle_blockscale on the
    device and [E, 2] weight_scale_2, through from_layer, against the oracle."""
    nu = pytest.importorskip("vllm.model_executor.layers.quantization.utils.nvfp4_utils")
    E, K, I, T, top_k = 10, 512, 256, 40, 4
    L, ts = _layer_tensors(oracle, cuda, E, K, I, seed=51)

    class FakeLayer:
        pass

    layer = FakeLayer()
    layer.w13_weight, layer.w2_weight = ts[0], ts[3]
    layer.w13_weight_scale = nu.swizzle_blockscale(ts[1].view(torch.float8_e4m3fn))
    layer.w2_weight_scale = nu.swizzle_blockscale(ts[4].view(torch.float8_e4m3fn))
    layer.w13_weight_scale_2 = torch.stack([ts[2], ts[2]], 1)
    layer.w2_weight_scale_2 = torch.stack([ts[5], ts[5]], 1)
    ex = plugin.RoutedExpertsB200.from_layer(layer)
    hidden = oracle.make_hidden(T, K, seed=52)
    ids, w = oracle.route_logits(T, E, top_k, seed=53)
    x = torch.from_numpy(hidden).to(cuda).view(torch.bfloat16)
    y = ex.forward_modular(x, torch.from_numpy(w).to(cuda), torch.from_numpy(ids).to(cuda))
    _check(y.float().cpu().numpy(), oracle.moe_forward(hidden, ids, w, L))
    assert ex.device_errors() == 0
