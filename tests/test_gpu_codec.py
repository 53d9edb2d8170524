"""Device NVFP4 codec vs the CPU oracle: dequant and quantise bit-exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from gpu_util import dev

pytestmark = pytest.mark.gpu


def test_dequant_bit_exact_random_planes(sbb, oracle, cuda):
    rng = np.random.default_rng(11)
    for rows, cols in ((1, 16), (7, 48), (256, 4096), (1280, 512)):
        q = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
        sf = rng.integers(0, 256, size=(rows, cols // 16), dtype=np.uint8)
        sf[sf == 0x7F] = 0x7E  # keep NaN scales out of the equality check
        sf[sf == 0xFF] = 0xFE
        g = np.float32(rng.uniform(1e-4, 2.0))
        want = oracle.dequant(q, sf, g)
        got = sbb.nvfp4_dequant(dev(q, cuda), dev(sf, cuda),
                                torch.tensor([g], device=cuda), rows).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (rows, cols)


def test_dequant_matches_vllm_golden(sbb, cuda):
    g = golden("expert_planes.npz")
    I = g["w13"].shape[1] // 2
    got = sbb.nvfp4_dequant(dev(g["w13"][0], cuda), dev(g["s13"][0], cuda),
                            dev(g["g13"], cuda), 2 * I).cpu().numpy()
    assert np.array_equal(got[:I], g["dq_gate"]) and np.array_equal(got[I:], g["dq_up"])


def test_dequant_per_expert_globals(sbb, oracle, cuda):
    L = oracle.make_layer(3, 256, 64, seed=5)
    got = sbb.nvfp4_dequant(dev(L.w13, cuda), dev(L.s13, cuda), dev(L.g13, cuda),
                            2 * L.I).cpu().numpy()
    for e in range(L.E):
        assert np.array_equal(got[e], oracle.dequant(L.w13[e], L.s13[e], L.g13[e]))


def test_quantize_bit_exact_vs_oracle_and_vllm(sbb, oracle, cuda):
    g = golden("quant.npz")
    x = g["x"]
    G = g["G"]
    q, sf = sbb.nvfp4_quantize(dev(x, cuda), dev(G, cuda), x.shape[0])
    q, sf = q.cpu().numpy(), sf.cpu().numpy()
    q_o, sf_o = oracle.quantize_nvfp4(x, G[0])
    assert np.array_equal(q, q_o) and np.array_equal(sf, sf_o)
    codes = oracle.unpack_fp4(q)
    vals = np.where(codes & 8, -1.0, 1.0).astype(np.float32) * oracle.E2M1_VALUES[codes & 7]
    assert np.array_equal(vals, g["vals"])


def test_quantize_bf16_input_layers(sbb, oracle, cuda):
    rng = np.random.default_rng(3)
    w = rng.standard_normal((2, 96, 256), dtype=np.float32) * np.float32(0.02)
    bits = oracle.f32_to_bf16_bits(w)
    wf = oracle.bf16_bits_to_f32(bits)
    G = np.array([np.float32(2688.0) / np.float32(np.abs(wf[e]).max()) for e in range(2)],
                 np.float32)
    q, sf = sbb.nvfp4_quantize(dev(bits, cuda, torch.bfloat16), dev(G, cuda), 96)
    for e in range(2):
        q_o, sf_o = oracle.quantize_nvfp4(wf[e], G[e])
        assert np.array_equal(q[e].cpu().numpy(), q_o)
        assert np.array_equal(sf[e].cpu().numpy(), sf_o)
