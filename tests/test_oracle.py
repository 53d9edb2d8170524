"""The CPU oracle pinned against the reference: its own CPU expert tier
(compiled from source), the fp32 loop of its device test, vLLM's NVFP4
dequantiser and quantiser. No GPU."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from conftest import cosine, golden, rel_err

# The oracle differs from the reference CPU tier only in fp32 rounding order
# (FMA contraction in the -O3 -march=native reference build): a few ulps.
ORACLE_VS_REF = 2e-6


def _digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _layer_digest(L) -> str:
    return _digest(L.w13, L.s13, L.g13, L.w2, L.s2, L.g2)


@pytest.mark.parametrize("kind", ["moe", "blocks"])
def test_known_answer_fixture(oracle, kind):
    fx = oracle.kat_fixture(kind)
    gold = golden(f"kat_{kind}.npz")
    assert str(gold["digest"]) == _digest(fx["hidden"], fx["ids"], fx["weights"]) + _layer_digest(fx["layer"])
    got = oracle.moe_forward(fx["hidden"], fx["ids"], fx["weights"], fx["layer"])
    assert rel_err(got, gold["out_ref"]) <= ORACLE_VS_REF
    # the device test's own tolerance against its fp32 loop (xpu_ops_smoke.cpp:2366)
    assert np.abs(got - gold["out_loop"]).max() <= 8e-4
    assert np.array_equal(oracle.kat_reference_loop(fx), gold["out_loop"])


def test_blocks_fixture_topology(oracle):
    """Lopsided routing of xpu_ops_smoke.cpp:2454-2552: expert 0 spans several
    32-row blocks, expert E-1 is empty, partial blocks and -1 ids exist."""
    fx = oracle.kat_fixture("blocks")
    plan = oracle.route_plan(fx["ids"], fx["layer"].E)
    c = plan["counts"]
    assert (c[0] + 31) // 32 > 1 and c[-1] == 0
    assert any(x % 32 for x in c if x)
    assert (fx["ids"] == -1).any()
    got = oracle.moe_forward(fx["hidden"], fx["ids"], fx["weights"], fx["layer"])
    routed = (fx["ids"] >= 0).any(axis=1)
    assert np.all(np.abs(got[routed]).max(axis=1) > 0)
    assert np.all(got[~routed] == 0)


def test_config0_golden(oracle):
    E, K, I, T, top_k = 16, 1024, 512, 64, 2
    L = oracle.make_layer(E, K, I, seed=0)
    hidden = oracle.make_hidden(T, K, seed=1)
    ids, w = oracle.route_logits(T, E, top_k, seed=2)
    gold = golden("c0.npz")
    assert str(gold["digest"]) == _digest(hidden, ids, w) + _layer_digest(L)
    got = oracle.moe_forward(hidden, ids, w, L)
    assert rel_err(got, gold["out_ref"]) <= ORACLE_VS_REF
    assert cosine(got, gold["out_ref"]) >= 1 - 1e-9


def test_dequant_matches_vllm_dequantizer(oracle):
    g = golden("expert_planes.npz")
    I = g["w13"].shape[1] // 2
    dq = oracle.dequant(g["w13"][0], g["s13"][0], g["g13"][0])
    assert np.array_equal(dq[:I], g["dq_gate"])
    assert np.array_equal(dq[I:], g["dq_up"])
    assert np.array_equal(oracle.dequant(g["w2"][0], g["s2"][0], g["g2"][0]), g["dq_down"])


def test_single_expert_ffn_matches_reference_tier(oracle):
    g = golden("expert_planes.npz")
    K = g["w2"].shape[1]
    I = g["w13"].shape[1] // 2
    L = oracle.Layer(1, K, I, g["w13"], g["s13"], g["g13"], g["w2"], g["s2"], g["g2"])
    for M in (1, 3, 16):
        x = g[f"x{M}"]
        ids = np.zeros((M, 1), np.int32)
        w = np.ones((M, 1), np.float32)
        got = oracle.moe_forward(x, ids, w, L)
        assert rel_err(got, g[f"y{M}"]) <= ORACLE_VS_REF


def test_quantizer_matches_vllm_ref_nvfp4_quant(oracle):
    g = golden("quant.npz")
    q, sf = oracle.quantize_nvfp4(g["x"], g["G"][0])
    codes = oracle.unpack_fp4(q)
    vals = np.where(codes & 8, -1.0, 1.0).astype(np.float32) * oracle.E2M1_VALUES[codes & 7]
    assert np.array_equal(vals, g["vals"])
    assert np.array_equal(oracle.e4m3_decode(sf), g["scales"])


def test_e4m3_and_e2m1_tables(oracle):
    lib = oracle.oracle_lib()
    for v in range(256):
        a = lib.sbo_e4m3(v)
        b = float(oracle.e4m3_decode(np.array([v], np.uint8))[0])
        assert (np.isnan(a) and np.isnan(b)) or a == b
    assert [lib.sbo_e2m1(n) for n in range(16)] == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                                                    -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]
    # e4m3 encode round-trips every finite non-negative code
    v = np.arange(0x7F, dtype=np.uint8)
    assert np.array_equal(oracle.e4m3_encode_rne(oracle.e4m3_decode(v)), v)


@pytest.mark.parametrize("M,top_k,E", [(1, 8, 170), (64, 8, 170), (700, 8, 170), (5, 3, 4)])
def test_route_plan_oracle_properties(oracle, M, top_k, E):
    rng = np.random.default_rng(M * 1000 + E)
    ids = rng.integers(-1, E, size=(M, top_k)).astype(np.int32)
    ids[0, 0] = E + 3      # out of range: dropped and counted
    ids[-1, -1] = -5       # out of range: dropped and counted
    p = oracle.route_plan(ids, E)
    flat = ids.ravel()
    valid = (flat >= 0) & (flat < E)
    assert p["bad_ids"] == 2
    assert np.array_equal(p["counts"], np.bincount(flat[valid], minlength=E))
    assert p["offsets"][-1] == valid.sum()
    # stable: sorted is the stable argsort of valid routes by expert
    r = np.nonzero(valid)[0]
    want = r[np.argsort(flat[r], kind="stable")]
    assert np.array_equal(p["sorted"], want)
    assert np.array_equal(p["slot_of"][want], np.arange(len(want)))
    assert np.all(p["slot_of"][~valid] == -1)


@pytest.mark.skipif("not __import__('oracle.nvfp4', fromlist=['x']).reference_available()")
@pytest.mark.parametrize("E,K,I,T,top_k,seed", [(8, 256, 64, 17, 4, 3), (12, 512, 160, 9, 3, 4)])
def test_oracle_vs_live_reference_tier(oracle, E, K, I, T, top_k, seed):
    L = oracle.make_layer(E, K, I, seed=seed)
    hidden = oracle.make_hidden(T, K, seed=seed + 1)
    ids, w = oracle.route_logits(T, E, top_k, seed=seed + 2)
    ids[0, 0] = -1
    ref = oracle.ReferenceCpuTier(L, threads=4)
    want = ref.forward(hidden, ids, w)
    ref.close()
    got = oracle.moe_forward(hidden, ids, w, L)
    assert rel_err(got, want) <= ORACLE_VS_REF
