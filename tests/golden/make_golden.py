"""Generate the golden fixtures under tests/golden/ from the REFERENCE itself.

Run in a container that has the reference tree (its CPU expert tier is
compiled from source by oracle/Makefile into oracle/_ref/) and vLLM:

    python tests/golden/make_golden.py

Inputs are regenerated at test time by the seeded generators of
oracle/nvfp4.py; each fixture stores a sha256 of its inputs so drift in a
generator is caught rather than silently compared. Outputs stored here come
from the reference's code, never from this repository's oracle:

* kat_moe.npz / kat_blocks.npz -- the known-answer fixtures of the reference's
  device test (src/QuixiCore-XPU/tests/xpu_ops_smoke.cpp:2260-2304 and
  :2454-2510), outputs of the reference's CPU expert tier (sb_cpu_moe_forward)
  and of the test's own fp32 loop (xpu_ops_smoke.cpp:2316-2348, restated).
* c0.npz -- benchmark config 0 (E=16, d=1024, I=512, top-2, T=64, seed 0)
  through sb_cpu_moe_forward.
* expert_planes.npz -- random-byte NVFP4 planes in the style of
  src/phase7/nvfp4_testutil.py:33-51 (all 16 nibble codes, scale exponents
  4..10), single-expert FFN outputs of sb_cpu_expert_forward at M in {1, 3, 16}
  and vLLM dequantize_to_dtype of the planes.
* quant.npz -- vLLM ref_nvfp4_quant codes and scales of a seeded matrix.
* w4a4.npz -- a W4A4 routed-expert layer through vLLM's NVFP4 linear
  emulation (run_nvfp4_emulations), static and dynamic activation globals.
"""

from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import nvfp4 as O  # noqa: E402


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def layer_digest(L: O.Layer) -> str:
    return digest(L.w13, L.s13, L.g13, L.w2, L.s2, L.g2)


def kat(kind: str) -> None:
    fx = O.kat_fixture(kind)
    L = fx["layer"]
    ref = O.ReferenceCpuTier(L, threads=4)
    out_ref = ref.forward(fx["hidden"], fx["ids"], fx["weights"])
    ref.close()
    out_loop = O.kat_reference_loop(fx)
    np.savez_compressed(HERE / f"kat_{kind}.npz", out_ref=out_ref, out_loop=out_loop,
                        digest=digest(fx["hidden"], fx["ids"], fx["weights"]) + layer_digest(L))


def c0() -> None:
    E, K, I, T, top_k = 16, 1024, 512, 64, 2
    L = O.make_layer(E, K, I, seed=0)
    hidden = O.make_hidden(T, K, seed=1)
    ids, w = O.route_logits(T, E, top_k, seed=2)
    ref = O.ReferenceCpuTier(L, threads=8)
    out = ref.forward(hidden, ids, w)
    ref.close()
    np.savez_compressed(HERE / "c0.npz", out_ref=out, ids=ids, weights=w,
                        digest=digest(hidden, ids, w) + layer_digest(L))


def random_plane(rng, rows, cols):
    q = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    exp = rng.integers(4, 11, size=(rows, cols // 16))
    man = rng.integers(0, 8, size=(rows, cols // 16))
    sf = ((exp << 3) | man).astype(np.uint8)
    return q, sf


def expert_planes() -> None:
    import torch
    from vllm.model_executor.layers.quantization.utils.nvfp4_emulation_utils import (
        dequantize_to_dtype,
    )

    K, I = 256, 128
    rng = np.random.default_rng(20260807)
    gq, gs = random_plane(rng, I, K)
    uq, us = random_plane(rng, I, K)
    dq, ds = random_plane(rng, K, I)
    g13 = np.float32(0.75)
    g2 = np.float32(1.25)
    # one expert in the op layout
    L = O.Layer(1, K, I, np.concatenate([gq, uq])[None], np.concatenate([gs, us])[None],
                np.array([g13], np.float32), dq[None], ds[None], np.array([g2], np.float32))
    ref = O.ReferenceCpuTier(L, threads=4)
    outs = {}
    for M in (1, 3, 16):
        x = O.f32_to_bf16_bits(rng.standard_normal((M, K), dtype=np.float32) * np.float32(0.5))
        out = np.zeros((M, K), np.float32)
        rc = ref.lib.sb_cpu_expert_forward(ref.h, 0, 0, x.ctypes.data, out.ctypes.data, M)
        assert rc == 0
        outs[f"x{M}"] = x
        outs[f"y{M}"] = out
    ref.close()

    def vdq(q, sf, g):
        return dequantize_to_dtype(torch.from_numpy(q), torch.from_numpy(sf).view(torch.float8_e4m3fn),
                                   torch.tensor(g, dtype=torch.float32), torch.float32,
                                   block_size=16, swizzle=False).numpy()

    np.savez_compressed(HERE / "expert_planes.npz", w13=L.w13, s13=L.s13, w2=L.w2, s2=L.s2,
                        g13=L.g13, g2=L.g2, dq_gate=vdq(gq, gs, g13), dq_up=vdq(uq, us, g13),
                        dq_down=vdq(dq, ds, g2), **outs)


def quant() -> None:
    import torch
    from vllm.model_executor.layers.quantization.utils.nvfp4_emulation_utils import (
        ref_nvfp4_quant,
    )

    rng = np.random.default_rng(7)
    x = O.bf16_bits_to_f32(O.f32_to_bf16_bits(
        rng.standard_normal((128, 512), dtype=np.float32) * np.float32(0.02)))
    # a few blocks that exercise ties, zeros and the clamp
    x[0, :16] = 0.0
    x[1, :16] = np.linspace(-1, 1, 16, dtype=np.float32) * np.float32(0.05)
    amax = np.float32(np.abs(x).max())
    G = np.float32(np.float32(2688.0) / amax)
    vals, scales = ref_nvfp4_quant(torch.from_numpy(x), torch.tensor([G]), 16)
    np.savez_compressed(HERE / "quant.npz", x=x, G=np.array([G], np.float32),
                        vals=vals.numpy(), scales=scales.numpy())


def w4a4() -> None:
    """A W4A4 routed-expert layer computed with vLLM's own NVFP4 linear
    emulation (run_nvfp4_emulations: the activations quantised and
    dequantised by ref_nvfp4_quant with the given global, the weights by
    dequantize_to_dtype, an fp32 matmul), SwiGLU in fp32 and the routes summed
    with their weights: the static per-expert a1/a2_gscale convention and the
    dynamic per-row one (global 448 * 6 / max|row|)."""
    import torch
    from vllm.model_executor.layers.quantization.utils.nvfp4_emulation_utils import (
        run_nvfp4_emulations,
    )

    E, K, I, T, top_k = 8, 512, 256, 12, 3
    L = O.make_layer(E, K, I, seed=41)
    hidden = O.make_hidden(T, K, seed=42)
    ids, w = O.route_logits(T, E, top_k, seed=43)
    ids[2, 1] = -1
    x = O.bf16_bits_to_f32(hidden)
    amax = np.float32(np.abs(x).max())
    a13 = np.full(E, np.float32(2688.0) / amax, np.float32)
    a2 = np.full(E, np.float32(2688.0) / (amax / np.float32(8.0)), np.float32)

    def emu(rows, G, q, sf, g):
        return run_nvfp4_emulations(
            torch.from_numpy(rows), torch.tensor([G], dtype=torch.float32),
            torch.from_numpy(q), torch.from_numpy(sf).view(torch.float8_e4m3fn),
            torch.tensor(g, dtype=torch.float32), swizzle=False).numpy()

    def dyn(row):
        m = np.float32(np.abs(row).max())
        return np.float32(2688.0) / m if m > 0 else np.float32(1.0)

    outs = {}
    for mode in ("static", "dynamic"):
        out = np.zeros((T, K), np.float32)
        for t in range(T):
            for k in range(top_k):
                e = int(ids[t, k])
                if e < 0 or e >= E:
                    continue
                xr = x[t:t + 1]
                G1 = a13[e] if mode == "static" else dyn(xr)
                gu = emu(xr, G1, L.w13[e], L.s13[e], L.g13[e])
                g, u = gu[:, :I], gu[:, I:]
                h = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
                G2 = a2[e] if mode == "static" else dyn(h)
                y = emu(h, G2, L.w2[e], L.s2[e], L.g2[e])
                out[t] += np.float32(w[t, k]) * y[0]
        outs[mode] = out
    np.savez_compressed(HERE / "w4a4.npz", out_static=outs["static"], out_dynamic=outs["dynamic"],
                        ids=ids, weights=w, a13=a13, a2=a2,
                        digest=digest(hidden, ids, w) + layer_digest(L))


if __name__ == "__main__":
    O.build(ref=True)
    if not O.reference_available():
        raise SystemExit("the reference CPU tier is not built; run where the reference tree exists")
    kat("moe")
    kat("blocks")
    c0()
    expert_planes()
    quant()
    w4a4()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)
