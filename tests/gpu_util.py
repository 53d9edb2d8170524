"""Helpers shared by the GPU parity tests."""

from __future__ import annotations

import numpy as np
import torch


def dev(a: np.ndarray, device, dtype: torch.dtype | None = None) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return t.view(dtype) if dtype is not None else t


def layer_to(L, device) -> tuple:
    return tuple(dev(x, device) for x in (L.w13, L.s13, L.g13, L.w2, L.s2, L.g2))


def run_moe(sbb, hidden_bits, ids, w, L, device, act=torch.bfloat16, out_dtype=torch.float32,
            multiply_router_weight=True):
    h = dev(hidden_bits, device, torch.bfloat16).to(act)
    out = sbb.nvfp4_moe(h, dev(ids, device), dev(w, device), *layer_to(L, device),
                        multiply_router_weight=multiply_router_weight, out_dtype=out_dtype)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


def random_layer(E, K, I, seed, device):
    """Random NVFP4 expert planes generated on the device: all 16 e2m1 codes,
    e4m3 scale exponents 4..10 as in the reference's fixtures
    (src/phase7/nvfp4_testutil.py:33-51), globals in [0.001, 0.003)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def plane(rows, cols):
        q = torch.randint(0, 256, (E, rows, cols // 2), generator=g, device=device,
                          dtype=torch.int32).to(torch.uint8)
        ex = torch.randint(4, 11, (E, rows, cols // 16), generator=g, device=device,
                           dtype=torch.int32)
        man = torch.randint(0, 8, (E, rows, cols // 16), generator=g, device=device,
                            dtype=torch.int32)
        return q, ((ex << 3) | man).to(torch.uint8)

    w13, s13 = plane(2 * I, K)
    w2, s2 = plane(K, I)
    g13 = (torch.rand(E, generator=g, device=device) * 0.002 + 0.001).float()
    g2 = (torch.rand(E, generator=g, device=device) * 0.002 + 0.001).float()
    return w13, s13, g13, w2, s2, g2


def host_layer(oracle, t, E, K, I):
    """The oracle's Layer of device tensors from random_layer."""
    w13, s13, g13, w2, s2, g2 = (x.cpu().numpy() for x in t)
    return oracle.Layer(E, K, I, w13, s13, g13, w2, s2, g2)
