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
