"""SBEXP001 expert banks: the reference's on-disk NVFP4 format
(``src/phase1/extract_experts.py:51-128, 234-281``; read by
``src/phase1/b70_provider.cpp:866-934`` and ``src/phase4/src/
shooting_brake_vllm/expert_bank.py:54-120``) loaded straight into the device
layout of :func:`shooting_brake_b200.nvfp4_moe`.

The file is mapped read-only by the library; a layer load reads only the
experts asked for, so an expert-parallel rank loads just its shard.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import torch

from . import Sbb200Error, _check, last_error, lib


class ExpertBank:
    def __init__(self, path: str | Path):
        self.h = lib().sbb200_bank_open(str(path).encode())
        if not self.h:
            raise Sbb200Error(-1, last_error())
        vals = [ctypes.c_size_t(0) for _ in range(4)]
        _check(lib().sbb200_bank_info(self.h, *(ctypes.addressof(v) for v in vals)))
        self.layers, self.experts, self.hidden, self.intermediate = (int(v.value) for v in vals)

    def read_expert(self, layer: int, expert: int) -> dict:
        """One expert's host planes (numpy uint8 / float32)."""
        H, I = self.hidden, self.intermediate
        w13 = np.empty((2 * I, H // 2), np.uint8)
        s13 = np.empty((2 * I, H // 16), np.uint8)
        w2 = np.empty((H, I // 2), np.uint8)
        s2 = np.empty((H, I // 16), np.uint8)
        g = np.zeros(2, np.float32)
        _check(lib().sbb200_bank_read_expert(
            self.h, layer, expert, w13.ctypes.data, s13.ctypes.data, g.ctypes.data,
            w2.ctypes.data, s2.ctypes.data, g.ctypes.data + 4))
        return {"w13": w13, "s13": s13, "g13": g[0], "w2": w2, "s2": s2, "g2": g[1]}

    def load_layer(self, layer: int, device: torch.device | str = "cuda",
                   experts: tuple[int, int] | None = None) -> tuple:
        """(w13, w13_scales, w13_global_scales, w2, w2_scales, w2_global_scales)
        device tensors of experts [begin, begin + count) (all by default)."""
        begin, count = experts if experts is not None else (0, self.experts)
        H, I = self.hidden, self.intermediate
        dev = torch.device(device)
        w13 = torch.empty((count, 2 * I, H // 2), dtype=torch.uint8, device=dev)
        s13 = torch.empty((count, 2 * I, H // 16), dtype=torch.uint8, device=dev)
        g13 = torch.empty(count, dtype=torch.float32, device=dev)
        w2 = torch.empty((count, H, I // 2), dtype=torch.uint8, device=dev)
        s2 = torch.empty((count, H, I // 16), dtype=torch.uint8, device=dev)
        g2 = torch.empty(count, dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        _check(lib().sbb200_bank_load(self.h, stream, layer, begin, count, w13.data_ptr(),
                                      s13.data_ptr(), g13.data_ptr(), w2.data_ptr(),
                                      s2.data_ptr(), g2.data_ptr()))
        return w13, s13, g13, w2, s2, g2

    def close(self) -> None:
        if self.h:
            lib().sbb200_bank_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
