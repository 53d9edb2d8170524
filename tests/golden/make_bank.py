"""Generate tests/golden/bank_small.bin (an SBEXP001 expert bank) and
bank_small_expect.npz with the REFERENCE's own bank writer and reader.

Run where the reference tree exists (found like the oracle's build finds it:
the SBB200_REFERENCE_DIR environment variable, else a directory named
``reference`` beside this repository):

    python tests/golden/make_bank.py

The planes come from this repository's seeded generator
(oracle.nvfp4.make_layer, 2 layers x 4 experts, hidden 256, intermediate 128);
the file itself is written by the reference's BankShape.header() and
write_layer() (src/phase1/extract_experts.py:99-104, 234-281), and the
expected planes are read back with the reference's ExpertBank reader
(src/phase4/src/shooting_brake_vllm/expert_bank.py:54-122), so the fixture
pins the library's reader to the reference's format on both sides.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import nvfp4 as O  # noqa: E402

LAYERS, EXPERTS, HIDDEN, INTER = 2, 4, 256, 128


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    ref = O.reference_dir()
    if ref is None:
        raise SystemExit("reference tree not found: set SBB200_REFERENCE_DIR")
    writer = _load(ref / "src/phase1/extract_experts.py", "sb_ref_extract_experts")
    pkg = ref / "src/phase4/src"
    sys.path.insert(0, str(pkg))
    reader = importlib.import_module("shooting_brake_vllm.expert_bank")

    shape = writer.BankShape(HIDDEN, INTER, EXPERTS, list(range(LAYERS)), "model")
    out_path = HERE / "bank_small.bin"
    with out_path.open("wb") as out:
        out.write(shape.header())
        for layer in range(LAYERS):
            L = O.make_layer(EXPERTS, HIDDEN, INTER, seed=900 + layer)
            tensors = {}
            for e in range(EXPERTS):
                p = f"model.layers.{layer}.mlp.experts.{e}"
                tensors[f"{p}.gate_proj.weight_packed"] = torch.from_numpy(L.w13[e][:INTER].copy())
                tensors[f"{p}.up_proj.weight_packed"] = torch.from_numpy(L.w13[e][INTER:].copy())
                tensors[f"{p}.gate_proj.weight_scale"] = torch.from_numpy(L.s13[e][:INTER].copy())
                tensors[f"{p}.up_proj.weight_scale"] = torch.from_numpy(L.s13[e][INTER:].copy())
                tensors[f"{p}.down_proj.weight_packed"] = torch.from_numpy(L.w2[e].copy())
                tensors[f"{p}.down_proj.weight_scale"] = torch.from_numpy(L.s2[e].copy())
                # the checkpoint stores the quantisation global, 1 / dequant multiplier
                q13 = torch.tensor(np.float32(1.0) / L.g13[e], dtype=torch.float32)
                tensors[f"{p}.gate_proj.weight_global_scale"] = q13
                tensors[f"{p}.up_proj.weight_global_scale"] = q13.clone()
                tensors[f"{p}.down_proj.weight_global_scale"] = torch.tensor(
                    np.float32(1.0) / L.g2[e], dtype=torch.float32)
            writer.write_layer(out, layer, shape, tensors)

    bank = reader.ExpertBank(out_path)
    expect = {}
    for layer in range(LAYERS):
        for e in range(EXPERTS):
            pl = bank.expert(layer, e)
            expect[f"w13_{layer}_{e}"] = np.concatenate([pl.gate, pl.up], axis=0)
            expect[f"s13_{layer}_{e}"] = np.concatenate([pl.gate_sf, pl.up_sf], axis=0).view(np.uint8)
            expect[f"w2_{layer}_{e}"] = np.asarray(pl.down)
            expect[f"s2_{layer}_{e}"] = np.asarray(pl.down_sf).view(np.uint8)
            expect[f"g_{layer}_{e}"] = np.array([pl.w13_inv_global, pl.w2_inv_global], np.float32)
    bank.close()
    np.savez_compressed(HERE / "bank_small_expect.npz", **expect)
    print("wrote", out_path, out_path.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
