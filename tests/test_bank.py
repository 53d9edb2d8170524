"""SBEXP001 expert banks: the library's reader against a bank written and
read back by the reference's own code (tests/golden/make_bank.py), its
validation of damaged files, and a device load feeding the forward."""

from __future__ import annotations

import importlib
import shutil
import struct

import numpy as np
import pytest

from conftest import GOLDEN, cosine, rel_err

BANK = GOLDEN / "bank_small.bin"
LAYERS, EXPERTS, HIDDEN, INTER = 2, 4, 256, 128


@pytest.fixture(scope="module")
def bankmod(sbb):
    return importlib.import_module(sbb.__name__ + ".bank")


@pytest.fixture(scope="module")
def expect():
    return np.load(GOLDEN / "bank_small_expect.npz")


def test_header_and_records_match_reference_reader(bankmod, expect, oracle):
    with bankmod.ExpertBank(BANK) as b:
        assert (b.layers, b.experts, b.hidden, b.intermediate) == (LAYERS, EXPERTS, HIDDEN, INTER)
        for layer in range(LAYERS):
            L = oracle.make_layer(EXPERTS, HIDDEN, INTER, seed=900 + layer)
            for e in range(EXPERTS):
                r = b.read_expert(layer, e)
                for k in ("w13", "s13", "w2", "s2"):
                    assert np.array_equal(r[k], expect[f"{k}_{layer}_{e}"]), (layer, e, k)
                assert np.array_equal(np.array([r["g13"], r["g2"]], np.float32),
                                      expect[f"g_{layer}_{e}"])
                # and the planes are the seeded layer the fixture was made from
                assert np.array_equal(r["w13"], L.w13[e]) and np.array_equal(r["s2"], L.s2[e])


def _damaged(tmp_path, edit) -> str:
    p = tmp_path / "bank.bin"
    shutil.copy(BANK, p)
    raw = bytearray(p.read_bytes())
    raw = edit(raw)
    p.write_bytes(bytes(raw))
    return str(p)


@pytest.mark.parametrize("what,edit,msg", [
    ("magic", lambda r: b"SBINT401" + r[8:], "magic 'SBINT401' is unsupported"),
    ("reserved", lambda r: r[:24] + struct.pack("<I", 1) + r[28:], "reserved"),
    ("geometry", lambda r: r[:20] + struct.pack("<I", 250) + r[24:], "inconsistent or unsupported geometry"),
    ("truncated", lambda r: r[:-7], "size does not match"),
    ("short", lambda r: r[:40], "large enough to hold a header"),
])
def test_damaged_banks_are_rejected(sbb, bankmod, tmp_path, what, edit, msg):
    path = _damaged(tmp_path, edit)
    with pytest.raises(sbb.Sbb200Error) as ei:
        bankmod.ExpertBank(path)
    assert msg in str(ei.value), str(ei.value)


def test_out_of_range_reads_are_rejected(sbb, bankmod):
    with bankmod.ExpertBank(BANK) as b:
        with pytest.raises(sbb.Sbb200Error):
            b.read_expert(LAYERS, 0)
        with pytest.raises(sbb.Sbb200Error):
            b.read_expert(0, EXPERTS)


@pytest.mark.gpu
def test_device_load_shard_and_forward(sbb, bankmod, oracle, expect, cuda):
    import torch
    from gpu_util import dev
    with bankmod.ExpertBank(BANK) as b:
        full = b.load_layer(1, cuda)
        shard = b.load_layer(1, cuda, experts=(1, 2))
    torch.cuda.synchronize()
    for e in range(EXPERTS):
        assert np.array_equal(full[0][e].cpu().numpy(), expect[f"w13_1_{e}"])
        assert np.array_equal(full[4][e].cpu().numpy(), expect[f"s2_1_{e}"])
        assert full[2][e].item() == expect[f"g_1_{e}"][0] and full[5][e].item() == expect[f"g_1_{e}"][1]
    for i in range(2):
        for t_full, t_shard in zip(full, shard):
            assert torch.equal(t_full[1 + i], t_shard[i])
    # the loaded layer through the forward
    L = oracle.make_layer(EXPERTS, HIDDEN, INTER, seed=901)
    L.g13 = np.array([expect[f"g_1_{e}"][0] for e in range(EXPERTS)], np.float32)
    L.g2 = np.array([expect[f"g_1_{e}"][1] for e in range(EXPERTS)], np.float32)
    T, k = 16, 2
    hidden = oracle.make_hidden(T, HIDDEN, seed=5)
    ids, w = oracle.route_logits(T, EXPERTS, k, seed=6)
    got = sbb.nvfp4_moe(dev(hidden, cuda, torch.bfloat16), dev(ids, cuda), dev(w, cuda), *full)
    torch.cuda.synchronize()
    want = oracle.moe_forward(hidden, ids, w, L)
    got = got.cpu().numpy()
    assert rel_err(got, want) <= 1e-2 and cosine(got, want) >= 0.9999
