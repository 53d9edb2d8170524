"""The tcgen05 path at the benchmark shapes (E=170, d=4096, I=1280, top-8),
checked against the CPU oracle on sampled tokens: a token's output depends
only on its own routes, so a sample checks a full-size batch exactly.

Weights here are random NVFP4 bytes generated on the device (all 16 e2m1
codes, e4m3 scale exponents 4..10 as in the reference's fixtures,
src/phase7/nvfp4_testutil.py:33-51). Tolerance: max relative error <= 1e-2
(max|got-want| / max|want|) and cosine >= 0.9999."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cosine, rel_err
from gpu_util import dev, host_layer, random_layer

pytestmark = pytest.mark.gpu

REL_TOL = 1e-2
COS_TOL = 0.9999


def run_and_check(sbb, oracle, cuda, E, K, I, ids, w, hidden_bits, tensors, sample=48, seed=0,
                  act=torch.bfloat16):
    T = ids.shape[0]
    h = dev(hidden_bits, cuda, torch.bfloat16).to(act)
    out = sbb.nvfp4_moe(h, dev(ids, cuda), dev(w, cuda), *tensors)
    torch.cuda.synchronize()
    assert sbb.nvfp4_moe_device_errors(cuda) == 0
    got = out.cpu().numpy()
    rng = np.random.default_rng(seed)
    toks = np.sort(rng.choice(T, size=min(sample, T), replace=False)).astype(np.int32)
    L = host_layer(oracle, tensors, E, K, I)
    want = oracle.moe_forward(hidden_bits, ids, w, L, tokens=toks)
    assert rel_err(got[toks], want) <= REL_TOL, rel_err(got[toks], want)
    assert cosine(got[toks], want) >= COS_TOL, cosine(got[toks], want)
    return got


@pytest.fixture(scope="module")
def big_layer(cuda):
    return random_layer(170, 4096, 1280, seed=5, device=cuda)


@pytest.mark.parametrize("T", [1, 2, 8, 64, 200])
def test_decode_shapes(sbb, oracle, cuda, big_layer, T):
    ids, w = oracle.route_logits(T, 170, 8, seed=T)
    hidden = oracle.make_hidden(T, 4096, seed=T + 1)
    run_and_check(sbb, oracle, cuda, 170, 4096, 1280, ids, w, hidden, big_layer, seed=T)


def test_prefill_chunk_8k(sbb, oracle, cuda, big_layer):
    T = 8192
    ids, w = oracle.route_logits(T, 170, 8, seed=9, bias_std=0.5)
    hidden = oracle.make_hidden(T, 4096, seed=10)
    run_and_check(sbb, oracle, cuda, 170, 4096, 1280, ids, w, hidden, big_layer, sample=24)


def test_skewed_zipf_routing(sbb, oracle, cuda, big_layer):
    T = 1024
    ids, w = oracle.route_zipf(T, 170, 8, seed=11)
    hidden = oracle.make_hidden(T, 4096, seed=12)
    run_and_check(sbb, oracle, cuda, 170, 4096, 1280, ids, w, hidden, big_layer, sample=32)


@pytest.mark.parametrize("T,E,top_k", [(40, 16, 2), (90, 8, 4), (300, 8, 8), (2000, 16, 4)])
def test_token_tile_widths(sbb, oracle, cuda, T, E, top_k):
    """Routes per expert from ~5 to ~500 select every token-tile width and
    experts that span several tiles."""
    K, I = 1024, 512
    tensors = random_layer(E, K, I, seed=T, device=cuda)
    ids, w = oracle.route_logits(T, E, top_k, seed=T + 3)
    ids[::7, 0] = -1
    hidden = oracle.make_hidden(T, K, seed=T + 4)
    run_and_check(sbb, oracle, cuda, E, K, I, ids, w, hidden, tensors, sample=40)


def test_single_hot_expert(sbb, oracle, cuda):
    K, I, E, T = 512, 256, 4, 700
    tensors = random_layer(E, K, I, seed=3, device=cuda)
    ids = np.full((T, 2), 2, np.int32)
    ids[:, 1] = -1
    ids[::3, 1] = 1
    w = np.full((T, 2), 0.5, np.float32)
    hidden = oracle.make_hidden(T, K, seed=4)
    run_and_check(sbb, oracle, cuda, E, K, I, ids, w, hidden, tensors, sample=60)


@pytest.mark.parametrize("scale", [1e-4, 1.0, 3000.0])
def test_activation_range(sbb, oracle, cuda, scale):
    """Activations far from unit scale: the 4-term split takes each row's
    global from the row's own maximum, so a uniform scale of the whole row
    changes nothing but that global."""
    K, I, E, T = 512, 256, 8, 33
    tensors = random_layer(E, K, I, seed=7, device=cuda)
    ids, w = oracle.route_logits(T, E, 3, seed=8)
    hidden = oracle.make_hidden(T, K, seed=9, scale=scale)
    run_and_check(sbb, oracle, cuda, E, K, I, ids, w, hidden, tensors, sample=T)


def test_f16_activations_tc(sbb, oracle, cuda):
    K, I, E, T = 1024, 512, 8, 50
    tensors = random_layer(E, K, I, seed=21, device=cuda)
    ids, w = oracle.route_logits(T, E, 4, seed=22)
    hidden = oracle.make_hidden(T, K, seed=23)
    run_and_check(sbb, oracle, cuda, E, K, I, ids, w, hidden, tensors, sample=T,
                  act=torch.float16)


def test_deterministic_repeat(sbb, oracle, cuda, big_layer):
    T = 64
    ids, w = oracle.route_logits(T, 170, 8, seed=31)
    hidden = dev(oracle.make_hidden(T, 4096, seed=32), cuda, torch.bfloat16)
    a = sbb.nvfp4_moe(hidden, dev(ids, cuda), dev(w, cuda), *big_layer)
    b = sbb.nvfp4_moe(hidden, dev(ids, cuda), dev(w, cuda), *big_layer)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def per_token_check(got, want):
    """The bar applied token by token: for every token t,
    max|got_t - want_t| / max|want_t| <= 1e-2 and cos(got_t, want_t) >= 0.9999.
    Returns the worst of each."""
    worst_rel, worst_cos = 0.0, 1.0
    for t in range(want.shape[0]):
        if not np.any(want[t]):
            assert not np.any(got[t])
            continue
        worst_rel = max(worst_rel, rel_err(got[t], want[t]))
        worst_cos = min(worst_cos, cosine(got[t], want[t]))
    assert worst_rel <= REL_TOL, worst_rel
    assert worst_cos >= COS_TOL, worst_cos
    return worst_rel, worst_cos


def _outlier_hidden(oracle, T, K, seed, kind):
    """bf16 bits of hidden rows with the dynamic range of real hidden states:
    'one1e3' one channel per row 10^3 x the rest; 'few1e4' four fixed
    channels 10^4 x; 'tiny_blocks' every 16-element block but the first at
    2^-14 (and some at 2^-20) of the row maximum."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, K)).astype(np.float32)
    if kind == "one1e3":
        ch = rng.integers(0, K, T)
        x[np.arange(T), ch] *= 1e3
    elif kind == "few1e4":
        for ch in (7, 300, 301, K - 5):
            x[:, ch] = np.sign(x[:, ch] + 1e-3) * (1e4 + 100 * rng.random(T))
    elif kind == "tiny_blocks":
        x[:, 16:] *= 2.0 ** -14
        x[:, 16 * 9:16 * 20] *= 2.0 ** -6  # these blocks end at 2^-20
    else:
        raise ValueError(kind)
    b = x.view(np.uint32)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even
    return b


@pytest.mark.parametrize("T", [48, 512])
@pytest.mark.parametrize("kind", ["one1e3", "few1e4", "tiny_blocks"])
def test_outlier_channels_per_token(sbb, oracle, cuda, kind, T):
    """W4A16 numerics of the 4-term activation split under outliers and
    blocks far below their row maximum, judged token by token rather than
    over the batch, at the decode shape's K and I. T = 48 runs four terms as
    interleaved N rows (decode tiles), T = 512 (128 routes per expert) three
    term planes along K under one global per row (prefill tiles), where a
    block 2^-14 below its row maximum keeps fewer terms; 48 sampled tokens
    are checked."""
    E, K, I, top_k = 16, 4096, 1280, 4
    tensors = random_layer(E, K, I, seed=71, device=cuda)
    ids, w = oracle.route_logits(T, E, top_k, seed=72)
    hidden = _outlier_hidden(oracle, T, K, seed=73, kind=kind)
    h = dev(hidden, cuda, torch.bfloat16)
    out = sbb.nvfp4_moe(h, dev(ids, cuda), dev(w, cuda), *tensors)
    torch.cuda.synchronize()
    assert sbb.nvfp4_moe_device_errors(cuda) == 0
    L = host_layer(oracle, tensors, E, K, I)
    toks = np.sort(np.random.default_rng(T).choice(T, size=min(48, T), replace=False))
    want = oracle.moe_forward(hidden, ids, w, L, tokens=toks.astype(np.int32))
    worst = per_token_check(out.cpu().numpy()[toks], want)
    print(f"{kind} T={T}: worst per-token rel {worst[0]:.3e}, cos {worst[1]:.7f}")
