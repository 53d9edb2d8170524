"""Device-side failure reporting of the tcgen05 GEMMs, without a GPU fault.

Every pipeline wait inside the grouped GEMM kernels is bounded. Here the
bound is set to 1 ns from the host (sbb200_set_kernel_wait_ns), so waits that
are not already satisfied give up at once: the kernel raises its error bit,
drains its own TMA loads and tensor-core work, frees tensor memory and
returns. The test checks that the bit reaches the host through both the
per-call word (sbb200_nvfp4_moe_device_errors), the library-wide sticky word
(sbb200_device_errors) and the provider's health, and that the CUDA context
stays usable: the next call with the default bound is right."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cosine, rel_err
from gpu_util import dev

pytestmark = pytest.mark.gpu


def _inputs(oracle, cuda):
    # the block-scaled (tcgen05) path, with units long enough that the
    # epilogue's first wait for an accumulator cannot succeed at once
    E, K, I, T, top_k = 16, 4096, 1280, 64, 2
    L = oracle.make_layer(E, K, I, seed=81)
    hidden = oracle.make_hidden(T, K, seed=82)
    ids, w = oracle.route_logits(T, E, top_k, seed=83)
    tensors = [torch.from_numpy(np.ascontiguousarray(x)).to(cuda)
               for x in (L.w13, L.s13, L.g13, L.w2, L.s2, L.g2)]
    return L, hidden, ids, w, tensors


def test_wait_limit_raises_error_bit_and_context_survives(sbb, oracle, cuda):
    L, hidden, ids, w, tensors = _inputs(oracle, cuda)
    h, di, dw = dev(hidden, cuda, torch.bfloat16), dev(ids, cuda), dev(w, cuda)
    sbb.device_errors(cuda)  # start from a clear sticky word
    prev = sbb.set_kernel_wait_ns(1)
    try:
        sbb.nvfp4_moe(h, di, dw, *tensors)
        torch.cuda.synchronize()
        assert sbb.nvfp4_moe_device_errors(cuda) & 1
    finally:
        sbb.set_kernel_wait_ns(prev)
    assert sbb.device_errors(cuda) & 1
    assert sbb.device_errors(cuda) == 0  # read clears it
    # the context is intact: the next call, with the default bound, is right
    out = sbb.nvfp4_moe(h, di, dw, *tensors)
    torch.cuda.synchronize()
    assert sbb.nvfp4_moe_device_errors(cuda) == 0
    assert sbb.device_errors(cuda) == 0
    got = out.cpu().numpy()
    want = oracle.moe_forward(hidden, ids, w, L)
    assert rel_err(got, want) <= 1e-2 and cosine(got, want) >= 0.9999


def test_provider_health_reports_device_errors(sbb, oracle, cuda):
    L, hidden, ids, w, tensors = _inputs(oracle, cuda)
    T, top_k = ids.shape
    p = sbb.Provider(0, T, top_k, L.E, L.K, L.I)
    try:
        p.register_layer(0, *tensors)
        h, di, dw = dev(hidden, cuda, torch.bfloat16), dev(ids, cuda), dev(w, cuda)
        prev = sbb.set_kernel_wait_ns(1)
        try:
            p.forward(0, h, di, dw)
            torch.cuda.synchronize()
        finally:
            sbb.set_kernel_wait_ns(prev)
        health, _ = p.health()
        assert health["device_errors"] & 1
        p.forward(0, h, di, dw)
        health, _ = p.health()
        assert health["device_errors"] == 0 and health["dispatches"] == 2
    finally:
        p.close()
        sbb.device_errors(cuda)
