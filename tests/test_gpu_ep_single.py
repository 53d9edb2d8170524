"""The expert-parallel step with one rank: every kernel of the exchange
(publish or in-split exchange, gather, pulled rows, pushed route rows, final
sum in k order) runs against this GPU's own buffer, so the expert-parallel
kernels are checked on any single B200, not only when several are free.
Bar: normwise relative error <= 1e-2 and cosine >= 0.9999 against the CPU
oracle; with a full batch the step's output must also equal the single-GPU
op's (same tiles, and the final sum adds the routes in the combine's
order)."""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from conftest import cosine, rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [
    (16, 1024, 512, 8, 24),    # 192 virtual routes: exchange inside the activation split
    (16, 1024, 512, 8, 256),   # 2,048 routes: publish/gather path, K-layout tiles
])
def test_single_rank_step_matches_oracle_and_op(sbb, oracle, cuda, shape):
    E, K, I, top_k, T = shape
    ep_mod = importlib.import_module(sbb.__name__ + ".ep")
    L = oracle.make_layer(E, K, I, seed=300 + T)
    ep = ep_mod.ExpertParallel(rank=0, world=1, device=cuda.index or 0, max_tokens=T,
                               top_k=top_k, E=E, K=K, I=I)
    try:
        ws = [torch.from_numpy(np.ascontiguousarray(x)).to(cuda)
              for x in (L.w13, L.s13, L.g13, L.w2, L.s2, L.g2)]
        for step, n in enumerate((T, T // 3, T)):  # buffers reused across steps
            hidden = oracle.make_hidden(n, K, seed=10 * step + T)
            ids, w = oracle.route_logits(n, E, top_k, seed=10 * step + T + 1)
            ids[0, 1] = -1
            h = torch.from_numpy(hidden).to(cuda).view(torch.bfloat16)
            di, dw = torch.from_numpy(ids).to(cuda), torch.from_numpy(w).to(cuda)
            got = ep.forward(h, di, dw, *ws, out_dtype=torch.float32)
            op = sbb._nvfp4_moe_impl(h, di, dw, *ws, True, torch.float32)
            torch.cuda.synchronize()
            assert ep.device_errors() == 0
            got = got.cpu().numpy()
            want = oracle.moe_forward(hidden, ids, w, L)
            assert rel_err(got, want) <= 1e-2, (step, rel_err(got, want))
            assert cosine(got, want) >= 0.9999, (step, cosine(got, want))
            if n == T:  # same routes per expert as the op's call: the same tiles
                assert np.array_equal(got, op.cpu().numpy()), step
    finally:
        ep.close()
