"""Child-process bodies for the expert-parallel tests (started with the
``spawn`` method; one process per rank, 127.0.0.1 rendezvous, gloo process
group with a short timeout). Not collected by pytest."""

from __future__ import annotations

import datetime
import os
import sys
import traceback
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _init(rank: int, world: int, store_path: str):
    """gloo process group through a file store at store_path (a fresh path
    per test): no TCP port to race another process for."""
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"file://{store_path}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    return dist


def handles_worker(rank: int, world: int, store: str, q):
    """exchange_handles over gloo: every rank gets all handles in rank order
    (host logic only; the CUDA library is not loaded)."""
    try:
        dist = _init(rank, world, store)
        import importlib
        import __graft_entry__ as g
        ep_mod = importlib.import_module(g.load_package().__name__ + ".ep")
        got = ep_mod.exchange_handles(bytes([rank + 1]) * ep_mod.HANDLE_BYTES)
        q.put((rank, got))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, traceback.format_exc()))


def ep_forward_worker(rank: int, world: int, store: str, shape: tuple, steps: list, w4a4: bool, q):
    """Expert-parallel forward on GPU `rank` vs the oracle, several steps."""
    try:
        dist = _init(rank, world, store)
        import numpy as np
        import torch
        import __graft_entry__ as g
        from oracle import nvfp4 as O
        from conftest import cosine, rel_err

        torch.cuda.set_device(rank)
        sbb = g.load_package()
        import importlib
        ep_mod = importlib.import_module(sbb.__name__ + ".ep")
        E, K, I, top_k, max_tokens = shape
        L = O.make_layer(E, K, I, seed=500)
        ep = ep_mod.ExpertParallel(rank=rank, world=world, device=rank, max_tokens=max_tokens,
                                   top_k=top_k, E=E, K=K, I=I, w4a4=w4a4)
        dev = torch.device("cuda", rank)
        b, c = ep.expert_begin, ep.expert_count
        ws = [torch.from_numpy(np.ascontiguousarray(x[b:b + c])).to(dev)
              for x in (L.w13, L.s13, L.g13, L.w2, L.s2, L.g2)]
        # every step first, back to back like a serving engine's layers; the
        # oracle runs afterwards, so host work between steps cannot hold one
        # rank past another's bounded waits
        runs = []
        for i, counts in enumerate(steps):
            T = counts[rank]
            seed = 1000 * i + 10 * rank
            hidden = O.make_hidden(max(T, 1), K, seed=seed)[:T]
            ids, w = O.route_logits(max(T, 1), E, top_k, seed=seed + 1)
            ids, w = ids[:T], w[:T]
            if T > 2:
                ids[1, 0] = -1          # a dropped route
                ids[2, :] = ids[2, 0]   # one expert repeated
            h = torch.from_numpy(np.ascontiguousarray(hidden)).to(dev).view(torch.bfloat16)
            out = ep.forward(h, torch.from_numpy(ids).to(dev), torch.from_numpy(w).to(dev), *ws,
                             out_dtype=torch.float32)
            runs.append((T, hidden, ids, w, out))
        torch.cuda.synchronize()
        results = []
        for T, hidden, ids, w, out in runs:
            got = out.cpu().numpy()
            if T:
                want = (O.moe_forward_w4a4(hidden, ids, w, L) if w4a4
                        else O.moe_forward(hidden, ids, w, L))
                results.append((T, rel_err(got, want), cosine(got, want)))
            else:
                results.append((0, 0.0, 1.0))
        errs = ep.device_errors()
        ep.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, {"results": results, "errors": errs}))
    except Exception:
        q.put((rank, traceback.format_exc()))


def ep_skip_worker(rank: int, world: int, store: str, q):
    """One step together, then rank 1 skips a step: rank 0's waits for it
    must give up after their deadline, raise the error bit and return; the
    context stays usable (a host synchronise and a device read follow).
    Rank 1 stays in the group (its memory stays mapped) until rank 0 is done."""
    try:
        dist = _init(rank, world, store)
        import time
        import numpy as np
        import torch
        import __graft_entry__ as g
        from oracle import nvfp4 as O

        torch.cuda.set_device(rank)
        sbb = g.load_package()
        import importlib
        ep_mod = importlib.import_module(sbb.__name__ + ".ep")
        E, K, I, top_k, T = 8, 512, 256, 4, 8
        L = O.make_layer(E, K, I, seed=77)
        ep = ep_mod.ExpertParallel(rank=rank, world=world, device=rank, max_tokens=T,
                                   top_k=top_k, E=E, K=K, I=I)
        dev = torch.device("cuda", rank)
        b, c = ep.expert_begin, ep.expert_count
        ws = [torch.from_numpy(np.ascontiguousarray(x[b:b + c])).to(dev)
              for x in (L.w13, L.s13, L.g13, L.w2, L.s2, L.g2)]
        hidden = torch.from_numpy(O.make_hidden(T, K, seed=rank)).to(dev).view(torch.bfloat16)
        ids, w = O.route_logits(T, E, top_k, seed=10 + rank)
        ids, w = torch.from_numpy(ids).to(dev), torch.from_numpy(w).to(dev)
        ep.forward(hidden, ids, w, *ws)
        torch.cuda.synchronize()
        first = ep.device_errors()
        dist.barrier()
        result = {"first": first}
        if rank == 0:
            t0 = time.time()
            ep.forward(hidden, ids, w, *ws)  # rank 1 does not take part
            torch.cuda.synchronize()
            result["seconds"] = time.time() - t0
            result["errors"] = ep.device_errors()
            result["after"] = float(torch.ones(4, device=dev).sum().item())  # context alive
        dist.barrier()  # rank 1 leaves only after rank 0's step has ended
        ep.close()
        dist.destroy_process_group()
        q.put((rank, result))
    except Exception:
        q.put((rank, traceback.format_exc()))
