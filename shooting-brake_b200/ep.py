"""Expert parallelism over NVLink for the routed-expert NVFP4 MoE.

One process per GPU of one node. The E routed experts of a layer are sharded
contiguously over the ranks (the first E % world ranks hold one extra expert,
``sbb200_ep_shard``); every rank keeps its own tokens and calls
:meth:`ExpertParallel.forward` once per step. Inside, the exchange is
device-resident (``include/sbb200.h``, ``csrc/ep.cu``): each destination reads
the rows routed to its experts straight from the source GPUs, runs its shard,
and stores each route's output row back into the source's buffer, which sums
its tokens' routes in ascending k with the router weights (the single-GPU
combine's order, so the result does not depend on the sharding). This replaces the reference's multi-card
split, where each card receives every route with foreign experts as -1 and
the host adds the per-card outputs (``src/phase4/src/shooting_brake_vllm/
routed_experts.py:354-382, 2460-2463, 2522-2524``).

``torch.distributed`` (any backend) is used once, to swap the CUDA IPC
handles of the exchange buffers; no collective runs on the data path.
"""

from __future__ import annotations

import ctypes

import torch

from . import DTYPE_CODE, Sbb200Error, _check, _check_cuda, _p, _stream, last_error, lib

HANDLE_BYTES = 64
STAGE_EVENTS = 8
STAGE_NAMES = ("publish", "gather+wait", "exchange+route_plan+split(pull)", "gate_up",
               "h_split+down(push)", "combine(none)", "final+wait")


def expert_shard(E: int, world: int, rank: int) -> tuple[int, int]:
    """(first expert, expert count) of ``rank``'s contiguous shard."""
    b, c = ctypes.c_size_t(0), ctypes.c_size_t(0)
    _check(lib().sbb200_ep_shard(E, world, rank, ctypes.addressof(b), ctypes.addressof(c)))
    return int(b.value), int(c.value)


def exchange_handles(handle: bytes, group=None) -> bytes:
    """All ranks' handles concatenated in rank order (one all_gather_object)."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return bytes(handle)  # a single process: its own handle is the whole table
    world = dist.get_world_size(group)
    got = [None] * world
    dist.all_gather_object(got, bytes(handle), group=group)
    for r, h in enumerate(got):
        if not isinstance(h, (bytes, bytearray)) or len(h) != HANDLE_BYTES:
            raise Sbb200Error(-1, f"rank {r} sent a malformed exchange handle")
    return b"".join(bytes(h) for h in got)


class ExpertParallel:
    """Exchange state of one rank; create it on every rank of ``group``
    (collectively: the constructor swaps handles)."""

    def __init__(self, *, rank: int, world: int, device: int, max_tokens: int, top_k: int,
                 E: int, K: int, I: int, act_dtype: torch.dtype = torch.bfloat16, group=None,
                 w4a4: bool = False):
        self.rank, self.world, self.E = rank, world, E
        self.max_tokens, self.top_k, self.K, self.I = max_tokens, top_k, K, I
        self.device = torch.device("cuda", device)
        self.act_dtype = act_dtype
        self.expert_begin, self.expert_count = expert_shard(E, world, rank)
        self.w4a4 = bool(w4a4)
        self.h = lib().sbb200_ep_create(device, rank, world, max_tokens, top_k, E, K, I,
                                        DTYPE_CODE[act_dtype], int(self.w4a4))
        if not self.h:
            raise Sbb200Error(-1, last_error())
        buf = ctypes.create_string_buffer(HANDLE_BYTES)
        _check(lib().sbb200_ep_ipc_handle(self.h, buf, HANDLE_BYTES))
        handles = exchange_handles(buf.raw, group)
        _check(lib().sbb200_ep_connect(self.h, handles, len(handles)))

    def local_experts(self, t: torch.Tensor) -> torch.Tensor:
        """This rank's slice of a tensor indexed by global expert id."""
        return t[self.expert_begin:self.expert_begin + self.expert_count]

    def forward(self, hidden: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                w13: torch.Tensor, w13_scales: torch.Tensor, w13_global_scales: torch.Tensor,
                w2: torch.Tensor, w2_scales: torch.Tensor, w2_global_scales: torch.Tensor,
                out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
                multiply_router_weight: bool = True,
                stage_events: list | None = None) -> torch.Tensor:
        """This rank's tokens through all E experts. The weights are this
        rank's shard (``local_experts`` of the full layer). ``stage_events``
        (STAGE_EVENTS recorded CUDA events, see STAGE_NAMES) times the step's
        phases."""
        for name, t in (("hidden", hidden), ("topk ids", topk_ids), ("router weights", topk_weights),
                        ("w13", w13), ("w13 scales", w13_scales),
                        ("w13 global scales", w13_global_scales), ("w2", w2),
                        ("w2 scales", w2_scales), ("w2 global scales", w2_global_scales)):
            _check_cuda(name, t)
        M = hidden.shape[0]
        if hidden.dtype != self.act_dtype or hidden.shape != (M, self.K):
            raise ValueError(f"sbb200 ep: hidden must be {self.act_dtype} [M,{self.K}]")
        if topk_ids.dtype != torch.int32 or topk_ids.shape != (M, self.top_k):
            raise ValueError(f"sbb200 ep: topk ids must be int32 [M,{self.top_k}]")
        if topk_weights.dtype != torch.float32 or topk_weights.shape != (M, self.top_k):
            raise ValueError(f"sbb200 ep: router weights must be float32 [M,{self.top_k}]")
        if w13.size(0) != self.expert_count or w2.size(0) != self.expert_count:
            raise ValueError(f"sbb200 ep: rank {self.rank} holds {self.expert_count} experts")
        if out is None:
            out = torch.empty((M, self.K), dtype=out_dtype, device=hidden.device)
        args = (self.h, _stream(hidden), _p(hidden), _p(topk_ids), _p(topk_weights), M, _p(w13),
                _p(w13_scales), _p(w13_global_scales), _p(w2), _p(w2_scales),
                _p(w2_global_scales), _p(out), DTYPE_CODE[out.dtype],
                int(bool(multiply_router_weight)))
        if stage_events is None:
            _check(lib().sbb200_ep_forward(*args))
        else:
            arr = (ctypes.c_void_p * STAGE_EVENTS)(*[ev.cuda_event for ev in stage_events])
            _check(lib().sbb200_ep_forward_staged(*args, arr, STAGE_EVENTS))
        return out

    def kernels_per_step(self) -> int:
        """Kernels one forward step launches on this rank (the library's own
        count: publish, gather, the shard's expert step, final sum)."""
        n = int(lib().sbb200_ep_launches(self.h))
        if n < 0:
            raise RuntimeError("expert-parallel handle is closed")
        return n

    def device_errors(self) -> int:
        """Error bits since the last read (bit 0: a wait for another rank
        timed out); synchronises the current stream."""
        v = ctypes.c_uint32(0)
        _check(lib().sbb200_ep_device_errors(self.h, torch.cuda.current_stream(self.device).cuda_stream,
                                             ctypes.addressof(v)))
        return int(v.value)

    def close(self) -> None:
        if self.h:
            lib().sbb200_ep_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
