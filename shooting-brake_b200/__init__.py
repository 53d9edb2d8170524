"""shooting_brake_b200 -- B200-native routed-expert NVFP4 MoE.

Python host side of the library. The compute lives in ``libsbb200.so``
(hand-written sm_100a CUDA kernels + a C++ host C-ABI, ``include/sbb200.h``);
this module reaches it through ctypes and exposes:

* :func:`nvfp4_moe` -- the operator of the reference's PyTorch extension
  (``src/QuixiCore-XPU/bindings/pytorch/tk_xpu_ext.sycl:296-410``): same
  arguments, same checks and messages, fp32 ``[M, K]`` output by default,
  registered as the custom op ``torch.ops.sbb200.nvfp4_moe``;
* building blocks used by the parity tests (:func:`route_plan`,
  :func:`nvfp4_dequant`, :func:`nvfp4_quantize`);
* :class:`Provider` -- registered layers with an owned workspace
  (the device-resident replacement of the B70 provider C-ABI);
* :mod:`.plugin` -- the vLLM ``RoutedExperts`` hook adapter;
* :mod:`.ep` -- expert parallelism over NVLink (one process per GPU);
* :mod:`.bank` -- the reference's SBEXP001 expert-bank files.

There is no CPU fallback: every entry point raises if the CUDA library is
missing or the tensors are not on a CUDA device.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

__all__ = [
    "Sbb200Error", "lib", "nvfp4_moe", "nvfp4_moe_workspace_bytes", "route_plan",
    "nvfp4_dequant", "nvfp4_quantize", "Provider", "DTYPE_CODE",
]

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libsbb200.so"

# sbb200_dtype (the reference's DType {f32, f16, bf16})
DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


class Sbb200Error(RuntimeError):
    """A C-ABI call returned an error status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"sbb200 error {status}: {message}")
        self.status = status


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded C-ABI library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with shooting-brake_b200/build.py "
                "(the CUDA path has no fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        P, S, I, F = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_float
        L.sbb200_abi_version.restype = S
        L.sbb200_abi_version.argtypes = []
        L.sbb200_last_error.restype = S
        L.sbb200_last_error.argtypes = [ctypes.c_char_p, S]
        L.sbb200_nvfp4_moe_workspace_bytes.restype = S
        L.sbb200_nvfp4_moe_workspace_bytes.argtypes = [S, S, S, S, S, I]
        L.sbb200_nvfp4_moe_launches.restype = I
        L.sbb200_nvfp4_moe_launches.argtypes = [S, S, S, S, S, I]
        L.sbb200_nvfp4_moe.restype = I
        L.sbb200_nvfp4_moe.argtypes = [P, P, P, P, P, P, P, P, P, P, P, S, P, I, S, S, S, S, S, I, I]
        L.sbb200_nvfp4_moe_staged.restype = I
        L.sbb200_nvfp4_moe_staged.argtypes = [P, P, P, P, P, P, P, P, P, P, P, S, P, I, S, S, S, S,
                                              S, I, I, P, S]
        L.sbb200_nvfp4_moe_bad_ids.restype = I
        L.sbb200_nvfp4_moe_bad_ids.argtypes = [P, P, P]
        L.sbb200_nvfp4_moe_device_errors.restype = I
        L.sbb200_nvfp4_moe_device_errors.argtypes = [P, P, P]
        L.sbb200_device_errors.restype = I
        L.sbb200_device_errors.argtypes = [P, P]
        L.sbb200_set_kernel_wait_ns.restype = ctypes.c_uint64
        L.sbb200_set_kernel_wait_ns.argtypes = [ctypes.c_uint64]
        L.sbb200_route_plan_scratch_bytes.restype = S
        L.sbb200_route_plan_scratch_bytes.argtypes = [S, S]
        L.sbb200_route_plan.restype = I
        L.sbb200_route_plan.argtypes = [P, P, S, S, S, P, P, P, P, P, P]
        L.sbb200_nvfp4_dequant.restype = I
        L.sbb200_nvfp4_dequant.argtypes = [P, P, P, P, S, P, S, S]
        L.sbb200_nvfp4_quantize.restype = I
        L.sbb200_nvfp4_quantize.argtypes = [P, P, I, P, S, P, P, S, S]
        L.sbb200_create.restype = P
        L.sbb200_create.argtypes = [I, S, S, S, S, S]
        L.sbb200_destroy.restype = None
        L.sbb200_destroy.argtypes = [P]
        L.sbb200_register_layer.restype = I
        L.sbb200_register_layer.argtypes = [P, S, S, P, P, P, P, P, P]
        L.sbb200_moe_forward.restype = I
        L.sbb200_moe_forward.argtypes = [P, S, P, P, I, P, P, P, I, S, I]
        L.sbb200_health.restype = I
        L.sbb200_health.argtypes = [P, P, ctypes.c_char_p, S]
        L.sbb200_nvfp4_moe_w4a4.restype = I
        L.sbb200_nvfp4_moe_w4a4.argtypes = [P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, S, P, I,
                                            S, S, S, S, S, I, I, P, S]
        L.sbb200_router_topk.restype = I
        L.sbb200_router_topk.argtypes = [P, P, I, S, S, S, P, P]
        L.sbb200_nvfp4_moe_from_logits.restype = I
        L.sbb200_nvfp4_moe_from_logits.argtypes = [P, P, P, I, P, P, P, P, P, P, P, P, P, S, P, I,
                                                   S, S, S, S, S, I, I]
        L.sbb200_bank_open.restype = P
        L.sbb200_bank_open.argtypes = [ctypes.c_char_p]
        L.sbb200_bank_info.restype = I
        L.sbb200_bank_info.argtypes = [P, P, P, P, P]
        L.sbb200_bank_read_expert.restype = I
        L.sbb200_bank_read_expert.argtypes = [P, S, S, P, P, P, P, P, P]
        L.sbb200_bank_load.restype = I
        L.sbb200_bank_load.argtypes = [P, P, S, S, S, P, P, P, P, P, P]
        L.sbb200_bank_close.restype = None
        L.sbb200_bank_close.argtypes = [P]
        L.sbb200_ep_shard.restype = I
        L.sbb200_ep_shard.argtypes = [S, I, I, P, P]
        L.sbb200_ep_create.restype = P
        L.sbb200_ep_create.argtypes = [I, I, I, S, S, S, S, S, I, I]
        L.sbb200_ep_ipc_handle.restype = I
        L.sbb200_ep_ipc_handle.argtypes = [P, P, S]
        L.sbb200_ep_connect.restype = I
        L.sbb200_ep_connect.argtypes = [P, P, S]
        L.sbb200_ep_forward.restype = I
        L.sbb200_ep_forward.argtypes = [P, P, P, P, P, S, P, P, P, P, P, P, P, I, I]
        L.sbb200_ep_forward_staged.restype = I
        L.sbb200_ep_forward_staged.argtypes = [P, P, P, P, P, S, P, P, P, P, P, P, P, I, I, P, S]
        L.sbb200_ep_device_errors.restype = I
        L.sbb200_ep_device_errors.argtypes = [P, P, P]
        L.sbb200_ep_launches.restype = I
        L.sbb200_ep_launches.argtypes = [P]
        L.sbb200_ep_destroy.restype = None
        L.sbb200_ep_destroy.argtypes = [P]
        _lib = L
    return _lib


def last_error() -> str:
    L = lib()
    n = L.sbb200_last_error(None, 0)
    buf = ctypes.create_string_buffer(n)
    L.sbb200_last_error(buf, n)
    return buf.value.decode(errors="replace")


def _check(rc: int) -> None:
    if rc != 0:
        raise Sbb200Error(rc, last_error())


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check_cuda(name: str, t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise ValueError(f"sbb200: {name} must be a CUDA tensor (there is no CPU path)")
    if not t.is_contiguous():
        raise ValueError(f"sbb200: {name} must be contiguous")


# --------------------------------------------------------------------------
# the operator
# --------------------------------------------------------------------------

def nvfp4_moe_workspace_bytes(M: int, E: int, top_k: int, K: int, I: int,
                              act_dtype: torch.dtype = torch.bfloat16) -> int:
    return int(lib().sbb200_nvfp4_moe_workspace_bytes(M, E, top_k, K, I, DTYPE_CODE[act_dtype]))


_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A per-(device, stream) workspace that only grows. Reused across calls on
    one stream, which is what keeps stream-ordered calls race-free."""
    key = (device.index or 0, torch.cuda.current_stream(device).cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("sbb200: graph-captured nvfp4_moe needs a workspace allocated "
                               "by an eager call of at least the same shape first")
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def _validate(hidden, topk_ids, topk_weights, w13, w13_scales, w13_global_scales, w2,
              w2_scales, w2_global_scales):
    """The shape and dtype checks of tk_xpu_ext.sycl:308-371, same messages."""
    for name, t in (("hidden", hidden), ("topk ids", topk_ids), ("router weights", topk_weights),
                    ("w13", w13), ("w13 scales", w13_scales),
                    ("w13 global scales", w13_global_scales), ("w2", w2),
                    ("w2 scales", w2_scales), ("w2 global scales", w2_global_scales)):
        _check_cuda(name, t)
        if t.device != hidden.device:
            raise ValueError(f"sbb200: {name} must be on the same device as hidden")

    def req(ok, msg):
        if not ok:
            raise ValueError("sbb200: " + msg)

    req(hidden.dim() == 2, "hidden must be [M,K]")
    req(hidden.dtype in DTYPE_CODE, "hidden must be float32, float16 or bfloat16")
    req(topk_ids.dim() == 2 and topk_ids.dtype == torch.int32, "topk ids must be int32 [M,top_k]")
    req(topk_weights.dtype == torch.float32 and topk_weights.shape == topk_ids.shape,
        "router weights must be float32 [M,top_k]")
    req(w13.dim() == 3 and w13.dtype == torch.uint8 and w13.size(1) % 2 == 0,
        "w13 must be byte [E,2I,K/2]")
    req(w2.dim() == 3 and w2.dtype == torch.uint8, "w2 must be byte [E,K,I/2]")
    req(w13_scales.dim() == 3 and w13_scales.element_size() == 1,
        "w13 scales must be byte [E,2I,K/16]")
    req(w2_scales.dim() == 3 and w2_scales.element_size() == 1, "w2 scales must be byte [E,K,I/16]")
    req(w13_global_scales.dtype == torch.float32 and w2_global_scales.dtype == torch.float32,
        "NVFP4 global scales must be float32")
    M, K = hidden.shape
    E = w13.size(0)
    top_k = topk_ids.size(1)
    I = w13.size(1) // 2
    req(M > 0 and E > 0 and top_k > 0 and I > 0, "NVFP4 MoE dimensions must be nonzero")
    req(topk_ids.size(0) == M, "topk ids must be int32 [M,top_k]")
    req(w13.size(2) == K // 2, "w13 must be byte [E,2I,K/2]")
    req(w2.size(0) == E and w2.size(1) == K and w2.size(2) == I // 2, "w2 must be byte [E,K,I/2]")
    req(w13_scales.size(0) == E and w13_scales.size(1) == 2 * I and w13_scales.size(2) == K // 16,
        "w13 scales must be byte [E,2I,K/16]")
    req(w2_scales.size(0) == E and w2_scales.size(1) == K and w2_scales.size(2) == I // 16,
        "w2 scales must be byte [E,K,I/16]")
    req(w13_global_scales.numel() == E and w2_global_scales.numel() == E,
        "NVFP4 global scales must contain E values")
    req(K % 32 == 0 and I % 32 == 0, "NVFP4 MoE K/I must be multiples of 32")
    return M, K, E, top_k, I


def _nvfp4_moe_impl(hidden: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                    w13: torch.Tensor, w13_scales: torch.Tensor, w13_global_scales: torch.Tensor,
                    w2: torch.Tensor, w2_scales: torch.Tensor, w2_global_scales: torch.Tensor,
                    multiply_router_weight: bool, out_dtype: torch.dtype,
                    out: torch.Tensor | None = None,
                    stage_events: list | None = None) -> torch.Tensor:
    M, K, E, top_k, I = _validate(hidden, topk_ids, topk_weights, w13, w13_scales,
                                  w13_global_scales, w2, w2_scales, w2_global_scales)
    if out is None:
        out = torch.empty((M, K), dtype=out_dtype, device=hidden.device)
    else:
        _check_cuda("out", out)
        if out.shape != (M, K) or out.dtype not in DTYPE_CODE:
            raise ValueError("sbb200: out must be [M,K] float32, float16 or bfloat16")
    nbytes = nvfp4_moe_workspace_bytes(M, E, top_k, K, I, hidden.dtype)
    ws = _workspace(hidden.device, nbytes)
    args = (_stream(hidden), _p(hidden), _p(topk_ids), _p(topk_weights), _p(w13), _p(w13_scales),
            _p(w13_global_scales), _p(w2), _p(w2_scales), _p(w2_global_scales), _p(ws),
            ws.numel(), _p(out), DTYPE_CODE[out.dtype], M, E, top_k, K, I,
            DTYPE_CODE[hidden.dtype], int(bool(multiply_router_weight)))
    if stage_events is None:
        rc = lib().sbb200_nvfp4_moe(*args)
    else:
        arr = (ctypes.c_void_p * STAGE_EVENTS)(*[ev.cuda_event for ev in stage_events])
        rc = lib().sbb200_nvfp4_moe_staged(*args, arr, STAGE_EVENTS)
    _check(rc)
    return out


def kernels_per_call(M: int, E: int, top_k: int, K: int, I: int,
                     act_dtype: torch.dtype = torch.bfloat16) -> int:
    """Kernels of this library one nvfp4_moe call of this shape launches (the
    driver's own count: route plan, activation split, gate/up, SwiGLU split,
    down, combine on the block-scaled path; up to 1,024 routes the split
    computes the route plan itself)."""
    return int(lib().sbb200_nvfp4_moe_launches(M, E, top_k, K, I, DTYPE_CODE[act_dtype]))


STAGE_EVENTS = 5
STAGE_NAMES = ("route_plan+x_split", "gate_up", "h_split+down", "combine")


def stage_events(stream: torch.cuda.Stream | None = None) -> list:
    """SBB200_STAGE_EVENTS timing events, created (recorded once) so their
    handles exist before being handed to the C-ABI."""
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(STAGE_EVENTS)]
    for ev in evs:
        ev.record(stream)
    return evs


_OUT_CODES = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}


def _check_split_scratch(split_scratch, split, topk_ids, w13):
    """The split-scratch check of tk_xpu_ext.sycl:378-388, same message."""
    if split and split_scratch is not None:
        _check_cuda("split scratch", split_scratch)
        M, top_k = topk_ids.shape
        I = w13.size(1) // 2
        if (split_scratch.dtype != torch.float32 or split_scratch.dim() != 2
                or split_scratch.size(0) != M * top_k or split_scratch.size(1) != 2 * I):
            raise ValueError("sbb200: split scratch must be float32 [M*top_k,2I]")


@torch.library.custom_op("sbb200::nvfp4_moe", mutates_args=())
def _nvfp4_moe_op(hidden: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                  w13: torch.Tensor, w13_scales: torch.Tensor, w13_global_scales: torch.Tensor,
                  w2: torch.Tensor, w2_scales: torch.Tensor, w2_global_scales: torch.Tensor,
                  split_scratch: torch.Tensor | None, split: bool,
                  multiply_router_weight: bool) -> torch.Tensor:
    """The reference extension's op, argument for argument and in the same
    order (tk_xpu_ext.sycl:296-302): fp32 [M, K] out. ``split`` and
    ``split_scratch`` pick a kernel shape on the reference's Arc cards; the
    B200 driver picks its kernels itself, so they are validated and leave the
    result unchanged."""
    _check_split_scratch(split_scratch, split, topk_ids, w13)
    return _nvfp4_moe_impl(hidden, topk_ids, topk_weights, w13, w13_scales, w13_global_scales,
                           w2, w2_scales, w2_global_scales, multiply_router_weight,
                           torch.float32)


@_nvfp4_moe_op.register_fake
def _(hidden, topk_ids, topk_weights, w13, w13_scales, w13_global_scales, w2, w2_scales,
      w2_global_scales, split_scratch, split, multiply_router_weight):
    return hidden.new_empty(hidden.shape, dtype=torch.float32)


@torch.library.custom_op("sbb200::nvfp4_moe_typed", mutates_args=())
def _nvfp4_moe_typed_op(hidden: torch.Tensor, topk_ids: torch.Tensor,
                        topk_weights: torch.Tensor, w13: torch.Tensor, w13_scales: torch.Tensor,
                        w13_global_scales: torch.Tensor, w2: torch.Tensor,
                        w2_scales: torch.Tensor, w2_global_scales: torch.Tensor,
                        multiply_router_weight: bool, out_dtype_code: int) -> torch.Tensor:
    """sbb200::nvfp4_moe with the output in the model dtype (out_dtype_code
    0 f32, 1 f16, 2 bf16): the hook's path, which skips the fp32 round trip
    the reference's plugin makes before casting (routed_experts.py:3004-3007)."""
    return _nvfp4_moe_impl(hidden, topk_ids, topk_weights, w13, w13_scales, w13_global_scales,
                           w2, w2_scales, w2_global_scales, multiply_router_weight,
                           _OUT_CODES[out_dtype_code])


@_nvfp4_moe_typed_op.register_fake
def _(hidden, topk_ids, topk_weights, w13, w13_scales, w13_global_scales, w2, w2_scales,
      w2_global_scales, multiply_router_weight, out_dtype_code):
    return hidden.new_empty(hidden.shape, dtype=_OUT_CODES[out_dtype_code])


def nvfp4_moe(hidden: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
              w13: torch.Tensor, w13_scales: torch.Tensor, w13_global_scales: torch.Tensor,
              w2: torch.Tensor, w2_scales: torch.Tensor, w2_global_scales: torch.Tensor,
              split_scratch: torch.Tensor | None = None, split: bool = False,
              multiply_router_weight: bool = True,
              out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Routed-expert NVFP4 MoE with the reference op's signature
    (tk_xpu_ext.sycl:296-302). ``split``/``split_scratch`` select a kernel
    shape on the reference's Arc cards; the B200 driver picks its kernels
    itself, so they are accepted and validated but do not change the result.
    Returns ``out_dtype`` [M, K] (fp32 like the reference op by default):
    fp32 goes through ``torch.ops.sbb200.nvfp4_moe``, other dtypes through
    ``torch.ops.sbb200.nvfp4_moe_typed``."""
    if out_dtype == torch.float32:
        return torch.ops.sbb200.nvfp4_moe(hidden, topk_ids, topk_weights, w13, w13_scales,
                                          w13_global_scales, w2, w2_scales, w2_global_scales,
                                          split_scratch, bool(split),
                                          bool(multiply_router_weight))
    _check_split_scratch(split_scratch, split, topk_ids, w13)
    return torch.ops.sbb200.nvfp4_moe_typed(hidden, topk_ids, topk_weights, w13, w13_scales,
                                            w13_global_scales, w2, w2_scales, w2_global_scales,
                                            bool(multiply_router_weight), DTYPE_CODE[out_dtype])


def nvfp4_moe_bad_ids(device: torch.device | None = None) -> int:
    """Count of ids outside [-1, E) seen by the last nvfp4_moe call on the
    current stream of ``device`` (synchronises that stream)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    key = (device.index or 0, torch.cuda.current_stream(device).cuda_stream)
    ws = _workspaces.get(key)
    if ws is None:
        return 0
    v = ctypes.c_uint32(0)
    _check(lib().sbb200_nvfp4_moe_bad_ids(key[1], _p(ws), ctypes.addressof(v)))
    return int(v.value)


def nvfp4_moe_device_errors(device: torch.device | None = None) -> int:
    """Device error word of the last nvfp4_moe call on the current stream of
    ``device`` (bit 0: a kernel wait passed its deadline; synchronises)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    key = (device.index or 0, torch.cuda.current_stream(device).cuda_stream)
    ws = _workspaces.get(key)
    if ws is None:
        return 0
    v = ctypes.c_uint32(0)
    _check(lib().sbb200_nvfp4_moe_device_errors(key[1], _p(ws), ctypes.addressof(v)))
    return int(v.value)


def device_errors(device: torch.device | None = None) -> int:
    """Error bits raised on ``device`` by any call of this library since the
    last read (bit 0: a tcgen05 GEMM wait passed its limit and that call's
    result is not valid), across workspaces, streams and graph replays.
    Reads and clears; synchronises the current stream."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    v = ctypes.c_uint32(0)
    with torch.cuda.device(device):
        _check(lib().sbb200_device_errors(torch.cuda.current_stream(device).cuda_stream,
                                          ctypes.addressof(v)))
    return int(v.value)


def set_kernel_wait_ns(ns: int) -> int:
    """Limit of the tcgen05 GEMMs' pipeline waits for later launches (0: the
    2 s default); returns the previous limit. A wait that runs out makes the
    kernel abandon its work and raise the device error bit instead of
    hanging."""
    return int(lib().sbb200_set_kernel_wait_ns(int(ns)))


# --------------------------------------------------------------------------
# building blocks
# --------------------------------------------------------------------------

def nvfp4_moe_w4a4(hidden: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                   w13: torch.Tensor, w13_scales: torch.Tensor, w13_global_scales: torch.Tensor,
                   w2: torch.Tensor, w2_scales: torch.Tensor, w2_global_scales: torch.Tensor,
                   a13_gscale: torch.Tensor | None = None, a2_gscale: torch.Tensor | None = None,
                   alpha13: torch.Tensor | None = None, alpha2: torch.Tensor | None = None,
                   multiply_router_weight: bool = True,
                   out_dtype: torch.dtype = torch.float32, out: torch.Tensor | None = None,
                   stage_events: list | None = None) -> torch.Tensor:
    """W4A4 routed-expert forward (see sbb200_nvfp4_moe_w4a4): activations
    quantised once to NVFP4, dynamically per row, or with vLLM's static
    per-expert a1/a2_gscale and g1/g2_alphas when all four are given."""
    M, K, E, top_k, I = _validate(hidden, topk_ids, topk_weights, w13, w13_scales,
                                  w13_global_scales, w2, w2_scales, w2_global_scales)
    static = [a13_gscale, a2_gscale, alpha13, alpha2]
    for name, t in zip(("a13_gscale", "a2_gscale", "alpha13", "alpha2"), static):
        if t is not None:
            _check_cuda(name, t)
            if t.dtype != torch.float32 or t.numel() != E:
                raise ValueError(f"sbb200: {name} must be float32 [E]")
    if out is None:
        out = torch.empty((M, K), dtype=out_dtype, device=hidden.device)
    nbytes = nvfp4_moe_workspace_bytes(M, E, top_k, K, I, hidden.dtype)
    ws = _workspace(hidden.device, nbytes)
    evs = None
    if stage_events is not None:
        evs = (ctypes.c_void_p * STAGE_EVENTS)(*[ev.cuda_event for ev in stage_events])
    _check(lib().sbb200_nvfp4_moe_w4a4(
        _stream(hidden), _p(hidden), _p(topk_ids), _p(topk_weights), _p(w13), _p(w13_scales),
        _p(w13_global_scales), _p(w2), _p(w2_scales), _p(w2_global_scales), *map(_p, static),
        _p(ws), ws.numel(), _p(out), DTYPE_CODE[out.dtype], M, E, top_k, K, I,
        DTYPE_CODE[hidden.dtype], int(bool(multiply_router_weight)), evs,
        STAGE_EVENTS if evs is not None else 0))
    return out


def router_topk(router_logits: torch.Tensor, top_k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k expert ids (int32, selection order) and softmax weights (fp32)
    of router logits [M, E] (ops::moe_route_topk of the reference, ops.hpp:262-272)."""
    _check_cuda("router logits", router_logits)
    if router_logits.dim() != 2 or router_logits.dtype not in DTYPE_CODE:
        raise ValueError("sbb200: router logits must be float32/float16/bfloat16 [M,E]")
    M, E = router_logits.shape
    ids = torch.empty((M, top_k), dtype=torch.int32, device=router_logits.device)
    w = torch.empty((M, top_k), dtype=torch.float32, device=router_logits.device)
    _check(lib().sbb200_router_topk(_stream(router_logits), _p(router_logits),
                                    DTYPE_CODE[router_logits.dtype], M, E, top_k, _p(ids), _p(w)))
    return ids, w


def nvfp4_moe_from_logits(hidden: torch.Tensor, router_logits: torch.Tensor, top_k: int,
                          w13: torch.Tensor, w13_scales: torch.Tensor,
                          w13_global_scales: torch.Tensor, w2: torch.Tensor,
                          w2_scales: torch.Tensor, w2_global_scales: torch.Tensor,
                          multiply_router_weight: bool = True,
                          out_dtype: torch.dtype = torch.float32):
    """The routed-expert forward with top-k routing fused in front of the
    permute: returns (out, topk_ids, topk_weights)."""
    _check_cuda("router logits", router_logits)
    M = hidden.shape[0]
    if router_logits.dim() != 2 or router_logits.shape[0] != M or router_logits.dtype not in DTYPE_CODE:
        raise ValueError("sbb200: router logits must be float32/float16/bfloat16 [M,E]")
    dev = hidden.device
    ids = torch.empty((M, top_k), dtype=torch.int32, device=dev)
    w = torch.empty((M, top_k), dtype=torch.float32, device=dev)
    _, K, E, _, I = _validate(hidden, ids, w, w13, w13_scales, w13_global_scales, w2,
                              w2_scales, w2_global_scales)
    if router_logits.shape[1] != E:
        raise ValueError("sbb200: router logits must have one column per expert")
    out = torch.empty((M, K), dtype=out_dtype, device=dev)
    nbytes = nvfp4_moe_workspace_bytes(M, E, top_k, K, I, hidden.dtype)
    ws = _workspace(dev, nbytes)
    _check(lib().sbb200_nvfp4_moe_from_logits(
        _stream(hidden), _p(hidden), _p(router_logits), DTYPE_CODE[router_logits.dtype], _p(ids),
        _p(w), _p(w13), _p(w13_scales), _p(w13_global_scales), _p(w2), _p(w2_scales),
        _p(w2_global_scales), _p(ws), ws.numel(), _p(out), DTYPE_CODE[out.dtype], M, E, top_k, K,
        I, DTYPE_CODE[hidden.dtype], int(bool(multiply_router_weight))))
    return out, ids, w


def route_plan(topk_ids: torch.Tensor, E: int) -> dict:
    """Stable device routing permutation; see sbb200_route_plan."""
    _check_cuda("topk ids", topk_ids)
    if topk_ids.dtype != torch.int32 or topk_ids.dim() != 2:
        raise ValueError("sbb200: topk ids must be int32 [M,top_k]")
    M, top_k = topk_ids.shape
    R = M * top_k
    dev = topk_ids.device
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    sorted_routes = torch.full((max(R, 1),), -7, dtype=torch.int32, device=dev)
    slot_of = torch.empty(max(R, 1), dtype=torch.int32, device=dev)
    scratch = torch.zeros(int(lib().sbb200_route_plan_scratch_bytes(R, E)), dtype=torch.uint8,
                          device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    _check(lib().sbb200_route_plan(_stream(topk_ids), _p(topk_ids), M, top_k, E, _p(counts),
                                   _p(offsets), _p(sorted_routes), _p(slot_of), _p(scratch),
                                   _p(bad)))
    return {"counts": counts, "offsets": offsets, "sorted": sorted_routes, "slot_of": slot_of[:R],
            "bad_ids": bad}


def nvfp4_dequant(q: torch.Tensor, sf: torch.Tensor, g: torch.Tensor,
                  rows_per_scale: int) -> torch.Tensor:
    """Bit-exact fp32 dequant of a [rows, cols/2] plane (see sbb200_nvfp4_dequant)."""
    for name, t in (("q", q), ("sf", sf), ("g", g)):
        _check_cuda(name, t)
    half = q.shape[-1]
    rows = q.numel() // half
    out = torch.empty(q.shape[:-1] + (half * 2,), dtype=torch.float32, device=q.device)
    _check(lib().sbb200_nvfp4_dequant(_stream(q), _p(q), _p(sf), _p(g), rows_per_scale, _p(out),
                                      rows, half * 2))
    return out


def nvfp4_quantize(x: torch.Tensor, gq: torch.Tensor,
                   rows_per_scale: int) -> tuple[torch.Tensor, torch.Tensor]:
    """vLLM ref_nvfp4_quant semantics on the device; returns (q, sf) bytes."""
    _check_cuda("x", x)
    _check_cuda("gq", gq)
    cols = x.shape[-1]
    rows = x.numel() // cols
    q = torch.empty(x.shape[:-1] + (cols // 2,), dtype=torch.uint8, device=x.device)
    sf = torch.empty(x.shape[:-1] + (cols // 16,), dtype=torch.uint8, device=x.device)
    _check(lib().sbb200_nvfp4_quantize(_stream(x), _p(x), DTYPE_CODE[x.dtype], _p(gq),
                                       rows_per_scale, _p(q), _p(sf), rows, cols))
    return q, sf


# --------------------------------------------------------------------------
# provider
# --------------------------------------------------------------------------

class Health(ctypes.Structure):
    _fields_ = [("generation", ctypes.c_uint64), ("dispatches", ctypes.c_uint64),
                ("allocations", ctypes.c_uint64), ("last_error_bytes", ctypes.c_uint64),
                ("loaded", ctypes.c_uint32), ("pending", ctypes.c_uint32),
                ("stopped", ctypes.c_uint32), ("device_errors", ctypes.c_uint32)]


class Provider:
    """Registered layers + an owned workspace (sbb200_create / register_layer /
    moe_forward / health)."""

    def __init__(self, device: int, max_tokens: int, top_k: int, max_E: int, K: int, I: int):
        self.h = lib().sbb200_create(device, max_tokens, top_k, max_E, K, I)
        if not self.h:
            raise Sbb200Error(-1, last_error())
        self.device = torch.device("cuda", device)
        self.K = K
        self._keep: dict[int, tuple] = {}

    def register_layer(self, layer: int, w13, w13_scales, w13_global_scales, w2, w2_scales,
                       w2_global_scales) -> None:
        ts = (w13, w13_scales, w13_global_scales, w2, w2_scales, w2_global_scales)
        for t in ts:
            _check_cuda("weight", t)
        self._keep[layer] = ts  # the provider keeps pointers, not copies
        _check(lib().sbb200_register_layer(self.h, layer, w13.size(0), *(_p(t) for t in ts)))

    def forward(self, layer: int, hidden: torch.Tensor, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor, out: torch.Tensor | None = None,
                out_dtype: torch.dtype = torch.float32,
                multiply_router_weight: bool = True) -> torch.Tensor:
        M = hidden.shape[0]
        if out is None:
            out = torch.empty((M, self.K), dtype=out_dtype, device=hidden.device)
        _check(lib().sbb200_moe_forward(self.h, layer, _stream(hidden), _p(hidden),
                                        DTYPE_CODE[hidden.dtype], _p(topk_ids), _p(topk_weights),
                                        _p(out), DTYPE_CODE[out.dtype], M,
                                        int(bool(multiply_router_weight))))
        return out

    def health(self) -> tuple[dict, str]:
        """(health fields, last error). ``device_errors`` is the device error
        word of the last forward (bit 0: a kernel wait passed its limit and
        that result is not valid); reading it synchronises the device."""
        h = Health()
        buf = ctypes.create_string_buffer(4096)
        lib().sbb200_health(self.h, ctypes.byref(h), buf, 4096)
        return {f: getattr(h, f) for f, _ in Health._fields_}, buf.value.decode(errors="replace")

    def close(self) -> None:
        if self.h:
            lib().sbb200_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
