"""CPU oracle driver for the routed-expert NVFP4 MoE path.

TEST INFRASTRUCTURE ONLY: the checker, never the product. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline / reference legs
import this module.

Contents
--------
* ctypes bindings to ``libsb_oracle.so`` (the C restatement in
  ``nvfp4_oracle.c``) and to ``_ref/libsb_cpu_expert.so`` (the reference's own
  CPU expert tier, ``src/phase7/cpu_expert_capi.h:70-135`` of the reference,
  compiled from its source by ``oracle/Makefile``).
* A numpy restatement of the NVFP4 quantiser the reference's tests and the
  benchmark configurations use: vLLM ``ref_nvfp4_quant`` / ``cast_to_fp4``
  (``vllm/model_executor/layers/quantization/utils/nvfp4_emulation_utils.py``,
  the library the reference's fixtures call, ``src/phase7/nvfp4_testutil.py:53-71``).
* Seeded generators for the benchmark configurations (weights bf16 N(0, 0.02) quantised
  with a per-tensor global multiplier ``amax / (448 * 6)``; activations bf16
  N(0, 1); softmax top-k routing renormalised over the selected k).
* The deterministic known-answer fixture of the reference's device test
  (``src/QuixiCore-XPU/tests/xpu_ops_smoke.cpp:93-96, 2229-2304``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libsb_oracle.so"
REF_SO = HERE / "_ref" / "libsb_cpu_expert.so"

BLOCK = 16
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


# --------------------------------------------------------------------------
# building / loading
# --------------------------------------------------------------------------

def reference_dir() -> Path | None:
    """Root of the reference source tree: ``SBB200_REFERENCE_DIR`` when set,
    else a directory named ``reference`` beside this repository, else None."""
    env = os.environ.get("SBB200_REFERENCE_DIR")
    if env:
        return Path(env)
    sibling = HERE.parent.parent / "reference"
    return sibling if (sibling / "src" / "phase7").is_dir() else None


def build(ref: bool = True) -> None:
    """Compile the C oracle (and, where the reference tree is found, the
    reference CPU tier) with ``oracle/Makefile``."""
    targets = ["oracle"] + (["ref"] if ref else [])
    cmd = ["make", "-s", "-C", str(HERE)] + targets
    rdir = reference_dir() if ref else None
    if rdir is not None:
        cmd.append(f"REF={rdir}")
    subprocess.run(cmd, check=True)


def reference_isa() -> str | None:
    """The -march the reference CPU tier in _ref was compiled for."""
    f = REF_SO.parent / "isa.txt"
    return f.read_text().strip() if f.exists() else None


_oracle_lib = None
_ref_lib = None


def oracle_lib() -> ctypes.CDLL:
    global _oracle_lib
    if _oracle_lib is None:
        if not ORACLE_SO.exists():
            build(ref=False)
        lib = ctypes.CDLL(str(ORACLE_SO))
        P = ctypes.c_void_p
        S = ctypes.c_size_t
        lib.sbo_e2m1.restype = ctypes.c_float
        lib.sbo_e2m1.argtypes = [ctypes.c_uint32]
        lib.sbo_e4m3.restype = ctypes.c_float
        lib.sbo_e4m3.argtypes = [ctypes.c_uint32]
        lib.sbo_nvfp4_dequant.restype = None
        lib.sbo_nvfp4_dequant.argtypes = [P, P, ctypes.c_float, P, S, S]
        lib.sbo_route_plan.restype = ctypes.c_int64
        lib.sbo_route_plan.argtypes = [P, S, S, S, P, P, P, P]
        lib.sbo_moe_forward_tokens.restype = ctypes.c_int
        lib.sbo_moe_forward_tokens.argtypes = [P, P, P, P, P, P, P, P, P, S, S, S, S,
                                               ctypes.c_int, P, S, P, ctypes.c_int]
        _oracle_lib = lib
    return _oracle_lib


def reference_available() -> bool:
    return REF_SO.exists()


def ref_lib() -> ctypes.CDLL:
    """The reference's CPU expert tier (sb_cpu_* C-ABI)."""
    global _ref_lib
    if _ref_lib is None:
        if not REF_SO.exists():
            build(ref=True)
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} not built (reference tree absent)")
        lib = ctypes.CDLL(str(REF_SO))
        P = ctypes.c_void_p
        S = ctypes.c_size_t
        lib.sb_cpu_create.restype = P
        lib.sb_cpu_create.argtypes = [S, S, S, S, S, S]
        lib.sb_cpu_load_expert.restype = ctypes.c_int
        lib.sb_cpu_load_expert.argtypes = [P, S, S, P, P, ctypes.c_float, P, P,
                                           ctypes.c_float, P, P, ctypes.c_float]
        lib.sb_cpu_moe_forward.restype = ctypes.c_int
        lib.sb_cpu_moe_forward.argtypes = [P, S, P, P, P, S, S, P]
        lib.sb_cpu_expert_forward.restype = ctypes.c_int
        lib.sb_cpu_expert_forward.argtypes = [P, S, S, P, P, S]
        lib.sb_cpu_skipped_routes.restype = ctypes.c_uint64
        lib.sb_cpu_skipped_routes.argtypes = [P]
        lib.sb_cpu_destroy.restype = None
        lib.sb_cpu_destroy.argtypes = [P]
        _ref_lib = lib
    return _ref_lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data


# --------------------------------------------------------------------------
# number formats
# --------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest-even), returned as uint16 bit patterns."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def e4m3_decode(v: np.ndarray) -> np.ndarray:
    """float8_e4m3fn byte -> fp32 (NaN for 0x7F/0xFF)."""
    v = v.astype(np.int32)
    sign = np.where(v & 0x80, -1.0, 1.0).astype(np.float32)
    exp = (v >> 3) & 0xF
    man = (v & 7).astype(np.float32)
    mag = np.where(exp == 0, np.ldexp(man, -9),
                   np.ldexp(1.0 + man / 8.0, exp - 7)).astype(np.float32)
    mag = np.where((exp == 15) & ((v & 7) == 7), np.float32(np.nan), mag)
    return sign * mag


def e4m3_encode_rne(x: np.ndarray) -> np.ndarray:
    """Non-negative fp32 (already clamped to <= 448) -> e4m3fn byte, rounding to
    nearest even like ``torch.Tensor.to(torch.float8_e4m3fn)``."""
    x = np.asarray(x, dtype=np.float64)
    out = np.zeros(x.shape, dtype=np.uint8)
    pos = x > 0
    xs = x[pos]
    _, e2 = np.frexp(xs)            # xs = m * 2**e2, m in [0.5, 1)
    e = e2 - 1                      # xs in [2**e, 2**(e+1))
    e = np.maximum(e, -6)           # below 2**-6 the step is the subnormal 2**-9
    step = np.ldexp(1.0, e - 3)
    q = np.round(xs / step) * step  # numpy rounds half to even
    q = np.minimum(q, 448.0)
    _, qe2 = np.frexp(q)
    qe = qe2 - 1
    sub = q < 2.0 ** -6
    code = np.where(
        sub,
        np.round(q / 2.0 ** -9).astype(np.int64),
        ((qe + 7) << 3) | np.round((q / np.ldexp(1.0, qe) - 1.0) * 8).astype(np.int64),
    )
    out[pos] = code.astype(np.uint8)
    return out


def cast_to_fp4_codes(x: np.ndarray) -> np.ndarray:
    """fp32 in [-6, 6] -> e2m1 codes (uint8 0..15), with vLLM ``cast_to_fp4``'s
    thresholds (round to nearest, ties to the even code). A value that rounds
    to zero gets code 0 regardless of sign."""
    a = np.abs(x)
    mag = np.zeros(x.shape, dtype=np.uint8)
    mag = np.where((a > 0.25) & (a < 0.75), 1, mag)
    mag = np.where((a >= 0.75) & (a <= 1.25), 2, mag)
    mag = np.where((a > 1.25) & (a < 1.75), 3, mag)
    mag = np.where((a >= 1.75) & (a <= 2.5), 4, mag)
    mag = np.where((a > 2.5) & (a < 3.5), 5, mag)
    mag = np.where((a >= 3.5) & (a <= 5.0), 6, mag)
    mag = np.where(a > 5.0, 7, mag).astype(np.uint8)
    sign = ((x < 0) & (mag != 0)).astype(np.uint8) << 3
    return sign | mag


def pack_fp4(codes: np.ndarray) -> np.ndarray:
    """[rows, cols] codes -> [rows, cols/2] bytes, low nibble = even column."""
    c = codes.astype(np.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


def unpack_fp4(packed: np.ndarray) -> np.ndarray:
    lo = packed & 0x0F
    hi = packed >> 4
    out = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


def quantize_nvfp4(w: np.ndarray, global_quant_scale) -> tuple[np.ndarray, np.ndarray]:
    """Restatement of vLLM ``ref_nvfp4_quant`` for a [rows, cols] fp32 matrix.

    ``global_quant_scale`` is the checkpoint's ``weight_global_scale``
    (448*6/amax); the dequant multiplier stored beside the weights is its
    inverse, amax/(448*6). A [rows] array gives each row its own global (the
    same arithmetic per row). Returns (packed e2m1 [rows, cols/2],
    e4m3 block scales [rows, cols/16]) as uint8.
    """
    rows, cols = w.shape
    assert cols % BLOCK == 0
    G = np.asarray(global_quant_scale, dtype=np.float32)
    if G.ndim == 1:
        G = G.reshape(rows, 1, 1)
    x = np.asarray(w, dtype=np.float32).reshape(rows, cols // BLOCK, BLOCK)
    vec_max = np.max(np.abs(x), axis=-1, keepdims=True).astype(np.float32)
    scale = (G * (vec_max * np.float32(1.0 / 6.0))).astype(np.float32)
    scale = np.clip(scale, -448.0, 448.0).astype(np.float32)
    sf = e4m3_encode_rne(scale)
    scale_q = e4m3_decode(sf)
    inv_g = np.float32(1.0) / (G + np.float32(G == 0) * np.float32(1e8))
    t = (scale_q * inv_g).astype(np.float32)
    out_scale = (np.float32(1.0) / (t + (t == 0).astype(np.float32) * np.float32(1e8))).astype(np.float32)
    scaled = np.clip((x * out_scale).astype(np.float32), -6.0, 6.0).reshape(rows, cols)
    codes = cast_to_fp4_codes(scaled)
    return pack_fp4(codes), sf.reshape(rows, cols // BLOCK)


def dequant(q: np.ndarray, sf: np.ndarray, g: float) -> np.ndarray:
    """W = e2m1 * fp32(e4m3 * g) via the C oracle (bit-exact reference)."""
    q = np.ascontiguousarray(q, dtype=np.uint8)
    sf = np.ascontiguousarray(sf, dtype=np.uint8)
    rows, half = q.shape
    out = np.empty((rows, half * 2), dtype=np.float32)
    oracle_lib().sbo_nvfp4_dequant(_ptr(q), _ptr(sf), float(np.float32(g)), _ptr(out),
                                   rows, half * 2)
    return out


# --------------------------------------------------------------------------
# layers and routing
# --------------------------------------------------------------------------

@dataclass
class Layer:
    """One routed-expert layer in the op's layout.

    w13 [E, 2I, K/2] (gate rows then up rows), s13 [E, 2I, K/16],
    g13 [E] fp32, w2 [E, K, I/2], s2 [E, K, I/16], g2 [E] fp32."""
    E: int
    K: int
    I: int
    w13: np.ndarray
    s13: np.ndarray
    g13: np.ndarray
    w2: np.ndarray
    s2: np.ndarray
    g2: np.ndarray

    @property
    def expert_bytes(self) -> int:
        return (self.w13[0].nbytes + self.s13[0].nbytes + self.w2[0].nbytes
                + self.s2[0].nbytes + 8)


def _quantize_plane(w: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.float32]:
    amax = np.float32(np.max(np.abs(w)))
    G = np.float32(np.float32(448.0 * 6.0) / amax)
    g = np.float32(amax / np.float32(448.0 * 6.0))
    q, sf = quantize_nvfp4(w, G)
    return q, sf, g


def make_layer(E: int, K: int, I: int, seed: int, std: float = 0.02) -> Layer:
    """Benchmark weights: bf16 N(0, std) per expert gate/up [2I, K] and down
    [K, I], quantised to NVFP4 with one global per w13 and one per w2."""
    rng = np.random.default_rng(seed)
    w13 = np.empty((E, 2 * I, K // 2), np.uint8)
    s13 = np.empty((E, 2 * I, K // 16), np.uint8)
    w2 = np.empty((E, K, I // 2), np.uint8)
    s2 = np.empty((E, K, I // 16), np.uint8)
    g13 = np.empty(E, np.float32)
    g2 = np.empty(E, np.float32)
    for e in range(E):
        a = bf16_bits_to_f32(f32_to_bf16_bits(
            rng.standard_normal((2 * I, K), dtype=np.float32) * np.float32(std)))
        w13[e], s13[e], g13[e] = _quantize_plane(a)
        b = bf16_bits_to_f32(f32_to_bf16_bits(
            rng.standard_normal((K, I), dtype=np.float32) * np.float32(std)))
        w2[e], s2[e], g2[e] = _quantize_plane(b)
    return Layer(E, K, I, w13, s13, g13, w2, s2, g2)


def make_hidden(T: int, K: int, seed: int, scale: float = 1.0) -> np.ndarray:
    """bf16 N(0, scale) activations as uint16 bit patterns [T, K]."""
    rng = np.random.default_rng(seed)
    return f32_to_bf16_bits(rng.standard_normal((T, K), dtype=np.float32) * np.float32(scale))


def softmax_topk(logits: np.ndarray, top_k: int) -> tuple[np.ndarray, np.ndarray]:
    """top-k of softmax(logits) renormalised over the selected k (equivalently a
    softmax over the k selected logits), ids int32 / weights fp32 [T, top_k]."""
    order = np.argsort(-logits, axis=1, kind="stable")[:, :top_k]
    sel = np.take_along_axis(logits, order, axis=1).astype(np.float64)
    sel = sel - sel.max(axis=1, keepdims=True)
    w = np.exp(sel)
    w = w / w.sum(axis=1, keepdims=True)
    return order.astype(np.int32), w.astype(np.float32)


def route_logits(T: int, E: int, top_k: int, seed: int,
                 bias_std: float = 0.0) -> tuple[np.ndarray, np.ndarray]:
    """Router logits N(0, 1) (plus an optional per-expert bias N(0, bias_std)),
    softmax top-k renormalised."""
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    if bias_std:
        logits = logits + rng.standard_normal(E).astype(np.float32) * np.float32(bias_std)
    return softmax_topk(logits, top_k)


def route_zipf(T: int, E: int, top_k: int, seed: int, s: float = 1.2) -> tuple[np.ndarray, np.ndarray]:
    """Skewed routing: each token draws top_k distinct experts with probability
    proportional to rank**-s over a seeded random permutation of the experts;
    weights are a softmax over N(0, 1) logits of the chosen k."""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(E)
    p = 1.0 / np.arange(1, E + 1, dtype=np.float64) ** s
    p /= p.sum()
    ids = np.empty((T, top_k), np.int32)
    for t in range(T):
        ids[t] = perm[rng.choice(E, size=top_k, replace=False, p=p)]
    lg = rng.standard_normal((T, top_k)).astype(np.float64)
    w = np.exp(lg - lg.max(axis=1, keepdims=True))
    w /= w.sum(axis=1, keepdims=True)
    return ids, w.astype(np.float32)


# --------------------------------------------------------------------------
# oracle entry points
# --------------------------------------------------------------------------

def router_topk(logits: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """fp32 restatement of the reference's top-k router
    (src/QuixiCore-XPU/kernels/moe/moe_route/variants/xpu_sycl/
    moe_route.sycl.cpp:16-50): k rounds of argmax over the untaken experts with
    a strict '>' from -inf (lowest index wins ties; a round that finds nothing
    picks expert 0), then exp(v - max) of the chosen logits summed in
    selection order, times 1/sum. Pure-Python loops over the k rounds, numpy
    over tokens: for test sizes."""
    x = np.asarray(logits, dtype=np.float32)
    M, E = x.shape
    ids = np.zeros((M, k), np.int32)
    val = np.zeros((M, k), np.float32)
    taken = np.zeros((M, E), bool)
    cols = np.arange(E)
    for i in range(k):
        cand = np.where(taken, np.float32(-np.inf), x)
        cand = np.where(np.isnan(cand), np.float32(-np.inf), cand)
        best = cand.max(axis=1)
        # lowest index among the maxima; rows whose best is -inf pick expert 0
        first = np.argmax(cand == best[:, None], axis=1)
        first = np.where(np.isneginf(best), 0, first)
        ids[:, i] = first
        val[:, i] = np.where(np.isneginf(best), np.float32(-np.inf), best)
        taken[np.arange(M), first] = True
    m = val.max(axis=1, keepdims=True)
    ex = np.exp(val - m).astype(np.float32)
    s = np.zeros(M, np.float32)
    for i in range(k):
        s = (s + ex[:, i]).astype(np.float32)
    inv = (np.float32(1.0) / s).astype(np.float32)
    return ids, (ex * inv[:, None]).astype(np.float32)


def kat_router_reference(logits: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """The double-precision check loop of the reference's router test
    (src/QuixiCore-XPU/tests/xpu_ops_smoke.cpp:436-450): argmax with strict
    '>' from -1e30, softmax over the chosen k in double."""
    x = np.asarray(logits, dtype=np.float64)
    M, E = x.shape
    ids = np.zeros((M, k), np.int32)
    w = np.zeros((M, k), np.float64)
    for t in range(M):
        taken = np.zeros(E, bool)
        rv = []
        for i in range(k):
            best, be = -1e30, 0
            for e in range(E):
                if not taken[e] and x[t, e] > best:
                    best, be = x[t, e], e
            taken[be] = True
            ids[t, i] = be
            rv.append(best)
        m = max(rv)
        ex = [np.exp(v - m) for v in rv]
        tot = sum(ex)
        w[t] = [v / tot for v in ex]
    return ids, w


def route_plan(ids: np.ndarray, E: int) -> dict:
    """Stable routing permutation: counts, offsets, sorted route ids (expert,
    then token*top_k + k ascending) and each route's slot (-1 if dropped)."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    M, top_k = ids.shape
    counts = np.zeros(E, np.int32)
    offsets = np.zeros(E + 1, np.int32)
    sorted_routes = np.zeros(max(M * top_k, 1), np.int32)
    slot_of = np.zeros(max(M * top_k, 1), np.int32)
    bad = oracle_lib().sbo_route_plan(_ptr(ids), M, top_k, E, _ptr(counts), _ptr(offsets),
                                      _ptr(sorted_routes), _ptr(slot_of))
    valid = int(offsets[E])
    return {"counts": counts, "offsets": offsets, "sorted": sorted_routes[:valid].copy(),
            "slot_of": slot_of[:M * top_k].copy(), "bad_ids": int(bad)}


def moe_forward(hidden_bf16: np.ndarray, ids: np.ndarray, weights: np.ndarray,
                layer: Layer, tokens: np.ndarray | None = None,
                multiply_router_weight: bool = True, threads: int | None = None) -> np.ndarray:
    """fp32 routed-expert output for ``tokens`` (all tokens when None)."""
    hidden_bf16 = np.ascontiguousarray(hidden_bf16, dtype=np.uint16)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    weights = np.ascontiguousarray(weights, dtype=np.float32)
    M, K = hidden_bf16.shape
    top_k = ids.shape[1]
    if tokens is None:
        tokens = np.arange(M, dtype=np.int32)
    tokens = np.ascontiguousarray(tokens, dtype=np.int32)
    out = np.zeros((len(tokens), K), np.float32)
    L = layer
    arrs = [np.ascontiguousarray(a) for a in (L.w13, L.s13, L.g13, L.w2, L.s2, L.g2)]
    rc = oracle_lib().sbo_moe_forward_tokens(
        _ptr(hidden_bf16), _ptr(ids), _ptr(weights), _ptr(arrs[0]), _ptr(arrs[1]),
        _ptr(arrs[2]), _ptr(arrs[3]), _ptr(arrs[4]), _ptr(arrs[5]), L.E, top_k, K, L.I,
        int(multiply_router_weight), _ptr(tokens), len(tokens), _ptr(out),
        int(threads or os.cpu_count() or 1))
    if rc != 0:
        raise RuntimeError(f"oracle moe_forward failed rc={rc}")
    return out


def moe_forward_w4a4(hidden_bf16: np.ndarray, ids: np.ndarray, weights: np.ndarray,
                     layer: Layer, a13: np.ndarray | None = None, a2: np.ndarray | None = None,
                     alpha13: np.ndarray | None = None, alpha2: np.ndarray | None = None,
                     multiply_router_weight: bool = True) -> np.ndarray:
    """W4A4 expert path: every activation row entering a GEMM is quantised to
    NVFP4 with ``quantize_nvfp4`` (vLLM ref_nvfp4_quant, pinned against vLLM's
    own output) and the products e2m1*e4m3 x e2m1*e4m3 are summed in fp64,
    then scaled. Static (a13/a2/alpha13/alpha2 given, vLLM's a1/a2_gscale and
    g1/g2_alphas per expert): G = a13[e] or a2[e], result * alpha. Dynamic:
    G = 448*6/max|row| (fp32), result * (1/G) * g13[e] or g2[e]. SwiGLU in
    fp32 as ``moe_forward``. Routes outside [0, E) contribute nothing."""
    x = bf16_bits_to_f32(np.asarray(hidden_bf16, np.uint16))
    T, K = x.shape
    E, I = layer.E, layer.I
    top_k = ids.shape[1]
    static = a13 is not None
    out = np.zeros((T, K), np.float64)

    def quant_rows(rows: np.ndarray, G: np.ndarray):
        q, sf = quantize_nvfp4(rows, G)
        return dequant(q, sf, 1.0).astype(np.float64)

    def dyn_g(rows: np.ndarray) -> np.ndarray:
        amax = np.abs(rows).max(axis=1).astype(np.float32)
        return np.where(amax > 0, np.float32(2688.0) / np.where(amax > 0, amax, 1), np.float32(1.0)).astype(np.float32)

    for e in range(E):
        t_idx, k_idx = np.nonzero(ids == e)
        if len(t_idx) == 0:
            continue
        w13 = dequant(layer.w13[e], layer.s13[e], 1.0).astype(np.float64)
        w2 = dequant(layer.w2[e], layer.s2[e], 1.0).astype(np.float64)
        xr = x[t_idx]
        G1 = np.full(len(t_idx), a13[e], np.float32) if static else dyn_g(xr)
        d13 = quant_rows(xr, G1) @ w13.T
        s1 = (np.full(len(t_idx), alpha13[e], np.float32) if static
              else (np.float32(1.0) / G1).astype(np.float32) * np.float32(layer.g13[e]))
        gu = (d13 * s1[:, None].astype(np.float64)).astype(np.float32)
        g, u = gu[:, :I], gu[:, I:]
        h = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
        G2 = np.full(len(t_idx), a2[e], np.float32) if static else dyn_g(h)
        d2 = quant_rows(h, G2) @ w2.T
        s2 = (np.full(len(t_idx), alpha2[e], np.float32) if static
              else (np.float32(1.0) / G2).astype(np.float32) * np.float32(layer.g2[e]))
        y = (d2 * s2[:, None].astype(np.float64))
        wr = weights[t_idx, k_idx].astype(np.float64) if multiply_router_weight else 1.0
        np.add.at(out, t_idx, y * (wr[:, None] if multiply_router_weight else 1.0))
    return out.astype(np.float32)


class ReferenceCpuTier:
    """The reference's own CPU expert tier (compiled from its source),
    driven through its C-ABI ``sb_cpu_*`` exactly as its host wrapper does
    (``src/phase4/src/shooting_brake_vllm/cpu_expert_host.py``). Gate and up
    share ``g13`` (``src/phase1/extract_experts.py:254-260``); the raw
    dequant multiplier is passed directly."""

    def __init__(self, layer: Layer, threads: int | None = None):
        self.lib = ref_lib()
        self.layer = layer
        L = layer
        self.threads = int(threads or os.cpu_count() or 1)
        self.h = self.lib.sb_cpu_create(1, L.E, L.K, L.I, L.E, self.threads)
        if not self.h:
            raise RuntimeError("sb_cpu_create failed")
        I, K = L.I, L.K
        for e in range(L.E):
            gq = np.ascontiguousarray(L.w13[e, :I])
            uq = np.ascontiguousarray(L.w13[e, I:])
            gs = np.ascontiguousarray(L.s13[e, :I])
            us = np.ascontiguousarray(L.s13[e, I:])
            dq = np.ascontiguousarray(L.w2[e])
            ds = np.ascontiguousarray(L.s2[e])
            rc = self.lib.sb_cpu_load_expert(self.h, 0, e, _ptr(gq), _ptr(gs), float(L.g13[e]),
                                             _ptr(uq), _ptr(us), float(L.g13[e]),
                                             _ptr(dq), _ptr(ds), float(L.g2[e]))
            if rc != 0:
                raise RuntimeError(f"sb_cpu_load_expert({e}) rc={rc}")

    def forward(self, hidden_bf16: np.ndarray, ids: np.ndarray, weights: np.ndarray) -> np.ndarray:
        hidden_bf16 = np.ascontiguousarray(hidden_bf16, dtype=np.uint16)
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        weights = np.ascontiguousarray(weights, dtype=np.float32)
        M, K = hidden_bf16.shape
        out = np.zeros((M, K), np.float32)
        rc = self.lib.sb_cpu_moe_forward(self.h, 0, _ptr(hidden_bf16), _ptr(ids), _ptr(weights),
                                         M, ids.shape[1], _ptr(out))
        if rc != 0:
            raise RuntimeError(f"sb_cpu_moe_forward rc={rc}")
        return out

    def close(self) -> None:
        if self.h:
            self.lib.sb_cpu_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# --------------------------------------------------------------------------
# the reference device test's deterministic fixture
# --------------------------------------------------------------------------

KAT_BLOCK_SCALES = np.array([0x3B, 0x2D, 0x35, 0x43], np.uint8)


def kat_sample(i: np.ndarray) -> np.ndarray:
    """``sample(i)`` of xpu_ops_smoke.cpp:93-96."""
    i = np.asarray(i, dtype=np.uint64)
    t = ((i * np.uint64(2654435761)) % np.uint64(10007)).astype(np.float64) / 10007.0
    return (-2.0 + 4.0 * t).astype(np.float32)


def kat_fp4(index: np.ndarray) -> np.ndarray:
    """``deterministic_fp4`` of xpu_ops_smoke.cpp:2229-2233."""
    index = np.asarray(index, dtype=np.uint64)
    mag = ((index * np.uint64(5) + np.uint64(1)) & np.uint64(7)).astype(np.uint8)
    sign = np.where(index % np.uint64(5) == 0, 8, 0).astype(np.uint8)
    return sign | mag


def kat_packed(elements: int) -> np.ndarray:
    """``fill_packed_fp4`` of xpu_ops_smoke.cpp:2235-2240."""
    i = np.arange(elements // 2, dtype=np.uint64)
    return (kat_fp4(2 * i) | (kat_fp4(2 * i + 1) << 4)).astype(np.uint8)


def kat_fixture(kind: str = "moe") -> dict:
    """Inputs of ``check_nvfp4_moe`` (xpu_ops_smoke.cpp:2260-2304, kind="moe")
    or of ``check_nvfp4_moe_grouped_blocks`` (:2454-2510, kind="blocks"),
    with bf16 activations."""
    if kind == "moe":
        M, E, top_k, K, I = 8, 8, 8, 256, 32
        hid_off, s2_off = 307, 2
    elif kind == "blocks":
        M, E, top_k, K, I = 100, 8, 4, 256, 64
        hid_off, s2_off = 911, 1
    else:
        raise ValueError(kind)
    hidden = f32_to_bf16_bits(kat_sample(np.arange(M * K) + hid_off) * np.float32(0.1)).reshape(M, K)
    ids = np.zeros((M, top_k), np.int32)
    w = np.zeros((M, top_k), np.float32)
    for m in range(M):
        for r in range(top_k):
            pair = m * top_k + r
            if kind == "moe":
                ids[m, r] = (m + r) % E
                w[m, r] = np.float32(1.0) / np.float32(top_k)
            else:
                e = 0 if pair % 5 < 3 else 1 + (pair % (E - 2))
                if pair % 37 == 0:
                    e = -1
                ids[m, r] = e
                w[m, r] = np.float32(0.1) + np.float32(0.05) * np.float32(r)
    if kind == "moe":
        ids[M - 1, top_k - 1] = -1
    w13 = kat_packed(E * 2 * I * K).reshape(E, 2 * I, K // 2)
    w2 = kat_packed(E * K * I).reshape(E, K, I // 2)
    s13 = KAT_BLOCK_SCALES[np.arange(E * 2 * I * K // 16) % 4].reshape(E, 2 * I, K // 16)
    s2 = KAT_BLOCK_SCALES[(np.arange(E * K * I // 16) + s2_off) % 4].reshape(E, K, I // 16)
    e = np.arange(E, dtype=np.float32)
    g13 = (np.float32(0.02) + np.float32(0.002) * e).astype(np.float32)
    g2 = (np.float32(0.03) + np.float32(0.002) * e).astype(np.float32)
    layer = Layer(E, K, I, w13, s13, g13, w2, s2, g2)
    return {"hidden": hidden, "ids": ids, "weights": w, "layer": layer, "top_k": top_k}


def kat_reference_loop(fx: dict) -> np.ndarray:
    """The fp32 CPU loop of check_nvfp4_moe (xpu_ops_smoke.cpp:2316-2348):
    W = (e2m1 * e4m3) * g, route outputs summed in (token, k) order."""
    L = fx["layer"]
    hidden = bf16_bits_to_f32(fx["hidden"])
    ids, w = fx["ids"], fx["weights"]
    M, K = hidden.shape
    ref = np.zeros((M, K), np.float32)

    def wmat(q, sf, g):
        codes = unpack_fp4(q)
        v = np.where(codes & 8, -1.0, 1.0).astype(np.float32) * E2M1_VALUES[codes & 7]
        s = np.repeat(e4m3_decode(sf), BLOCK, axis=-1)
        return ((v * s).astype(np.float32) * np.float32(g)).astype(np.float32)

    for m in range(M):
        for r in range(ids.shape[1]):
            e = int(ids[m, r])
            if e < 0 or e >= L.E:
                continue
            W13 = wmat(L.w13[e], L.s13[e], L.g13[e])
            # np.cumsum in float32 accumulates sequentially, as the C loop does
            gu = np.cumsum((W13 * hidden[m][None, :]).astype(np.float32), axis=1,
                           dtype=np.float32)[:, -1]
            g = gu[:L.I].astype(np.float64)
            act = ((g * (1.0 / (1.0 + np.exp(-g)))).astype(np.float32) * gu[L.I:]).astype(np.float32)
            W2 = wmat(L.w2[e], L.s2[e], L.g2[e])
            y = np.cumsum((W2 * act[None, :]).astype(np.float32), axis=1, dtype=np.float32)[:, -1]
            ref[m] = (ref[m] + (w[m, r] * y).astype(np.float32)).astype(np.float32)
    return ref
