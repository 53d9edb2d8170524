"""vLLM routed-experts hook adapter for the B200 path.

The reference reaches its expert kernels from vLLM through
``HybridRoutedExperts(RoutedExperts).forward_modular(x, topk_weights,
topk_ids, shared_experts=None, shared_experts_input=None)``
(``src/phase4/src/shooting_brake_vllm/routed_experts.py:2312-2397``),
registered out of tree as ``RoutedExperts`` through the
``vllm.general_plugins`` entry point (``src/phase4/src/shooting_brake_vllm/
__init__.py:318-344``, ``pyproject.toml:45-46``).

:class:`RoutedExpertsB200` keeps that call shape. Its forward is the custom op
``torch.ops.sbb200.nvfp4_moe`` on device-resident weights, stream-ordered
with no host synchronisation, so a vLLM decode step that holds it can be
captured and replayed as a CUDA graph. Weights are taken in the bank layout
(w13 rows ``[gate; up]``, linear e4m3 scales, per-expert fp32 dequant
multiplier); a layer whose w13 halves are stored ``[up; gate]`` (the
FlashInfer ordering the reference checks at ``routed_experts.py:1757-1760``)
is reordered once at construction.

:func:`register` installs the adapter into vLLM when vLLM provides the
``RoutedExperts`` pluggable layer with a ``forward_modular`` method (the
reference pins vLLM 0.26, ``pyproject.toml:36``); releases without
it (0.22 aliases ``RoutedExperts`` to ``FusedMoE``) return False.
"""

from __future__ import annotations

import torch

from . import nvfp4_moe


class RoutedExpertsB200:
    """One MoE layer's routed experts on a B200.

    Args (E experts, d hidden, I intermediate):
      w13: uint8 [E, 2I, d/2] packed e2m1, rows [gate; up] (or [up; gate] with
        ``w13_is_up_gate=True``).
      w13_scale: uint8 [E, 2I, d/16] e4m3 block scales, linear layout.
      w13_global: float32 [E] dequant multiplier (W = e2m1 * e4m3 * g).
      w2, w2_scale, w2_global: the down projection, [E, d, I/2], [E, d, I/16], [E].
      expert_map: optional int32 [n_global] mapping a global expert id to its
        local row here, -1 where the expert lives elsewhere (the reference's
        per-card slot map, ``routed_experts.py:354-382``); routes mapped to -1
        contribute nothing.
      multiply_router_weight: scale each route by its router weight.
    """

    def __init__(self, w13: torch.Tensor, w13_scale: torch.Tensor, w13_global: torch.Tensor,
                 w2: torch.Tensor, w2_scale: torch.Tensor, w2_global: torch.Tensor, *,
                 w13_is_up_gate: bool = False, expert_map: torch.Tensor | None = None,
                 multiply_router_weight: bool = True, shared: tuple | None = None):
        if w13.dim() != 3 or w13.size(1) % 2:
            raise ValueError("sbb200: w13 must be uint8 [E,2I,d/2]")
        if w13_is_up_gate:
            half = w13.size(1) // 2
            w13 = torch.cat([w13[:, half:], w13[:, :half]], dim=1).contiguous()
            w13_scale = torch.cat([w13_scale[:, half:], w13_scale[:, :half]], dim=1).contiguous()
        self.w13, self.w13_scale = w13.contiguous(), w13_scale.contiguous()
        self.w13_global = w13_global.float().contiguous()
        self.w2, self.w2_scale = w2.contiguous(), w2_scale.contiguous()
        self.w2_global = w2_global.float().contiguous()
        if expert_map is not None:
            expert_map = expert_map.to(device=w13.device, dtype=torch.int32).contiguous()
            if expert_map.dim() != 1:
                raise ValueError("sbb200: expert map must be int32 [n_global]")
        self.expert_map = expert_map
        self.multiply_router_weight = multiply_router_weight
        self.num_routed = self.w13.size(0)
        self.shared_chunks = 0
        if shared is not None:
            self._append_shared(*shared)

    def _append_shared(self, w13, w13_scale, w13_global, w2, w2_scale, w2_global) -> None:
        """Fuse one NVFP4 shared expert (w13 [2Is, d/2] gate rows then up
        rows, w2 [d, Is/2], with their scales and scalar globals) into the
        routed weights. SwiGLU is elementwise over the intermediate dimension,
        so with Is = n * I the shared expert is exactly n experts of
        intermediate I (gate/up row blocks, down column blocks on 16-element
        scale boundaries); they are appended after the routed experts and
        every token routes to all n with weight 1 (or its shared gate)."""
        I = self.w13.size(1) // 2
        Is = w13.size(0) // 2
        if Is % I:
            raise ValueError(f"sbb200: shared intermediate {Is} is not a multiple of {I}")
        n = Is // I
        dev = self.w13.device
        g13 = w13_global.reshape(-1)[:1].float().to(dev)
        g2 = w2_global.reshape(-1)[:1].float().to(dev)
        cw13, cs13, cw2, cs2 = [], [], [], []
        for c in range(n):
            rows = slice(c * I, (c + 1) * I)
            up = slice(Is + c * I, Is + (c + 1) * I)
            cw13.append(torch.cat([w13[rows], w13[up]]).to(dev))
            cs13.append(torch.cat([w13_scale[rows], w13_scale[up]]).to(dev))
            cw2.append(w2[:, c * (I // 2):(c + 1) * (I // 2)].to(dev))
            cs2.append(w2_scale[:, c * (I // 16):(c + 1) * (I // 16)].to(dev))
        self.w13 = torch.cat([self.w13, torch.stack(cw13)]).contiguous()
        self.w13_scale = torch.cat([self.w13_scale, torch.stack(cs13)]).contiguous()
        self.w2 = torch.cat([self.w2, torch.stack(cw2)]).contiguous()
        self.w2_scale = torch.cat([self.w2_scale, torch.stack(cs2)]).contiguous()
        self.w13_global = torch.cat([self.w13_global, g13.expand(n)]).contiguous()
        self.w2_global = torch.cat([self.w2_global, g2.expand(n)]).contiguous()
        self.shared_chunks = n
        self._shared_ids = torch.arange(self.num_routed, self.num_routed + n, dtype=torch.int32,
                                        device=dev)

    @classmethod
    def from_layer(cls, layer, scale_layout: str = "swizzled", **kw) -> "RoutedExpertsB200":
        """Build from a vLLM NVFP4 MoE layer after weight loading: ``w13_weight``
        [E, 2I, d/2], ``w13_weight_scale``, ``w2_weight``, ``w2_weight_scale``
        and the per-expert globals (``routed_experts.py:1529-1552, 1744-1753``).

        Block scales: vLLM keeps them swizzled for its CUTLASS/FlashInfer
        kernels (128-row x 4-column tiles, padded; ``swizzle_blockscale``), so
        by default they are converted to linear order once, here, as the
        reference's hook does before its CPU tier reads them
        (``routed_experts.py:1926-1938``, vLLM ``convert_swizzled_to_linear``).
        ``scale_layout="linear"`` takes them as they are (bank layout).

        Globals: the dequant multiplier g (W = e2m1 * e4m3 * g) comes from
        the quant config when the layer has one: ``alpha_or_gscale`` of w1/w2
        is g divided by the activation global (vLLM's g1/g2 alphas,
        ``expert_bank.py:270-295``), so g = alpha * a_gscale. Otherwise from
        ``w13_weight_scale_2`` / ``w2_weight_scale_2`` ([E], or [E, 2] with
        separate w1/w3 globals, of which vLLM keeps the first column and
        warns when they differ; the same is done here).

        A ``_w13_is_reordered()`` method, when present, says whether the w13
        halves are ``[up; gate]``."""
        reordered = getattr(layer, "_w13_is_reordered", None)
        kw.setdefault("w13_is_up_gate", bool(reordered()) if callable(reordered) else False)

        def t(name):
            v = getattr(layer, name)
            return v.data if hasattr(v, "data") else v

        w13, w2 = t("w13_weight"), t("w2_weight")
        E, two_i, half_d = w13.shape
        d, I = half_d * 2, two_i // 2
        s13, s2 = t("w13_weight_scale"), t("w2_weight_scale")
        if scale_layout == "swizzled":
            s13 = unswizzle_block_scales(s13, two_i, d // 16)
            s2 = unswizzle_block_scales(s2, d, I // 16)
        elif scale_layout != "linear":
            raise ValueError("sbb200: scale_layout must be 'swizzled' or 'linear'")
        g13, g2 = layer_globals(layer, E)
        return cls(w13, s13, g13.to(w13.device), w2, s2, g2.to(w13.device), **kw)

    def device_errors(self) -> int:
        """Device error word of this layer's last forward on the current
        stream (bit 0: a kernel wait passed its limit and that result is not
        valid). Synchronises the stream."""
        from . import nvfp4_moe_device_errors
        return nvfp4_moe_device_errors(self.w13.device)

    @property
    def num_experts(self) -> int:
        return self.num_routed

    def forward_modular(self, x: torch.Tensor, topk_weights: torch.Tensor,
                        topk_ids: torch.Tensor, shared_experts=None,
                        shared_experts_input: torch.Tensor | None = None,
                        shared_gate: torch.Tensor | None = None) -> torch.Tensor:
        """Routed-expert output [M, d] in x's dtype, plus the shared expert's:
        a fused NVFP4 shared expert (``shared=`` at construction) runs inside
        the same grouped call, weighted by ``shared_gate`` [M] (1 if None); a
        shared-expert module given here is run beside it and added (the
        hook's ``Y_local + Y_routed`` sum, ``routed_experts.py:2517-2531``)."""
        ids = topk_ids if topk_ids.dtype == torch.int32 else topk_ids.to(torch.int32)
        if self.expert_map is not None:
            valid = (ids >= 0) & (ids < self.expert_map.numel())
            ids = torch.where(valid, self.expert_map[ids.clamp(0, self.expert_map.numel() - 1)],
                              torch.full_like(ids, -1))
        w = topk_weights if topk_weights.dtype == torch.float32 else topk_weights.float()
        if self.shared_chunks:
            M, n = ids.shape[0], self.shared_chunks
            ids = torch.cat([ids, self._shared_ids.expand(M, n)], dim=1)
            sw = (torch.ones((M, 1), dtype=torch.float32, device=w.device) if shared_gate is None
                  else shared_gate.reshape(M, 1).float())
            w = torch.cat([w, sw.expand(M, n)], dim=1)
        y = nvfp4_moe(x, ids.contiguous(), w.contiguous(), self.w13, self.w13_scale,
                      self.w13_global, self.w2, self.w2_scale, self.w2_global,
                      multiply_router_weight=self.multiply_router_weight, out_dtype=x.dtype)
        if shared_experts is not None:
            y = y + shared_experts(shared_experts_input if shared_experts_input is not None
                                   else x)
        return y

    __call__ = forward_modular


def unswizzle_block_scales(sf: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """Linear [E, rows, cols] e4m3 block scales (uint8) from vLLM's swizzled
    layout (``swizzle_blockscale``: per expert, rows padded to 128 and
    columns to 4, stored as [rows/128, cols/4, 32, 4, 4] with element
    (m, k, r, q, c) = linear[128 m + 32 q + r, 4 k + c]); the inverse of
    vLLM's ``convert_swizzled_to_linear``, expert by expert. Runs once, with
    torch ops on the tensor's device."""
    if sf.dim() == 2:
        sf = sf.unsqueeze(0)
    E = sf.shape[0]
    rp, cp = -(-rows // 128) * 128, -(-cols // 4) * 4
    flat = sf.reshape(E, -1)
    if flat.shape[1] != rp * cp:
        raise ValueError(f"sbb200: swizzled block scales of {tuple(sf.shape)} do not cover "
                         f"[{E}, {rp}, {cp}] (rows {rows}, cols {cols} padded to 128 x 4)")
    raw = flat.view(torch.uint8) if flat.dtype != torch.uint8 else flat
    tiles = raw.reshape(E, rp // 128, cp // 4, 32, 4, 4)
    lin = tiles.permute(0, 1, 4, 3, 2, 5).reshape(E, rp, cp)
    return lin[:, :rows, :cols].contiguous()


def layer_globals(layer, E: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-expert fp32 dequant multipliers (g13, g2) of a vLLM NVFP4 MoE layer:
    alpha * a_gscale from the quant config when present (vLLM's alphas are the
    weight global divided by the activation global), else the
    ``*_weight_scale_2`` tensors ([E] or [E, 2] -> first column)."""
    import warnings

    qc = getattr(getattr(layer, "quant_method", None), "moe_quant_config", None)
    desc = [getattr(qc, n, None) for n in ("_w1", "_w2", "_a1", "_a2")] if qc else []
    vals = [getattr(x, "alpha_or_gscale", None) for x in desc]
    if len(vals) == 4 and all(v is not None for v in vals):
        out = []
        for alpha, a_g in ((vals[0], vals[2]), (vals[1], vals[3])):
            alpha = alpha.detach().float().reshape(-1)
            a_g = a_g.detach().float().reshape(-1).to(alpha.device)
            if alpha.numel() != E or a_g.numel() not in (1, E):
                raise ValueError("sbb200: quant config alphas must be [E] and activation "
                                 "globals [1] or [E]")
            out.append((alpha * a_g).contiguous())
        return out[0], out[1]

    def g(name):
        v = getattr(layer, name)
        v = (v.data if hasattr(v, "data") else v).detach().float()
        if v.dim() == 2 and v.shape == (E, 2):
            if not torch.equal(v[:, 0], v[:, 1]):
                warnings.warn(f"sbb200: {name} holds different w1 and w3 globals; using the "
                              "first (as vLLM does)", stacklevel=3)
            v = v[:, 0]
        v = v.reshape(-1)
        if v.numel() != E:
            raise ValueError(f"sbb200: {name} must hold E (or E x 2) values")
        return v.contiguous()

    return g("w13_weight_scale_2"), g("w2_weight_scale_2")


_registered = None


def register() -> bool:
    """Register a vLLM ``RoutedExperts`` subclass whose ``forward_modular``
    runs this path, when the installed vLLM has that pluggable layer. Returns
    False (and changes nothing) when it does not. Calling it again is a no-op."""
    global _registered
    try:
        from vllm.model_executor.custom_op import PluggableLayer, op_registry_oot
    except ImportError:
        return False
    try:  # the module the reference imports it from (routed_experts.py:13)
        from vllm.model_executor.layers.fused_moe.routed_experts import RoutedExperts
    except ImportError:
        try:
            from vllm.model_executor.layers.fused_moe import RoutedExperts  # type: ignore
        except ImportError:
            return False
    if not hasattr(RoutedExperts, "forward_modular"):
        # older vLLM (e.g. 0.22): RoutedExperts is FusedMoE without the
        # modular forward the hook overrides
        return False

    if _registered is None:
        class B200RoutedExperts(RoutedExperts):  # pragma: no cover - needs that vLLM layer
            def forward_modular(self, x, topk_weights, topk_ids, shared_experts=None,
                                shared_experts_input=None):
                impl = getattr(self, "_sbb200", None)
                if impl is None:
                    impl = self._sbb200 = RoutedExpertsB200.from_layer(self)
                return impl.forward_modular(x, topk_weights, topk_ids, shared_experts,
                                            shared_experts_input)

        _registered = B200RoutedExperts

    existing = op_registry_oot.get("RoutedExperts")
    if existing is None:
        PluggableLayer.register_oot(_registered, name="RoutedExperts")
    elif existing is not _registered:
        raise RuntimeError("cannot install the B200 adapter: RoutedExperts is already replaced")
    return True
