"""A drop-in for the reference's routed-expert GEMM pair.

``RoutedExpertGemm`` here takes the constructor and call signatures of
sgl_nvidia_mega.deepseek_v41.sm103.moe.routed_expert_gemm.RoutedExpertGemm
(routed_expert_gemm.py:537-554, __call__ :703, gate_topk_and_gemms :776) and
the members its caller, MoeSlot (deepseek_v41/moe/routed.py:82-239), reads, so
that routed.py can construct this class in place of the reference's with the
same arguments (routed.py:391-404) and call it as it does (routed.py:209-230):

    gemm(x_q, x_s, ids, w)                               -> (rows, weights, permuted)
    gemm.gate_topk_and_gemms(x_q, x_s, logits, bias, scale, num_valid, alt=...,
                             renormalize_epsilon=..., ids_out=..., x=..., early=...)
                                                         -> (rows, weights, permuted, ids)

The weights are the ones SGLang hands the reference: the processed TRT-LLM-gen
MXFP4 layout (rows permuted, [w3; w1] halves, scales interleaved), re-laid once
into canonical copies at construction (``megamoe.layouts``); ``layout="canonical"``
takes SGLang's unprocessed FusedMoE layout as is. Routing scores with the
reference's DSV4.1 rule, sqrt(softplus) + bias, renormalized, scaled; at the
reference gate's top-6 / top-3 with that gate's own numerics
(score="sqrtsoftplus_dsv41": ids and weights bit-equal to gate_topk.cu's).

The reference's slot options (gate_topk, gate_route, gate_route_quant,
gemm2_pipe, gemm2_registers) choose among its kernel builds; this library has
one chain that serves all of them (top-k, route and quantization in its own
front launches), so they are accepted and recorded, and the ``serves_*`` /
``supports*`` answers follow the chain's limits instead.
"""

from __future__ import annotations

from typing import Optional

import torch

from .moe import RoutedMoE


class RoutedExpertGemm:
    """The reference's RoutedExpertGemm interface over ``megamoe.RoutedMoE``."""

    def __init__(
        self,
        w13,
        w13_scale,
        w2,
        w2_scale,
        clamp,
        top_k: int,
        max_rows: int,
        gate_topk: bool = False,
        router_experts: Optional[int] = None,
        expert_offset: int = 0,
        gemm2_pipe: bool = False,
        gemm2_registers: int = 0,
        gate_route: bool = False,
        gate_route_quant: bool = False,
        deal_group: int = -1,
        *,
        layout: str = "trtllm",
        halves: str = "w3_w1",
        score: Optional[str] = None,
    ):
        if layout not in ("trtllm", "canonical"):
            raise ValueError(f"layout {layout!r}: 'trtllm' (processed) or 'canonical'")
        w13, w13_scale = w13.view(torch.uint8), w13_scale.view(torch.uint8)
        w2, w2_scale = w2.view(torch.uint8), w2_scale.view(torch.uint8)
        kwargs = dict(clamp=clamp, router_experts=router_experts, expert_offset=expert_offset, deal_group=deal_group)
        if layout == "trtllm":
            self.moe = RoutedMoE.from_trtllm(w13, w13_scale, w2, w2_scale, top_k, max_rows, halves=halves, **kwargs)
        else:
            self.moe = RoutedMoE(w13, w13_scale, w2, w2_scale, top_k, max_rows, **kwargs)
        self.clamp = clamp
        self.top_k, self.max_rows = int(top_k), int(max_rows)
        self.experts = self.moe.experts
        self.router_experts = self.moe.router_experts
        self.expert_offset = self.moe.expert_offset
        self.deal_group = self.moe.deal_group
        self.hidden = self.moe.hidden
        # the reference gate's own numerics where its gate_topk.cu has a build
        # (top-6 / top-3: ids and weights equal bit for bit), else sqrt(softplus)
        # with this library's IEEE numerics
        self.score = score if score is not None else (
            "sqrtsoftplus_dsv41" if self.top_k in (3, 6) else "sqrtsoftplus")
        self.gemm2_pipe, self.gemm2_registers = bool(gemm2_pipe), int(gemm2_registers)
        # markers MoeSlot tests for "this build exists": the chain serves every slot
        self.gate_topk_kernel = self.gate_route_kernel = self.gate_route_quant_kernel = self.moe
        self.slots = dict(gate_topk=bool(gate_topk), gate_route=bool(gate_route),
                          gate_route_quant=bool(gate_route_quant))

    # ---------------------------------------------------------------- the calls
    def _scale_2d(self, x_quant, x_scale):
        rows = x_quant.size(0)
        need = rows * self.hidden // 32
        if x_scale.dim() == 2 and tuple(x_scale.shape) == (rows, self.hidden // 32):
            return x_scale
        return x_scale.reshape(-1)[:need].view(rows, self.hidden // 32)

    def __call__(self, x_quant, x_scale, topk_ids, topk_weights):
        """Route + gate_up + down on the current stream (routed_expert_gemm.py:703):
        the deferred-finalize triple (rows, weights, slot -> permuted row)."""
        return self.moe(x_quant, self._scale_2d(x_quant, x_scale), topk_ids, topk_weights)

    def gate_topk_and_gemms(self, x_quant, x_scale, logits, bias, routed_scaling_factor: float, num_valid,
                            alt=None, renormalize_epsilon: float = 0.0, ids_out=None, x=None, early: bool = False):
        """``__call__`` from the router's fp32 logits (routed_expert_gemm.py:776):
        (rows, top-k weights, slot -> row, top-k ids). With ``x`` (bf16) the
        chain quantizes the routed input itself and x_quant / x_scale are unused."""
        if x is None:
            x_scale = self._scale_2d(x_quant, x_scale)
        else:
            x_quant = x_scale = None
        return self.moe.gate_topk_and_gemms(x_quant, x_scale, logits, bias, routed_scaling_factor, num_valid, alt,
                                            renormalize_epsilon, ids_out, x, early, score=self.score)

    def bind_early_release(self, release: int) -> None:
        """The reference's early-router hand-off (routed_expert_gemm.py:872): the
        front launch here is always released early by its predecessor (PDL)."""

    # ------------------------------------------------------------- capabilities
    def _rows_ok(self, rows: int) -> bool:
        return 1 <= rows <= self.max_rows

    def supports_inputs(self, x_quant, x_scale) -> bool:
        rows = x_quant.size(0)
        return (self._rows_ok(rows) and tuple(x_quant.shape) == (rows, self.hidden) and x_quant.element_size() == 1
                and x_quant.is_contiguous() and x_scale is not None and x_scale.element_size() == 1
                and x_scale.is_contiguous() and x_scale.numel() >= rows * self.hidden // 32)

    def supports(self, x_quant, x_scale, topk_ids, topk_weights) -> bool:
        return (self.supports_inputs(x_quant, x_scale) and topk_ids.dim() == 2 and topk_ids.size(1) == self.top_k
                and topk_ids.size(0) == x_quant.size(0) and topk_weights.dtype == torch.float32)

    def supports_gate_topk(self, logits: torch.Tensor, bias: torch.Tensor) -> bool:
        return (logits.dtype == torch.float32 and logits.dim() == 2 and logits.is_contiguous()
                and logits.size(1) == self.router_experts and self._rows_ok(logits.size(0))
                and (bias is None or (bias.dtype == torch.float32 and bias.numel() == self.router_experts)))

    def serves_gate_route(self, rows: int, input_ids=None) -> bool:
        return self._rows_ok(rows) and (input_ids is None or input_ids.numel() >= rows)

    def serves_gate_route_quant(self, rows: int, input_ids=None, x=None) -> bool:
        return self.serves_gate_route(rows, input_ids) and (
            x is None or (x.dtype == torch.bfloat16 and tuple(x.shape) == (rows, self.hidden) and x.is_contiguous()
                          and x.data_ptr() % 16 == 0))
