"""A step of consecutive routed-MoE layers chained through the decoder hop.

Layer l takes the normalized input x_l and the bf16 residual stream r; its
combine is all-reduced over the group and followed, in the same launch, by the
hop epilogue: r <- bf16(group sum + r), x_{l+1} = RMSNorm(r) * gamma_l
(``qwen3_5/sm103/hop/__init__.py:431``). The whole step is one C call
(``mm_stack_forward``) issuing every layer's PDL-chained launches on one stream,
as the reference's megakernel forward calls ``moe.step`` once per MoE layer
(``deepseek_v41/moe/step.py:101``). The layers share the per-step buffers (logits,
top-k, route record, rows): every kernel writes them only after its PDL wait,
i.e. after the previous layer's last launch has completed.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import check, lib
from .moe import RoutedMoE, _ptr, _stream


class MoEStack:
    """``layers[i]`` (a ``RoutedMoE``, full or an EP window) with router weight
    ``router_weights[i]`` (bf16 [E, H]), bias ``biases[i]`` (fp32 [E] or None)
    and RMSNorm weight ``gammas[i]`` (bf16 [H], the norm after layer i)."""

    def __init__(self, layers: Sequence[RoutedMoE], router_weights: Sequence[torch.Tensor],
                 gammas: Sequence[torch.Tensor], comm, *, biases: Optional[Sequence[Optional[torch.Tensor]]] = None,
                 routed_scaling_factor: float = 1.0, score: str = "sigmoid", renormalize=True,
                 renormalize_epsilon: float = 0.0):
        n = len(layers)
        if n < 1 or len(router_weights) != n or len(gammas) != n or (biases is not None and len(biases) != n):
            raise ValueError("layers, router_weights, gammas (and biases) must have one entry per layer")
        first = layers[0]
        for m in layers:
            if (m.hidden, m.top_k, m.router_experts, m.max_rows) != (first.hidden, first.top_k, first.router_experts,
                                                                      first.max_rows):
                raise ValueError("every layer of a stack needs the same hidden, top_k, router_experts and max_rows")
        if comm.hidden != first.hidden or comm.max_tokens < first.max_rows:
            raise ValueError("comm must serve the stack's hidden size and max_rows tokens")
        if score not in _lib.SCORES:
            raise ValueError(f"unknown score function {score!r}")
        for i, (w, g) in enumerate(zip(router_weights, gammas)):
            if w.dtype != torch.bfloat16 or tuple(w.shape) != (first.router_experts, first.hidden):
                raise ValueError(f"router_weights[{i}]: expected bf16 [{first.router_experts}, {first.hidden}]")
            if g.dtype != torch.bfloat16 or tuple(g.shape) != (first.hidden,):
                raise ValueError(f"gammas[{i}]: expected bf16 [{first.hidden}]")
        self.layers, self.router_weights, self.gammas = list(layers), list(router_weights), list(gammas)
        self.biases = list(biases) if biases is not None else [None] * n
        self.comm = comm
        self.scale, self.score, self.renormalize, self.eps = (float(routed_scaling_factor), score,
                                                              renormalize, float(renormalize_epsilon))
        self.hidden, self.top_k, self.max_rows = first.hidden, first.top_k, first.max_rows
        dev = first.device
        self.device = dev
        tmax, k, h = self.max_rows, self.top_k, self.hidden
        self.logits = torch.empty((tmax, first.router_experts), dtype=torch.float32, device=dev)
        self.weights = torch.empty((tmax, k), dtype=torch.float32, device=dev)
        self.ids = torch.empty((tmax, k), dtype=torch.int32, device=dev)
        self.permuted = torch.empty((tmax, k), dtype=torch.int32, device=dev)
        self.record = torch.empty((max(m.route_words_max for m in layers),), dtype=torch.int32, device=dev)
        self.rows = torch.empty((max(m.rows_capacity for m in layers), h), dtype=torch.bfloat16, device=dev)
        self.norm = [torch.empty((tmax, h), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self._arr = None
        self._key = None

    def _args(self, tokens: int, x: torch.Tensor, residual: torch.Tensor):
        key = (tokens, x.data_ptr(), residual.data_ptr())
        if self._key == key:
            return self._arr
        n = len(self.layers)
        arr = (_lib.MMStackLayer * n)()
        for i, m in enumerate(self.layers):
            a = arr[i].args
            arr[i].layer = m._handle
            a.x = x.data_ptr() if i == 0 else self.norm[(i - 1) & 1].data_ptr()
            a.router_w = self.router_weights[i].data_ptr()
            a.logits = None
            a.logits_out = self.logits.data_ptr()
            a.bias = _ptr(self.biases[i])
            a.num_valid = None
            a.score_func = _lib.SCORES[self.score]
            a.renormalize = _lib.renorm_code(self.renormalize)
            a.routed_scaling = self.scale
            a.renorm_eps = self.eps
            a.tokens = tokens
            a.weights, a.ids, a.permuted = self.weights.data_ptr(), self.ids.data_ptr(), self.permuted.data_ptr()
            a.record, a.rows = self.record.data_ptr(), self.rows.data_ptr()
            a.out = self.norm[i & 1].data_ptr()
            a.partial = None
            a.comm = self.comm.handle
            a.residual = residual.data_ptr()
            a.gamma = self.gammas[i].data_ptr()
            a.norm_eps = self.comm.eps
            a.residual_out = residual.data_ptr()
        self._arr, self._key = arr, key
        return arr

    def forward(self, x: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        """One step: ``x`` bf16 [T, H] is layer 0's normalized input, ``residual``
        bf16 [T, H] is updated in place. Returns the normalized output of the
        last layer (a view of a stack-owned buffer, valid until the next call)."""
        for name, t in (("x", x), ("residual", residual)):
            if t.dtype != torch.bfloat16 or t.dim() != 2 or t.size(1) != self.hidden or not t.is_contiguous():
                raise ValueError(f"{name}: expected a contiguous bf16 [T, {self.hidden}] tensor")
        tokens = x.size(0)
        if residual.size(0) != tokens or not 1 <= tokens <= self.max_rows:
            raise ValueError(f"{tokens} tokens (residual {residual.size(0)}) outside 1..{self.max_rows}")
        arr = self._args(tokens, x, residual)
        check(lib().mm_stack_forward(arr, len(self.layers), _stream(self.device)), "mm_stack_forward")
        return self.norm[(len(self.layers) - 1) & 1][:tokens]

    def check(self) -> None:
        """Synchronize and raise if any layer's or the hop's bounded device wait timed out."""
        for m in self.layers:
            m.check()
        self.comm.check()
