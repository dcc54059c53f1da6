"""Host-side mirror of the reference's routed-MoE step API over libmegamoe.

RoutedMoE keeps the shape of sgl-nvidia-mega's RoutedExpertGemm
(deepseek_v41/sm103/moe/routed_expert_gemm.py:534-870) and of the deferred
finalize that consumes its output (deepseek_v41/sm103/all_reduce_mhc.py:1484,
glm5_3/sm103/moe/finalize.py):

  * ``__call__(x_quant, x_scale, topk_ids, topk_weights)`` -> the
    deferred-finalize triple (gemm2 rows, weights, slot -> row), positionally
    like RoutedExpertGemm.__call__ (routed_expert_gemm.py:703);
  * ``gate_topk_and_gemms(x_quant, x_scale, logits, bias, routed_scaling_factor,
    num_valid, alt=None, renormalize_epsilon=0.0, ids_out=None, x=None,
    early=False)`` -> (rows, weights, permuted, ids), like
    RoutedExpertGemm.gate_topk_and_gemms (:776);
  * ``finalize(rows, weights, permuted)`` -> the combined bf16 MoE output;
  * ``forward(x, router_weight=..., bias=...)`` -> one whole MoE step.

The routed input is MXFP8 (x_quant E4M3 codes [T, H], x_scale E8M0 [T, H/32],
as SGLang's quantize_routed_input hands it to the reference) or bf16 (x_quant a
bf16 [T, H] tensor with x_scale None, or ``x=`` in gate_topk_and_gemms: the
chain quantizes it itself, as the reference's gate_route_quant slot does).
Weights are the canonical layout (FlashInfer-shuffled ones go through
``from_trtllm``); errors raise ValueError (shape/argument) or RuntimeError
(device), as the reference's do.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import check, lib


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _expect(t: torch.Tensor, shape: Sequence[int], name: str, nbytes: int = 1) -> torch.Tensor:
    if tuple(t.shape) != tuple(shape) or t.element_size() != nbytes or not t.is_contiguous():
        raise ValueError(
            f"{name}: expected a contiguous {tuple(shape)} {nbytes}-byte tensor, "
            f"got {tuple(t.shape)} {t.dtype}"
        )
    return t


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8) if t.element_size() == 1 and t.dtype != torch.uint8 else t


class RoutedMoE:
    """The routed-MoE chain bound to one MoE layer's FP4 weights.

    Weights (canonical layout, read in place; see include/megamoe.h):
      w13 u8 [E, 2I, H/2], w13_scale u8 [E, 2I, H/32], w2 u8 [E, H, I/2],
      w2_scale u8 [E, H, I/32]; ``shared`` = the same four tensors with E = 1.
    ``weight_format="nvfp4"``: the scales are E4M3 per 16 ([E, 2I, H/16],
    [E, H, I/16]), ``w13_scale_2`` / ``w2_scale_2`` are the fp32 [E] per-expert
    second-level scales, ``input_scale`` the static (FC1, FC2) input scales,
    and ``shared`` carries six tensors (the four, then its two scale_2 [1]).
    ``router_experts``: the router's expert count (default: the local ones);
    ``expert_offset``: router id of local expert 0 (expert parallelism);
    ``deal_group`` (0 or 1; -1 off): balanced dealing, the layer holds every
    expert and keeps the step's distinct experts of even (0) or odd (1) rank
    in id order (routed_expert_gemm.py:557-599, route.cuh:39-46);
    ``clamp``: fp32 [E] SwiGLU clamp limits or None;
    ``act_terms``: MXFP4 terms per activation (1..3, default 3: each term
    quantizes the residual of the previous ones; about 1e-3 relative).
    """

    def __init__(
        self,
        w13: torch.Tensor,
        w13_scale: torch.Tensor,
        w2: torch.Tensor,
        w2_scale: torch.Tensor,
        top_k: int,
        max_rows: int,
        *,
        clamp: Optional[torch.Tensor] = None,
        router_experts: Optional[int] = None,
        expert_offset: int = 0,
        deal_group: int = -1,
        shared: Optional[Sequence[torch.Tensor]] = None,
        shared_clamp: Optional[torch.Tensor] = None,
        act_terms: int = 3,
        weight_format: str = "mxfp4",
        w13_scale_2: Optional[torch.Tensor] = None,
        w2_scale_2: Optional[torch.Tensor] = None,
        input_scale: Optional[Sequence[float]] = None,
    ):
        if weight_format not in ("mxfp4", "nvfp4"):
            raise ValueError(f"unknown weight format {weight_format!r}")
        nv = weight_format == "nvfp4"
        block = 16 if nv else 32
        w13, w13_scale, w2, w2_scale = (_u8(t) for t in (w13, w13_scale, w2, w2_scale))
        if w13.dim() != 3:
            raise ValueError(f"w13: expected [E, 2I, H/2], got {tuple(w13.shape)}")
        experts, two_i, half_h = w13.shape
        hidden, inter = 2 * half_h, two_i // 2
        _expect(w13, (experts, 2 * inter, hidden // 2), "w13")
        _expect(w13_scale, (experts, 2 * inter, hidden // block), "w13_scale")
        _expect(w2, (experts, hidden, inter // 2), "w2")
        _expect(w2_scale, (experts, hidden, inter // block), "w2_scale")
        if nv:
            if w13_scale_2 is None or w2_scale_2 is None or input_scale is None or len(input_scale) != 2:
                raise ValueError("nvfp4 needs w13_scale_2, w2_scale_2 and input_scale=(fc1, fc2)")
            for name, t in (("w13_scale_2", w13_scale_2), ("w2_scale_2", w2_scale_2)):
                _expect(t, (experts,), name, 4)
                if t.dtype != torch.float32 or t.device != w13.device:
                    raise ValueError(f"{name} must be fp32 [E] on the weights' device")
        self.weight_format = weight_format
        if not w13.is_cuda:
            raise ValueError("weights must be CUDA tensors")
        self.device = w13.device
        self.hidden, self.inter, self.experts = hidden, inter, experts
        self.router_experts = experts if router_experts is None else int(router_experts)
        self.expert_offset = int(expert_offset)
        self.deal_group = int(deal_group)
        if self.deal_group not in (-1, 0, 1):
            raise ValueError(f"deal_group {deal_group}: 0, 1 or -1 (off)")
        if self.deal_group >= 0 and (self.expert_offset != 0 or experts != self.router_experts):
            raise ValueError(f"balanced dealing needs all {self.router_experts} experts and expert_offset 0")
        self.top_k = int(top_k)
        self.max_rows = int(max_rows)
        self.act_terms = int(act_terms)
        if clamp is not None:
            _expect(clamp, (experts,), "clamp", 4)
            if clamp.dtype != torch.float32:
                raise ValueError("clamp must be fp32 [E]")
        keep = [w13, w13_scale, w2, w2_scale, clamp]
        desc = _lib.MMLayerDesc()
        desc.hidden, desc.intermediate, desc.experts = hidden, inter, experts
        desc.router_experts = self.router_experts
        # the library's expert_offset: negative selects balanced dealing
        desc.expert_offset = -1 - self.deal_group if self.deal_group >= 0 else self.expert_offset
        desc.top_k = self.top_k
        desc.max_tokens = self.max_rows
        desc.weight_format = _lib.MM_WEIGHT_NVFP4 if nv else _lib.MM_WEIGHT_MXFP4
        desc.act_terms = self.act_terms
        desc.device = self.device.index if self.device.index is not None else torch.cuda.current_device()
        desc.routed = _lib.MMExpertWeights(*(t.data_ptr() for t in (w13, w13_scale, w2, w2_scale)),
                                           _ptr(w13_scale_2) if nv else None, _ptr(w2_scale_2) if nv else None)
        self.w13_scale_2, self.w2_scale_2 = (w13_scale_2, w2_scale_2) if nv else (None, None)
        self.input_scale = (float(input_scale[0]), float(input_scale[1])) if nv else None
        if nv:
            desc.input_scale[0], desc.input_scale[1] = self.input_scale
            keep += [w13_scale_2, w2_scale_2]
        self.has_shared = shared is not None
        if shared is not None:
            if len(shared) != (6 if nv else 4):
                raise ValueError(f"shared: expected {6 if nv else 4} tensors")
            s13, s13s, s2, s2s = (_u8(t) for t in shared[:4])
            _expect(s13, (1, 2 * inter, hidden // 2), "shared w13")
            _expect(s13s, (1, 2 * inter, hidden // block), "shared w13_scale")
            _expect(s2, (1, hidden, inter // 2), "shared w2")
            _expect(s2s, (1, hidden, inter // block), "shared w2_scale")
            extra = [None, None]
            if nv:
                extra = list(shared[4:6])
                for t in extra:
                    _expect(t, (1,), "shared scale_2", 4)
            desc.shared = _lib.MMExpertWeights(*(t.data_ptr() for t in (s13, s13s, s2, s2s)),
                                               *(_ptr(t) for t in extra))
            keep += [s13, s13s, s2, s2s, shared_clamp] + extra
        desc.clamp = _ptr(clamp)
        desc.shared_clamp = _ptr(shared_clamp)
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(lib().mm_layer_create(ctypes.byref(desc), ctypes.byref(handle)), "mm_layer_create")
        self._handle = handle
        self._tensors = keep  # the layer reads them in place
        info = _lib.MMLayerInfo()
        check(lib().mm_layer_get_info(handle, ctypes.byref(info)), "mm_layer_get_info")
        self.rows_capacity = int(info.rows_capacity)
        self.shared_row_base = int(info.shared_row_base)
        self.route_words_max = int(info.route_words)
        self.expert_weight_bytes = int(info.weight_bytes)

    @classmethod
    def from_trtllm(cls, w13, w13_scale, w2, w2_scale, top_k: int, max_rows: int, *, halves: str = "w3_w1",
                    **kwargs) -> "RoutedMoE":
        """A layer from SGLang's processed TRT-LLM-gen MXFP4 weights (the layout
        the reference's RoutedExpertGemm takes), or NVFP4 ones with
        weight_format="nvfp4" (plus its scale_2 / input_scale arguments):
        re-laid once into canonical copies (megamoe.layouts.trtllm_to_canonical);
        the processed tensors are not read afterwards."""
        from .layouts import trtllm_to_canonical

        c13, c13s, c2, c2s = trtllm_to_canonical(w13, w13_scale, w2, w2_scale, halves=halves,
                                                 weight_format=kwargs.get("weight_format", "mxfp4"))
        return cls(c13, c13s, c2, c2s, top_k, max_rows, **kwargs)

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            try:
                lib().mm_layer_destroy(handle)
            except Exception:
                pass
            self._handle = None

    # ------------------------------------------------------------------ helpers
    def _check_xq(self, x_quant: torch.Tensor, x_scale: torch.Tensor) -> int:
        """Rows of an MXFP8 routed input (E4M3 codes [T, H], E8M0 scales [T, H/32])."""
        for name, t, cols in (("x_quant", x_quant, self.hidden), ("x_scale", x_scale, self.hidden // 32)):
            if t.element_size() != 1 or t.dim() != 2 or t.size(1) != cols or not t.is_contiguous() \
                    or t.device != self.device:
                raise ValueError(f"{name}: expected a contiguous 1-byte [T, {cols}] tensor on {self.device}, "
                                 f"got {tuple(t.shape)} {t.dtype}")
        rows = x_quant.size(0)
        if x_scale.size(0) != rows or not 1 <= rows <= self.max_rows:
            raise ValueError(f"x_quant / x_scale: {rows} / {x_scale.size(0)} rows (1..{self.max_rows})")
        return rows

    def _check_x(self, x: torch.Tensor) -> int:
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.size(1) != self.hidden or not x.is_contiguous():
            raise ValueError(f"x: expected a contiguous bf16 [T, {self.hidden}] tensor, got {tuple(x.shape)} {x.dtype}")
        rows = x.size(0)
        if not 1 <= rows <= self.max_rows:
            raise ValueError(f"{rows} rows outside 1..{self.max_rows}")
        return rows

    def _outputs(self, rows: int):
        dev = self.device
        permuted = torch.empty((rows, self.top_k), dtype=torch.int32, device=dev)
        record = torch.empty(route_words(rows, self.top_k, self.experts), dtype=torch.int32, device=dev)
        out_rows = torch.empty((self.rows_capacity, self.hidden), dtype=torch.bfloat16, device=dev)
        return permuted, record, out_rows

    def shared_rows(self, rows: torch.Tensor, tokens: int) -> Optional[torch.Tensor]:
        """The shared expert's bf16 [T, H] output inside a rows buffer."""
        if not self.has_shared:
            return None
        return rows[self.shared_row_base : self.shared_row_base + tokens]

    # ------------------------------------------------------------------ API
    def __call__(self, x_quant: torch.Tensor, x_scale: Optional[torch.Tensor], topk_ids: torch.Tensor,
                 topk_weights: Optional[torch.Tensor] = None):
        """Route + gate_up + down on the current stream from given top-k ids
        (RoutedExpertGemm.__call__(x_quant, x_scale, topk_ids, topk_weights)).
        ``x_quant``/``x_scale``: the MXFP8 routed input, or a bf16 [T, H]
        ``x_quant`` with ``x_scale`` None. Returns (rows, weights, permuted):
        rows[permuted[t, k]] is slot (t, k)'s expert output (-1: an expert
        another rank holds)."""
        mx = x_scale is not None
        rows = self._check_xq(x_quant, x_scale) if mx else self._check_x(x_quant)
        if topk_ids.dim() != 2 or tuple(topk_ids.shape) != (rows, self.top_k):
            raise ValueError(f"topk_ids: expected [{rows}, {self.top_k}], got {tuple(topk_ids.shape)}")
        ids = topk_ids.to(torch.int32).contiguous()
        permuted, record, out_rows = self._outputs(rows)
        if mx:
            rc = lib().mm_layer_experts_mxfp8(self._handle, x_quant.data_ptr(), x_scale.data_ptr(), ids.data_ptr(),
                                              rows, permuted.data_ptr(), record.data_ptr(), out_rows.data_ptr(),
                                              _stream(self.device))
        else:
            rc = lib().mm_layer_experts(self._handle, x_quant.data_ptr(), ids.data_ptr(), rows, permuted.data_ptr(),
                                        record.data_ptr(), out_rows.data_ptr(), _stream(self.device))
        check(rc, "mm_layer_experts_mxfp8" if mx else "mm_layer_experts")
        self.last_record = record
        w = None if topk_weights is None else topk_weights.contiguous().view(rows, self.top_k)
        return out_rows, w, permuted

    def gate_topk_and_gemms(
        self,
        x_quant: Optional[torch.Tensor],
        x_scale: Optional[torch.Tensor],
        logits: torch.Tensor,
        bias: Optional[torch.Tensor],
        routed_scaling_factor: float,
        num_valid: Optional[torch.Tensor] = None,
        alt=None,
        renormalize_epsilon: float = 0.0,
        ids_out: Optional[torch.Tensor] = None,
        x: Optional[torch.Tensor] = None,
        early: bool = False,
        *,
        score: str = "sigmoid",
        renormalize=True,
    ):
        """Top-k from fp32 router logits, then route + gate_up + down, in the
        reference's positional order (routed_expert_gemm.py:776-870). The
        routed input is ``x_quant``/``x_scale`` (MXFP8), or ``x`` (bf16, which
        then takes their place: pass None for both). ``alt`` = (bias_alt,
        input_ids, token id): rows whose token is that id rank with bias_alt
        (vision routing). ``early`` is accepted for the reference's signature;
        the router launch here always releases this one early. ``score``:
        sigmoid (default), softmax or sqrtsoftplus (the reference's DSV4.1
        router); ``renormalize``: True (score / sum), False, or "scaled_bf16"
        (GLM-5.3's bf16(scale * s / (sum + eps))). Returns (rows, weights,
        permuted, ids)."""
        del early
        mx = x is None
        if mx:
            if x_quant is None or x_scale is None:
                raise ValueError("gate_topk_and_gemms: pass x_quant and x_scale, or x")
            rows = self._check_xq(x_quant, x_scale)
        else:
            rows = self._check_x(x)
        if logits.dtype != torch.float32 or tuple(logits.shape) != (rows, self.router_experts) or not logits.is_contiguous():
            raise ValueError(f"logits: expected contiguous fp32 [{rows}, {self.router_experts}]")
        weights = torch.empty((rows, self.top_k), dtype=torch.float32, device=self.device)
        ids = ids_out[:rows] if ids_out is not None else torch.empty((rows, self.top_k), dtype=torch.int32, device=self.device)
        g = gate_args(logits, bias, num_valid, score, renormalize, routed_scaling_factor, renormalize_epsilon, weights, ids,
                      alt)
        permuted, record, out_rows = self._outputs(rows)
        if mx:
            rc = lib().mm_layer_gate_experts_mxfp8(self._handle, x_quant.data_ptr(), x_scale.data_ptr(), ctypes.byref(g),
                                                   rows, permuted.data_ptr(), record.data_ptr(), out_rows.data_ptr(),
                                                   _stream(self.device))
        else:
            rc = lib().mm_layer_gate_experts(self._handle, x.data_ptr(), ctypes.byref(g), rows, permuted.data_ptr(),
                                             record.data_ptr(), out_rows.data_ptr(), _stream(self.device))
        check(rc, "mm_layer_gate_experts_mxfp8" if mx else "mm_layer_gate_experts")
        self.last_record = record
        return out_rows, weights, permuted, ids

    def finalize(self, rows: torch.Tensor, weights: torch.Tensor, permuted: torch.Tensor,
                 shared_output: Optional[torch.Tensor] = None, partial: bool = False):
        """Slot-order weighted combine (+ the shared expert). ``shared_output``
        defaults to the shared expert's rows inside ``rows``. With ``partial``
        returns the fp32 [2, T, H] un-rounded (routed, shared) sums instead."""
        tokens = permuted.size(0)
        if shared_output is None:
            shared_output = self.shared_rows(rows, tokens)
        return finalize(rows, weights, permuted, shared_output, partial=partial)

    def forward(
        self,
        x: torch.Tensor,
        *,
        router_weight: Optional[torch.Tensor] = None,
        logits: Optional[torch.Tensor] = None,
        bias: Optional[torch.Tensor] = None,
        routed_scaling_factor: float = 1.0,
        num_valid: Optional[torch.Tensor] = None,
        score: str = "sigmoid",
        renormalize: bool = True,
        renormalize_epsilon: float = 0.0,
        partial: bool = False,
        buffers: Optional[dict] = None,
        comm=None,
        residual: Optional[torch.Tensor] = None,
        gamma: Optional[torch.Tensor] = None,
        alt=None,
    ):
        """One whole MoE step on the current stream. Returns the bf16 [T, H]
        output (or the fp32 [2, T, H] partial sums with ``partial``; with
        ``comm``, a ``megamoe.PeerAllReduce`` of this rank's group, the output
        all-reduced over the group in the same launch as the combine; with
        ``comm`` and ``residual`` (bf16 [T, H]), the decoder hop's epilogue too:
        returns (norm_out, residual_out) as ``comm.moe_finalize_all_reduce_rms_norm``
        does, norm_out None without ``gamma``; residual_out may be ``residual``
        itself via buffers["residual_out"]). ``buffers``
        (optional dict) receives the intermediate tensors and may carry
        preallocated ones (keys: logits, weights, ids, permuted, record, rows,
        out, partial) so repeated calls allocate nothing."""
        tokens = self._check_x(x)
        if comm is not None and partial:
            raise ValueError("forward: comm and partial are exclusive")
        if residual is not None:
            if comm is None:
                raise ValueError("forward: residual needs comm (a PeerAllReduce, a group of one on one GPU)")
            if residual.dtype != torch.bfloat16 or tuple(residual.shape) != (tokens, self.hidden) \
                    or not residual.is_contiguous():
                raise ValueError("residual must be contiguous bf16 [T, H]")
            if gamma is not None and (gamma.dtype != torch.bfloat16 or tuple(gamma.shape) != (self.hidden,)):
                raise ValueError("gamma must be bf16 [H]")
        b = {} if buffers is None else buffers
        dev = self.device
        if router_weight is not None:
            if router_weight.dtype != torch.bfloat16 or tuple(router_weight.shape) != (self.router_experts, self.hidden):
                raise ValueError(f"router_weight: expected bf16 [{self.router_experts}, {self.hidden}]")
            if b.get("logits") is None or b["logits"].shape[0] != tokens:
                b["logits"] = torch.empty((tokens, self.router_experts), dtype=torch.float32, device=dev)
        elif logits is None:
            raise ValueError("forward needs router_weight or logits")

        def buf(name, shape, dtype):
            t = b.get(name)
            if t is None or tuple(t.shape) != tuple(shape) or t.dtype != dtype:
                t = torch.empty(shape, dtype=dtype, device=dev)
                b[name] = t
            return t

        weights = buf("weights", (tokens, self.top_k), torch.float32)
        ids = buf("ids", (tokens, self.top_k), torch.int32)
        permuted = buf("permuted", (tokens, self.top_k), torch.int32)
        record = buf("record", (route_words(tokens, self.top_k, self.experts),), torch.int32)
        rows = buf("rows", (self.rows_capacity, self.hidden), torch.bfloat16)
        out = None if partial or (residual is not None and gamma is None) else \
            buf("out", (tokens, self.hidden), torch.bfloat16)
        res_out = buf("residual_out", (tokens, self.hidden), torch.bfloat16) if residual is not None else None
        part = buf("partial", (2, tokens, self.hidden), torch.float32) if partial else None
        a = _lib.MMForwardArgs()
        a.x = x.data_ptr()
        a.router_w = _ptr(router_weight)
        a.logits = _ptr(logits)
        a.logits_out = _ptr(b.get("logits")) if router_weight is not None else None
        a.bias = _ptr(bias)
        a.num_valid = _ptr(num_valid)
        a.score_func = _lib.SCORES[score]
        a.renormalize = _lib.renorm_code(renormalize)
        a.routed_scaling = float(routed_scaling_factor)
        a.renorm_eps = float(renormalize_epsilon)
        a.tokens = tokens
        a.weights, a.ids, a.permuted, a.record = (t.data_ptr() for t in (weights, ids, permuted, record))
        a.rows = rows.data_ptr()
        a.out = _ptr(out)
        a.partial = _ptr(part)
        a.comm = None if comm is None else comm.handle
        _alt_fields(a, alt)
        a.residual = _ptr(residual)
        a.gamma = _ptr(gamma)
        a.norm_eps = 0.0 if comm is None else comm.eps
        a.residual_out = _ptr(res_out)
        check(lib().mm_layer_forward(self._handle, ctypes.byref(a), _stream(dev)), "mm_layer_forward")
        if residual is not None:
            return out, res_out
        return part if partial else out

    def rearm_experts(self) -> None:
        """Re-arm the last front pass's work tables for another rerun_experts."""
        check(lib().mm_layer_rearm_experts(self._handle, _stream(self.device)), "mm_layer_rearm_experts")

    def rerun_experts(self, tokens: int, record: torch.Tensor, rows: torch.Tensor, rearm: bool = True) -> None:
        """Launch the expert kernel again on the last front pass's work tables
        (benchmark hook: times the dominant kernel alone). ``rearm=False``
        when rearm_experts was called since the last launch."""
        if rearm:
            self.rearm_experts()
        check(lib().mm_layer_rerun_experts(self._handle, tokens, record.data_ptr(), rows.data_ptr(),
                                            _stream(self.device)), "mm_layer_rerun_experts")

    def check(self) -> None:
        """Synchronize and raise (DeviceTimeoutError) if a bounded device wait of
        this layer timed out."""
        check(lib().mm_layer_check(self._handle), "mm_layer_check")

    def set_wait_budget(self, microseconds: int) -> None:
        """Budget of every bounded device wait of this layer's expert launches
        (default 1.5 s)."""
        check(lib().mm_layer_set_wait_budget(self._handle, int(microseconds)), "mm_layer_set_wait_budget")

    def block_downs(self) -> None:
        """Test hook for the timeout path: re-arm the last front pass's work
        tables with every gate_up -> down mailbox out of reach, so that the next
        ``rerun_experts(..., rearm=False)`` ends on its bounded waits and
        ``check`` raises DeviceTimeoutError."""
        check(lib().mm_layer_block_downs(self._handle, _stream(self.device)), "mm_layer_block_downs")

    def read_scratch(self, which: str) -> torch.Tensor:
        """A uint8 copy of one of the layer's quantized-activation buffers:
        "x_codes" [3, max_rows, H/2], "x_scales" [3, max_rows, H/block],
        "h_codes" [3, rows_capacity, h_row], "h_scales" [3, rows_capacity,
        h_scale_row] (terms past act_terms unused; h rows in permuted order)."""
        code = {"x_codes": _lib.MM_SCRATCH_X_CODES, "x_scales": _lib.MM_SCRATCH_X_SCALES,
                "h_codes": _lib.MM_SCRATCH_H_CODES, "h_scales": _lib.MM_SCRATCH_H_SCALES}[which]
        n = int(lib().mm_layer_scratch_bytes(self._handle, code))
        out = torch.empty(n, dtype=torch.uint8, device=self.device)
        check(lib().mm_layer_read_scratch(self._handle, code, out.data_ptr(), n, _stream(self.device)),
              "mm_layer_read_scratch")
        info = _lib.MMLayerInfo()
        check(lib().mm_layer_get_info(self._handle, ctypes.byref(info)), "mm_layer_get_info")
        return out.view(3, -1, {"x_codes": self.hidden // 2,
                                "x_scales": self.hidden // (16 if self.weight_format == "nvfp4" else 32),
                                "h_codes": int(info.h_row_bytes),
                                "h_scales": int(info.h_scale_row_bytes)}[which])


# ---------------------------------------------------------------------- stateless ops
def route_words(rows: int, top_k: int, experts: int) -> int:
    """int32 length of the route record (routed_expert_gemm.py:107-120)."""
    return int(lib().mm_route_words(rows, top_k, experts))


def _alt_fields(obj, alt) -> None:
    """Set the vision-routing fields of a gate / forward args struct from ``alt``
    = (bias_alt fp32 [E] or None, input_ids int32/int64 [T], token id), the
    reference's gate_topk_and_gemms ``alt`` (routed_expert_gemm.py:776-812)."""
    if alt is None:
        obj.bias_alt, obj.input_ids, obj.input_ids64, obj.alt_token_id = None, None, 0, -1
        return
    bias_alt, input_ids, token = alt
    if bias_alt is not None and (bias_alt.dtype != torch.float32 or not bias_alt.is_contiguous()):
        raise ValueError("bias_alt must be a contiguous fp32 tensor")
    if input_ids.dtype not in (torch.int32, torch.int64) or not input_ids.is_contiguous():
        raise ValueError("input_ids must be a contiguous int32 or int64 tensor")
    obj.bias_alt = _ptr(bias_alt)
    obj.input_ids = input_ids.data_ptr()
    obj.input_ids64 = int(input_ids.dtype == torch.int64)
    obj.alt_token_id = int(token)


def gate_args(logits, bias, num_valid, score, renormalize, scale, eps, weights, ids, alt=None) -> _lib.MMGateArgs:
    if score not in _lib.SCORES:
        raise ValueError(f"unknown score function {score!r}")
    if bias is not None and (bias.dtype != torch.float32 or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous fp32 tensor")
    g = _lib.MMGateArgs()
    _alt_fields(g, alt)
    g.logits = logits.data_ptr()
    g.bias = _ptr(bias)
    g.num_valid = _ptr(num_valid)
    g.score_func = _lib.SCORES[score]
    g.renormalize = _lib.renorm_code(renormalize)
    g.routed_scaling = float(scale)
    g.renorm_eps = float(eps)
    g.weights = weights.data_ptr()
    g.ids = ids.data_ptr()
    return g


def router_gemv(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """fp32 logits [T, E] = x bf16 [T, H] @ weight bf16 [E, H]^T (fixed summation order)."""
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError("router_gemv takes bf16 x and weight")
    x, weight = x.contiguous(), weight.contiguous()
    tokens, hidden = x.shape
    experts = weight.size(0)
    logits = torch.empty((tokens, experts), dtype=torch.float32, device=x.device)
    check(
        lib().mm_router_gemv(x.data_ptr(), weight.data_ptr(), logits.data_ptr(), tokens, experts, hidden, _stream(x.device)),
        "mm_router_gemv",
    )
    return logits


def gate_topk(logits: torch.Tensor, bias: Optional[torch.Tensor], top_k: int, *, score: str = "sigmoid",
              renormalize: bool = True, routed_scaling_factor: float = 1.0, renormalize_epsilon: float = 0.0,
              num_valid: Optional[torch.Tensor] = None, alt=None):
    """(weights fp32 [T, k], ids int32 [T, k]) of the router top-k; ``alt`` =
    (bias_alt, input_ids, token id) for vision routing."""
    logits = logits.contiguous()
    tokens, experts = logits.shape
    weights = torch.empty((tokens, top_k), dtype=torch.float32, device=logits.device)
    ids = torch.empty((tokens, top_k), dtype=torch.int32, device=logits.device)
    g = gate_args(logits, bias, num_valid, score, renormalize, routed_scaling_factor, renormalize_epsilon, weights, ids,
                  alt)
    check(lib().mm_gate_topk(ctypes.byref(g), tokens, experts, top_k, _stream(logits.device)), "mm_gate_topk")
    return weights, ids


def route(ids: torch.Tensor, experts: int, expert_offset: int = 0):
    """(permuted int32 [T, k], record int32) of given top-k ids (route.cu / route_wide.cu)."""
    ids = ids.to(torch.int32).contiguous()
    tokens, top_k = ids.shape
    permuted = torch.empty_like(ids)
    record = torch.empty(route_words(tokens, top_k, experts), dtype=torch.int32, device=ids.device)
    check(
        lib().mm_route(ids.data_ptr(), permuted.data_ptr(), record.data_ptr(), tokens, top_k, experts, expert_offset,
                       _stream(ids.device)),
        "mm_route",
    )
    return permuted, record


def finalize(rows: torch.Tensor, weights: torch.Tensor, permuted: torch.Tensor,
             shared_output: Optional[torch.Tensor] = None, partial: bool = False) -> torch.Tensor:
    """out[t] = bf16(bf16(sum_k w * rows[perm]) + shared[t]) in slot order."""
    tokens, top_k = permuted.shape
    hidden = rows.size(1)
    dev = rows.device
    out = None if partial else torch.empty((tokens, hidden), dtype=torch.bfloat16, device=dev)
    part = torch.empty((2, tokens, hidden), dtype=torch.float32, device=dev) if partial else None
    w = weights.to(torch.float32).contiguous()
    perm = permuted.to(torch.int32).contiguous()
    check(
        lib().mm_finalize(rows.data_ptr(), w.data_ptr(), perm.data_ptr(), _ptr(shared_output), _ptr(out), _ptr(part),
                          tokens, top_k, hidden, _stream(dev)),
        "mm_finalize",
    )
    return part if partial else out


def finalize_partial(partial: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 output from an all-reduced fp32 [2, T, H] partial."""
    _, tokens, hidden = partial.shape
    if out is None:
        out = torch.empty((tokens, hidden), dtype=torch.bfloat16, device=partial.device)
    check(lib().mm_finalize_partial(partial.data_ptr(), out.data_ptr(), tokens, hidden, _stream(partial.device)),
          "mm_finalize_partial")
    return out
