"""Partitions of one MoE layer's canonical MXFP4 weights across ranks.

Tensor parallel on the expert intermediate (the reference's MoE TP,
``routed_expert_gemm.py:37-40`` slices): rank r of n holds, of every expert, the
gate rows [r I/n, (r+1) I/n) and the matching up rows of w13, and the same K
columns of w2; the partial outputs of the ranks sum to the full output (the
SwiGLU is element-wise in the intermediate, so it commutes with the split).

Expert parallel (``deepseek_v41/spec.py:126-128``, ``route.cuh:17-23``): rank r
of n holds experts [r E/n, (r+1) E/n); the router stays replicated and slots
routed to another rank map to row -1.
"""

from __future__ import annotations

from typing import Sequence, Tuple

import torch


def tp_slice(w13: torch.Tensor, w13_scale: torch.Tensor, w2: torch.Tensor, w2_scale: torch.Tensor,
             rank: int, world: int, block: int = 32) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Rank ``rank``'s TP slice of canonical [n, 2I, H/2] / [n, 2I, H/block] /
    [n, H, I/2] / [n, H, I/block] weights (contiguous copies); block 32 for
    MXFP4, 16 for NVFP4 (whose per-expert scale_2 is not sliced)."""
    two_i = w13.shape[1]
    inter = two_i // 2
    if inter % world or (inter // world) % 64:
        raise ValueError(f"intermediate {inter} does not split into {world} slices of a multiple of 64")
    part = inter // world
    g0, u0 = rank * part, inter + rank * part
    s13 = torch.cat([w13[:, g0:g0 + part], w13[:, u0:u0 + part]], dim=1).contiguous()
    s13s = torch.cat([w13_scale[:, g0:g0 + part], w13_scale[:, u0:u0 + part]], dim=1).contiguous()
    s2 = w2[:, :, rank * part // 2:(rank + 1) * part // 2].contiguous()
    s2s = w2_scale[:, :, rank * part // block:(rank + 1) * part // block].contiguous()
    return s13, s13s, s2, s2s


def ep_window(experts: int, rank: int, world: int) -> Tuple[int, int]:
    """(expert_offset, local experts) of EP rank ``rank``: a consecutive window."""
    if experts % world:
        raise ValueError(f"{experts} experts do not split over {world} ranks")
    local = experts // world
    return rank * local, local


def ep_slice(tensors: Sequence[torch.Tensor], rank: int, world: int) -> Tuple[torch.Tensor, ...]:
    """The EP window of per-expert tensors (first dimension = experts)."""
    offset, local = ep_window(tensors[0].shape[0], rank, world)
    return tuple(t[offset:offset + local].contiguous() for t in tensors)
