"""Weight-layout adapters: SGLang's processed FlashInfer / TRT-LLM-gen MXFP4 and
NVFP4 layouts -> the canonical layout this library reads.

SGLang's ``Mxfp4FlashinferTrtllmMoEMethod`` hands the TRT-LLM-gen MoE (and the
reference's ``RoutedExpertGemm``, whose test builds the same layout:
``test/kernels/test_deepseek_v41_moe.py:62-104``) weights processed per expert:

  * w13 ([w3; w1] halves, TRT-LLM's gated-activation order): rows permuted by
    ``_maybe_get_cached_w3_w1_permute_indices(..., epilogue_tile_m=128)`` (the
    gated-activation row interleave, then the 128-row epilogue-tile shuffle);
  * w13 scales: the same row permutation, then ``block_scale_interleave`` (the
    128 x 4 scale-factor swizzle);
  * w2 and its scales: ``get_w2_permute_indices_with_cache`` rows, then the
    same swizzle for the scales.

The NVFP4 processing (the TRT-LLM NVFP4 tensors of GLM-5.3's engine,
``glm5_3/sm103/moe/weights.py:1-30``: the same row maps, E4M3 scales per 16
elements in the same 128 x 4 interleave) differs only in the scale block.
``trtllm_to_canonical`` inverts all of it once, at build time, into the
canonical [w1; w3] rows with row-major scales; the row permutations come from
FlashInfer's own index helpers (host code, evaluated on the CPU), the swizzle is
restated here (``interleave_scales`` / ``deinterleave_scales``: a 512-byte atom
per 128 rows x 4 columns, byte 16 (r % 32) + 4 ((r / 32) % 4) + c % 4).
"""

from __future__ import annotations

from typing import Tuple

import torch


def interleave_scales(s: torch.Tensor) -> torch.Tensor:
    """The 128 x 4 scale swizzle of a [R, C] byte matrix (R padded to 128 and C
    to 4 with zeros): returns the flat swizzled bytes, atom (R/128, C/4) major."""
    R, C = s.shape
    Rp, Cp = (R + 127) // 128 * 128, (C + 3) // 4 * 4
    p = torch.zeros((Rp, Cp), dtype=s.dtype, device=s.device)
    p[:R, :C] = s
    # [rt, m1, m0, ct, kk] -> [rt, ct, m0, m1, kk]
    t = p.view(Rp // 128, 4, 32, Cp // 4, 4).permute(0, 3, 2, 1, 4)
    return t.contiguous().view(-1)


def deinterleave_scales(flat: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """Inverse of ``interleave_scales``: the [rows, cols] byte matrix."""
    Rp, Cp = (rows + 127) // 128 * 128, (cols + 3) // 4 * 4
    t = flat.reshape(-1)[: Rp * Cp].view(Rp // 128, Cp // 4, 32, 4, 4).permute(0, 3, 2, 1, 4)
    return t.contiguous().view(Rp, Cp)[:rows, :cols]


def _perms(two_i: int, half_h: int, hidden: int, half_i: int, block: int = 32):
    """Row permutations of the processed w13 / w13 scales / w2 / w2 scales
    (FlashInfer's host-side index helpers; the scale matrices have 2 K / block
    columns: block 32 for MXFP4, 16 for NVFP4)."""
    from flashinfer.fused_moe.core import (  # host-side index helpers
        _maybe_get_cached_w3_w1_permute_indices,
        get_w2_permute_indices_with_cache,
    )

    cache: dict = {}
    per_byte = block // 2  # packed code bytes per scale
    p13 = _maybe_get_cached_w3_w1_permute_indices(cache, torch.empty((two_i, half_h), dtype=torch.uint8), 128)
    p13s = _maybe_get_cached_w3_w1_permute_indices(
        cache, torch.empty((two_i, half_h // per_byte), dtype=torch.uint8), 128, num_elts_per_sf=16)
    p2 = get_w2_permute_indices_with_cache(cache, torch.empty((hidden, half_i), dtype=torch.uint8), 128)
    p2s = get_w2_permute_indices_with_cache(cache, torch.empty((hidden, half_i // per_byte), dtype=torch.uint8), 128,
                                            num_elts_per_sf=16)
    return p13.cpu(), p13s.cpu(), p2.cpu(), p2s.cpu()


def _block(weight_format: str) -> int:
    if weight_format not in ("mxfp4", "nvfp4"):
        raise ValueError(f"weight_format must be 'mxfp4' or 'nvfp4', not {weight_format!r}")
    return 32 if weight_format == "mxfp4" else 16


def trtllm_to_canonical(w13: torch.Tensor, w13_scale: torch.Tensor, w2: torch.Tensor, w2_scale: torch.Tensor,
                        *, halves: str = "w3_w1",
                        weight_format: str = "mxfp4") -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Canonical (w13 u8 [E, 2I, H/2] as [w1; w3], w13_scale u8 [E, 2I, H/block],
    w2 u8 [E, H, I/2], w2_scale u8 [E, H, I/block]) copies of processed
    TRT-LLM-gen weights; block 32 (MXFP4, E8M0 scales) or 16 (NVFP4, E4M3
    scales). ``halves``: the order of the processed w13's two halves, "w3_w1"
    (TRT-LLM's, up first) or "w1_w3"."""
    block = _block(weight_format)
    if halves not in ("w3_w1", "w1_w3"):
        raise ValueError(f"halves must be 'w3_w1' or 'w1_w3', not {halves!r}")
    w13, w2 = (t.view(torch.uint8) for t in (w13, w2))
    E, two_i, half_h = w13.shape
    hidden, half_i = w2.shape[1], w2.shape[2]
    inter, H = two_i // 2, 2 * half_h
    if tuple(w2.shape) != (E, H, inter // 2):
        raise ValueError(f"w2: expected [{E}, {H}, {inter // 2}], got {tuple(w2.shape)}")
    p13, p13s, p2, p2s = _perms(two_i, half_h, hidden, half_i, block)
    dev = w13.device
    inv13, inv13s = torch.argsort(p13).to(dev), torch.argsort(p13s).to(dev)
    inv2, inv2s = torch.argsort(p2).to(dev), torch.argsort(p2s).to(dev)
    c13 = w13[:, inv13].contiguous()
    c2 = w2[:, inv2].contiguous()
    s13f, s2f = w13_scale.reshape(E, -1).view(torch.uint8), w2_scale.reshape(E, -1).view(torch.uint8)
    c13s = torch.stack([deinterleave_scales(s13f[e], two_i, H // block)[inv13s] for e in range(E)]).contiguous()
    c2s = torch.stack([deinterleave_scales(s2f[e], hidden, inter // block)[inv2s] for e in range(E)]).contiguous()
    if halves == "w3_w1":  # canonical is [w1 (gate); w3 (up)]
        c13 = torch.cat([c13[:, inter:], c13[:, :inter]], dim=1).contiguous()
        c13s = torch.cat([c13s[:, inter:], c13s[:, :inter]], dim=1).contiguous()
    return c13, c13s, c2, c2s


def canonical_to_trtllm(w13: torch.Tensor, w13_scale: torch.Tensor, w2: torch.Tensor, w2_scale: torch.Tensor,
                        *, halves: str = "w3_w1", weight_format: str = "mxfp4"):
    """The processing ``trtllm_to_canonical`` inverts (for tests and tools):
    canonical [w1; w3] MXFP4 / NVFP4 weights -> processed TRT-LLM-gen layout."""
    block = _block(weight_format)
    w13, w2, w13_scale, w2_scale = (t.view(torch.uint8) for t in (w13, w2, w13_scale, w2_scale))
    E, two_i, half_h = w13.shape
    hidden, half_i = w2.shape[1], w2.shape[2]
    inter = two_i // 2
    if halves == "w3_w1":
        w13 = torch.cat([w13[:, inter:], w13[:, :inter]], dim=1)
        w13_scale = torch.cat([w13_scale[:, inter:], w13_scale[:, :inter]], dim=1)
    p13, p13s, p2, p2s = (p.to(w13.device) for p in _perms(two_i, half_h, hidden, half_i, block))
    g13 = w13[:, p13].contiguous()
    g2 = w2[:, p2].contiguous()
    g13s = torch.stack([interleave_scales(w13_scale[e][p13s]) for e in range(E)]).reshape(E, two_i, -1)
    g2s = torch.stack([interleave_scales(w2_scale[e][p2s]) for e in range(E)]).reshape(E, hidden, -1)
    return g13, g13s.contiguous(), g2, g2s.contiguous()
