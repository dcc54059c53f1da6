#!/usr/bin/env python
"""B1: the reference's own SM100 routed-expert pair and this library, on the same
B200, the same weights, routings and inputs.

The reference arm is sgl-nvidia-mega's RoutedExpertGemm
(deepseek_v41/sm103/moe/routed_expert_gemm.py:534), unmodified: route.cu /
route_wide.cu, gemm1.cu (tcgen05 kind::mxf8f6f4, MXFP8 activations x MXFP4
weights, clamped SwiGLU, MXFP8 requant of h) and gemm2.cu, compiled by NVRTC for
the device's sm_XXXa, from the files baseline/stage_ref_sm100.py copied into
baseline/_ref/. Its weights are the layout it reads: FlashInfer's processed
MXFP4 (the gated-activation row shuffle and the 128 x 4 scale interleave,
test/kernels/test_deepseek_v41_moe.py:62-104) of the same canonical weights this
library reads in place, padded from the 576-wide slice to 640 with zeros as the
reference requires (routed_expert_gemm.py:495-531).

Geometry: DeepSeek-V4.1's routed half as the reference serves it (hidden 5120,
384 experts, top-6, intermediate slice 576, clamp 10; routed_expert_gemm.py:36-49),
rows 1 / 6 / 16 / 48, D distinct experts per half. Weights: E2M1 codes uniform
over all bytes, E8M0 scales uniform in [118, 125] (the reference test's
distribution). Routed input: bf16 x ~ N(0, 1) quantized to MXFP8 by the MX rule
(a power-of-two scale per 32 with amax / scale <= 448, E4M3 codes).

Timing: the method of benchmark/bench_deepseek_v41_routed_moe.py:233-275 — a
CUDA graph of 39 halves alternating two layers' weights (cold: every half
routes its own experts), each half behind a one-element spacer kernel so no
half overlaps its predecessor; µs per half = (graph time - a graph of the
spacers alone) / 39, median over repeats, the two arms interleaved.
A half is what each arm's __call__(x_quant, x_scale, topk_ids, topk_weights)
launches: the reference's route + GEMM1 + GEMM2; this library's MXFP8 input
conversion + route + expert kernel.

Checks on every case: the slot -> row map and the route record equal, both
arms' rows (gathered by that map) within --tol of each other (max|a - b| /
max|b|; default 6e-2: the reference rounds h to MXFP8 between its GEMMs, about
4e-2 of the largest row value here, where this library carries h as three
MXFP4 terms; tests/test_gpu_ref_sm100.py holds each arm to the CPU oracle of
its own numerics within 2e-2).

Usage (on the GPU box, after staging):
  python baseline/ref_sm100.py [--rows 1 6 16 48] [--distinct 6 16 32 384] [--json]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref")
for _p in (REPO, os.path.join(REPO, "sgl-nvidia-mega_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

HIDDEN, SLICE, PADDED, EXPERTS, TOP_K, CLAMP, SCALE = 5120, 576, 640, 384, 6, 10.0, 1.5
HALVES = 39


def reference_module():
    """The staged reference module, or None with the reason."""
    if not os.path.isdir(os.path.join(REF, "sgl_nvidia_mega")):
        return None, "baseline/_ref is not staged (python baseline/stage_ref_sm100.py --reference <checkout>)"
    if REF not in sys.path:
        sys.path.insert(0, REF)
    try:
        from sgl_nvidia_mega.deepseek_v41.sm103.moe import routed_expert_gemm as reg
    except Exception as e:  # noqa: BLE001
        return None, f"the staged reference does not import: {e!r}"
    return reg, None


def make_layer(seed: int, device, experts: int = EXPERTS):
    """One layer: the canonical MXFP4 tensors this library reads ([w1; w3] rows,
    row-major E8M0 scales, slice 576) and the reference's processed, padded copy."""
    from megamoe.layouts import canonical_to_trtllm

    g = torch.Generator().manual_seed(seed)

    def rnd(shape, lo, hi):
        return torch.randint(lo, hi, shape, dtype=torch.uint8, generator=g).to(device)

    e, h, s, p = experts, HIDDEN, SLICE, PADDED
    c13, c13s = rnd((e, 2 * s, h // 2), 0, 256), rnd((e, 2 * s, h // 32), 118, 126)
    c2, c2s = rnd((e, h, s // 2), 0, 256), rnd((e, h, s // 32), 118, 126)
    clamp = torch.full((e,), CLAMP, dtype=torch.float32, device=device)
    # the reference's padded slice: [w1 | 0; w3 | 0] rows, zero K columns of w2 past 576
    p13 = torch.zeros((e, 2 * p, h // 2), dtype=torch.uint8, device=device)
    p13s = torch.full((e, 2 * p, h // 32), 127, dtype=torch.uint8, device=device)
    p13[:, :s], p13[:, p:p + s] = c13[:, :s], c13[:, s:]
    p13s[:, :s], p13s[:, p:p + s] = c13s[:, :s], c13s[:, s:]
    p2 = torch.zeros((e, h, p // 2), dtype=torch.uint8, device=device)
    p2s = torch.full((e, h, p // 32), 127, dtype=torch.uint8, device=device)
    p2[:, :, :s // 2], p2s[:, :, :s // 32] = c2, c2s
    g13, g13s, g2, g2s = canonical_to_trtllm(p13, p13s, p2, p2s, halves="w3_w1")
    del p13, p13s, p2, p2s
    return dict(canonical=(c13, c13s, c2, c2s), processed=(g13, g13s, g2, g2s), clamp=clamp)


def routing(rows: int, distinct: int, gen: torch.Generator, experts: int = EXPERTS, top_k: int = TOP_K):
    """ids [rows, top_k] over min(distinct, rows * top_k) experts: a shuffled pool
    of `distinct` experts dealt round-robin, so a row's k ids are distinct and
    every pooled expert is used when the slots allow."""
    distinct = max(top_k, min(distinct, experts))
    pool = torch.randperm(experts, generator=gen)[:distinct]
    order = torch.randperm(distinct, generator=gen)
    slot = torch.arange(rows * top_k).view(rows, top_k)
    start = torch.randint(0, distinct, (1,), generator=gen)
    return pool[order[(slot + start) % distinct]].to(torch.int32)


def mxfp8(x: torch.Tensor):
    """MXFP8 of bf16 x [T, H]: per 32 elements the E8M0 power of two 2^e with
    e = ceil(log2(amax / 448)) (so |x| / 2^e <= 448), codes E4M3 of x / 2^e."""
    T, H = x.shape
    xf = x.float().view(T, H // 32, 32)
    amax = xf.abs().amax(-1, keepdim=True).clamp_min(2.0 ** -126)
    e = torch.ceil(torch.log2(amax / 448.0)).clamp(-127, 127)
    q = (xf / torch.exp2(e)).to(torch.float8_e4m3fn).view(T, H)
    s = (e.squeeze(-1) + 127).to(torch.uint8)
    return q.view(torch.uint8).contiguous(), s.contiguous()


class Pair:
    """Both arms bound to the same layers."""

    def __init__(self, reg, layers, max_rows: int = 64):
        import megamoe

        self.reg = reg
        self.ref = [reg.RoutedExpertGemm(*L["processed"], L["clamp"], top_k=TOP_K, max_rows=max_rows)
                    for L in layers]
        self.mm = [megamoe.RoutedMoE(*L["canonical"], TOP_K, max_rows, clamp=L["clamp"]) for L in layers]

    def half(self, arm: str, i: int, x_q, x_s, ids, w):
        obj = (self.ref if arm == "reference" else self.mm)[i % len(self.ref)]
        return obj(x_q, x_s, ids, w)


def gathered(rows, permuted):
    return rows[permuted.clamp(min=0).long()].float()


def check_case(pair: Pair, rows: int, distinct: int, seed: int, dev):
    """One half on layer 0 through both arms: (permuted equal, route record
    equal, max-abs-rel of this library's rows against the reference's)."""
    g = torch.Generator().manual_seed(seed)
    ids = routing(rows, distinct, g).to(dev)
    w = torch.softmax(torch.randn(rows, TOP_K, generator=g), -1).to(dev)
    x_q, x_s = mxfp8(torch.randn(rows, HIDDEN, generator=g).to(torch.bfloat16).to(dev))
    r_rows, _, r_perm = pair.half("reference", 0, x_q, x_s, ids, w)
    m_rows, _, m_perm = pair.half("mm", 0, x_q, x_s, ids, w)
    ctas = pair.reg.max_ctas(rows, TOP_K, EXPERTS)
    r_perm2, r_record = pair.ref[0]._route(ids, rows, ctas)
    torch.cuda.synchronize()
    m_record = pair.mm[0].last_record
    same_perm = bool(torch.equal(r_perm, m_perm)) and bool(torch.equal(r_perm2, m_perm))
    same_record = bool(torch.equal(r_record, m_record[: r_record.numel()]))
    a, b = gathered(m_rows, m_perm), gathered(r_rows, r_perm)
    err = float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))
    return same_perm, same_record, err


def graph_of(pair: Pair, arm: str, rows: int, distinct: int, seed: int, dev, spacers_only=False):
    g = torch.Generator().manual_seed(seed)
    ids = [routing(rows, distinct, g).to(dev) for _ in range(HALVES)]
    ws = [torch.softmax(torch.randn(rows, TOP_K, generator=g), -1).to(dev) for _ in range(HALVES)]
    x_q, x_s = mxfp8(torch.randn(rows, HIDDEN, generator=g).to(torch.bfloat16).to(dev))
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    keep = []

    def body():
        keep.clear()
        for i in range(HALVES):
            flag.add_(1)  # spacer: the next half starts after it, not beside its predecessor
            if not spacers_only:
                keep.append(pair.half(arm, i, x_q, x_s, ids[i], ws[i]))

    body()  # warm-up (and the reference's NVRTC builds) outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        body()
    torch.cuda.synchronize()
    return graph, (ids, ws, x_q, x_s, flag, keep)


def replay_us(graph, replays: int) -> float:
    start, end = torch.cuda.Event(True), torch.cuda.Event(True)
    graph.replay()
    torch.cuda.synchronize()
    start.record()
    for _ in range(replays):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) * 1e3 / replays / HALVES


def weight_bytes(distinct_used: float) -> float:
    """Algorithmic weight bytes of a half: the unpadded slice of every used expert
    (3 x 5120 x 576 E2M1 codes + an E8M0 scale per 32)."""
    return distinct_used * (3 * HIDDEN * SLICE // 2 + 3 * HIDDEN * SLICE // 32)


def run(rows_list, distinct_list, repeats=5, replays=20, tol=6e-2, seed=7, log=print):
    reg, why = reference_module()
    if reg is None:
        raise RuntimeError(why)
    dev = torch.device("cuda", torch.cuda.current_device())
    layers = [make_layer(seed + i, dev) for i in range(2)]
    pair = Pair(reg, layers)
    results = []
    for rows in rows_list:
        for distinct in distinct_list:
            d_used = min(max(distinct, TOP_K), rows * TOP_K, EXPERTS)
            if distinct > rows * TOP_K and distinct != EXPERTS:
                continue  # the same case as distinct = rows * top_k
            same_perm, same_record, err = check_case(pair, rows, distinct, 900 + rows + distinct, dev)
            graphs = {arm: graph_of(pair, arm, rows, distinct, 1000 + distinct, dev)
                      for arm in ("reference", "mm")}
            spacer = graph_of(pair, "mm", rows, distinct, 1000 + distinct, dev, spacers_only=True)
            times = {"reference": [], "mm": []}
            for r in range(repeats):
                arms = ("reference", "mm") if r % 2 == 0 else ("mm", "reference")
                base = replay_us(spacer[0], replays)
                for arm in arms:
                    times[arm].append(replay_us(graphs[arm][0], replays) - base)
            ref_us, mm_us = (statistics.median(times[a]) for a in ("reference", "mm"))
            wb = weight_bytes(d_used)
            res = dict(rows=rows, distinct=d_used, reference_us=ref_us, mm_us=mm_us,
                       speedup=ref_us / mm_us, weight_bytes=wb,
                       reference_tbs=wb / (ref_us * 1e-6) / 1e12, mm_tbs=wb / (mm_us * 1e-6) / 1e12,
                       same_permuted=same_perm, same_record=same_record, rows_max_abs_rel=err,
                       rows_within_tol=err <= tol)
            results.append(res)
            log(json.dumps(res))
            del graphs, spacer
            torch.cuda.empty_cache()
    return results


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, nargs="+", default=[1, 6, 16, 48])
    ap.add_argument("--distinct", type=int, nargs="+", default=[6, 16, 32, 384])
    ap.add_argument("--repeats", type=int, default=5)
    ap.add_argument("--replays", type=int, default=20)
    ap.add_argument("--tol", type=float, default=6e-2)
    args = ap.parse_args()
    results = run(args.rows, args.distinct, args.repeats, args.replays, args.tol)
    print("rows distinct | reference us | this library us | speed-up | TB/s ref / mm | perm record | rows err")
    for r in results:
        print(f"{r['rows']:4d} {r['distinct']:4d} | {r['reference_us']:8.2f} | {r['mm_us']:8.2f} | "
              f"{r['speedup']:5.2f}x | {r['reference_tbs']:.2f} / {r['mm_tbs']:.2f} | "
              f"{r['same_permuted']} {r['same_record']} | {r['rows_max_abs_rel']:.2e}")
    return 0 if all(r["same_permuted"] and r["same_record"] and r["rows_within_tol"] for r in results) else 1


if __name__ == "__main__":
    sys.exit(main())
