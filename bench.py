#!/usr/bin/env python
"""Routed-MoE µs/layer and tokens/s on B200 (BASELINE.json metric).

Workload (all synthetic, seeded; random-init MXFP4 weights of the named shape):
  N = 1: BASELINE config 2 — one routed-MoE layer, hidden 7168, 384 routed experts
         + 1 shared (intermediate 2048), sigmoid + fp32 bias top-8, routed scale
         2.5, MXFP4 weights (E2M1 codes uniform over 16 nibbles, E8M0 exponents
         uniform in [-10, -6]), 8 tokens of bf16 x ~ N(0, 1).
  N > 1: the same layer tensor-parallel on the expert intermediate (2048 / N per
         rank, shared expert split alike), routing replicated on every rank; the
         combine fused with the all-reduce over NVLink peer memory (one launch:
         each rank pushes its combined rows to every peer by P2P stores, waits on
         per-tile flags, sums in rank order), or with --combine nccl the fp32
         partial sums all-reduced by NCCL; total work fixed ("scaling": "strong").
A step is one MoE layer over one batch: router GEMV -> top-k -> route ->
gate_up -> SwiGLU + requant -> down -> combine (-> all-reduce). Each step takes
the next of 64 resident token batches (distinct routings); one step streams
~1.4 GB of expert weights, far above the 126 MB L2, so no flush is needed.
The e2e figure goes through the public API call with host buffers.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mm|reference|flashinfer|ref-sm100]
Under torchrun each rank drives one GPU; rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
for _p in (REPO, os.path.join(REPO, "sgl-nvidia-mega_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

H, I, E, K, SCALE = 7168, 2048, 384, 8, 2.5
CONFIGS = {  # BASELINE configs this bench runs: (hidden, intermediate, routed experts, weight format)
    "2": (7168, 2048, 384, "mxfp4"),
    "4": (6144, 2048, 256, "nvfp4"),
}
METRIC = "routed-MoE tokens/s per layer (us/layer = 1e3 * ms_per_step)"
POOL = 64


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--tokens", type=int, default=None, help="default: 8 (config 2), 80 (config 4)")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="2",
                    help="BASELINE config: 2 (MXFP4, hidden 7168, 384 + 1 experts) or 4 (NVFP4, hidden 6144, "
                         "256 + 1 experts; TP x EP2 at N > 1)")
    ap.add_argument("--experts", type=int, default=None,
                    help="routed experts (default: the config's; fewer only for small profiling cases)")
    ap.add_argument("--impl", choices=["mm", "reference", "flashinfer", "ref-sm100"], default="mm",
                    help="mm: this library; reference: the CPU oracle port; flashinfer: SGLang's stock GPU path "
                         "(FlashInfer TRT-LLM-gen fused MoE, a library) on the same workload, N = 1; ref-sm100: the "
                         "reference's own SM100 routed pair beside this library at DeepSeek-V4.1 geometry, N = 1 "
                         "(baseline/ref_sm100.py; needs baseline/stage_ref_sm100.py run first)")
    ap.add_argument("--fi-act", choices=["bf16", "mxfp8"], default="bf16",
                    help="--impl flashinfer: activations bf16, or MXFP8 quantized before the timed region")
    ap.add_argument("--combine", choices=["peer", "nccl"], default="peer",
                    help="N > 1: fused combine + peer all-reduce (default) or NCCL all-reduce of fp32 partials")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--slice", type=int, default=0,
                    help="one GPU only: run rank 0's share of an N-way sharded layer (TP-N for config 2) with no "
                         "exchange, to measure and profile narrow slices")
    ap.add_argument("--stack", action="store_true",
                    help="BASELINE config 5: a step of --layers EP8 MoE layers chained through the fused hop")
    ap.add_argument("--layers", type=int, default=60)
    return ap.parse_args()


def routing_rule(config):
    """(renormalize, eps) of a BASELINE config's routing weights: config 4 follows
    GLM-5.3 (bf16(scale * s / (sum + 1e-20)), glm5_3/sm103/moe/routing.py:3-11);
    the others renormalize by the plain sum."""
    return ("scaled_bf16", 1e-20) if config == "4" else (True, 0.0)


def workload_name(config, T, shards, hidden, inter, experts):
    """The workload string both arms report for one layer of BASELINE `config`."""
    tp, ep = partition(shards, CONFIGS[config][3])
    fmt_name = "MXFP4" if CONFIGS[config][3] == "mxfp4" else "NVFP4"
    if shards <= 1:
        split = ""
    elif config == "2":
        split = f" (TP{shards}: {inter // shards} per rank)"
    else:
        split = f" (TP{tp} x EP{ep}: {experts // ep} experts x {inter // tp} per rank)"
    rule = ", GLM-5.3 bf16 weights" if config == "4" else ""
    return (f"BASELINE config {config}: one routed-MoE layer, hidden {hidden}, {experts} routed + 1 shared experts, "
            f"intermediate {inter}{split}, sigmoid+bias top-{K}{rule}, scale {SCALE}, {fmt_name}, {T} tokens")


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def expert_bytes(hidden, inter, block=32):
    """Algorithmic bytes of one expert's FP4 weights: 3 matrices of H x I, half
    a byte per element plus one scale byte per block (32: MXFP4's E8M0, 16:
    NVFP4's E4M3; NVFP4's per-expert fp32 scale_2 is negligible)."""
    return 3 * hidden * inter // 2 + 3 * hidden * inter // block


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (every 200 ms) during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
        except Exception:
            pass
        finally:
            if self.path and os.path.exists(self.path):
                os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------- layer
def partition(world, fmt):
    """(tp, ep) of the bench's layer over `world` ranks: config 2 is TP-N on the
    intermediate; config 4 is TP (N/2) x EP2 at N >= 2 (BASELINE: TP4 x EP2 at 8)."""
    if fmt == "nvfp4" and world >= 2:
        return world // 2, 2
    return world, 1


def build_layer(rank, world, tokens, device, fmt="mxfp4"):
    """This rank's part of the seeded random layer: (moe, routed weights,
    shared weights or None, router, bias, x pool, info). Rank r holds EP
    window r // tp with the TP slice r % tp of the intermediate; the shared
    expert is TP-split within EP group 0."""
    import megamoe

    tp, ep = partition(world, fmt)
    ep_rank = rank // tp
    local = E // ep
    offset = ep_rank * local
    ir = I // tp
    g = torch.Generator(device=device).manual_seed(1000 + rank)

    def rnd(shape, lo, hi):
        return torch.randint(lo, hi + 1, shape, dtype=torch.uint8, device=device, generator=g)

    has_shared = ep_rank == 0
    extra = {}
    if fmt == "mxfp4":
        w = [rnd((local, 2 * ir, H // 2), 0, 255), rnd((local, 2 * ir, H // 32), 117, 121),
             rnd((local, H, ir // 2), 0, 255), rnd((local, H, ir // 32), 117, 121)]
        shared = [rnd((1, 2 * ir, H // 2), 0, 255), rnd((1, 2 * ir, H // 32), 117, 121),
                  rnd((1, H, ir // 2), 0, 255), rnd((1, H, ir // 32), 117, 121)] if has_shared else None
    else:
        # NVFP4: E2M1 codes uniform, E4M3 scales of values ~U[0.5, 4] per 16,
        # per-expert fp32 scale_2 = 2^-8 (1 + u/4), static input scales
        def sf(shape):
            v = 0.5 + 3.5 * torch.rand(shape, device=device, generator=g)
            return v.to(torch.float8_e4m3fn).view(torch.uint8)

        def s2(n):
            return (2.0 ** -8 * (1.0 + 0.25 * torch.rand((n,), device=device, generator=g))).float()

        w = [rnd((local, 2 * ir, H // 2), 0, 255), sf((local, 2 * ir, H // 16)),
             rnd((local, H, ir // 2), 0, 255), sf((local, H, ir // 16))]
        w13_s2, w2_s2 = s2(local), s2(local)
        shared = [rnd((1, 2 * ir, H // 2), 0, 255), sf((1, 2 * ir, H // 16)), rnd((1, H, ir // 2), 0, 255),
                  sf((1, H, ir // 16)), s2(1), s2(1)] if has_shared else None
        # FC2's input scale from twice the largest |h| of 8 rows through expert 0
        lut = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], device=device)
        codes, scales = w[0][0], w[1][0]
        vals = torch.stack([lut[(codes & 15).long()], lut[(codes >> 4).long()]], -1).reshape(2 * ir, H)
        sc = scales.view(torch.float8_e4m3fn).float().repeat_interleave(16, dim=1)
        w13_0 = vals * sc * w13_s2[0]
        xs0 = torch.randn((8, H), device=device, generator=g)
        gu = xs0 @ w13_0.T
        hh = gu[:, ir:] * (gu[:, :ir] * torch.sigmoid(gu[:, :ir]))
        fc2 = 2.0 * float(hh.abs().max()) / (6.0 * 448.0)
        extra = dict(weight_format="nvfp4", w13_scale_2=w13_s2, w2_scale_2=w2_s2,
                     input_scale=(8.0 / (6.0 * 448.0), fc2))
    moe = megamoe.RoutedMoE(*w, K, max(tokens, 8), router_experts=E, expert_offset=offset, shared=shared,
                            **extra)
    gx = torch.Generator(device=device).manual_seed(7)  # identical on every rank: replicated routing
    router = (torch.randn((E, H), device=device, generator=gx) * 0.02).to(torch.bfloat16)
    bias = (torch.randn((E,), device=device, generator=gx) * 0.01).float()
    xs = torch.randn((POOL, tokens, H), device=device, generator=gx).to(torch.bfloat16)
    info = dict(tp=tp, ep=ep, offset=offset, local=local, ir=ir, has_shared=has_shared,
                block=16 if fmt == "nvfp4" else 32)
    return moe, w, shared, router, bias, xs, info


def run_mm(args):
    import megamoe

    global H, I, E
    H, I, E, fmt = CONFIGS[args.config]
    if args.experts is not None:
        E = args.experts
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    T = args.tokens if args.tokens is not None else (80 if args.config == "4" else 8)
    if args.slice > 1 and world > 1:
        raise SystemExit("--slice runs on one GPU")
    shards = args.slice if args.slice > 1 else world  # ranks the layer is sharded over
    moe, w, shared, router, bias, xs, info = build_layer(rank, shards, T, dev, fmt)
    bufs = {}
    peer = world > 1 and args.combine == "peer"
    comm = megamoe.PeerAllReduce(T, H) if peer else None

    renorm, eps = routing_rule(args.config)

    def step(x, b=None):
        b = bufs if b is None else b
        if world == 1 or peer:
            return moe.forward(x, router_weight=router, bias=bias, routed_scaling_factor=SCALE, buffers=b,
                               comm=comm, renormalize=renorm, renormalize_epsilon=eps)
        part = moe.forward(x, router_weight=router, bias=bias, routed_scaling_factor=SCALE, partial=True,
                           buffers=b, renormalize=renorm, renormalize_epsilon=eps)
        dist.all_reduce(part)
        out = b.setdefault("final", torch.empty((T, H), dtype=torch.bfloat16, device=dev))
        megamoe.finalize_partial(part, out=out)
        return out

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def check():
        moe.check()
        if comm is not None:
            comm.check()

    for i in range(max(args.warmup, 3)):
        step(xs[i % POOL])
    check()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for i in range(args.steps):
            step(xs[i % POOL])
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    barrier()
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    check()
    ms_step = ms / args.steps
    value = T * args.steps / (ms / 1e3)

    # distinct local experts per step (seeded routings, averaged over the pool)
    distinct = []
    lo, hi = info["offset"], info["offset"] + info["local"]
    for i in range(POOL):
        step(xs[i])
        ids = bufs["ids"]
        distinct.append(int(torch.unique(ids[(ids >= lo) & (ids < hi)]).numel()))
    torch.cuda.synchronize()
    d_mean = float(np.mean(distinct))
    eb = expert_bytes(H, info["ir"], info["block"])
    n_shared = 1 if info["has_shared"] else 0
    layer_bytes = (d_mean + n_shared) * eb + E * H * 2
    if dist is not None:  # the roofline of a sharded layer is its busiest rank's bytes
        t = torch.tensor([layer_bytes], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        layer_bytes = float(t.item())

    # dominant kernel alone: the expert kernel relaunched on the last step's tables
    last_d = distinct[-1]
    reps = 200
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for i in range(3):
        moe.rerun_experts(T, bufs["record"], bufs["rows"])
    for a, b in evs:
        moe.rearm_experts()  # outside the timed pair: only the kernel is timed
        a.record()
        moe.rerun_experts(T, bufs["record"], bufs["rows"], rearm=False)
        b.record()
    torch.cuda.synchronize()
    k_ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
    moe.check()
    k_bytes = (last_d + n_shared) * eb
    peak, peak_kind = peaks()
    achieved = k_bytes / (k_ms / 1e3) / 1e9

    # end to end through the public API with host buffers: every step copies its
    # x from pinned host memory and its output back, pipelined on a copy stream
    host_x = torch.empty((POOL, T, H), dtype=torch.bfloat16).pin_memory()
    host_x.copy_(xs.cpu())
    e2e_steps = min(args.steps, 1000)
    barrier()
    e2e_ms = e2e_pipelined(step, host_x, e2e_steps, dev)
    if dist is not None:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = T * e2e_steps / (e2e_ms / 1e3)

    # DRAM bytes of the dominant kernel: measured per streamed expert in one ncu
    # capture of a smaller case (profiles/expert_kernel_traffic.json), scaled by
    # the experts this launch streams; only where the capture's shape applies
    traffic = None
    tpath = os.path.join(REPO, "profiles", "expert_kernel_traffic.json")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                entries = json.load(f)
            for tj in entries if isinstance(entries, list) else [entries]:
                if (int(tj["world"]) == shards and int(tj["hidden"]) == H and int(tj["intermediate"]) == I
                        and tj.get("format", "mxfp4") == fmt):
                    traffic = float(tj["traffic_bytes_per_expert"]) * (last_d + n_shared)
        except Exception:
            traffic = None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, shared, router, bias, xs, T, moe if fmt == "nvfp4" else None,
                           max_experts=None if args.config == "2" else 6, renorm=(renorm, eps))
    fmt_name = "MXFP4" if fmt == "mxfp4" else "NVFP4"
    if args.config == "2":
        par = f"tp{shards}" if shards > 1 else "single"
    else:
        par = f"tp{info['tp']}xep{info['ep']}" if shards > 1 else "single"
    if shards != world:
        par = f"slice of {par} (rank 0's share on one GPU, no exchange)"

    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "us_per_layer": ms_step * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": f"{fmt} weights x {fmt}(3-term) activations, fp32 accumulate",
        "data": f"synthetic (seeded random {fmt_name} weights, bf16 x ~ N(0,1))",
        "config": {
            "workload": workload_name(args.config, T, shards, H, I, E),
            "tokens": T,
            "parallelism": par,
            "l2": f"inputs larger than L2 (~{layer_bytes / 1e9:.2f} GB of expert weights per step, "
                  f"{POOL} distinct token batches)",
            "launch": "eager, PDL-chained launches",
            "combine": ("fused combine + all-reduce over NVLink peer memory" if peer else
                        "NCCL all-reduce of fp32 partials + round" if world > 1 else "combine"),
            "distinct_experts_per_step": d_mean,
            "layer_weight_bytes": layer_bytes,
            "layer_roofline_frac": (layer_bytes / (ms_step / 1e3) / 1e9) / peak,
        },
        "roofline": {
            "bound": "hbm",
            "kernel": "mm::expert_kernel",
            "achieved": achieved,
            "peak": peak,
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": traffic,
            "algorithmic_bytes_per_launch": k_bytes,
            "launch_ms": k_ms,
        },
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2, "steps": e2e_steps,
                "copies": "per step: x H2D from pinned memory and the output D2H, on a copy stream overlapping the "
                          "neighbouring steps (double-buffered)"},
        "gpu_launches": args.steps * (4 if world == 1 or peer else 5),
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    check()
    if dist is not None:
        dist.barrier()
        if comm is not None:
            comm.close()
        dist.barrier()
        dist.destroy_process_group()


def e2e_pipelined(step, host_x, n, dev):
    """Device time (ms, CUDA events on the compute stream) of n steps through the
    public API with host buffers. Step i copies x from pinned host memory
    (host_x[i % pool]) and its output back to pinned host memory; the copies
    run on a copy stream, double-buffered, so that step i's output copy and
    step i+1's input copy overlap the neighbouring steps' kernels. The region
    opens before the first input copy and closes after the last output copy."""
    comp = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(device=dev)
    T, Hh = host_x.shape[1], host_x.shape[2]
    xdev = [torch.zeros((T, Hh), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    host_out = torch.empty((2, T, Hh), dtype=torch.bfloat16).pin_memory()
    bufs = [{}, {}]
    step(xdev[0], bufs[0])  # allocate each slot's buffers outside the timed region
    step(xdev[1], bufs[1])
    torch.cuda.synchronize()
    ev = lambda: torch.cuda.Event()  # noqa: E731
    h2d, done, d2h = [ev(), ev()], [ev(), ev()], [ev(), ev()]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pool = host_x.shape[0]
    start.record(comp)
    copy.wait_event(start)
    with torch.cuda.stream(copy):
        xdev[0].copy_(host_x[0], non_blocking=True)
        h2d[0].record(copy)
    for i in range(n):
        slot = i & 1
        if i + 1 < n:  # the next step's input, once step i - 1 has consumed that slot
            with torch.cuda.stream(copy):
                if i >= 1:
                    copy.wait_event(done[slot ^ 1])
                xdev[slot ^ 1].copy_(host_x[(i + 1) % pool], non_blocking=True)
                h2d[slot ^ 1].record(copy)
        comp.wait_event(h2d[slot])
        if i >= 2:
            comp.wait_event(d2h[slot])  # step i - 2's output has left this slot's buffer
        out = step(xdev[slot], bufs[slot])
        done[slot].record(comp)
        with torch.cuda.stream(copy):
            copy.wait_event(done[slot])
            host_out[slot].copy_(out, non_blocking=True)
            d2h[slot].record(copy)
    comp.wait_event(d2h[(n - 1) & 1])
    end.record(comp)
    torch.cuda.synchronize()
    return start.elapsed_time(end)


# --------------------------------------------------------------------------- config 5
def run_stack(args):
    """a step of `layers` routed-MoE layers (hidden 7168, 384
    experts, top-8, intermediate 2048, MXFP4, no shared expert) at EP8: rank r
    holds the EP8 window r (48 experts per layer per GPU); routing is replicated;
    each layer's combine is all-reduced over the ranks and followed by the
    residual + RMSNorm hop in the same launch, whose output is the next layer's
    input (bf16 residual stream carried through the step). With fewer than 8
    ranks each rank still holds one EP8 window, so its per-layer work is that of
    an EP8 rank (routes to absent windows are skipped)."""
    import megamoe

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    ep = 8
    if world > ep:
        raise SystemExit("--stack runs at most 8 ranks (EP8)")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    T, L = (args.tokens if args.tokens is not None else 8), args.layers
    per = E // ep
    offset = rank * per
    moes, routers, biases, gammas = [], [], [], []
    for layer in range(L):
        g = torch.Generator(device=dev).manual_seed(1000 + 97 * layer + rank)

        def rnd(shape, lo, hi):
            return torch.randint(lo, hi + 1, shape, dtype=torch.uint8, device=dev, generator=g)

        w = [rnd((per, 2 * I, H // 2), 0, 255), rnd((per, 2 * I, H // 32), 117, 121),
             rnd((per, H, I // 2), 0, 255), rnd((per, H, I // 32), 117, 121)]
        moes.append(megamoe.RoutedMoE(*w, K, max(T, 8), router_experts=E, expert_offset=offset))
        gx = torch.Generator(device=dev).manual_seed(7 + layer)  # replicated on every rank
        routers.append((torch.randn((E, H), device=dev, generator=gx) * 0.02).to(torch.bfloat16))
        biases.append((torch.randn((E,), device=dev, generator=gx) * 0.01).float())
        gammas.append((1 + 0.1 * torch.randn((H,), device=dev, generator=gx)).to(torch.bfloat16))
    comm = megamoe.PeerAllReduce(max(T, 8), H)
    stack = megamoe.MoEStack(moes, routers, gammas, comm, biases=biases, routed_scaling_factor=SCALE)
    gx = torch.Generator(device=dev).manual_seed(5)
    xs = torch.randn((POOL, T, H), device=dev, generator=gx).to(torch.bfloat16)
    res_pool = torch.randn((POOL, T, H), device=dev, generator=gx).to(torch.bfloat16)
    residual = torch.empty((T, H), dtype=torch.bfloat16, device=dev)

    def step(i, x=None):
        residual.copy_(res_pool[i % POOL])
        return stack.forward(xs[i % POOL] if x is None else x, residual)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(max(args.warmup, 3)):
        step(i)
    stack.check()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for i in range(args.steps):
            step(i)
        end.record()
        torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end))
    barrier()
    stack.check()
    ms_step = ms / args.steps
    value = T * args.steps / (ms / 1e3)

    # local distinct experts per layer (layer by layer through the same hop, 4 pool entries)
    d_local = []
    for i in range(4):
        cur = xs[i]
        residual.copy_(res_pool[i])
        for li, m in enumerate(moes):
            bufs = {}
            cur, _ = m.forward(cur, router_weight=routers[li], bias=biases[li], routed_scaling_factor=SCALE,
                               buffers=bufs, comm=comm, residual=residual, gamma=gammas[li])
            ids = bufs["ids"]
            d_local.append(int(torch.unique(ids[(ids >= offset) & (ids < offset + per)]).numel()))
            residual.copy_(bufs["residual_out"])
    torch.cuda.synchronize()
    stack.check()
    eb = expert_bytes(H, I)
    d_mean = float(np.mean(d_local))
    step_bytes = L * (d_mean * eb + E * H * 2)
    step_bytes_max = max_over_ranks(step_bytes)

    # the dominant kernel alone: layer 0's expert kernel relaunched on its last tables
    bufs = {}
    moes[0].forward(xs[0], router_weight=routers[0], bias=biases[0], routed_scaling_factor=SCALE, buffers=bufs,
                    comm=comm, residual=residual, gamma=gammas[0])
    ids = bufs["ids"]
    k_d = int(torch.unique(ids[(ids >= offset) & (ids < offset + per)]).numel())
    reps = 200
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in evs:
        moes[0].rearm_experts()
        a.record()
        moes[0].rerun_experts(T, bufs["record"], bufs["rows"], rearm=False)
        b.record()
    torch.cuda.synchronize()
    k_ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
    stack.check()
    peak, peak_kind = peaks()
    k_bytes = k_d * eb
    achieved = k_bytes / (k_ms / 1e3) / 1e9 if k_d else 0.0

    # end to end: the step's x and residual from pinned host memory, output read back
    host_x = torch.empty((POOL, T, H), dtype=torch.bfloat16).pin_memory()
    host_x.copy_(xs.cpu())
    host_r = torch.empty((POOL, T, H), dtype=torch.bfloat16).pin_memory()
    host_r.copy_(res_pool.cpu())
    host_out = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
    xdev = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    e2e_steps = min(args.steps, 200)
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for i in range(e2e_steps):
        xdev.copy_(host_x[i % POOL], non_blocking=True)
        residual.copy_(host_r[i % POOL], non_blocking=True)
        out = stack.forward(xdev, residual)
        host_out.copy_(out, non_blocking=True)
    e2.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2))
    stack.check()

    line = {
        "metric": f"{L}-layer routed-MoE stack tokens/s per step (us/layer = 1e3 * ms_per_step / {L})",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "us_per_layer": ms_step * 1e3 / L,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "mxfp4 weights x mxfp4(3-term) activations, fp32 accumulate",
        "data": "synthetic (seeded random MXFP4 weights, bf16 x and residual ~ N(0,1))",
        "config": {
            "workload": f"BASELINE config 5: {L} routed-MoE layers, hidden {H}, {E} experts (EP8: {per} per GPU, "
                        f"window {rank}), intermediate {I}, sigmoid+bias top-{K}, scale {SCALE}, MXFP4, "
                        f"{T} tokens, bf16 residual + RMSNorm hop between layers",
            "tokens": T,
            "layers": L,
            "parallelism": f"ep8 windows on {world} GPU(s)",
            "l2": f"inputs larger than L2 (~{step_bytes / 1e9:.1f} GB of expert weights per step)",
            "launch": "one mm_stack_forward call per step (eager, PDL-chained across layers)",
            "local_distinct_experts_per_layer": d_mean,
            "step_weight_bytes_max_rank": step_bytes_max,
            "step_roofline_frac": (step_bytes_max / (ms_step / 1e3) / 1e9) / peak,
        },
        "roofline": {
            "bound": "hbm",
            "kernel": "mm::expert_kernel (layer 0)",
            "achieved": achieved,
            "peak": peak,
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": None,
            "algorithmic_bytes_per_launch": k_bytes,
            "launch_ms": k_ms,
        },
        "e2e": {"value": T * e2e_steps / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 2 * T * H * 2,
                "d2h_bytes_per_step": T * H * 2, "steps": e2e_steps},
        "gpu_launches": args.steps * L * 4,
        "clocks": clocks.summary(),
        "cpu_baseline": None,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------- CPU legs
def _cpu_layer_step(x_bf16, router_bf16, bias, experts_w, shared_w, oracle, max_experts=None,
                    renorm=(True, 0.0)):
    """One layer on the CPU oracle: routing, then the activated experts (all of
    them, or the first max_experts) and the shared expert. Returns (seconds of
    routing, seconds per expert MLP, distinct experts)."""
    t0 = time.perf_counter()
    logits = oracle.router_gemv(oracle.bf16_bits(x_bf16), oracle.bf16_bits(router_bf16))
    w, ids = oracle.gate_topk(logits, bias.numpy(), K, scale=SCALE, renormalize=renorm[0], eps=renorm[1])
    t1 = time.perf_counter()
    x = x_bf16.float()
    out = torch.zeros_like(x)
    experts = sorted(set(ids.flatten().tolist()))
    ran = experts if max_experts is None else experts[:max_experts]
    for e in ran:
        toks = [t for t in range(ids.shape[0]) if e in ids[t]]
        ws = [float(w[t][list(ids[t]).index(e)]) for t in toks]
        y = oracle.expert_mlp(x[toks], *experts_w(e))
        for j, t in enumerate(toks):
            out[t] += ws[j] * y[j]
    out += oracle.expert_mlp(x, *shared_w)
    t2 = time.perf_counter()
    return t1 - t0, (t2 - t1) / (len(ran) + 1), len(experts)


def cpu_baseline(w, shared, router, bias, xs, T, nv_moe=None, max_experts=None, renorm=(True, 0.0)):
    """The oracle port timed on this host's cores on the same workload, after
    one warm-up step: a full layer step (every activated expert + shared), or
    with max_experts a bounded sample whose layer time is routing + (distinct
    + 1) x the mean expert time."""
    from oracle import oracle

    threads = torch.get_num_threads()
    router_c, bias_c = router.cpu(), bias.cpu()
    xc = [xs[i].cpu() for i in range(2)]
    needed = set()
    for xi in xc:
        logits = oracle.router_gemv(oracle.bf16_bits(xi), oracle.bf16_bits(router_c))
        _, ids = oracle.gate_topk(logits, bias_c.numpy(), K, scale=SCALE, renormalize=renorm[0], eps=renorm[1])
        ex = sorted(set(ids.flatten().tolist()))
        needed |= set(ex if max_experts is None else ex[:max_experts])
    if nv_moe is None:
        cache = {e: tuple(t[e].cpu() for t in w) + (None, "exact") for e in needed}
        sh = tuple(t[0].cpu() for t in shared) + (None, "exact")
    else:  # NVFP4: scale_2 per expert and the layer's static input scales
        s13, s2 = nv_moe.w13_scale_2.cpu(), nv_moe.w2_scale_2.cpu()
        ins = nv_moe.input_scale
        cache = {e: tuple(t[e].cpu() for t in w) + (None, "exact", 3, (float(s13[e]), float(s2[e]), ins))
                 for e in needed}
        sh = tuple(t[0].cpu() for t in shared[:4]) + (None, "exact", 3,
                                                       (float(shared[4][0]), float(shared[5][0]), ins))
    _cpu_layer_step(xc[0], router_c, bias_c, lambda e: cache[e], sh, oracle, max_experts, renorm)  # warm-up
    route_s, per_expert_s, d = _cpu_layer_step(xc[1], router_c, bias_c, lambda e: cache[e], sh, oracle,
                                               max_experts, renorm)
    layer_s = route_s + (d + 1) * per_expert_s
    sample = (f"1 full layer step ({T} tokens, every activated expert + shared) after 1 warm-up"
              if max_experts is None else
              f"routing + {max_experts} of {d} activated experts + shared ({T} tokens) after 1 warm-up; layer "
              f"time = routing + (distinct + 1) x mean expert time")
    return {"value": T / layer_s, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{sample}; {layer_s:.1f} s per layer"}


def run_reference(args):
    """The reference path's CPU implementation (the oracle port: the reference
    itself has no CPU MoE path) on all host threads, on this arm's workload
    (or 4 with --config 4): every step is one full layer
    step, router GEMV -> top-k -> every activated expert's MLP (dequantized
    FP4 weights, fp32) -> weighted combine + the shared expert, on the next of 4
    seeded token batches. Each expert's weights are generated once (seeded by
    its id) and kept resident, as on the GPU. The run stops early, with the
    steps it completed reported, when it would outlast a few minutes."""
    from oracle import oracle

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    global H, I, E
    H, I, E, fmt = CONFIGS[args.config]
    torch.set_num_threads(os.cpu_count() or 1)
    threads = torch.get_num_threads()
    T = args.tokens if args.tokens is not None else (80 if args.config == "4" else 8)
    renorm = routing_rule(args.config)
    nv = fmt == "nvfp4"
    ins = (8.0 / (6.0 * 448.0), 2.0 ** -4)  # NVFP4 static input scales (FC1 for |x| <= 8)

    def expert(seed):
        g = torch.Generator().manual_seed(seed)
        codes = lambda shape: torch.randint(0, 256, shape, dtype=torch.uint8, generator=g)  # noqa: E731
        if not nv:
            sc = lambda shape: torch.randint(117, 122, shape, dtype=torch.uint8, generator=g)  # noqa: E731
            return (codes((2 * I, H // 2)), sc((2 * I, H // 32)), codes((H, I // 2)), sc((H, I // 32)), None,
                    "exact")
        sf = lambda shape: (0.5 + 3.5 * torch.rand(shape, generator=g)).to(torch.float8_e4m3fn).view(  # noqa: E731
            torch.uint8)
        s2 = 2.0 ** -8 * (1.0 + 0.25 * float(torch.rand((), generator=g)))
        return (codes((2 * I, H // 2)), sf((2 * I, H // 16)), codes((H, I // 2)), sf((H, I // 16)), None, "exact",
                3, (s2, s2, ins))

    cache = {}

    def weights_of(e):
        if e not in cache:
            cache[e] = expert(1000 + e)
        return cache[e]

    shared_w = expert(999)
    gx = torch.Generator().manual_seed(7)
    router = (torch.randn((E, H), generator=gx) * 0.02).to(torch.bfloat16)
    bias = (torch.randn((E,), generator=gx) * 0.01).float()
    xs = [torch.randn((T, H), generator=gx).to(torch.bfloat16) for _ in range(4)]
    for xb in xs:  # every batch's experts resident before the timed steps (set-up)
        logits = oracle.router_gemv(oracle.bf16_bits(xb), oracle.bf16_bits(router))
        _, ids = oracle.gate_topk(logits, bias.numpy(), K, scale=SCALE, renormalize=renorm[0], eps=renorm[1])
        for e in set(ids.flatten().tolist()):
            weights_of(e)
    budget = 240.0
    step_s, distinct = [], []
    t_begin = time.perf_counter()
    for i in range(args.warmup + args.steps):
        r_s, e_s, d = _cpu_layer_step(xs[i % 4], router, bias, weights_of, shared_w, oracle, None, renorm)
        t1 = time.perf_counter()
        if i >= args.warmup:
            step_s.append(r_s + e_s * (d + 1))
            distinct.append(d)
        if t1 - t_begin > budget and len(step_s) >= 1:
            break
    done = len(step_s)
    ms = float(np.mean(step_s)) * 1e3
    value = T / (ms / 1e3)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": done,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "us_per_layer": ms * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": f"fp32 (dequantized {fmt.upper()} weights, bf16 x)",
        "data": "synthetic (seeded)",
        "config": {"workload": workload_name(args.config, T, args.gpus, H, I, E), "tokens": T,
                   "parallelism": "single" if args.gpus <= 1 else f"the whole layer on rank 0's host cores",
                   "distinct_experts_per_step": float(np.mean(distinct)) if distinct else None},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{done} full layer steps of {T} tokens (router GEMV, top-k, every activated "
                                   f"expert's MLP + the shared expert, combine) after {args.warmup} warm-up; "
                                   f"at most {budget:.0f} s"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- flashinfer
def run_flashinfer(args):
    """SGLang's stock GPU path for this layer, as a same-box comparison: torch's router
    GEMM (bf16 in, fp32 logits), FlashInfer's TRT-LLM-gen fused MoE with its own
    DeepSeekV3-style routing (sigmoid + bias, one group, top-8, renormalize, x 2.5) and
    finalize over the same MXFP4 weights (bf16 activations), the shared expert as a
    second FlashInfer call, the sum. FlashInfer's tactic is autotuned once for the shape
    (as a server does at warm-up). Also reports how far its output is from this
    library's on the same inputs. Config 2, one GPU."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 or args.config != "2":
        if rank == 0:
            print(json.dumps({"impl": "flashinfer", "unavailable": "the FlashInfer comparison runs config 2 on one GPU"}),
                  flush=True)
        return
    if args.tokens is not None and args.tokens < 8:
        # FlashInfer 0.6.11's autotuner crashed on the host (a segfault in
        # cuModuleGetFunction) at 1 token on this B200; the case is not run
        print(json.dumps({"impl": "flashinfer", "unavailable": "FlashInfer's autotuner crashed on the host below 8 "
                                                               "tokens (segfault in cuModuleGetFunction)"}), flush=True)
        return
    sys.path.insert(0, os.path.join(REPO, "baseline"))
    import flashinfer_moe  # sets FlashInfer's cache directory before flashinfer is imported

    global E
    if args.experts is not None:
        E = args.experts
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    T = args.tokens if args.tokens is not None else 8
    moe, w, shared, router, bias, xs, info = build_layer(0, 1, T, dev)
    fl = flashinfer_moe.FlashInferLayer(*w, shared, bias, K, SCALE, T)
    router_t = router.t()
    try:
        torch.mm(xs[0], router_t, out_dtype=torch.float32)

        def logits_of(x):
            return torch.mm(x, router_t, out_dtype=torch.float32)
        router_kind = "torch.mm bf16 -> fp32 out"
    except Exception:
        router_f = router.float().t().contiguous()

        def logits_of(x):
            return torch.mm(x.float(), router_f)
        router_kind = "torch.mm fp32"

    mx = args.fi_act == "mxfp8"
    xq = [flashinfer_moe.mxfp8_quantize(xs[i]) for i in range(POOL)] if mx else None

    def step(x, i=None):
        if mx:
            return fl.forward(x, logits_of(x), *xq[i])
        return fl.forward(x, logits_of(x))

    from flashinfer.autotuner import autotune

    with autotune(True):
        step(xs[0], 0)
    torch.cuda.synchronize()

    # agreement with this library (both are checked separately: this one against the oracle)
    errs = []
    for i in range(8):
        a = step(xs[i], i).float()
        b = moe.forward(xs[i], router_weight=router, bias=bias, routed_scaling_factor=SCALE).float()
        errs.append(float((a - b).abs().max() / b.abs().max()))
    torch.cuda.synchronize()

    for i in range(max(args.warmup, 3)):
        step(xs[i % POOL], i % POOL)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        start.record()
        for i in range(args.steps):
            step(xs[i % POOL], i % POOL)
        end.record()
        torch.cuda.synchronize()
    ms_step = start.elapsed_time(end) / args.steps

    host_x = torch.empty((POOL, T, H), dtype=torch.bfloat16).pin_memory()
    host_x.copy_(xs.cpu())
    host_out = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
    xdev = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    e2e_steps = min(args.steps, 1000)
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for i in range(e2e_steps):
        xdev.copy_(host_x[i % POOL], non_blocking=True)
        host_out.copy_(step(xdev, i % POOL), non_blocking=True)
    e2.record()
    torch.cuda.synchronize()
    e2e_value = T * e2e_steps / (s2.elapsed_time(e2) / 1e3)

    distinct = []
    bufs = {}
    for i in range(POOL):
        moe.forward(xs[i], router_weight=router, bias=bias, routed_scaling_factor=SCALE, buffers=bufs)
        distinct.append(int(torch.unique(bufs["ids"]).numel()))
    torch.cuda.synchronize()
    d_mean = float(np.mean(distinct))
    layer_bytes = (d_mean + 1) * expert_bytes(H, I) + E * H * 2
    peak, peak_kind = peaks()
    line = {
        "impl": "flashinfer",
        "metric": METRIC,
        "value": T / (ms_step / 1e3),
        "unit": "tokens/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "us_per_layer": ms_step * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": ("mxfp4 weights x mxfp8 activations (FlashInfer MxE2m1 x MxE4m3; x quantized before the timed "
                  "region, e2e reuses the pool's codes)" if mx else
                  "mxfp4 weights x bf16 activations (FlashInfer MxE2m1 x Bfloat16)"),
        "data": "synthetic (the mm arm's seeded weights and token batches)",
        "config": {
            "workload": f"BASELINE config 2: one routed-MoE layer, hidden {H}, {E} routed + 1 shared experts, "
                        f"intermediate {I}, sigmoid+bias top-{K}, scale {SCALE}, MXFP4, {T} tokens",
            "tokens": T,
            "parallelism": "single",
            "path": f"{router_kind}; flashinfer.fused_moe.trtllm_fp4_block_scale_moe (routing_method DeepSeekV3, "
                    f"n_group 1, do_finalize); shared expert via trtllm_fp4_block_scale_routed_moe; add",
            "flashinfer": __import__("flashinfer").__version__,
            "distinct_experts_per_step": d_mean,
            "layer_weight_bytes": layer_bytes,
            "layer_roofline_frac": (layer_bytes / (ms_step / 1e3) / 1e9) / peak,
            "peak": peak,
            "peak_kind": peak_kind,
            "max_abs_rel_vs_mm": {"max": max(errs), "median": float(np.median(errs)), "batches": len(errs)},
        },
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2, "steps": e2e_steps},
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)
    moe.check()


def run_ref_sm100(args):
    """B1: the reference's own SM100 routed pair (RoutedExpertGemm: route +
    GEMM1 + GEMM2) and this library's __call__ on the same weights, routings and
    MXFP8 inputs at DeepSeek-V4.1 geometry (hidden 5120, 384 experts, top-6,
    slice 576), timed by the reference benchmark's CUDA-graph method; one JSON
    line with both arms' µs per routed half per case (baseline/ref_sm100.py)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    sys.path.insert(0, os.path.join(REPO, "baseline"))
    import ref_sm100

    reg, why = ref_sm100.reference_module()
    if reg is None:
        print(json.dumps({"impl": "ref-sm100", "unavailable": why}), flush=True)
        return
    torch.cuda.set_device(0)
    rows = [args.tokens] if args.tokens is not None else [1, 6, 16, 48]
    cases = ref_sm100.run(rows, [6, 16, 32, 384], repeats=max(3, args.warmup), replays=20, log=lambda _: None)
    main_case = next((c for c in cases if c["rows"] == 6 and c["distinct"] == 16), cases[0])
    line = {
        "impl": "ref-sm100",
        "metric": "routed-MoE half us (route + gate_up + down), DeepSeek-V4.1 geometry",
        "value": main_case["mm_us"],
        "unit": "us",
        "higher_is_better": False,
        "reference_value": main_case["reference_us"],
        "n_gpus": 1,
        "config": {"workload": "DeepSeek-V4.1 routed half: hidden 5120, 384 experts, top-6, intermediate slice 576 "
                               "(reference padded to 640), MXFP4 weights, MXFP8 routed input; headline case 6 rows, "
                               "16 distinct experts; CUDA graph of 39 halves over two layers, spacer-corrected"},
        "cases": cases,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "ref-sm100":
        run_ref_sm100(args)
    elif args.impl == "flashinfer":
        run_flashinfer(args)
    elif args.stack:
        run_stack(args)
    else:
        run_mm(args)


if __name__ == "__main__":
    main()
