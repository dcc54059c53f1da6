"""Parity at the BASELINE geometries the benchmark times, through the whole step
(router GEMV -> top-k -> route -> experts -> combine) on the bench's own seeded
layer (bench.build_layer: weights generated on the GPU):

  * config 2: hidden 7168, 384 routed + 1 shared experts, intermediate 2048,
    MXFP4, sigmoid + bias top-8, scale 2.5, at 8 and 32 tokens;
  * config 3's tensor-parallel slice: rank 0 of TP8 (intermediate 256 per
    rank, its share of the shared expert) at 32 tokens, its partial output;
  * config 4: hidden 6144, 256 routed + 1 shared experts, intermediate 2048,
    NVFP4 weights and activations, GLM-5.3 routing weights
    (bf16(scale * s / (sum + 1e-20))), 80 tokens.

Ids bit-exact against the CPU oracle's router GEMV + top-k; the slot -> row map
against the oracle's route; the output within 2e-2 (max-abs-rel, BASELINE's
bar) of the oracle's dequantize-then-fp32 layer, checked on up to 8 tokens so
that the CPU oracle multiplies only their activated experts."""

import numpy as np
import pytest
import torch

import oracle.oracle as O

pytestmark = pytest.mark.gpu

OUT_TOL = 2e-2


def _bench():
    import bench

    return bench


def _sub_layer(w, shared, needed, moe, fmt):
    """CPU copies of the needed experts (and the shared expert) for the oracle."""
    idx = torch.tensor(needed, device=w[0].device, dtype=torch.long)
    sub = {"w13": w[0][idx].cpu(), "w13_scale": w[1][idx].cpu(), "w2": w[2][idx].cpu(),
           "w2_scale": w[3][idx].cpu(), "clamp": None, "shared": None}
    if shared is not None:
        sub["shared"] = tuple(t.cpu() for t in shared)
    if fmt == "nvfp4":
        sub.update(fmt="nvfp4", w13_scale_2=moe.w13_scale_2[idx].cpu(), w2_scale_2=moe.w2_scale_2[idx].cpu(),
                   input_scale=moe.input_scale)
    return sub


def _check_layer(config, tokens, world=1, renorm=True, eps=0.0):
    b = _bench()
    saved = (b.H, b.I, b.E)
    b.H, b.I, b.E, fmt = b.CONFIGS[config]
    try:
        dev = torch.device("cuda", 0)
        moe, w, shared, router, bias, xs, info = b.build_layer(0, world, tokens, dev, fmt)
        H, E, K = b.H, b.E, b.K
        bufs = {}
        for i in (0, 1):  # two batches in a row through the same buffers
            x = xs[i]
            out = moe.forward(x, router_weight=router, bias=bias, routed_scaling_factor=b.SCALE, buffers=bufs,
                              renormalize=renorm, renormalize_epsilon=eps)
            torch.cuda.synchronize()
            moe.check()
            xc = x.cpu()
            logits = O.router_gemv(O.bf16_bits(xc), O.bf16_bits(router.cpu()))
            ow, oids = O.gate_topk(logits, bias.cpu().numpy(), K, scale=b.SCALE,
                                   renormalize="scaled_bf16" if renorm == "scaled_bf16" else renorm, eps=eps)
            assert np.array_equal(bufs["ids"].cpu().numpy(), oids), (config, tokens, i)
            assert np.array_equal(bufs["weights"].cpu().numpy().view(np.uint32), ow.view(np.uint32))
            operm, _ = O.route(oids, info["local"], info["offset"])
            assert np.array_equal(bufs["permuted"].cpu().numpy(), operm)
            check = list(range(0, tokens, max(1, tokens // 8)))[:8]
            sel = oids[check]
            needed = sorted({int(e) for e in sel.flatten() if e >= 0})
            remap = {e: j for j, e in enumerate(needed)}
            ids_sub = np.vectorize(lambda e: remap.get(int(e), -1))(sel).astype(np.int32)
            sub = _sub_layer(w, shared, needed, moe, fmt)
            ref, _, _ = O.moe_layer(xc[check], ids_sub, ow[check], sub, numerics="exact")
            err = O.max_abs_rel(out.float().cpu().numpy()[check], ref.numpy())
            assert err <= OUT_TOL, (config, tokens, i, err)
        del moe, w, shared
        torch.cuda.empty_cache()
    finally:
        b.H, b.I, b.E = saved


@pytest.mark.parametrize("tokens", [8, 32])
def test_config2_layer(tokens):
    _check_layer("2", tokens)


@pytest.mark.parametrize("tokens", [8, 32])
def test_config3_tp8_slice(tokens):
    """Rank 0's TP8 slice (intermediate 256: one-stage down tiles, two per unit
    sharing one activation copy); at 8 tokens the gate_up tiles also split K."""
    _check_layer("2", tokens, world=8)


def test_config4_nvfp4_layer_with_glm_weights():
    _check_layer("4", 80, renorm="scaled_bf16", eps=1e-20)
