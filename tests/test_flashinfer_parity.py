"""Expert-MLP parity against the reference's own parity target: FlashInfer's
TRT-LLM-gen routed MoE (the call of test/kernels/test_deepseek_v41_moe.py:116-153
in the reference), run on the B200 as a library over the same MXFP4 weights
(processed into its layout by ``megamoe.layouts.canonical_to_trtllm``), with bf16
activations. Both FlashInfer and this library are held to the CPU oracle's
dequantize-then-fp32 layer (max|got - ref| / max|ref| <= 2e-2) and to each other.

Opt-in (MM_FLASHINFER_TESTS=1) and needs FlashInfer's prebuilt launcher
(``python baseline/flashinfer_moe.py build``): FlashInfer is a comparison here,
never part of the product path."""

import os
import sys

import numpy as np
import pytest
import torch

import oracle.oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("MM_FLASHINFER_TESTS") != "1",
                                 reason="FlashInfer comparison: set MM_FLASHINFER_TESTS=1")]
TOL = 2e-2


def _fi():
    path = os.path.join(REPO, "baseline")
    if path not in sys.path:
        sys.path.insert(0, path)
    import flashinfer_moe

    return flashinfer_moe


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max())


@pytest.mark.parametrize("T,E,I", [(8, 32, 2048), (32, 64, 2048)])
def test_flashinfer_and_megamoe_match_the_oracle(T, E, I):
    fi = _fi()
    import megamoe

    H, K, scale = 7168, 8, 2.5
    dev = torch.device("cuda", 0)
    layer = O.make_layer(H, I, E, shared=True, seed=31)
    x, router, bias = O.make_inputs(T, H, E, seed=32)
    logits = O.router_gemv(O.bf16_bits(x), O.bf16_bits(router))
    weights, ids = O.gate_topk(logits, bias.numpy(), K, scale=scale)
    ref, _, _ = O.moe_layer(x, ids, weights, layer)

    w = [layer[k].to(dev) for k in ("w13", "w13_scale", "w2", "w2_scale")]
    shared = [t.to(dev) for t in layer["shared"]]
    fl = fi.FlashInferLayer(*w, shared, bias.to(dev), K, scale, T)
    xd = x.to(dev)
    got_fi = fl.forward_routed(xd, torch.from_numpy(ids).to(dev), torch.from_numpy(weights).to(dev))
    got_fi_routing = fl.forward(xd, torch.from_numpy(logits).to(dev))
    moe = megamoe.RoutedMoE(*w, K, T, shared=shared)
    got_mm = moe.forward(xd, logits=torch.from_numpy(logits).to(dev), bias=bias.to(dev),
                         routed_scaling_factor=scale)
    torch.cuda.synchronize()
    moe.check()
    ref_t = torch.from_numpy(np.asarray(ref, dtype=np.float32)) if not torch.is_tensor(ref) else ref
    assert _rel(got_fi, ref_t) <= TOL
    assert _rel(got_fi_routing, ref_t) <= TOL
    assert _rel(got_mm, ref_t) <= TOL
    assert _rel(got_mm, got_fi) <= TOL
