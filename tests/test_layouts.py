"""The TRT-LLM-gen / FlashInfer processed-weight adapter (megamoe.layouts), MXFP4
and NVFP4:
exact round trips on the CPU; on the GPU, the restated scale swizzle against
FlashInfer's own block_scale_interleave and a layer built from processed
weights against the canonical one."""

import numpy as np
import pytest
import torch

import oracle.oracle as O


def _layouts():
    from megamoe import layouts

    return layouts


@pytest.mark.parametrize("R,C", [(128, 4), (256, 224), (1280, 160), (100, 6), (512, 7)])
def test_scale_swizzle_round_trip(R, C):
    L = _layouts()
    g = torch.Generator().manual_seed(R + C)
    s = torch.randint(0, 256, (R, C), dtype=torch.uint8, generator=g)
    flat = L.interleave_scales(s)
    assert flat.numel() == ((R + 127) // 128 * 128) * ((C + 3) // 4 * 4)
    assert torch.equal(L.deinterleave_scales(flat, R, C), s)
    # the atom: row r, column c of the first 128 x 4 tile lands at 16 (r % 32) + 4 (r / 32) + c
    if R >= 128 and C >= 4:
        assert int(flat[16 * 5 + 4 * 2 + 3]) == int(s[5 + 32 * 2, 3])


@pytest.mark.parametrize("halves", ["w3_w1", "w1_w3"])
def test_trtllm_layout_round_trip(halves):
    L = _layouts()
    layer = O.make_layer(512, 256, 3, shared=False, seed=4)
    w = [layer[k] for k in ("w13", "w13_scale", "w2", "w2_scale")]
    processed = L.canonical_to_trtllm(*w, halves=halves)
    assert not torch.equal(processed[0], w[0])
    back = L.trtllm_to_canonical(*processed, halves=halves)
    for a, b in zip(back, w):
        assert torch.equal(a, b)


@pytest.mark.parametrize("halves", ["w3_w1", "w1_w3"])
def test_trtllm_nvfp4_layout_round_trip(halves):
    """NVFP4 (E4M3 scale per 16): the same row maps, a scale block of 16."""
    L = _layouts()
    layer = O.make_nvfp4_layer(512, 256, 3, shared=False, seed=5)
    w = [layer[k] for k in ("w13", "w13_scale", "w2", "w2_scale")]
    assert w[1].shape[-1] == 512 // 16 and w[3].shape[-1] == 256 // 16
    processed = L.canonical_to_trtllm(*w, halves=halves, weight_format="nvfp4")
    assert not torch.equal(processed[0], w[0])
    back = L.trtllm_to_canonical(*processed, halves=halves, weight_format="nvfp4")
    for a, b in zip(back, w):
        assert torch.equal(a, b)
    with pytest.raises(ValueError):
        L.trtllm_to_canonical(*processed, weight_format="fp8")


def test_trtllm_w13_tile_holds_one_gate_up_feature_block():
    """A 128-row tile of processed w13 holds features [64m, 64m + 64) of both
    halves, the tile this library's gate_up unit multiplies."""
    L = _layouts()
    p13, _, _, _ = L._perms(2 * 256, 256, 512, 128)
    for m in range(4):
        rows = sorted(int(r) for r in p13[128 * m:128 * (m + 1)])
        assert rows == list(range(64 * m, 64 * m + 64)) + list(range(256 + 64 * m, 256 + 64 * m + 64))


@pytest.mark.gpu
def test_scale_swizzle_matches_flashinfer():
    from flashinfer.fp4_quantization import block_scale_interleave

    L = _layouts()
    g = torch.Generator().manual_seed(0)
    for R, C in ((128, 4), (1280, 160), (7168, 64), (256, 28)):
        s = torch.randint(0, 256, (R, C), dtype=torch.uint8, generator=g).cuda()
        want = block_scale_interleave(s).reshape(-1).cpu()
        got = L.interleave_scales(s).cpu()
        assert torch.equal(got, want), (R, C)


@pytest.mark.gpu
def test_layer_from_trtllm_weights_equals_canonical_layer():
    import megamoe

    H, I, E, K, T = 1024, 512, 8, 4, 6
    layer = O.make_layer(H, I, E, shared=False, seed=8)
    dev = torch.device("cuda", 0)
    w = [layer[k].to(dev) for k in ("w13", "w13_scale", "w2", "w2_scale")]
    processed = _layouts().canonical_to_trtllm(*w)
    a = megamoe.RoutedMoE(*w, K, 8)
    b = megamoe.RoutedMoE.from_trtllm(*processed, K, 8)
    x, _, _ = O.make_inputs(T, H, E, seed=8)
    g = torch.Generator().manual_seed(8)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).int().to(dev)
    wts = torch.rand((T, K), generator=g).to(dev)
    ra, _, pa = a(x.to(dev), None, ids, wts)
    rb, _, pb = b(x.to(dev), None, ids, wts)
    assert torch.equal(pa, pb)
    sel = pa.flatten().long()  # the rows the slots point to (padding rows are never written)
    assert torch.equal(ra[sel], rb[sel])


@pytest.mark.gpu
def test_nvfp4_layer_from_trtllm_weights_equals_canonical_layer():
    import megamoe

    H, I, E, K, T = 1024, 512, 8, 4, 6
    layer = O.make_nvfp4_layer(H, I, E, shared=False, seed=9)
    dev = torch.device("cuda", 0)
    w = [layer[k].to(dev) for k in ("w13", "w13_scale", "w2", "w2_scale")]
    nv = dict(weight_format="nvfp4", w13_scale_2=layer["w13_scale_2"].to(dev), w2_scale_2=layer["w2_scale_2"].to(dev),
              input_scale=layer["input_scale"])
    processed = _layouts().canonical_to_trtllm(*w, weight_format="nvfp4")
    a = megamoe.RoutedMoE(*w, K, 8, **nv)
    b = megamoe.RoutedMoE.from_trtllm(*processed, K, 8, **nv)
    x, _, _ = O.make_inputs(T, H, E, seed=9)
    g = torch.Generator().manual_seed(9)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).int().to(dev)
    wts = torch.rand((T, K), generator=g).to(dev)
    ra, _, pa = a(x.to(dev), None, ids, wts)
    rb, _, pb = b(x.to(dev), None, ids, wts)
    assert torch.equal(pa, pb)
    sel = pa.flatten().long()
    assert torch.equal(ra[sel], rb[sel])
