"""Byte-exact quantization on the GPU, read back from the layer's own buffers.

The chain carries each activation into its GEMMs as FP4 terms (MXFP4: E2M1 codes
with an E8M0 scale per 32; NVFP4: E2M1 with an E4M3 scale per 16 under the
layer's static input scale). These tests read the code and scale bytes the
kernels wrote (``RoutedMoE.read_scratch``) and compare them with the CPU
oracle's quantizer byte for byte:

  * the routed input x, quantized by the router launch, over blocks at amax 0,
    bf16 subnormals, the bf16 maximum (E4M3 scale saturation for NVFP4), single
    non-zeros, power-of-two amax boundaries and random magnitudes;
  * the routed input given as MXFP8 (the reference's x_quant / x_scale);
  * the SwiGLU output h, quantized by the expert kernel's gate_up epilogue. The
    layer is built so that h is exact in any summation order: every up row of
    w13 has one non-zero weight (its product with each activation term is
    exact), and the gate rows are clamped at L = 32, which they exceed, so that
    h = up * 32 / (1 + e^-32) = up * 32 exactly in fp32. The reference pins its
    own quantization bytes the same way (test_deepseek_v41_moe.py:858-905,
    rule in route_quant.cuh:1-15).

Also: GLM-5.3's routing weight rule on the GPU against the oracle, bit for bit."""

import numpy as np
import pytest
import torch

import oracle.oracle as O

pytestmark = pytest.mark.gpu

ROWS_TOL = 1e-2
OUT_TOL = 2e-2


def _special_x(T, H, seed, huge=3.3e38):
    """bf16 [T, H] whose 32-element blocks walk the quantizer's edge cases."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((T, H), generator=g)
    blocks = H // 32
    for t in range(T):
        for b in range(blocks):
            kind = (t * blocks + b) % 9
            blk = x[t, 32 * b:32 * b + 32]
            if kind == 0:
                blk.zero_()                                      # amax 0
            elif kind == 1:
                blk.mul_(1e-39)                                  # bf16 subnormals
            elif kind == 2:
                blk.copy_(torch.sign(blk) * huge)                # the bf16 range's top
            elif kind == 3:
                blk.zero_()
                blk[(t + b) % 32] = -0.75                        # one non-zero
            elif kind == 4:
                blk.clamp_(-5.0, 5.0)
                blk[3] = 6.0 * 2.0 ** ((t + b) % 7 - 3)          # amax at 6 * 2^k
            elif kind == 5:
                blk.mul_(2.0 ** ((t * 7 + b) % 40 - 20))         # wide exponents
            elif kind == 6:
                blk.copy_(torch.full((32,), 0.5) * (1 + (b % 3)))  # constant block
    return x.to(torch.bfloat16)


def _layer(fmt, H, I, E, seed, **kw):
    return O.make_nvfp4_layer(H, I, E, shared=False, seed=seed, **kw) if fmt == "nvfp4" else \
        O.make_layer(H, I, E, shared=False, seed=seed, **kw)


def _moe(layer, K, max_rows):
    import megamoe

    dev = torch.device("cuda", 0)
    w = [layer[k].to(dev) for k in ("w13", "w13_scale", "w2", "w2_scale")]
    nv = {}
    if layer.get("fmt") == "nvfp4":
        nv = dict(weight_format="nvfp4", w13_scale_2=layer["w13_scale_2"].to(dev),
                  w2_scale_2=layer["w2_scale_2"].to(dev), input_scale=layer["input_scale"])
    clamp = None if layer.get("clamp") is None else layer["clamp"].to(dev)
    return megamoe.RoutedMoE(*w, K, max_rows, clamp=clamp, **nv)


def _quant(v, fmt, layer, which):
    """The oracle's FP4 terms of fp32 v [..., K]: (codes, scales) with a leading terms axis."""
    if fmt == "nvfp4":
        return O.nvfp4_quant(v, 3, layer["input_scale"][which])
    return O.fp4_quant(v, 3)


@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4"])
@pytest.mark.parametrize("T", [1, 5, 16])
def test_routed_input_terms_bitexact(fmt, T):
    H, I, E, K = 2048, 256, 8, 2
    layer = _layer(fmt, H, I, E, seed=40 + T)
    moe = _moe(layer, K, 16)
    x = _special_x(T, H, seed=T)
    g = torch.Generator().manual_seed(T)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).int()
    moe(x.cuda(), None, ids.cuda())
    got_q = moe.read_scratch("x_codes")[:, :T].cpu().numpy()
    got_s = moe.read_scratch("x_scales")[:, :T].cpu().numpy()
    moe.check()
    want_q, want_s = _quant(x.float().numpy(), fmt, layer, 0)
    assert np.array_equal(got_q, want_q)
    assert np.array_equal(got_s, want_s)


@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4"])
def test_mxfp8_routed_input(fmt):
    """The reference's call shape: (x_quant E4M3 [T, H], x_scale E8M0 [T, H/32],
    topk_ids, topk_weights). Each element enters as e4m3 * 2^(scale - 127): the
    layer's FP4 terms of that value are the oracle's bit for bit, the rows
    match the oracle fed the same values, and gate_topk_and_gemms takes the
    same pair."""
    H, I, E, K, T = 2048, 256, 16, 4, 8
    layer = _layer(fmt, H, I, E, seed=77)
    moe = _moe(layer, K, 16)
    x, _, _ = O.make_inputs(T, H, E, seed=77)
    xv = x.float().numpy()
    xv[1, :64] *= 1e-30  # blocks whose MXFP8 scale is tiny
    qh, _, sh, _ = O.mxfp8_quant(xv, 1)
    xdeq = O.mxfp8_dequant(qh, sh).astype(np.float32)
    g = torch.Generator().manual_seed(77)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).int()
    w = torch.rand((T, K), generator=g)
    xq = torch.from_numpy(qh).cuda().view(torch.float8_e4m3fn)
    xs = torch.from_numpy(sh).cuda()
    rows, wo, perm = moe(xq, xs, ids.cuda(), w.cuda())
    got_q = moe.read_scratch("x_codes")[:, :T].cpu().numpy()
    got_s = moe.read_scratch("x_scales")[:, :T].cpu().numpy()
    want_q, want_s = _quant(xdeq, fmt, layer, 0)
    assert np.array_equal(got_q, want_q)
    assert np.array_equal(got_s, want_s)
    out = moe.finalize(rows, wo, perm)
    moe.check()
    xt = torch.from_numpy(xdeq)
    ex, _, _ = O.moe_layer(xt, ids.numpy(), w.numpy(), layer, numerics="exact")
    _, kn_rows, _ = O.moe_layer(xt, ids.numpy(), w.numpy(), layer, numerics="kernel")
    pc = perm.cpu().numpy()
    got_rows = np.stack([rows.float().cpu()[pc[t, k]].numpy() for (t, k) in kn_rows])
    want_rows = np.stack([v.numpy() for v in kn_rows.values()])
    assert O.max_abs_rel(got_rows, want_rows) <= ROWS_TOL
    assert O.max_abs_rel(out.float().cpu().numpy(), ex.numpy()) <= OUT_TOL
    # the gate path with the same MXFP8 input
    logits = torch.randn((T, E), generator=g).float()
    rows2, w2, perm2, ids2 = moe.gate_topk_and_gemms(xq, xs, logits.cuda(), None, 2.5)
    ow, oids = O.gate_topk(logits.numpy(), None, K, scale=2.5)
    assert np.array_equal(ids2.cpu().numpy(), oids)
    assert np.array_equal(moe.read_scratch("x_codes")[:, :T].cpu().numpy(), want_q)
    moe.check()


# ----------------------------------------------------------------------------- h terms
CLAMP = 32.0


def _exact_h_layer(fmt, H, I, E, seed):
    """A layer whose h = SwiGLU(x W13^T) is exact in any summation order (see the
    module docstring), and the recipe to recompute it. Returns (layer, cols,
    wvals): up feature f of expert e multiplies x[:, cols[e, f]] by wvals[e, f]
    (in the weights' own units: E2M1 x E8M0 for MXFP4, E2M1 x E4M3 for NVFP4)."""
    g = torch.Generator().manual_seed(seed)
    nv = fmt == "nvfp4"
    blk = 16 if nv else 32
    w13 = torch.zeros((E, 2 * I, H // 2), dtype=torch.uint8)
    e4m3 = O.e4m3_lut()
    if nv:
        # scales: E4M3 1.0 for the gate rows' block 0, random normal E4M3 codes elsewhere
        s13 = torch.randint(0x08, 0x77, (E, 2 * I, H // blk), dtype=torch.uint8, generator=g)
        s13[:, :I, 0] = 0x38  # 1.0
    else:
        s13 = torch.randint(117, 122, (E, 2 * I, H // blk), dtype=torch.uint8, generator=g)
        s13[:, :I, 0] = 127  # 1.0
    w13[:, :I, 0] = 0x07  # gate rows: +6 at element 0, zero elsewhere
    cols = np.zeros((E, I), dtype=np.int64)
    wvals = np.zeros((E, I), dtype=np.float64)
    e2m1 = O.E2M1.astype(np.float64)
    for e in range(E):
        for f in range(I):
            if e == 0 and f < 32:
                cols[e, f] = 32  # an all-zero up row (its h block has amax 0)
                continue
            c = 32 + int(torch.randint(0, H - 32, (1,), generator=g))
            nib = int(torch.randint(1, 16, (1,), generator=g))
            if nib == 8:
                nib = 9  # -0 -> -0.5
            byte = c // 2
            w13[e, I + f, byte] = nib if c % 2 == 0 else (nib << 4)
            group = f // 32
            if nv:
                code = int(s13[e, I + f, c // blk])
                sval = float(e4m3[code])
            else:
                # magnitudes that differ per 32-feature group: E8M0 127 + d, d in [-24, 2]
                d = (group * 5 + e) % 27 - 24
                s13[e, I + f, c // blk] = 127 + d
                sval = 2.0 ** d
            cols[e, f] = c
            wvals[e, f] = e2m1[nib] * sval
    w2 = torch.randint(0, 256, (E, H, I // 2), dtype=torch.uint8, generator=g)
    layer = {"w13": w13, "w13_scale": s13, "w2": w2, "clamp": torch.full((E,), CLAMP), "shared": None}
    if nv:
        layer["w2_scale"] = torch.full((E, H, I // 16), 0x38, dtype=torch.uint8)
        layer.update(fmt="nvfp4", w13_scale_2=torch.ones(E), w2_scale_2=torch.ones(E),
                     input_scale=(float(np.float32(8.0 / (6.0 * 448.0))), 0.25))
    else:
        layer["w2_scale"] = torch.full((E, H, I // 32), 120, dtype=torch.uint8)
    return layer, cols, wvals


def _x_for_exact_h(T, H, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((T, H), generator=g).clamp(-4.0, 4.0)
    x[:, 0] = 8.0  # every gate row's input: the gate is far above the clamp
    for b in range(1, H // 32):
        x[:, 32 * b:32 * b + 32] *= 2.0 ** ((b * 3) % 25 - 12)
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4"])
@pytest.mark.parametrize("H,T", [(1024, 3), (1024, 8), (1024, 24), (512, 8), (512, 24)])
def test_swiglu_output_terms_bitexact(fmt, H, T):
    """h's terms for every requantization path: hidden 1024 splits the gate_up
    tiles (K chunks; one- or two-row segments finish in the half's last warp,
    more rows are shared out over the chunks' warps), hidden 512 leaves them
    whole (a row or two one at a time, 3-4 rows in a group, more rows staged
    two lanes per MXFP4 block); 24 tokens over 4 experts give ~12 rows each."""
    I, E, K = 256, 4, 2
    layer, cols, wvals = _exact_h_layer(fmt, H, I, E, seed=11 + T + H)
    moe = _moe(layer, K, max(16, T))
    x = _x_for_exact_h(T, H, seed=T)
    g = torch.Generator().manual_seed(100 + T)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).int()
    _, _, perm = moe(x.cuda(), None, ids.cuda())
    hq = moe.read_scratch("h_codes").cpu().numpy()
    hs = moe.read_scratch("h_scales").cpu().numpy()
    moe.check()
    # the activation terms the kernel multiplies, each term separately
    xq, xsc = _quant(x.float().numpy(), fmt, layer, 0)
    terms = []
    for t in range(3):
        if fmt == "nvfp4":
            terms.append(O.nvfp4_dequant(xq[t:t + 1], xsc[t:t + 1], 1.0).astype(np.float64))
        else:
            terms.append(O.fp4_dequant(xq[t:t + 1], xsc[t:t + 1]).astype(np.float64))
    nv = fmt == "nvfp4"
    alpha = np.float32(np.float32(1.0) * np.float32(layer["input_scale"][0])) if nv else None
    pc = perm.cpu().numpy()
    for tok in range(T):
        for k in range(K):
            e = int(ids[tok, k])

            def acc(colv, wv):
                # exact products; each term's accumulator is a sum of K products from
                # +0, so a zero product of a negative weight accumulates to +0, not -0
                a = [np.float32(0.0) + np.float32(terms[t][tok, colv] * wv) for t in range(3)]
                s = (a[0] + a[1]) + a[2]
                return s * alpha if nv else s

            gate = acc(np.zeros(I, dtype=np.int64), 6.0)
            assert np.all(gate >= CLAMP), "the gate must exceed the clamp for h to be exact"
            up = acc(cols[e], wvals[e]).astype(np.float32)
            h = (np.clip(up, -CLAMP, CLAMP) * np.float32(CLAMP)).astype(np.float32)
            want_q, want_s = _quant(h[None, :], fmt, layer, 1)
            prow = pc[tok, k]
            assert np.array_equal(hq[:, prow, :I // 2], want_q[:, 0]), (tok, k)
            assert np.array_equal(hs[:, prow, :I // (16 if nv else 32)], want_s[:, 0]), (tok, k)


# ----------------------------------------------------------------------------- GLM rule
@pytest.mark.parametrize("E,K", [(256, 8), (384, 6), (64, 16)])
def test_scaled_bf16_weight_rule_bitexact(E, K):
    """GLM-5.3's routing weights, bf16(scale * s / (sum + 1e-20)) with the
    butterfly-order sum, from the stateless top-k and from the layer's front
    launch, equal the oracle's bit for bit; every weight is a bf16 value."""
    import megamoe

    g = torch.Generator().manual_seed(E + K)
    H, I = 1024, 256
    layer = O.make_layer(H, I, E, shared=False, seed=5)
    moe = _moe(layer, K, 32)
    for T in (1, 8, 16, 30):
        logits = torch.randn((T, E), generator=g).float()
        bias = (torch.randn(E, generator=g) * 0.05).float()
        valid = max(1, T - 3)
        nv = torch.tensor([valid], dtype=torch.int32, device="cuda")
        w, ids = megamoe.gate_topk(logits.cuda(), bias.cuda(), K, renormalize="scaled_bf16",
                                   routed_scaling_factor=2.5, renormalize_epsilon=1e-20, num_valid=nv)
        ow, oids = O.gate_topk(logits.numpy(), bias.numpy(), K, renormalize="scaled_bf16", scale=2.5, eps=1e-20,
                               num_valid=valid)
        assert np.array_equal(ids.cpu().numpy(), oids), T
        assert np.array_equal(w.cpu().numpy().view(np.uint32), ow.view(np.uint32)), T
        assert np.all((ow.view(np.uint32) & 0xffff) == 0)  # bf16 values
        x = torch.randn((T, H), generator=g).to(torch.bfloat16)
        _, w2, _, ids2 = moe.gate_topk_and_gemms(None, None, logits.cuda(), bias.cuda(), 2.5, nv, None, 1e-20,
                                                 x=x.cuda(), renormalize="scaled_bf16")
        assert np.array_equal(ids2.cpu().numpy(), oids), T
        assert np.array_equal(w2.cpu().numpy().view(np.uint32), ow.view(np.uint32)), T
    moe.check()
