"""The CPU oracle against the reference: golden route fixtures generated from the
reference's own route kernels, the live reference kernels when they are built
here, and known-answer cases of the reference's routing / quantization rules."""

import ctypes
import math
import os

import numpy as np
import pytest
import torch

import oracle.oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "route_cases.npz")


# ------------------------------------------------------------------ route record pins
def test_route_matches_golden_fixtures():
    data = np.load(GOLDEN)
    n = int(data["count"][0])
    assert n >= 50
    for i in range(n):
        ids = data[f"ids_{i}"]
        local, offset = (int(v) for v in data[f"meta_{i}"])
        perm, rec = O.route(ids, local, offset)
        assert np.array_equal(perm, data[f"perm_{i}"]), i
        assert np.array_equal(rec, data[f"rec_{i}"]), i


@pytest.mark.skipif(O.ref_route_lib() is None, reason="reference route kernels not built here")
def test_route_matches_live_reference():
    ref = O.ref_route_lib()
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    rng = np.random.default_rng(5)
    for _ in range(150):
        T = int(rng.integers(1, 65))
        K = int(rng.integers(1, 9))
        E = int(rng.choice([32, 96, 128, 384]))
        K = min(K, 512 // T)
        ids = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
        u = rng.random()
        if u < 0.45:
            local, offset = E, 0
        elif u < 0.8:
            local, offset = E // 2, int(rng.integers(0, 2)) * (E // 2)
        else:  # balanced dealing to group 0 or 1 (route.cuh:39-46)
            local, offset = E, -1 - int(rng.integers(0, 2))
        perm, rec = O.route(ids, local, offset)
        rp, rr = np.empty_like(perm), np.empty_like(rec)
        ref.ref_route_wide(P(ids), P(rp), P(rr), T, K, local, offset)
        assert np.array_equal(perm, rp) and np.array_equal(rec, rr)
        if T <= 8 and local % 32 == 0:
            barrier = np.zeros(1, np.uint32)
            ref.ref_route(P(ids), P(rp), P(rr), P(barrier), T, K, local, offset)
            assert np.array_equal(perm, rp) and np.array_equal(rec, rr)


def test_route_record_layout_known_answer():
    # two rows, top-2, 8 experts: row 0 -> {3, 1}, row 1 -> {1, 5}
    ids = np.array([[3, 1], [1, 5]], np.int32)
    perm, rec = O.route(ids, 8, 0)
    # experts 1 (rows 0, 1), 3 (row 0), 5 (row 1) -> tiles 0, 1, 2
    assert perm.tolist() == [[8, 0], [1, 16]]
    m = 4  # max_ctas: min(8, 4) + 0
    cw = 4
    assert rec[0] == 24 and rec[1] == 3 and rec[2] == 0 and rec[3] == 0
    assert rec[4:4 + 3].tolist() == [1, 3, 5]
    assert rec[4 + cw:4 + cw + 3].tolist() == [2, 9, 17]
    tok = rec[4 + 2 * cw:]
    assert len(tok) == 8 * m
    assert tok[0] == 0 and tok[1] == 1 and tok[8] == 0 and tok[16] == 1


def test_route_words_matches_reference_formula():
    # routed_expert_gemm.py:107-120
    for T, K, E in [(1, 6, 384), (8, 8, 384), (64, 8, 384), (48, 6, 192), (256, 16, 1024)]:
        slots = T * K
        filled = min(E, slots)
        m = filled + (slots - filled) // 8
        assert O.route_words(T, K, E) == 4 + 2 * ((m + 3) // 4 * 4) + 8 * m


# ------------------------------------------------------------------ scores and keys
def test_det_exp_accuracy():
    L = O.lib()
    xs = np.concatenate([np.linspace(-103.9, 88.7, 40001), [0.0, -0.0, 1e-30, -1e-30, 1e-7]]).astype(np.float32)
    got = np.array([L.or_det_exp(float(x)) for x in xs], dtype=np.float32)
    ref = np.exp(xs.astype(np.float64))
    ulp = np.abs(got.astype(np.float64) - ref) / np.spacing(ref.astype(np.float32)).astype(np.float64)
    assert np.nanmax(ulp[ref > 1e-37]) < 1.0
    assert L.or_det_exp(float("inf")) == float("inf")
    assert L.or_det_exp(-1e30) == 0.0
    assert math.isnan(L.or_det_exp(float("nan")))


def test_routing_key_orders_and_nan_last():
    L = O.lib()
    L.or_routing_key.restype = ctypes.c_uint32
    L.or_routing_key.argtypes = [ctypes.c_float]
    vals = [-math.inf, -3.0, -1e-30, -0.0, 0.0, 1e-30, 2.0, math.inf]
    keys = [L.or_routing_key(v) for v in vals]
    assert keys == sorted(keys)
    assert L.or_routing_key(-0.0) == L.or_routing_key(0.0)  # -0 ranks as +0
    assert L.or_routing_key(float("nan")) < L.or_routing_key(-math.inf)


def test_topk_ties_lowest_id_and_nan_rows():
    # ties go to the lower expert id (gate_topk.cuh:211-290, routing.py:32-70)
    logits = np.zeros((1, 16), np.float32)
    logits[0, [3, 7, 11]] = 1.0
    w, ids = O.gate_topk(logits, None, 4, score="sigmoid")
    assert ids.tolist() == [[3, 7, 11, 0]]
    # a NaN logit ranks below every number; an all-NaN row takes the lowest ids
    logits = np.full((2, 8), np.nan, np.float32)
    logits[0, 5] = -1e9
    w, ids = O.gate_topk(logits, None, 2, score="sigmoid")
    assert ids[0, 0] == 5 and ids[0, 1] == 0
    assert ids[1].tolist() == [0, 1]
    # padded rows: id -1, weight 0
    w, ids = O.gate_topk(np.random.default_rng(0).standard_normal((4, 16)).astype(np.float32), None, 3,
                         num_valid=2)
    assert (ids[2:] == -1).all() and (w[2:] == 0).all() and (ids[:2] >= 0).all()


def test_topk_weights_renormalized_and_scaled():
    rng = np.random.default_rng(1)
    logits = rng.standard_normal((5, 64)).astype(np.float32)
    bias = (rng.standard_normal(64) * 0.01).astype(np.float32)
    w, ids = O.gate_topk(logits, bias, 8, score="sigmoid", scale=2.5)
    assert np.allclose(w.sum(1), 2.5, rtol=1e-6)
    s = 1 / (1 + np.exp(-logits.astype(np.float64)))
    keys = s + bias
    for t in range(5):
        assert set(ids[t]) == set(np.argsort(-keys[t], kind="stable")[:8])
        assert np.allclose(w[t], 2.5 * s[t, ids[t]] / s[t, ids[t]].sum(), rtol=1e-5)
    w, ids = O.gate_topk(logits, None, 6, score="softmax")
    for t in range(5):
        top = np.argsort(-logits[t], kind="stable")[:6]
        assert ids[t].tolist() == top.tolist()
        e = np.exp(logits[t, top].astype(np.float64) - logits[t, top].max())
        assert np.allclose(w[t], e / e.sum(), rtol=1e-5)
    w, _ = O.gate_topk(logits, None, 4, score="sigmoid", renormalize=False, scale=2.0)
    assert (w <= 2.0).all()


# ------------------------------------------------------------------ MX quantization
def test_mx_scale_code_known_answers():
    L = O.lib()
    L.or_mx_scale_code.restype = ctypes.c_uint32
    L.or_mx_scale_code.argtypes = [ctypes.c_float]
    assert L.or_mx_scale_code(0.0) == 127     # zero block: scale 1
    assert L.or_mx_scale_code(448.0) == 127   # exactly representable maximum
    assert L.or_mx_scale_code(449.0) == 128   # rounded up: never saturates
    assert L.or_mx_scale_code(224.0) == 126
    assert L.or_mx_scale_code(1.0) == 119     # 1/448 -> 2^-9 * 1.14 -> exponent -8 after rounding up


def test_e4m3_matches_torch_in_range():
    L = O.lib()
    v = np.concatenate([np.random.default_rng(2).standard_normal(20000) * 60,
                        np.linspace(-0.05, 0.05, 4001), [448.0, -448.0, 0.0, -0.0]]).astype(np.float32)
    v = v[np.abs(v) <= 448]
    mine = np.array([L.or_e4m3(float(x)) for x in v], dtype=np.uint8)
    ref = torch.tensor(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(mine, ref)
    assert L.or_e4m3(1e6) == 0x7E and L.or_e4m3(-1e6) == 0xFE  # saturating
    assert L.or_e4m3(float("nan")) == 0x7F


def test_mxfp4_terms_converge():
    v = np.random.default_rng(3).standard_normal((8, 1024)).astype(np.float32)
    errs = [np.abs(O.act_roundtrip(v, t) - v).max() / np.abs(v).max() for t in (1, 2, 3)]
    assert errs[0] < 0.2 and errs[1] < 0.03 and errs[2] < 4e-3
    assert errs[0] > errs[1] > errs[2]


def test_e2m1_rounding_is_nearest_even():
    L = O.lib()
    L.or_e2m1.restype = ctypes.c_uint8
    L.or_e2m1.argtypes = [ctypes.c_float]
    grid = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6], dtype=np.float64)
    xs = np.concatenate([np.linspace(0, 7, 2801), [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 100.0]])
    for x in xs:
        code = L.or_e2m1(float(x))
        d = np.abs(grid - min(x, 6.0))
        best = np.flatnonzero(d == d.min())
        want = best[0] if len(best) == 1 else [b for b in best if b % 2 == 0][0]
        assert code == want, (x, code, want)
        assert L.or_e2m1(float(-x)) == (want | 8 if x > 0 else L.or_e2m1(float(-x)))


def test_mx4_scale_code_known_answers():
    L = O.lib()
    L.or_mx4_scale_code.restype = ctypes.c_uint32
    L.or_mx4_scale_code.argtypes = [ctypes.c_float]
    assert L.or_mx4_scale_code(0.0) == 127   # zero block: scale 1
    assert L.or_mx4_scale_code(6.0) == 127   # exactly E2M1's largest magnitude
    assert L.or_mx4_scale_code(6.5) == 128   # rounded up, never saturating
    assert L.or_mx4_scale_code(3.0) == 126


# ------------------------------------------------------------------ GEMV order, combine
def test_router_gemv_order_is_a_close_sum():
    g = torch.Generator().manual_seed(0)
    x = torch.randn((3, 1024), generator=g).to(torch.bfloat16)
    w = (torch.randn((16, 1024), generator=g) * 0.02).to(torch.bfloat16)
    got = O.router_gemv(O.bf16_bits(x), O.bf16_bits(w))
    ref = x.double() @ w.double().T
    assert np.allclose(got, ref.numpy(), rtol=1e-5, atol=1e-6)


def test_finalize_known_answer():
    def bf(a):
        return O.bf16_bits(torch.tensor(a, dtype=torch.float32).to(torch.bfloat16))

    rows = bf([[1.0, 2.0], [3.0, -4.0], [100.0, 0.5]])
    perm = np.array([[0, -1, 1]], np.int32)
    w = np.array([[0.5, 9.0, 0.25]], np.float32)
    shared = bf([[1.0, 1.0]])
    out = O.finalize(rows, w, perm, shared)
    vals = O.bits_to_f32(out)
    assert vals.tolist() == [[0.5 + 0.75 + 1.0, 1.0 - 1.0 + 1.0]]


def test_allreduce_ranks_sums_in_rank_order():
    def bf(a):
        return O.bf16_bits(torch.tensor(a, dtype=torch.float32).to(torch.bfloat16))

    big = 2.0 ** 30
    # fp32 absorbs 1 into 2^30, so only the order (2^30, -2^30, 1) keeps it
    assert O.bits_to_f32(O.allreduce_ranks([bf([big]), bf([1.0]), bf([-big])])).tolist() == [0.0]
    assert O.bits_to_f32(O.allreduce_ranks([bf([big]), bf([-big]), bf([1.0])])).tolist() == [1.0]
    # the fp32 sum is rounded to bf16 once, at the end (nearest even)
    ys = [bf([1.0]), bf([2.0 ** -8]), bf([2.0 ** -9])]
    assert O.bits_to_f32(O.allreduce_ranks(ys)).tolist() == [1.0 + 2.0 ** -7]
    one = O.allreduce_ranks([bf([[1.5, -2.0], [0.0, 3.0]])])
    assert np.array_equal(one, bf([[1.5, -2.0], [0.0, 3.0]]))


def test_allreduce_norm_known_answers():
    def bf(a):
        return O.bf16_bits(torch.tensor(a, dtype=torch.float32).to(torch.bfloat16))

    H = 7168
    gamma = bf(np.linspace(-2, 2, H, dtype=np.float32))
    # every pre value 2: sum of squares 4 H, inv = 1 / sqrt(4) = 1/2, norm = gamma
    res_out, norm = O.allreduce_norm([bf(np.zeros((2, H), np.float32))], bf(np.full((2, H), 2.0, np.float32)),
                                     gamma, 0.0)
    assert np.array_equal(res_out, bf(np.full((2, H), 2.0, np.float32)))
    assert np.array_equal(norm, np.stack([gamma, gamma]))
    # two ranks + residual: pre is one rounding of the fp32 sum (1 + 2^-8 + 2^-9 -> 1 + 2^-7)
    y0, y1 = bf(np.full((1, H), 1.0, np.float32)), bf(np.full((1, H), 2.0 ** -8, np.float32))
    res_out, none = O.allreduce_norm([y0, y1], bf(np.full((1, H), 2.0 ** -9, np.float32)), None, 1e-6)
    assert none is None
    assert np.all(O.bits_to_f32(res_out) == 1.0 + 2.0 ** -7)


def test_allreduce_norm_matches_float64():
    g = torch.Generator().manual_seed(4)
    for H in (1024, 6144, 7168):
        ys = [O.bf16_bits(torch.randn(5, H, generator=g).to(torch.bfloat16)) for _ in range(3)]
        res = O.bf16_bits(torch.randn(5, H, generator=g).to(torch.bfloat16))
        gam = O.bf16_bits((1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16))
        r, n = O.allreduce_norm(ys, res, gam, 1e-6)
        pre = sum(O.bits_to_f32(y).astype(np.float64) for y in ys) + O.bits_to_f32(res)
        assert np.abs(O.bits_to_f32(r) - pre).max() <= 2.0 ** -8 * np.abs(pre).max()
        p = O.bits_to_f32(r).astype(np.float64)
        ref = p / np.sqrt((p * p).mean(1, keepdims=True) + 1e-6) * O.bits_to_f32(gam)
        assert np.abs(O.bits_to_f32(n) - ref).max() <= 2.0 ** -7 * np.abs(ref).max()


def test_moe_layer_oracle_shapes_and_linearity():
    H, I, E, K, T = 256, 256, 4, 2, 3
    layer = O.make_layer(H, I, E, shared=True, seed=1)
    x, _, _ = O.make_inputs(T, H, E, seed=1, router=False)
    ids = np.array([[0, 1], [1, 2], [3, 0]], np.int32)
    w = np.ones((T, K), np.float32)
    out, rows, shared = O.moe_layer(x, ids, w, layer)
    assert out.shape == (T, H) and len(rows) == T * K and shared.shape == (T, H)
    out2, _, _ = O.moe_layer(x, ids, 2 * w, layer)
    assert torch.allclose(out2 - shared, 2 * (out - shared), rtol=1e-5, atol=1e-5)


def test_nvfp4_codec_known_answers():
    # scale rule: sf = e4m3(gs * amax / 6); a block whose amax maps to 6 * 448 / gs
    # saturates at 448, and codes use E2M1's nearest-even grid
    gs = 2.0
    v = np.zeros((1, 16), np.float32)
    v[0, :4] = [6.0, -3.0, 1.0, 0.75]  # amax 6 -> sf = e4m3(2) = 2.0, multiplier gs / sf = 1
    q, s = O.nvfp4_quant(v, 1, 1.0 / gs)
    assert O.e4m3_table()[s[0, 0, 0]] == 2.0
    codes = [(q[0, 0, i // 2] >> (4 * (i % 2))) & 15 for i in range(4)]
    assert [float(O.E2M1[c]) for c in codes] == [6.0, -3.0, 1.0, 1.0]  # 0.75 ties to even (1.0)
    big = np.full((1, 16), 1e6, np.float32)
    _, s = O.nvfp4_quant(big, 1, 1.0 / gs)
    assert O.e4m3_table()[s[0, 0, 0]] == 448.0
    # three terms converge on smooth data
    x = np.random.RandomState(1).randn(8, 256).astype(np.float32)
    errs = [np.abs(O.act_roundtrip(x, t, "nvfp4", 8.0 / 2688.0) - x).max() for t in (1, 2, 3)]
    assert errs[0] > errs[1] > errs[2] and errs[2] < 1e-2 * np.abs(x).max()


def test_nvfp4_weight_dequant_matches_definition():
    L = O.make_nvfp4_layer(256, 256, 2, shared=False, seed=9)
    W = O.dequant_nvfp4(L["w2"][1], L["w2_scale"][1], float(L["w2_scale_2"][1]))
    codes, sc = L["w2"][1].numpy(), L["w2_scale"][1].numpy()
    r, k = 5, 37
    byte = codes[r, k // 2]
    e2 = O.E2M1[(byte >> 4) if k % 2 else (byte & 15)]
    want = np.float64(e2) * np.float64(O.e4m3_table()[sc[r, k // 16]]) * np.float64(L["w2_scale_2"][1])
    assert abs(float(W[r, k]) - want) <= 1e-7 * max(1.0, abs(want))
    vals = O.e4m3_table()[L["w13_scale"].numpy()]
    assert vals.min() >= 0.5 and vals.max() <= 4.0


def test_sqrtsoftplus_known_answers_and_accuracy():
    h = O.lib()
    h.or_sqrtsoftplus.restype = ctypes.c_float
    h.or_sqrtsoftplus.argtypes = [ctypes.c_float]
    assert h.or_sqrtsoftplus(25.0) == 5.0                     # above 20: sqrt(x)
    assert h.or_sqrtsoftplus(-200.0) == 0.0                   # exp underflows
    assert math.isnan(h.or_sqrtsoftplus(float("nan")))
    xs = np.concatenate([np.linspace(-80, 20, 4001), np.random.default_rng(2).normal(0, 6, 4000).clip(-80, 20)])
    worst = 0.0
    for x in xs.astype(np.float32):
        want = math.sqrt(math.log1p(math.exp(float(x))))
        worst = max(worst, abs(h.or_sqrtsoftplus(float(x)) - want) / want)
    assert worst < 4 * 2.0 ** -24, worst                     # a couple of ulps


def test_gate_topk_sqrtsoftplus_and_alt_bias():
    rng = np.random.default_rng(3)
    T, E, K = 6, 64, 4
    logits = rng.normal(size=(T, E)).astype(np.float32)
    w, ids = O.gate_topk(logits, None, K, score="sqrtsoftplus", scale=2.0)
    s = np.sqrt(np.log1p(np.exp(logits.astype(np.float64))))
    assert np.array_equal(np.sort(ids, 1), np.sort(np.argsort(-s, 1)[:, :K], 1))
    sel = np.take_along_axis(s, ids.astype(np.int64), 1)
    assert np.allclose(w, 2.0 * sel / sel.sum(1, keepdims=True), rtol=1e-6)
    # image rows (token 7) rank with bias_alt: a huge alt bias on expert 9 wins
    bias_alt = np.zeros(E, np.float32)
    bias_alt[9] = 100.0
    toks = np.array([7, 1, 7, 2, 3, 7], np.int64)
    _, ids2 = O.gate_topk(logits, np.zeros(E, np.float32), K, score="sqrtsoftplus", bias_alt=bias_alt,
                          input_ids=toks, alt_token_id=7)
    assert [int(ids2[t, 0]) == 9 for t in range(T)] == [True, False, True, False, False, True]


def test_scaled_bf16_weight_rule_known_answers():
    """GLM-5.3's routing weights (glm5_3/sm103/moe/routing.py:3-11): the top-8 by
    sigmoid + bias, w = bf16(scale * s / (sum + 1e-20)) with the scale applied
    first and the sum in the order of a warp xor-butterfly over the slots,
    ((s0 + s4) + (s2 + s6)) + ((s1 + s5) + (s3 + s7))."""
    f32 = np.float32
    g = np.random.default_rng(3)
    E, K, T = 256, 8, 6
    logits = g.standard_normal((T, E)).astype(np.float32)
    bias = (g.standard_normal(E) * 0.01).astype(np.float32)
    w, ids = O.gate_topk(logits, bias, K, renormalize="scaled_bf16", scale=2.5, eps=1e-20)
    _, ids_sum = O.gate_topk(logits, bias, K, scale=2.5)
    assert np.array_equal(ids, ids_sum)  # the rule changes the weights, not the selection
    sig = O.lib().or_sigmoid
    for t in range(T):
        s = [f32(sig(float(logits[t, e]))) for e in ids[t]]
        total = ((s[0] + s[4]) + (s[2] + s[6])) + ((s[1] + s[5]) + (s[3] + s[7]))
        d = f32(total + f32(1e-20))
        for k in range(K):
            q = f32(f32(f32(2.5) * s[k]) / d)
            b = np.array([q], dtype=np.float32).view(np.uint32)[0]
            b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000  # bf16 round to nearest even
            assert w[t, k].view(np.uint32) == b, (t, k)
    # a sum whose order shows: slots whose scores differ by 2^-24 relative
    logits2 = np.full((1, 16), -30.0, dtype=np.float32)
    logits2[0, :8] = [20.0, 0.0, 20.0, 0.0, 20.0, 0.0, 20.0, 0.0]
    w2, ids2 = O.gate_topk(logits2, None, 8, renormalize="scaled_bf16", scale=1.0, eps=1e-20)
    assert sorted(ids2[0].tolist()) == list(range(8))
    assert np.all(w2.view(np.uint32) & 0xFFFF == 0)
