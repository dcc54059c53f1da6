"""GPU parity of the routed-MoE chain against the CPU oracle (calls go through
the C ABI via megamoe's ctypes binding).

Bit-exact: router GEMV logits, top-k ids and weights, the route record and
slot -> row map, the combine. Tolerance: the MoE output against the oracle's
dequantize-then-fp32 path (max|got - ref| / max|ref| <= 2e-2, BASELINE's bar),
and the deferred rows against the oracle fed the kernels' own MXFP4 activation
terms (<= 1e-2: only the fp32 accumulation order differs)."""

import numpy as np
import pytest
import torch

import oracle.oracle as O

pytestmark = pytest.mark.gpu

OUT_TOL = 2e-2     # MoE output vs the fp32 dequantize oracle
ROWS_TOL = 1e-2    # deferred rows vs the oracle with the kernels' activation quantization


def _mm():
    import megamoe

    return megamoe


def to_gpu_layer(layer, top_k, max_rows, act_terms=3, router_experts=None, expert_offset=0, window=None):
    mm = _mm()
    dev = torch.device("cuda", 0)
    sel = (lambda t: t[window]) if window is not None else (lambda t: t)
    w = [sel(layer[k]).contiguous().to(dev) for k in ("w13", "w13_scale", "w2", "w2_scale")]
    shared = None
    if layer.get("shared") is not None:
        shared = [t.to(dev) for t in layer["shared"]]
    clamp = None if layer.get("clamp") is None else sel(layer["clamp"]).to(dev)
    nv = {}
    if layer.get("fmt") == "nvfp4":
        nv = dict(weight_format="nvfp4", w13_scale_2=sel(layer["w13_scale_2"]).contiguous().to(dev),
                  w2_scale_2=sel(layer["w2_scale_2"]).contiguous().to(dev), input_scale=layer["input_scale"])
    return mm.RoutedMoE(*w, top_k, max_rows, clamp=clamp, router_experts=router_experts,
                        expert_offset=expert_offset, shared=shared, act_terms=act_terms, **nv)


# ----------------------------------------------------------------------------- routing
@pytest.mark.parametrize("T,E,H", [(4, 16, 1024), (8, 384, 7168), (33, 256, 6144)])
def test_router_gemv_bitexact(T, E, H):
    mm = _mm()
    x, w, _ = O.make_inputs(T, H, E, seed=T + E)
    got = mm.router_gemv(x.cuda(), w.cuda()).cpu().numpy()
    want = O.router_gemv(O.bf16_bits(x), O.bf16_bits(w))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _logits(kind, T, E, g):
    if kind == "normal":
        return torch.randn((T, E), generator=g)
    if kind == "wide":
        return torch.randn((T, E), generator=g) * 15
    if kind == "ties":
        return torch.randint(-3, 4, (T, E), generator=g).float() * 0.5
    if kind == "nan_rows":
        x = torch.randn((T, E), generator=g)
        x[0::3] = float("nan")
        x[1::3, ::5] = float("nan")
        x[1::3, 1::7] = float("inf")
        x[2::3, 2::11] = float("-inf")
        return x
    if kind == "tie_cutoff":
        x = torch.full((T, E), -2.0)
        x[:, torch.randperm(E, generator=g)[: E // 4]] = 0.75
        return x
    raise ValueError(kind)


@pytest.mark.parametrize("score", ["sigmoid", "softmax", "sqrtsoftplus"])
@pytest.mark.parametrize("kind", ["normal", "wide", "ties", "nan_rows", "tie_cutoff"])
@pytest.mark.parametrize("E,K", [(16, 2), (384, 8), (256, 8), (512, 10)])
def test_gate_topk_bitexact(score, kind, E, K):
    mm = _mm()
    g = torch.Generator().manual_seed(1234)
    for T in (1, 5, 8, 32):
        for trial in range(2):
            logits = _logits(kind, T, E, g).float().contiguous()
            bias = None if trial == 0 and kind != "ties" else (torch.randn(E, generator=g) * 0.05).float()
            valid = T if trial == 0 else max(1, T - 2)
            nv = torch.tensor([valid], dtype=torch.int32, device="cuda")
            w, ids = mm.gate_topk(logits.cuda(), None if bias is None else bias.cuda(), K, score=score,
                                  routed_scaling_factor=2.5, num_valid=nv)
            ow, oids = O.gate_topk(logits.numpy(), None if bias is None else bias.numpy(), K, score=score,
                                   scale=2.5, num_valid=valid)
            assert np.array_equal(ids.cpu().numpy(), oids), (kind, T, trial)
            assert _same_bits(w.cpu().numpy(), ow), (kind, T, trial)


@pytest.mark.parametrize("ids64", [False, True])
def test_gate_topk_vision_alt_bias_bitexact(ids64):
    """Rows whose input token is the image token rank with bias_alt (DSV4.1 VL
    routing, gate_topk.cuh:290-346); padded rows stay -1 whatever their token."""
    mm = _mm()
    g = torch.Generator().manual_seed(99)
    T, E, K, tok = 12, 384, 6, 128815
    logits = torch.randn((T, E), generator=g)
    bias = (torch.randn(E, generator=g) * 0.05).float()
    bias_alt = (torch.randn(E, generator=g) * 0.5).float()
    input_ids = torch.randint(0, 200000, (T,), generator=g)
    input_ids[[0, 3, 4, 11]] = tok
    input_ids = input_ids.to(torch.int64 if ids64 else torch.int32)
    for score in ("sqrtsoftplus", "sigmoid"):
        for valid in (T, T - 1):
            nv = torch.tensor([valid], dtype=torch.int32, device="cuda")
            w, ids = mm.gate_topk(logits.cuda(), bias.cuda(), K, score=score, routed_scaling_factor=2.5,
                                  num_valid=nv, alt=(bias_alt.cuda(), input_ids.cuda(), tok))
            ow, oids = O.gate_topk(logits.numpy(), bias.numpy(), K, score=score, scale=2.5, num_valid=valid,
                                   bias_alt=bias_alt.numpy(), input_ids=input_ids.numpy(), alt_token_id=tok)
            assert np.array_equal(ids.cpu().numpy(), oids), (score, valid)
            assert _same_bits(w.cpu().numpy(), ow), (score, valid)
            _, plain_ids = O.gate_topk(logits.numpy(), bias.numpy(), K, score=score, scale=2.5, num_valid=valid)
            assert not np.array_equal(oids, plain_ids)  # the image rows did rank with bias_alt


def _same_bits(a, b):
    """Bit-exact fp32 equality, except that any NaN equals any NaN (the payload
    of a NaN weight of an all-NaN row is not meaningful)."""
    both_nan = np.isnan(a) & np.isnan(b)
    return bool(np.all(both_nan | (a.view(np.uint32) == b.view(np.uint32))))


def _random_ids(T, K, E, g, distinct=None):
    distinct = E if distinct is None else max(min(distinct, E), K)
    pool = torch.randperm(E, generator=g)[:distinct]
    return torch.stack([pool[torch.randperm(distinct, generator=g)[:K]] for _ in range(T)]).int()


@pytest.mark.parametrize("T", [1, 4, 8, 9, 16, 48, 64, 100, 256])
@pytest.mark.parametrize("K,E", [(2, 16), (6, 384), (8, 384), (8, 256), (16, 1024)])
def test_route_bitexact(T, K, E):
    mm = _mm()
    g = torch.Generator().manual_seed(7 * T + K)
    for distinct, offset, local in ((None, 0, E), (K, 0, E), (None, E // 2, E // 2), (None, 0, E // 2),
                                    (None, -1, E), (None, -2, E), (K, -2, E)):  # -1/-2: balanced dealing
        ids = _random_ids(T, K, E, g, distinct)
        perm, rec = mm.route(ids.cuda(), local, offset)
        operm, orec = O.route(ids.numpy(), local, offset)
        assert np.array_equal(perm.cpu().numpy(), operm), (T, K, E, distinct, offset)
        assert np.array_equal(rec.cpu().numpy(), orec), (T, K, E, distinct, offset)


@pytest.mark.parametrize("T,K,E", [(1, 8, 384), (2, 6, 64), (4, 8, 16), (5, 6, 384), (3, 2, 8), (16, 2, 16)])
def test_route_decode_batches_and_foreign_ids(T, K, E):
    """Decode-sized steps (up to 32 slots) with padded ids (-1), ids of no
    local expert and every window / dealing mode, against the oracle. A row's
    ids are distinct, as the reference's route assumes (route.cuh)."""
    mm = _mm()
    g = torch.Generator().manual_seed(31 * T + K + E)
    for offset, local in ((0, E), (E // 2, E // 2), (0, E // 2), (-1, E), (-2, E)):
        for trial in range(4):
            ids = _random_ids(T, K, E, g, distinct=(None, K + 1, 2 * K, None)[trial])
            if trial & 1:
                ids[T - 1, K - 1] = -1                       # a padded slot
            if trial & 2 and offset >= 0:
                ids[T // 2, 0] = E + 3                       # no expert of the window
            perm, rec = mm.route(ids.cuda(), local, offset)
            operm, orec = O.route(ids.numpy(), local, offset)
            assert np.array_equal(perm.cpu().numpy(), operm), (T, K, E, offset, trial)
            assert np.array_equal(rec.cpu().numpy(), orec), (T, K, E, offset, trial)


def test_finalize_bitexact():
    mm = _mm()
    g = torch.Generator().manual_seed(3)
    T, K, H, P = 8, 8, 7168, 96
    rows = torch.randn((P, H), generator=g).to(torch.bfloat16)
    shared = torch.randn((T, H), generator=g).to(torch.bfloat16)
    w = torch.rand((T, K), generator=g)
    perm = torch.randint(-1, P, (T, K), generator=g).int()
    for sh in (None, shared):
        out = mm.finalize(rows.cuda(), w.cuda(), perm.cuda(), None if sh is None else sh.cuda())
        want = O.finalize(O.bf16_bits(rows), w.numpy(), perm.numpy(), None if sh is None else O.bf16_bits(sh))
        assert np.array_equal(O.bf16_bits(out.cpu()), want)


# ----------------------------------------------------------------------------- experts
def _run_and_check(layer, x, ids, weights, K, max_rows, act_terms=3, expert_offset=0, local=None,
                   router_experts=None, window=None):
    moe = to_gpu_layer(layer, K, max_rows, act_terms=act_terms, router_experts=router_experts,
                       expert_offset=expert_offset, window=window)
    xg = x.cuda()
    rows, _, perm = moe(xg, None, ids.cuda())
    out = moe.finalize(rows, weights.cuda(), perm)
    moe.check()
    rows_c = rows.float().cpu()
    perm_c = perm.cpu().numpy()
    ref_layer = dict(layer)
    ex_out, _, _ = O.moe_layer(x, ids.numpy(), weights.numpy(), ref_layer, numerics="exact",
                               expert_offset=expert_offset, local_experts=local)
    kn_out, kn_rows, kn_shared = O.moe_layer(x, ids.numpy(), weights.numpy(), ref_layer, numerics="kernel",
                                             terms=act_terms, expert_offset=expert_offset, local_experts=local)
    # the routing itself
    operm, _ = O.route(ids.numpy(), local if local is not None else layer["w13"].shape[0], expert_offset)
    assert np.array_equal(perm_c, operm)
    # deferred rows against the oracle with the kernels' quantization
    got_rows = np.stack([rows_c[perm_c[t, k]].numpy() for (t, k) in kn_rows])
    want_rows = np.stack([v.numpy() for v in kn_rows.values()])
    # with one term a code the fp32 accumulation order moves across a rounding
    # boundary is a whole E2M1 step of that activation, not a residual's
    rows_tol = ROWS_TOL if act_terms > 1 else 5e-2
    assert O.max_abs_rel(got_rows, want_rows) <= rows_tol
    if kn_shared is not None:
        sh = rows_c[moe.shared_row_base: moe.shared_row_base + x.shape[0]].numpy()
        assert O.max_abs_rel(sh, kn_shared.numpy()) <= rows_tol
    # one or two activation terms are coarser numerics: plain NVFP4 / MXFP4
    # activations sit about 1e-1 from the fp32 path (the oracle measures it)
    tol = {3: OUT_TOL, 2: 1e-1, 1: 2.5e-1}[act_terms]
    err = O.max_abs_rel(out.float().cpu().numpy(), ex_out.numpy())
    assert err <= tol, err
    return moe, out


def test_experts_config1():
    """H 1024, 16 experts, top-2 softmax, I 512, T 4."""
    mm = _mm()
    H, I, E, K, T = 1024, 512, 16, 2, 4
    layer = O.make_layer(H, I, E, shared=False, seed=0)
    x, wr, _ = O.make_inputs(T, H, E, seed=0)
    logits = mm.router_gemv(x.cuda(), wr.cuda())
    w, ids = mm.gate_topk(logits, None, K, score="softmax")
    _run_and_check(layer, x, ids.cpu(), w.cpu(), K, max_rows=8)


@pytest.mark.parametrize("T,distinct", [(1, None), (8, None), (8, 8), (24, 8), (40, 8), (64, None)])
def test_experts_shared_sigmoid(T, distinct):
    """Routed + shared expert, sigmoid routing; distinct = 8 makes experts take
    all the rows (segments of 16 rows, several tiles per expert)."""
    H, I, E, K = 1024, 256, 32, 8
    layer = O.make_layer(H, I, E, shared=True, seed=T)
    x, _, _ = O.make_inputs(T, H, E, seed=T)
    g = torch.Generator().manual_seed(T)
    ids = _random_ids(T, K, E, g, distinct)
    w = torch.rand((T, K), generator=g)
    _run_and_check(layer, x, ids, w, K, max_rows=64)


def test_experts_clamp_and_single_term():
    H, I, E, K, T = 2048, 512, 16, 4, 6
    layer = O.make_layer(H, I, E, shared=True, seed=11, clamp=0.5)
    layer["shared_clamp"] = None
    x, _, _ = O.make_inputs(T, H, E, seed=11)
    g = torch.Generator().manual_seed(11)
    ids = _random_ids(T, K, E, g)
    w = torch.rand((T, K), generator=g)
    _run_and_check(layer, x, ids, w, K, max_rows=8)
    _run_and_check(layer, x, ids, w, K, max_rows=8, act_terms=2)


# ----------------------------------------------------------------------------- NVFP4
def test_nvfp4_experts_config1_shape():
    """NVFP4 weights (E2M1 + E4M3 per 16 + per-expert scale_2, kind::mxf4nvf4
    block16) at the config-1 shape, softmax top-2, with a shared expert."""
    mm = _mm()
    H, I, E, K, T = 1024, 512, 16, 2, 4
    layer = O.make_nvfp4_layer(H, I, E, shared=True, seed=2)
    x, wr, _ = O.make_inputs(T, H, E, seed=2)
    logits = mm.router_gemv(x.cuda(), wr.cuda())
    w, ids = mm.gate_topk(logits, None, K, score="softmax")
    _run_and_check(layer, x, ids.cpu(), w.cpu(), K, max_rows=8)


@pytest.mark.parametrize("T,distinct", [(1, None), (16, None), (24, 8)])
def test_nvfp4_experts_config4_hidden(T, distinct):
    """NVFP4 at config 4's hidden size (6144) with a shared expert, sigmoid-style
    random routing; distinct = 8 gives experts segments of 16 rows."""
    H, I, E, K = 6144, 256, 32, 8
    layer = O.make_nvfp4_layer(H, I, E, shared=True, seed=60 + T)
    x, _, _ = O.make_inputs(T, H, E, seed=60 + T)
    g = torch.Generator().manual_seed(60 + T)
    ids = _random_ids(T, K, E, g, distinct)
    w = torch.rand((T, K), generator=g)
    _run_and_check(layer, x, ids, w, K, max_rows=32)


def test_nvfp4_single_term_and_ep_window():
    """NVFP4 with one activation term (plain NVFP4 activations, looser bar) and
    an EP window of 16 of 32 experts."""
    H, I, E, K, T = 2048, 256, 32, 4, 8
    layer = O.make_nvfp4_layer(H, I, E, shared=False, seed=71)
    x, _, _ = O.make_inputs(T, H, E, seed=71)
    g = torch.Generator().manual_seed(71)
    ids = _random_ids(T, K, E, g)
    w = torch.rand((T, K), generator=g)
    half = {k: (v[16:32] if k in ("w13", "w13_scale", "w2", "w2_scale", "w13_scale_2", "w2_scale_2") else v)
            for k, v in layer.items()}
    _run_and_check(half, x, ids, w, K, max_rows=8, expert_offset=16, local=16, router_experts=32)
    _run_and_check(layer, x, ids, w, K, max_rows=8, act_terms=1)


def test_experts_balanced_dealing_groups_sum_to_the_layer():
    """Balanced dealing (route.cuh:39-46): each group keeps alternate distinct
    experts; each group's rows match the oracle of its experts, and the two
    groups' combined outputs add up to the whole layer's."""
    mm = _mm()
    H, I, E, K, T = 1024, 256, 32, 6, 8
    layer = O.make_layer(H, I, E, shared=False, seed=13)
    x, _, _ = O.make_inputs(T, H, E, seed=13)
    g = torch.Generator().manual_seed(13)
    ids = _random_ids(T, K, E, g)
    w = torch.rand((T, K), generator=g)
    dev = torch.device("cuda", 0)
    wts = [layer[k].to(dev) for k in ("w13", "w13_scale", "w2", "w2_scale")]
    parts = []
    for group in (0, 1):
        moe = mm.RoutedMoE(*wts, K, 8, deal_group=group)
        rows, _, perm = moe(x.cuda(), None, ids.cuda())
        operm, orec = O.route(ids.numpy(), E, -1 - group)
        assert np.array_equal(perm.cpu().numpy(), operm)
        _, kn_rows, _ = O.moe_layer(x, ids.numpy(), w.numpy(), layer, numerics="kernel", deal_group=group)
        pc = perm.cpu().numpy()
        got = np.stack([rows.float().cpu()[pc[t, k]].numpy() for (t, k) in kn_rows])
        want = np.stack([v.numpy() for v in kn_rows.values()])
        assert O.max_abs_rel(got, want) <= ROWS_TOL
        parts.append(moe.finalize(rows, w.cuda(), perm, partial=True))
        moe.check()
    total = mm.finalize_partial(parts[0] + parts[1])
    ex, _, _ = O.moe_layer(x, ids.numpy(), w.numpy(), layer, numerics="exact")
    assert O.max_abs_rel(total.float().cpu().numpy(), ex.numpy()) <= OUT_TOL


@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4"])
@pytest.mark.parametrize("I", [320, 384, 576, 640])
@pytest.mark.parametrize("T,distinct", [(8, None), (40, 6)])
def test_experts_dsv41_geometry(fmt, I, T, distinct):
    """DeepSeek-V4.1's own geometry (routed_expert_gemm.py:31-40): hidden 5120,
    an intermediate slice of 576 (or its 640 padding), top-6; the down GEMM's K
    is not a multiple of the 256-wide pipeline stage, so its last stage is
    partial (zero-filled past K). I = 320 / 384 give two K stages per down tile,
    so MXFP4 takes two tiles per down unit with a partial second stage."""
    H, E, K = 5120, 32, 6
    if fmt == "nvfp4":
        layer = O.make_nvfp4_layer(H, I, E, shared=True, seed=I + T)
    else:
        layer = O.make_layer(H, I, E, shared=True, seed=I + T)
    x, _, _ = O.make_inputs(T, H, E, seed=I + T)
    g = torch.Generator().manual_seed(I + T)
    ids = _random_ids(T, K, E, g, distinct)
    w = torch.rand((T, K), generator=g)
    _run_and_check(layer, x, ids, w, K, max_rows=64)


def test_experts_expert_parallel_window():
    """EP: the rank holds experts [16, 32) of 32; other slots map to -1."""
    H, I, E, K, T = 1024, 256, 32, 4, 8
    layer = O.make_layer(H, I, E, shared=False, seed=5)
    x, _, _ = O.make_inputs(T, H, E, seed=5)
    g = torch.Generator().manual_seed(5)
    ids = _random_ids(T, K, E, g)
    w = torch.rand((T, K), generator=g)
    half = {k: (v[16:32] if k in ("w13", "w13_scale", "w2", "w2_scale") else v) for k, v in layer.items()}
    _run_and_check(half, x, ids, w, K, max_rows=8, expert_offset=16, local=16, router_experts=32)


def test_forward_matches_steps_and_graph():
    """The one-call forward (router -> combine) equals the step-by-step calls,
    and a CUDA-graph replay equals eager."""
    mm = _mm()
    H, I, E, K, T = 2048, 256, 64, 8, 8
    layer = O.make_layer(H, I, E, shared=True, seed=21)
    x, wr, bias = O.make_inputs(T, H, E, seed=21)
    moe = to_gpu_layer(layer, K, 16)
    xg, wg, bg = x.cuda(), wr.cuda(), bias.cuda()
    bufs = {}
    out = moe.forward(xg, router_weight=wg, bias=bg, routed_scaling_factor=2.5, buffers=bufs).clone()
    logits = mm.router_gemv(xg, wg)
    rows, w, perm, ids = moe.gate_topk_and_gemms(None, None, logits, bg, 2.5, x=xg)
    out2 = moe.finalize(rows, w, perm)
    assert torch.equal(out, out2)
    ow, oids = O.gate_topk(O.router_gemv(O.bf16_bits(x), O.bf16_bits(wr)), bias.numpy(), K, scale=2.5)
    assert np.array_equal(ids.cpu().numpy(), oids)
    ex_out, _, _ = O.moe_layer(x, oids, ow, layer, numerics="exact")
    assert O.max_abs_rel(out.float().cpu().numpy(), ex_out.numpy()) <= OUT_TOL
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        moe.forward(xg, router_weight=wg, bias=bg, routed_scaling_factor=2.5, buffers=bufs)
    bufs["out"].zero_()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(bufs["out"], out)
    moe.check()


# ----------------------------------------------------------------------------- peer combine
def test_peer_allreduce_group_of_one_matches_finalize():
    """The combine fused with the all-reduce, in a group of one: each call's
    output is bit-exact the oracle's combine, across calls whose token counts
    change (the per-slot flags, counters and parity must stay consistent) and
    across CUDA-graph replays (the state lives on the device)."""
    mm = _mm()
    g = torch.Generator().manual_seed(5)
    K, H, P, TMAX = 8, 7168, 160, 16
    comm = mm.PeerAllReduce(TMAX, H)
    rows = torch.randn((P, H), generator=g).to(torch.bfloat16)
    rg = rows.cuda()
    for T in (8, 3, 8, 16, 1, 5, 16, 16, 2):
        shared = torch.randn((T, H), generator=g).to(torch.bfloat16)
        w = torch.rand((T, K), generator=g)
        perm = torch.randint(-1, P, (T, K), generator=g).int()
        out = comm.finalize(rg, w.cuda(), perm.cuda(), shared.cuda())
        want = O.allreduce_ranks([O.finalize(O.bf16_bits(rows), w.numpy(), perm.numpy(), O.bf16_bits(shared))])
        assert np.array_equal(O.bf16_bits(out.cpu()), want), T
    comm.check()
    T = 8
    shared = torch.randn((T, H), generator=g).to(torch.bfloat16).cuda()
    w = torch.rand((T, K), generator=g).cuda()
    perm = torch.randint(-1, P, (T, K), generator=g).int().cuda()
    out = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    eager = comm.finalize(rg, w, perm, shared).clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        comm.finalize(rg, w, perm, shared, out=out)
    for _ in range(5):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    comm.check()
    comm.close()


def test_forward_with_peer_group_of_one():
    """forward(comm=...) runs the whole step with the fused combine and equals forward()."""
    mm = _mm()
    H, I, E, K, T = 2048, 256, 64, 8, 8
    layer = O.make_layer(H, I, E, shared=True, seed=23)
    x, wr, bias = O.make_inputs(T, H, E, seed=23)
    moe = to_gpu_layer(layer, K, 16)
    comm = mm.PeerAllReduce(16, H)
    xg, wg, bg = x.cuda(), wr.cuda(), bias.cuda()
    want = moe.forward(xg, router_weight=wg, bias=bg, routed_scaling_factor=2.5).clone()
    for _ in range(3):
        got = moe.forward(xg, router_weight=wg, bias=bg, routed_scaling_factor=2.5, comm=comm)
        assert torch.equal(got, want)
    with pytest.raises(ValueError):
        moe.forward(xg, router_weight=wg, bias=bg, partial=True, comm=comm)
    comm.check()
    moe.check()
    comm.close()


@pytest.mark.parametrize("H", [1024, 6144, 7168])
def test_peer_allreduce_norm_group_of_one(H):
    """The combine + all-reduce with the decoder hop's residual + RMSNorm
    epilogue (one cluster per token row): residual_out and norm_out bit-exact
    the oracle's fold, across calls of changing token counts, with residual
    updated in place, and without gamma."""
    mm = _mm()
    g = torch.Generator().manual_seed(H)
    K, P, TMAX, EPS = 8, 96, 16, 1e-6
    comm = mm.PeerAllReduce(TMAX, H, eps=EPS)
    rows = torch.randn((P, H), generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    rg, gg = rows.cuda(), gamma.cuda()
    for T in (8, 3, 16, 1, 8):
        shared = torch.randn((T, H), generator=g).to(torch.bfloat16)
        w = torch.rand((T, K), generator=g)
        perm = torch.randint(-1, P, (T, K), generator=g).int()
        res = torch.randn((T, H), generator=g).to(torch.bfloat16)
        y = O.finalize(O.bf16_bits(rows), w.numpy(), perm.numpy(), O.bf16_bits(shared))
        want_r, want_n = O.allreduce_norm([y], O.bf16_bits(res), O.bf16_bits(gamma), EPS)
        args = dict(routed_output=rg, expert_weights=w.cuda(), permuted_indices=perm.cuda(),
                    gated_shared_output=shared.cuda())
        norm, r_out = comm.moe_finalize_all_reduce_rms_norm(**args, residual=res.cuda(), gamma=gg)
        assert np.array_equal(O.bf16_bits(r_out.cpu()), want_r), T
        assert np.array_equal(O.bf16_bits(norm.cpu()), want_n), T
        inplace = res.cuda()
        none, r2 = comm.moe_finalize_all_reduce_rms_norm(**args, residual=inplace, gamma=None, residual_out=inplace)
        assert none is None and r2.data_ptr() == inplace.data_ptr()
        assert np.array_equal(O.bf16_bits(inplace.cpu()), want_r), T
    comm.check()
    comm.close()


def test_forward_hop_group_of_one():
    """forward(comm, residual, gamma): the whole step ending in the hop equals
    forward() followed by the oracle's residual + RMSNorm of its output."""
    mm = _mm()
    H, I, E, K, T = 2048, 256, 64, 8, 8
    layer = O.make_layer(H, I, E, shared=True, seed=29)
    x, wr, bias = O.make_inputs(T, H, E, seed=29)
    moe = to_gpu_layer(layer, K, 16)
    comm = mm.PeerAllReduce(16, H, eps=1e-5)
    g = torch.Generator().manual_seed(29)
    res = torch.randn((T, H), generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    xg, wg, bg = x.cuda(), wr.cuda(), bias.cuda()
    bufs = {}
    moe.forward(xg, router_weight=wg, bias=bg, routed_scaling_factor=2.5, buffers=bufs)
    shared = moe.shared_rows(bufs["rows"], T)
    y = O.finalize(O.bf16_bits(bufs["rows"].cpu()), bufs["weights"].cpu().numpy(), bufs["permuted"].cpu().numpy(),
                   O.bf16_bits(shared.cpu()))
    want_r, want_n = O.allreduce_norm([y], O.bf16_bits(res), O.bf16_bits(gamma), 1e-5)
    norm, r_out = moe.forward(xg, router_weight=wg, bias=bg, routed_scaling_factor=2.5, comm=comm,
                              residual=res.cuda(), gamma=gamma.cuda())
    assert np.array_equal(O.bf16_bits(r_out.cpu()), want_r)
    assert np.array_equal(O.bf16_bits(norm.cpu()), want_n)
    with pytest.raises(ValueError):
        moe.forward(xg, router_weight=wg, bias=bg, residual=res.cuda())
    comm.check()
    moe.check()
    comm.close()


# ----------------------------------------------------------------------------- stack
def _stack_parts(n, H, I, E, K, T, seed, window=None):
    g = torch.Generator().manual_seed(seed)
    layers = [O.make_layer(H, I, E, shared=False, seed=seed + 1 + i) for i in range(n)]
    routers = [(torch.randn((E, H), generator=g) * 0.02).to(torch.bfloat16) for _ in range(n)]
    biases = [(torch.randn((E,), generator=g) * 0.01).float() for _ in range(n)]
    gammas = [(1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16) for _ in range(n)]
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    res = torch.randn((T, H), generator=g).to(torch.bfloat16)
    return layers, routers, biases, gammas, x, res


def test_stack_matches_layer_loop_oracle_and_graph():
    """mm_stack_forward over 3 layers equals the per-layer forward loop bit for
    bit; each layer's ids and hop outputs equal the oracle's on the GPU's own
    layer inputs; a CUDA-graph replay of the step equals eager."""
    mm = _mm()
    n, H, I, E, K, T = 3, 1024, 256, 32, 8, 8
    layers, routers, biases, gammas, x, res = _stack_parts(n, H, I, E, K, T, seed=40)
    moes = [to_gpu_layer(L, K, 16) for L in layers]
    comm = mm.PeerAllReduce(16, H, eps=1e-6)
    rg, bg, gg = [t.cuda() for t in routers], [t.cuda() for t in biases], [t.cuda() for t in gammas]
    stack = mm.MoEStack(moes, rg, gg, comm, biases=bg, routed_scaling_factor=2.5)
    xs, r_stack = x.cuda(), res.cuda()
    out = stack.forward(xs, r_stack).clone()
    # the loop, checked layer by layer against the oracle on its own inputs
    cur, r = xs, res.cuda()
    for i, m in enumerate(moes):
        bufs = {}
        norm, r_new = m.forward(cur, router_weight=rg[i], bias=bg[i], routed_scaling_factor=2.5, buffers=bufs,
                                comm=comm, residual=r, gamma=gg[i])
        ow, oids = O.gate_topk(O.router_gemv(O.bf16_bits(cur.cpu()), O.bf16_bits(routers[i])), biases[i].numpy(),
                               K, scale=2.5)
        assert np.array_equal(bufs["ids"].cpu().numpy(), oids), i
        y = O.finalize(O.bf16_bits(bufs["rows"].cpu()), bufs["weights"].cpu().numpy(),
                       bufs["permuted"].cpu().numpy(), None)
        want_r, want_n = O.allreduce_norm([y], O.bf16_bits(r.cpu()), O.bf16_bits(gammas[i]), 1e-6)
        assert np.array_equal(O.bf16_bits(r_new.cpu()), want_r), i
        assert np.array_equal(O.bf16_bits(norm.cpu()), want_n), i
        cur, r = norm.clone(), r_new.clone()
    assert torch.equal(out, cur)
    assert torch.equal(r_stack, r)
    # graph replay of the whole step (residual restored before each replay)
    r_graph = res.cuda()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        stack.forward(xs, r_graph)
    for _ in range(3):
        r_graph.copy_(res.cuda())
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(r_graph, r)
        assert torch.equal(stack.norm[(n - 1) & 1][:T], out)
    stack.check()
    del graph
    comm.close()


@pytest.mark.parametrize("score", ["sigmoid", "softmax", "sqrtsoftplus"])
@pytest.mark.parametrize("kind", ["normal", "ties", "nan_rows", "tie_cutoff"])
@pytest.mark.parametrize("E,K", [(16, 2), (384, 8), (512, 10)])
def test_front_rank_and_route_bitexact(score, kind, E, K):
    """The layer's front launch (one CTA per row ranks it; the last builds the
    record) against the oracle: ids and weights bit for bit, the slot -> row
    map equal, padded rows included."""
    mm = _mm()
    H, I = 1024, 256
    layer = O.make_layer(H, I, E, shared=False, seed=81)
    moe = to_gpu_layer(layer, K, 64)
    g = torch.Generator().manual_seed(4321)
    for T in (1, 5, 8, 9, 16, 32):
        for trial in range(2):
            logits = _logits(kind, T, E, g).float().contiguous()
            bias = None if trial == 0 and kind != "ties" else (torch.randn(E, generator=g) * 0.05).float()
            valid = T if trial == 0 else max(1, T - 2)
            nv = torch.tensor([valid], dtype=torch.int32, device="cuda")
            x = torch.randn((T, H), generator=g).to(torch.bfloat16)
            _, w, perm, ids = moe.gate_topk_and_gemms(None, None, logits.cuda(),
                                                     None if bias is None else bias.cuda(), 2.5, nv, x=x.cuda(),
                                                     score=score)
            torch.cuda.synchronize()
            ow, oids = O.gate_topk(logits.numpy(), None if bias is None else bias.numpy(), K, score=score,
                                   scale=2.5, num_valid=valid)
            assert np.array_equal(ids.cpu().numpy(), oids), (kind, T, trial)
            assert _same_bits(w.cpu().numpy(), ow), (kind, T, trial)
            operm, _ = O.route(oids, E)
            assert np.array_equal(perm.cpu().numpy(), operm), (kind, T, trial)
    moe.check()


@pytest.mark.parametrize("T", [3, 8, 16])
def test_front_vision_alt_bias_and_ep(T):
    """The front launch with the vision alt-bias on an EP window: ids and
    weights equal the oracle's, non-local slots map to -1."""
    mm = _mm()
    H, I, E, K = 1024, 256, 384, 8
    layer = O.make_layer(H, I, E, shared=False, seed=91)
    moe = to_gpu_layer(layer, K, 64, router_experts=E, expert_offset=192, window=slice(192, 384))
    g = torch.Generator().manual_seed(92)
    logits = torch.randn((T, E), generator=g).float()
    bias = (torch.randn(E, generator=g) * 0.05).float()
    bias_alt = (torch.randn(E, generator=g) * 0.5).float()
    input_ids = torch.randint(0, 3, (T,), generator=g, dtype=torch.int32)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    _, w, perm, ids = moe.gate_topk_and_gemms(None, None, logits.cuda(), bias.cuda(), 2.5,
                                             alt=(bias_alt.cuda(), input_ids.cuda(), 1), x=x.cuda())
    torch.cuda.synchronize()
    ow, oids = O.gate_topk(logits.numpy(), bias.numpy(), K, scale=2.5, bias_alt=bias_alt.numpy(),
                           input_ids=input_ids.numpy(), alt_token_id=1)
    assert np.array_equal(ids.cpu().numpy(), oids)
    assert _same_bits(w.cpu().numpy(), ow)
    operm, _ = O.route(oids, 192, 192)
    assert np.array_equal(perm.cpu().numpy(), operm)
    moe.check()


def test_rerun_experts_after_rearm_reproduces_rows():
    """The benchmark hook: re-arming the work tables and relaunching the expert
    kernel on the last front pass recomputes the same rows, bit for bit, as
    often as it is repeated."""
    H, I, E, K, T = 2048, 512, 64, 8, 8
    layer = O.make_layer(H, I, E, shared=True, seed=101)
    x, wr, bias = O.make_inputs(T, H, E, seed=102)
    moe = to_gpu_layer(layer, K, 16)
    bufs = {}
    moe.forward(x.cuda(), router_weight=wr.cuda(), bias=bias.cuda(), routed_scaling_factor=2.5, buffers=bufs)
    torch.cuda.synchronize()
    want = bufs["rows"].clone()
    for _ in range(3):
        bufs["rows"].zero_()
        moe.rerun_experts(T, bufs["record"], bufs["rows"])
        torch.cuda.synchronize()
        moe.check()
        perm = bufs["permuted"].cpu().numpy()
        used = sorted({int(p) for p in perm.flatten() if p >= 0})
        assert torch.equal(bufs["rows"][used], want[used])
