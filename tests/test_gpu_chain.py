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
    return mm.RoutedMoE(*w, top_k, max_rows, clamp=clamp, router_experts=router_experts,
                        expert_offset=expert_offset, shared=shared, act_terms=act_terms)


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


@pytest.mark.parametrize("score", ["sigmoid", "softmax"])
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
    for distinct, offset, local in ((None, 0, E), (K, 0, E), (None, E // 2, E // 2), (None, 0, E // 2)):
        ids = _random_ids(T, K, E, g, distinct)
        perm, rec = mm.route(ids.cuda(), local, offset)
        operm, orec = O.route(ids.numpy(), local, offset)
        assert np.array_equal(perm.cpu().numpy(), operm), (T, K, E, distinct, offset)
        assert np.array_equal(rec.cpu().numpy(), orec), (T, K, E, distinct, offset)


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
    rows, _, perm = moe(xg, ids.cuda())
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
    assert O.max_abs_rel(got_rows, want_rows) <= ROWS_TOL
    if kn_shared is not None:
        sh = rows_c[moe.shared_row_base: moe.shared_row_base + x.shape[0]].numpy()
        assert O.max_abs_rel(sh, kn_shared.numpy()) <= ROWS_TOL
    tol = OUT_TOL if act_terms == 3 else 1e-1
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
    rows, w, perm, ids = moe.gate_topk_and_gemms(xg, logits, bg, 2.5)
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
