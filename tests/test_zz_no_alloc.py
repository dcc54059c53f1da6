"""The allocation-free router top-k + route record (mm_gate_route_noalloc)
against the allocating path (mm_gate_topk, then mm_route), through the C ABI.

mm_gate_route_noalloc serves callers that cannot call cudaMalloc: a serving
runtime that reserves the GPU's memory for its own pool at start-up, or plugin
code handed only its input and output pointers. Its scratch (a ticket and the
staged top-k ids) is a static device array of the library instead of memory
from mm_layer_create. It must give the same ids, weights, slot -> row
map and route record bit for bit, including on consecutive calls that reuse the
shared scratch, and reject requests larger than that scratch."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _gate(lib_mod, logits, bias, score, weights, ids, num_valid=None):
    g = lib_mod.MMGateArgs()
    g.logits = logits.data_ptr()
    g.bias = None if bias is None else bias.data_ptr()
    g.num_valid = None if num_valid is None else num_valid.data_ptr()
    g.score_func = lib_mod.SCORES[score]
    g.renormalize = 1
    g.routed_scaling = 2.5
    g.renorm_eps = 0.0
    g.weights = weights.data_ptr()
    g.ids = None if ids is None else ids.data_ptr()
    return g


def _noalloc(lib_mod, logits, bias, score, K, local, offset, want_ids, num_valid=None):
    L = lib_mod.lib()
    T, E = logits.shape
    dev = logits.device
    weights = torch.empty((T, K), dtype=torch.float32, device=dev)
    ids = torch.empty((T, K), dtype=torch.int32, device=dev) if want_ids else None
    permuted = torch.empty((T, K), dtype=torch.int32, device=dev)
    record = torch.empty(L.mm_route_words(T, K, local), dtype=torch.int32, device=dev)
    g = _gate(lib_mod, logits, bias, score, weights, ids, num_valid)
    stream = torch.cuda.current_stream().cuda_stream
    lib_mod.check(L.mm_gate_route_noalloc(ctypes.byref(g), T, E, K, local, offset, permuted.data_ptr(),
                                          record.data_ptr(), stream), "mm_gate_route_noalloc")
    return weights, ids, permuted, record


def _allocating(lib_mod, logits, bias, score, K, local, offset, num_valid=None):
    L = lib_mod.lib()
    T, E = logits.shape
    dev = logits.device
    weights = torch.empty((T, K), dtype=torch.float32, device=dev)
    ids = torch.empty((T, K), dtype=torch.int32, device=dev)
    g = _gate(lib_mod, logits, bias, score, weights, ids, num_valid)
    stream = torch.cuda.current_stream().cuda_stream
    lib_mod.check(L.mm_gate_topk(ctypes.byref(g), T, E, K, stream), "mm_gate_topk")
    permuted = torch.empty((T, K), dtype=torch.int32, device=dev)
    record = torch.empty(L.mm_route_words(T, K, local), dtype=torch.int32, device=dev)
    lib_mod.check(L.mm_route(ids.data_ptr(), permuted.data_ptr(), record.data_ptr(), T, K, local, offset, stream),
                  "mm_route")
    return weights, ids, permuted, record


@pytest.mark.parametrize("T,E,K,local,offset,score,valid", [
    (8, 384, 8, 384, 0, "sigmoid", None),     # BASELINE config 2 routing
    (32, 256, 8, 128, 128, "sigmoid", None),  # an expert-parallel window
    (5, 64, 6, 64, 0, "softmax", None),
    (64, 384, 8, 384, 0, "sigmoid", None),    # several tiles per expert
    (16, 384, 8, 384, 0, "sigmoid", 13),      # padded graph rows: ids -1, weights 0
])
def test_noalloc_matches_gate_topk_then_route_on_consecutive_calls(T, E, K, local, offset, score, valid):
    from megamoe import _lib

    gen = torch.Generator().manual_seed(1000 + T + E)
    bias = (torch.randn(E, generator=gen) * 0.05).float().cuda()
    nv = None if valid is None else torch.tensor([valid], dtype=torch.int32, device="cuda")
    for call in range(2):  # two calls in a row share the static scratch
        logits = torch.randn((T, E), generator=gen).float().cuda()
        got = _noalloc(_lib, logits, bias, score, K, local, offset, want_ids=call == 0, num_valid=nv)
        want = _allocating(_lib, logits, bias, score, K, local, offset, num_valid=nv)
        torch.cuda.synchronize()
        gw, gi, gp, gr = (None if t is None else t.cpu().numpy() for t in got)
        ww, wi, wp, wr = (t.cpu().numpy() for t in want)
        assert np.array_equal(gw.view(np.uint32), ww.view(np.uint32)), call
        if gi is not None:
            assert np.array_equal(gi, wi), call
        assert np.array_equal(gp, wp), call
        assert np.array_equal(gr, wr), call


def test_noalloc_rejects_requests_beyond_its_scratch():
    from megamoe import _lib

    L = _lib.lib()
    T, E, K = 256, 384, 16  # 4096 slots > the 2048 the static scratch holds
    logits = torch.zeros((T, E), dtype=torch.float32, device="cuda")
    weights = torch.empty((T, K), dtype=torch.float32, device="cuda")
    out = torch.empty((T, K), dtype=torch.int32, device="cuda")
    g = _gate(_lib, logits, None, "sigmoid", weights, None)
    rc = L.mm_gate_route_noalloc(ctypes.byref(g), T, E, K, E, 0, out.data_ptr(), out.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.MM_ERR_INVALID
    assert b"static scratch" in L.mm_last_error()
