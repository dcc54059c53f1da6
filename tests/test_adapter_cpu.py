"""The drop-in adapter (megamoe.adapter.RoutedExpertGemm) called exactly as the
reference's caller calls its RoutedExpertGemm (no GPU: the layer underneath is
replaced by a recorder, the tensors are CPU mocks of the right shapes).

  * construction as routed.py:391-404 builds the reference's;
  * ``gemm(x_q, x_s, ids, w)`` (routed.py:230) reaches RoutedMoE.__call__ as
    the MXFP8 input with the same ids and weights;
  * ``gemm.gate_topk_and_gemms(x_q, x_s, logits, bias, scale, num_valid,
    alt=..., renormalize_epsilon=..., ids_out=..., early=...)`` (routed.py:209-221),
    with and without ``x=`` (slot gate_route_quant), reaches
    RoutedMoE.gate_topk_and_gemms with every argument in its place;
  * the members MoeSlot reads (top_k, max_rows, clamp, router_experts, the
    serves_* / supports* answers) exist and answer by the chain's limits."""

import pytest
import torch

H, E, K, I, T = 512, 16, 6, 256, 5


class _Recorder:
    calls = []

    def __init__(self, w13, w13_scale, w2, w2_scale, top_k, max_rows, **kw):
        self.experts = w13.shape[0]
        self.hidden = 2 * w13.shape[2]
        self.router_experts = kw.get("router_experts") or self.experts
        self.expert_offset = kw.get("expert_offset", 0)
        self.deal_group = kw.get("deal_group", -1)
        _Recorder.calls.append(("init", (w13, w13_scale, w2, w2_scale, top_k, max_rows), kw))

    @classmethod
    def from_trtllm(cls, w13, w13_scale, w2, w2_scale, top_k, max_rows, *, halves, **kw):
        obj = cls(w13, w13_scale, w2, w2_scale, top_k, max_rows, **kw)
        _Recorder.calls.append(("from_trtllm", halves, kw))
        return obj

    def __call__(self, *args):
        _Recorder.calls.append(("call", args))
        return "triple"

    def gate_topk_and_gemms(self, *args, **kw):
        _Recorder.calls.append(("gate", args, kw))
        return "quad"


@pytest.fixture
def adapter(monkeypatch):
    from megamoe import adapter as A

    _Recorder.calls = []
    monkeypatch.setattr(A, "RoutedMoE", _Recorder)
    w13 = torch.zeros((E, 2 * I, H // 2), dtype=torch.uint8)
    w13_s = torch.zeros((E, 2 * I, H // 32), dtype=torch.uint8).view(torch.float8_e4m3fn)
    w2 = torch.zeros((E, H, I // 2), dtype=torch.uint8)
    w2_s = torch.zeros((E, H, I // 32), dtype=torch.uint8).view(torch.float8_e4m3fn)
    clamp = torch.full((E,), 10.0)
    # routed.py:391-404, positional weights then keywords
    gemm = A.RoutedExpertGemm(w13, w13_s, w2, w2_s, clamp, top_k=K, max_rows=48, gate_topk=True,
                              router_experts=2 * E, expert_offset=E, deal_group=-1, gate_route=True,
                              gate_route_quant=True, gemm2_pipe=False, gemm2_registers=0)
    return gemm


def test_construction_matches_the_reference_call(adapter):
    kind, args, kw = _Recorder.calls[0]
    assert kind == "init"
    assert all(a.dtype == torch.uint8 for a in args[:4])  # fp8-typed scales viewed as bytes
    assert args[4:] == (K, 48)
    assert kw["router_experts"] == 2 * E and kw["expert_offset"] == E and kw["clamp"] is not None
    assert _Recorder.calls[1] == ("from_trtllm", "w3_w1", {k: kw[k] for k in kw})
    assert adapter.top_k == K and adapter.max_rows == 48 and adapter.router_experts == 2 * E
    assert adapter.clamp is not None and adapter.gemm2_registers == 0


def test_call_with_the_reference_positional_arguments(adapter):
    x_q = torch.zeros((T, H), dtype=torch.uint8).view(torch.float8_e4m3fn)
    x_s = torch.zeros(T * H // 32 + 64, dtype=torch.uint8)  # a padded flat scale buffer
    ids = torch.zeros((T, K), dtype=torch.int32)
    w = torch.ones((T, K), dtype=torch.float32)
    assert adapter(x_q, x_s, ids, w) == "triple"  # routed.py:230: self.gemm(x_q, x_s, ids, w)
    kind, args = _Recorder.calls[-1]
    assert kind == "call"
    assert args[0] is x_q and args[2] is ids and args[3] is w
    assert tuple(args[1].shape) == (T, H // 32)  # the scale view the chain takes
    assert adapter.supports(x_q, x_s, ids, w)
    assert not adapter.supports(x_q, x_s, ids[:, :2], w)


def test_gate_topk_and_gemms_with_the_reference_arguments(adapter):
    x_q = torch.zeros((T, H), dtype=torch.uint8)
    x_s = torch.zeros((T, H // 32), dtype=torch.uint8)
    logits = torch.zeros((T, 2 * E), dtype=torch.float32)
    bias = torch.zeros(2 * E, dtype=torch.float32)
    nv = torch.tensor([T], dtype=torch.int32)
    ids_out = torch.zeros((64, K), dtype=torch.int32)
    alt = (bias, torch.zeros(T, dtype=torch.int64), 7)
    # routed.py:209-221
    out = adapter.gate_topk_and_gemms(x_q, x_s, logits, bias, 1.5, nv, alt=alt, renormalize_epsilon=1e-20,
                                      ids_out=ids_out, early=True)
    assert out == "quad"
    kind, args, kw = _Recorder.calls[-1]
    assert kind == "gate"
    assert args[0] is x_q and args[1] is x_s and args[2] is logits and args[3] is bias
    assert args[4:] == (1.5, nv, alt, 1e-20, ids_out, None, True)
    assert kw == {"score": "sqrtsoftplus_dsv41"}  # top-6: the reference gate's own numerics
    # slot gate_route_quant: the bf16 input replaces x_q / x_s
    x = torch.zeros((T, H), dtype=torch.bfloat16)
    adapter.gate_topk_and_gemms(None, None, logits, bias, 1.5, None, x=x)
    _, args, _ = _Recorder.calls[-1]
    assert args[0] is None and args[1] is None and args[9] is x
    assert adapter.serves_gate_route_quant(T, None, x)
    assert not adapter.serves_gate_route_quant(T, None, x[:, :16])
    assert adapter.supports_gate_topk(logits, bias)
    assert not adapter.supports_gate_topk(logits[:, :E].contiguous(), bias)
    adapter.bind_early_release(3)
