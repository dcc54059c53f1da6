"""SGLang's stock routed-MoE path on the B200, as a same-box GPU baseline: FlashInfer's
TRT-LLM-gen fused MoE (``flashinfer.fused_moe.trtllm_fp4_block_scale_moe`` /
``trtllm_fp4_block_scale_routed_moe``), run as a library.

This is what the reference serves with outside its own DSV4.1 kernels, and what it
checks its routed GEMM pair against: ``test/kernels/test_deepseek_v41_moe.py:116-153``
(``Mxfp4FlashinferTrtllmMoEMethod``'s call, ``do_finalize=False``). FlashInfer's kernels
are prebuilt cubins shipped in the ``flashinfer-cubin`` wheel; they are launched, never
inspected.

FlashInfer builds a host-side launcher library on first use (about 16 minutes of nvcc on
24 cores). ``python baseline/flashinfer_moe.py build`` builds it once, offline, into
``baseline/_flashinfer/`` (git-ignored; it ships with the repository snapshot to the GPU
box). ``load()`` then reuses that library and never compiles on the GPU box.

Nothing in the ``megamoe`` package imports this file: it is a measured comparison, used
only by ``bench.py --impl flashinfer``.
"""

from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CACHE = os.path.join(HERE, "_flashinfer")


def _env() -> None:
    if "flashinfer" in sys.modules and os.environ.get("FLASHINFER_WORKSPACE_BASE") != CACHE:
        raise RuntimeError("flashinfer was imported before baseline.flashinfer_moe set its cache directory")
    os.environ["FLASHINFER_WORKSPACE_BASE"] = CACHE
    os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", "10.0a")


def _spec():
    _env()
    from flashinfer.fused_moe.core import gen_trtllm_gen_fused_moe_sm100_module

    return gen_trtllm_gen_fused_moe_sm100_module()


def build() -> str:
    """Compile FlashInfer's TRT-LLM-gen MoE launcher for sm_100a into ``_flashinfer/``;
    object files are removed afterwards (only the shared library is kept)."""
    spec = _spec()
    spec.build(verbose=False)
    for name in os.listdir(spec.build_dir):
        if name.endswith(".o"):
            os.remove(os.path.join(spec.build_dir, name))
    return str(spec.jit_library_path)


def load():
    """Import FlashInfer's fused-MoE entry points over the prebuilt launcher; raises
    when the launcher has not been built."""
    spec = _spec()
    if not spec.jit_library_path.exists():
        raise RuntimeError(f"FlashInfer's MoE launcher is not built ({spec.jit_library_path}); "
                           "run `python baseline/flashinfer_moe.py build` first")
    import flashinfer.jit.core as jit_core

    compile_ = jit_core.JitSpec.build

    def build_if_missing(self, verbose, need_lock=True):
        if self.jit_library_path.exists():
            return None
        return compile_(self, verbose, need_lock)

    jit_core.JitSpec.build = build_if_missing
    from flashinfer.fused_moe import trtllm_fp4_block_scale_moe, trtllm_fp4_block_scale_routed_moe

    return trtllm_fp4_block_scale_moe, trtllm_fp4_block_scale_routed_moe


def pack_topk(ids, weights):
    """FlashInfer's packed routed-expert word, its routing kernels' ``PackedScoreIdx<bf16>``
    ({bf16 score; int16 idx}, RoutingKernel.h) read as one little-endian int32: expert id
    << 16 | bf16 weight bits."""
    import torch

    wb = weights.to(torch.bfloat16).view(torch.int16).to(torch.int32) & 0xFFFF
    return (ids.to(torch.int32) << 16) | wb


class FlashInferLayer:
    """One MXFP4 routed-MoE layer (+ one shared expert) on FlashInfer's TRT-LLM-gen
    kernels, from the canonical weights ``megamoe.RoutedMoE`` reads ([w1; w3] rows,
    row-major E8M0 scales). Activations stay bf16 (FlashInfer's MxE2m1 x Bfloat16 mode);
    routing is FlashInfer's DeepSeekV3 method with one group (sigmoid + bias -> top-k ->
    renormalize -> x routed scale), the rule of the bench's layer.

    ``forward(x, logits)`` is one step: the routed MoE with FlashInfer's own routing and
    finalize, the shared expert as a one-expert routed call, and their sum."""

    def __init__(self, w13, s13, w2, s2, shared, bias, top_k, scale, tokens):
        import torch

        from megamoe.layouts import canonical_to_trtllm

        self.moe, self.routed = load()
        E, two_i, _ = w13.shape
        self.E, self.I, self.k, self.scale, self.T = E, two_i // 2, top_k, scale, tokens
        g = canonical_to_trtllm(w13, s13, w2, s2)
        self.w = (g[0], g[1].view(torch.float8_e4m3fn), g[2], g[3].view(torch.float8_e4m3fn))
        self.sw = None
        if shared is not None:
            gs = canonical_to_trtllm(*shared[:4])
            self.sw = (gs[0], gs[1].view(torch.float8_e4m3fn), gs[2], gs[3].view(torch.float8_e4m3fn))
            one = torch.ones((tokens, 1), dtype=torch.float32, device=w13.device)
            self.shared_ids = pack_topk(torch.zeros((tokens, 1), dtype=torch.int32, device=w13.device), one)
        self.bias = bias.float().contiguous()

    def _call(self, fn, head, w, experts, top_k, local=None, **kw):
        return fn(*head, gemm1_weights=w[0], gemm1_weights_scale=w[1], gemm1_bias=None, gemm1_alpha=None,
                  gemm1_beta=None, gemm1_clamp_limit=None, gemm2_weights=w[2], gemm2_weights_scale=w[3],
                  gemm2_bias=None, output1_scale_scalar=None, output1_scale_gate_scalar=None,
                  output2_scale_scalar=None, num_experts=experts, top_k=top_k, intermediate_size=self.I,
                  local_expert_offset=0, local_num_experts=experts if local is None else local, enable_pdl=True,
                  tune_max_num_tokens=max(self.T, 8), **kw)[0]

    def forward(self, x, logits, x_q=None, x_s=None):
        """x bf16 [T, H] (bf16 activations), or with ``x_q``/``x_s`` its MXFP8 codes and
        linear-layout E8M0 scales (FlashInfer's MxE4m3 activations)."""
        if x_q is not None:
            x = x_q
        out = self._call(self.moe, (logits, self.bias, x, x_s), self.w, self.E, self.k, n_group=1,
                         topk_group=1, routed_scaling_factor=self.scale, routing_method_type=2,
                         do_finalize=True)
        if self.sw is None:
            return out
        # FlashInfer's routing wants >= 4 experts, a multiple of 4: the shared expert is
        # local expert 0 of 4, every token routed to it with weight 1 (TopK: weights as given)
        sh = self._call(self.routed, (self.shared_ids[: x.shape[0]], None, x, x_s), self.sw, 4, 1, local=1,
                        n_group=None, topk_group=None, routed_scaling_factor=None, routing_method_type=5,
                        do_finalize=True)
        return out + sh

    def forward_routed(self, x, ids, weights):
        """One step with given routing (ids int32 [T, k], weights fp32 [T, k], the
        routed scale already in the weights): FlashInfer's routed MoE over the packed
        (id, bf16 weight) words, finalized, plus the shared expert."""
        out = self._call(self.routed, (pack_topk(ids, weights), None, x, None), self.w, self.E, self.k,
                         n_group=None, topk_group=None, routed_scaling_factor=None, routing_method_type=5,
                         do_finalize=True)
        if self.sw is None:
            return out
        sh = self._call(self.routed, (self.shared_ids[: x.shape[0]], None, x, None), self.sw, 4, 1, local=1,
                        n_group=None, topk_group=None, routed_scaling_factor=None, routing_method_type=5,
                        do_finalize=True)
        return out + sh


def mxfp8_quantize(x):
    """MXFP8 codes (float8_e4m3fn [T, H]) and linear E8M0 scales ([T, H/32] viewed as
    float8_e4m3fn, as FlashInfer takes them) of bf16 x: per 32 elements the scale
    2^ceil(log2(amax / 448)), codes x / scale rounded to E4M3 (the OCP MX rule)."""
    import torch

    T, H = x.shape
    xf = x.float().view(T, H // 32, 32)
    amax = xf.abs().amax(-1, keepdim=True)
    e = torch.ceil(torch.log2(torch.clamp(amax / 448.0, min=2.0 ** -126)))
    q = (xf / torch.exp2(e)).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(T, H)
    s = (e + 127.0).to(torch.uint8).view(T, H // 32).view(torch.float8_e4m3fn)
    return q.contiguous(), s.contiguous()


if __name__ == "__main__":
    if sys.argv[1:] != ["build"]:
        sys.exit("usage: python baseline/flashinfer_moe.py build")
    print(build())
