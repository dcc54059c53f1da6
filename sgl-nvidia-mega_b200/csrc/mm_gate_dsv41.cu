// The router top-k with the DeepSeek-V4.1 gate's own numerics
// (MM_SCORE_SQRTSOFTPLUS_DSV41), for ids and weights equal bit for bit to the
// reference's gate_topk.cu on the same logits.
//
// The reference's gate (deepseek_v41/sm103/moe/src/gate_topk.cuh:99-198, built
// with DSV41_GATE_REFERENCE 0 when SGLang routes with its Triton kernel) is
// compiled by NVRTC with flush-to-zero and approximate square root and
// division (routed_expert_gemm.py:213-220, GATE_TOPK_NVRTC_OPTIONS). This file
// is its own translation unit so that it is compiled with the same three
// flags (megamoe/_build.py: -ftz=true -prec-sqrt=false -prec-div=false) and
// evaluates the same source-level operations:
//   score  s = sqrtf(x > 20 ? x : log1pf(expf(x)))        (CUDA's expf, log1pf, sqrtf)
//   key    v = s + bias, NaN as +inf (ranked first), v + 0 (-0 as +0),
//          the order-preserving u32 of v
//   sum    top-6: ((w0 + w2) + (w1 + w3)) + (w4 + w5); top-3: (w0 + w2) + w1
//          (the order of the Triton kernel's reduction over its 8 / 4 slots)
//   weight div.full(w, eps > 0 ? sum + eps : (sum > 0 ? sum : 1)) * scale
// Selection (the K largest keys, the lowest id winning a tie) and padded rows
// (id -1, weight 0) are shared with the other score functions (mm_gate.cuh).
// These bits cannot be replayed on the CPU (the functions' implementations
// are CUDA's); the GPU tests pin them against the reference kernel itself.
#include <cstdint>
#include <cuda_runtime.h>

#include "megamoe.h"
#include "mm_gate.cuh"
#include "mm_kernels.cuh"

namespace mm {

namespace {

// div.full.f32: the PTX ISA's full-range approximate division (the reference
// divides the routing weights with it).
__device__ __forceinline__ float div_full(float a, float b) {
  float q;
  asm("div.full.f32 %0, %1, %2;" : "=f"(q) : "f"(a), "f"(b));
  return q;
}

struct Dsv41Routing {
  static __device__ __forceinline__ float score(const GateArgs &, float x) {
    const float sp = x > 20.0f ? x : log1pf(expf(x));
    return sqrtf(sp);
  }
  static __device__ __forceinline__ uint32_t key(float s, float b) {
    const float biased = s + b;
    const float v = (biased == biased ? biased : __int_as_float(0x7f800000)) + 0.0f;
    const uint32_t bits = __float_as_uint(v);
    return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
  }
  static __device__ __forceinline__ float weight(const GateArgs &g, const GateSmem &sm, int k) {
    const int K = g.top_k;  // 3 or 6 (the host checks)
    float w[6];
#pragma unroll
    for (int i = 0; i < 6; ++i) w[i] = i < K ? sm.score[sm.sel[i]] : 0.0f;
    const float sum = K == 6 ? ((w[0] + w[2]) + (w[1] + w[3])) + (w[4] + w[5]) : (w[0] + w[2]) + w[1];
    const float eps = g.renorm_eps;
    const float norm = eps > 0.0f ? sum + eps : (sum > 0.0f ? sum : 1.0f);
    return div_full(sm.score[sm.sel[k]], norm) * g.routed_scaling;
  }
};

}  // namespace

__global__ void __launch_bounds__(512) gate_topk_dsv41_kernel(GateArgs g) {
  pdl_launch_dependents();
  __shared__ GateSmem sm;
  pdl_wait();
  const int valid = g.num_valid != nullptr ? *g.num_valid : static_cast<int>(gridDim.x);
  gate_row<Dsv41Routing>(g, blockIdx.x, valid, sm);
}

__global__ void __launch_bounds__(512) front_dsv41_kernel(FrontArgs f) {
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char front_smem[];
  front_body<Dsv41Routing, false>(f, front_smem);  // rows only: the quantization is IEEE (front_kernel)
}

}  // namespace mm
