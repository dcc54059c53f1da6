// Kernel argument blocks and the device helpers shared by several kernels.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "mm_numerics.cuh"

namespace mm {

struct GateArgs {
  const float *logits;       // [T, router_experts]
  const float *bias;         // [router_experts] or null
  const int *num_valid;      // [1] or null
  int score_func;            // 0 sigmoid, 1 softmax
  int renormalize;
  float routed_scaling;
  float renorm_eps;
  int router_experts;
  int top_k;
  float *weights_out;        // [T, top_k]
  int *ids_out;              // [T, top_k]
};

struct RouteArgs {
  const int *ids;            // [T, top_k] router ids
  int *permuted;             // [T, top_k]
  int *record;               // route record
  int tokens, top_k, experts, expert_offset;
  // expert-kernel work tables (segs null: record only)
  int4 *segs;
  int *ctrl;
  int *flags;
  int has_shared;
  int shared_row_base;
  int m1, m2;                // gate_up / down units per segment
};

struct FrontArgs {
  GateArgs gate;             // gate.logits null: ids are given in route.ids
  RouteArgs route;
  const uint16_t *x;         // bf16 [T, H]
  uint8_t *xq;               // [2][max_tokens][H]
  uint8_t *xs;               // [2][max_tokens][H/32]
  int hidden;
  int max_tokens;
  int terms;
};

struct alignas(64) ExpertArgs {
  CUtensorMap w13_map;       // routed gate_up codes, 3-D {H, 2I, E}, 16U4_ALIGN16B
  CUtensorMap w2_map;        // routed down codes, {I, H, E}
  CUtensorMap sw13_map;      // shared expert (same shapes, E = 1)
  CUtensorMap sw2_map;
  const uint8_t *sfa13;      // [E][I/64][H/256][1024] scale chunks
  const uint8_t *sfa2;       // [E][H/128][I/256][1024]
  const uint8_t *ssfa13;
  const uint8_t *ssfa2;
  const uint8_t *xq;         // [2][max_tokens][H]
  const uint8_t *xs;         // [2][max_tokens][H/32]
  uint8_t *hq;               // [2][rows_cap][I]
  uint8_t *hs;               // [2][rows_cap][I/32]
  uint16_t *rows_out;        // [rows_cap][H] bf16
  const int *record;
  const int4 *segs;
  int *ctrl;
  int *flags;
  uint32_t *err;
  const float *clamp;        // [E] or null
  const float *shared_clamp; // [1] or null
  int hidden, inter, max_tokens, rows_cap, terms, token_off;
  int m1, m2, ks1, ks2;
};

struct FinalizeArgs {
  const uint16_t *rows;
  const float *weights;
  const int *permuted;
  const uint16_t *shared_rows;
  uint16_t *out;
  float *partial;
  int tokens, top_k, hidden;
};

// Two-term MXFP8 quantization of 32 fp32 values (see quantize_row).
__device__ __forceinline__ void quantize_block32(const float (&v)[32], uint8_t *q_hi,
                                                 uint8_t *q_lo, uint8_t *s_hi, uint8_t *s_lo,
                                                 int terms) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const uint32_t c = mx_scale_code(amax);
  const float inv = mx_inverse(c);
  const float sv = mx_scale_value(c);
  uint32_t packed[8];
  float r[32];
  float amax2 = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const uint16_t q2 = e4m3x2(__fmul_rn(v[i], inv), __fmul_rn(v[i + 1], inv));
    const uint8_t c0 = static_cast<uint8_t>(q2 & 0xffu), c1 = static_cast<uint8_t>(q2 >> 8);
    if ((i & 2) == 0) packed[i >> 2] = q2;
    else packed[i >> 2] |= static_cast<uint32_t>(q2) << 16;
    r[i] = __fsub_rn(v[i], __fmul_rn(e4m3_value(c0), sv));
    r[i + 1] = __fsub_rn(v[i + 1], __fmul_rn(e4m3_value(c1), sv));
    amax2 = fmaxf(amax2, fmaxf(fabsf(r[i]), fabsf(r[i + 1])));
  }
  uint4 *dh = reinterpret_cast<uint4 *>(q_hi);
  dh[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  dh[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  *s_hi = static_cast<uint8_t>(c);
  if (terms < 2) return;
  const uint32_t c2 = mx_scale_code(amax2);
  const float inv2 = mx_inverse(c2);
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const uint16_t q2 = e4m3x2(__fmul_rn(r[i], inv2), __fmul_rn(r[i + 1], inv2));
    if ((i & 2) == 0) packed[i >> 2] = q2;
    else packed[i >> 2] |= static_cast<uint32_t>(q2) << 16;
  }
  uint4 *dl = reinterpret_cast<uint4 *>(q_lo);
  dl[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  dl[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  *s_lo = static_cast<uint8_t>(c2);
}

// kernels (definitions in mm_route.cu, mm_experts.cu, mm_finalize.cu)
__global__ void router_gemv_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ w,
                                   float *__restrict__ logits, int tokens, int experts, int hidden);
__global__ void gate_topk_kernel(GateArgs g);
__global__ void route_kernel(RouteArgs r);
__global__ void front_kernel(FrontArgs f);
__global__ void expert_kernel(const __grid_constant__ ExpertArgs p);
__global__ void repack_scales_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
                                     int n, int rows, int k, int gate_up, int inter);
__global__ void finalize_kernel(FinalizeArgs a);
__global__ void finalize_partial_kernel(const float *__restrict__ partial, uint16_t *__restrict__ out,
                                        int tokens, int hidden);

}  // namespace mm
