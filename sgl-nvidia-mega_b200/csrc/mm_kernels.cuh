// Kernel argument blocks and the device helpers shared by several kernels.
#pragma once
#include <utility>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "mm_numerics.cuh"

namespace mm {

struct GateArgs {
  const float *logits;       // [T, router_experts]
  const float *bias;         // [router_experts] or null
  const int *num_valid;      // [1] or null
  int score_func;            // 0 sigmoid, 1 softmax, 2 sqrt(softplus)
  int renormalize;
  float routed_scaling;
  float renorm_eps;
  int router_experts;
  int top_k;
  float *weights_out;        // [T, top_k]
  int *ids_out;              // [T, top_k]
  const float *bias_alt;     // [router_experts] or null (vision rows rank with it)
  const void *input_ids;     // [T] int32 / int64, or null
  int input_ids64;
  long long alt_token_id;
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
};

constexpr int kMaxRouterParts = 14;  // H <= 14336 for the router GEMV (x tile in shared memory)
constexpr int kMaxRouterHidden = 1024 * kMaxRouterParts;

struct RouterArgs {
  const uint16_t *x;         // bf16 [T, H] (GEMV input; quantized unless x8 is set)
  const uint8_t *x8;         // or MXFP8 [T, H] E4M3 codes (quantization only), with
  const uint8_t *s8;         //    [T, H/32] E8M0 block scales
  const uint16_t *w;         // bf16 [E, H] (null when gemv_ctas == 0)
  float *logits;             // [T, E]
  int tokens, experts, hidden;
  int gemv_ctas;             // E, or 0 for quantization only
  uint8_t *xq;               // [kMaxTerms][max_tokens][H/2] packed E2M1, or null
  uint8_t *xs;               // [kMaxTerms][max_tokens][H/32] E8M0 (NVFP4: [H/16] E4M3)
  int max_tokens;
  int terms;
  int fmt;                   // kFmtMx or kFmtNv
  float gs, inv_gs;          // NVFP4: 1 / input_scale[0] and input_scale[0]
};

struct alignas(64) ExpertArgs {
  CUtensorMap w13_map;       // routed gate_up codes, u8 3-D {H/2, 2I, E}, box {128, 64, 1}
  CUtensorMap w2_map;        // routed down codes, u8 {I/2, H, E}, box {128, 128, 1}
  CUtensorMap sw13_map;      // shared expert (same shapes, E = 1)
  CUtensorMap sw2_map;
  const uint8_t *sfa13;      // [E][I/64][H/256][scale chunks of a stage]
  const uint8_t *sfa2;       // [E][H/128][I/256][...]
  const uint8_t *ssfa13;
  const uint8_t *ssfa2;
  const uint8_t *xq;         // [kMaxTerms][max_tokens][H/2]
  const uint8_t *xs;         // [kMaxTerms][max_tokens][H/block]
  uint8_t *hq;               // [kMaxTerms][rows_cap][hq_row]
  uint8_t *hs;               // [kMaxTerms][rows_cap][hs_row]
  // NVFP4 only: accumulator multipliers per expert (weight scale_2 x the
  // GEMM's input scale) and the down GEMM's input quantization scale
  const float *alpha13;      // [E]
  const float *alpha2;       // [E]
  const float *salpha13;     // [1] shared expert
  const float *salpha2;      // [1]
  float gs2, inv_gs2;        // 1 / input_scale[1] and input_scale[1]
  uint16_t *rows_out;        // [rows_cap][H] bf16
  const int *record;
  const int4 *segs;
  int *ctrl;
  int *flags;
  uint32_t *err;
  const float *clamp;        // [E] or null
  const float *shared_clamp; // [1] or null
  int hidden, inter, max_tokens, rows_cap, terms, token_off;
  int hq_row, hs_row;        // bytes per h row / h scale row: I rounded up to 256 features, zero past I
  int m1, m2, ks1, ks2;      // gate_up units / down tiles per segment; K stages of each
  int tg2, u2;               // down tiles per down unit; down units per segment (ceil(m2 / tg2))
  unsigned long long wait_ns;  // budget of every bounded wait (mm_layer_set_wait_budget)
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

// MXFP4 terms of 32 fp32 values (one block): term t is the MXFP4 quantization
// of the residual left by terms 0..t-1 (E8M0 code by mx4_scale_code, codes
// e2m1(r * 2^(127-code)) RN saturating, residual r -= e2m1 * 2^(code-127)).
// Writes 16 bytes of codes per term at q + t * q_stride and the code at
// s + t * s_stride.
__device__ __forceinline__ void quantize_block32_fp4(const float (&v)[32], int terms, uint8_t *q,
                                                     size_t q_stride, uint8_t *s, size_t s_stride) {
  float r[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) r[i] = v[i];
  for (int t = 0; t < terms; ++t) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(r[i]));
    const uint32_t c = mx4_scale_code(amax);
    const float inv = mx_inverse(c);
    const float sv = mx_scale_value(c);
    uint32_t packed[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const uint32_t b = e2m1x2(__fmul_rn(r[i], inv), __fmul_rn(r[i + 1], inv));
      packed[i >> 3] |= b << (8 * ((i >> 1) & 3));
      r[i] = __fsub_rn(r[i], __fmul_rn(e2m1_value(b & 15u), sv));
      r[i + 1] = __fsub_rn(r[i + 1], __fmul_rn(e2m1_value(b >> 4), sv));
    }
    *reinterpret_cast<uint4 *>(q + t * q_stride) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    s[t * s_stride] = static_cast<uint8_t>(c);
  }
}

// NVFP4 terms of 16 fp32 values (one block) under the global scale gs: term t
// is the NVFP4 quantization of the residual left by terms 0..t-1 (E4M3 scale
// sf = nv4_scale_code(amax, gs), codes e2m1(r * gs / sf) RN saturating,
// residual r -= (e2m1 * sf) * inv_gs). Writes 8 bytes of codes per term at
// q + t * q_stride and the scale byte at s + t * s_stride.
__device__ __forceinline__ void quantize_block16_nvfp4(const float *v, int terms, float gs, float inv_gs,
                                                       uint8_t *q, size_t q_stride, uint8_t *s,
                                                       size_t s_stride) {
  float r[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) r[i] = v[i];
  for (int t = 0; t < terms; ++t) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(r[i]));
    const uint32_t c = nv4_scale_code(amax, gs);
    const float sv = e4m3_value(static_cast<uint8_t>(c));
    const float f = nv4_multiplier(sv, gs);
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const uint32_t b = e2m1x2(__fmul_rn(r[i], f), __fmul_rn(r[i + 1], f));
      packed[i >> 3] |= b << (8 * ((i >> 1) & 3));
      r[i] = __fsub_rn(r[i], __fmul_rn(__fmul_rn(e2m1_value(b & 15u), sv), inv_gs));
      r[i + 1] = __fsub_rn(r[i + 1], __fmul_rn(__fmul_rn(e2m1_value(b >> 4), sv), inv_gs));
    }
    *reinterpret_cast<uint2 *>(q + t * q_stride) = make_uint2(packed[0], packed[1]);
    s[t * s_stride] = static_cast<uint8_t>(c);
  }
}

// Launch with programmatic stream serialization: the kernel may start while its
// predecessor runs; it reads the predecessor's outputs after griddepcontrol.wait.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void *stream,
                   Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Host helpers shared by the .cu files (mm_api.cu defines them).
int set_error(int code, const char *fmt, ...);
// dynamic shared memory of the router launch for hidden size H: 8 token rows
// of x (bf16) and the part sums of a 4-expert x 8-token tile
inline size_t router_smem_bytes(int hidden) {
  return static_cast<size_t>(8) * hidden * 2 + static_cast<size_t>(4) * kMaxRouterParts * 8 * 4;
}
// dynamic shared memory of the route build for (tokens, local experts)
inline size_t route_smem_size(int tokens, int experts) {
  const int words = (tokens + 31) / 32;
  return static_cast<size_t>(experts) * words * 4 + static_cast<size_t>(experts) * 4 * 3 + 32 * 4;
}

// kernels (definitions in mm_route.cu, mm_experts.cu, mm_finalize.cu)
__global__ void router_quant_kernel(RouterArgs a);
__global__ void gate_topk_kernel(GateArgs g);
__global__ void route_kernel(RouteArgs r);
__global__ void front_kernel(FrontArgs f);
// The expert kernel of format fmt (kFmtMx / kFmtNv): the dynamic shared memory
// attribute (once per process and format) and a launch of `ctas` CTAs.
// Defined beside the kernel template, whose instantiations stay in that file.
cudaError_t expert_kernel_configure(int fmt);
cudaError_t expert_kernel_launch(int fmt, int ctas, const ExpertArgs &ea, void *stream);
__global__ void repack_scales_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
                                     int n, int rows, int k, int gate_up, int inter, int block);
__global__ void nv_alpha_kernel(const float *__restrict__ scale_2, float input_scale, float *__restrict__ alpha,
                                int n);
__global__ void finalize_kernel(FinalizeArgs a);
__global__ void finalize_partial_kernel(const float *__restrict__ partial, uint16_t *__restrict__ out,
                                        int tokens, int hidden);

}  // namespace mm
