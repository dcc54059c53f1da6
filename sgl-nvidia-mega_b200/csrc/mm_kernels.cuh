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
  int m1, m2;                // gate_up tiles / down units per segment
  int ks1;                   // K stages of a gate_up tile
  int grid;                  // the expert kernel's CTAs (the split-K choice)
  int *split_cnt;            // [2 x grid] split-K arrival counters, zeroed when split > 1
  int *seg_tok;              // [segments][kSegRows] the token of each segment row
};

// The routed input's quantization into FP4 terms (extra CTAs of the front launch).
struct QuantArgs {
  const uint16_t *x;         // bf16 [T, H], or null with
  const uint8_t *x8;         //    MXFP8 [T, H] E4M3 codes and
  const uint8_t *s8;         //    [T, H/32] E8M0 block scales
  uint8_t *xq;               // [kMaxTerms][max_tokens][H/2] packed E2M1
  uint8_t *xs;               // [kMaxTerms][max_tokens][H/32] E8M0 (NVFP4: [H/16] E4M3)
  int tokens, hidden, max_tokens, terms;
  int fmt;                   // kFmtMx or kFmtNv
  float gs, inv_gs;          // NVFP4: 1 / input_scale[0] and input_scale[0]
  int ctas;                  // quantization CTAs (after the T row CTAs); 0: none
};

struct FrontArgs {
  GateArgs gate;             // gate.logits null: ids are given in route.ids
  RouteArgs route;
  QuantArgs quant;
  int row_ctas;              // T with a gate (one per row), 1 with given ids, 0: quantization only
};

constexpr int kMaxRouterParts = 14;  // H <= 14336 for the router GEMV (x tile in shared memory)
constexpr int kMaxRouterHidden = 1024 * kMaxRouterParts;

struct RouterArgs {
  const uint16_t *x;         // bf16 [T, H]
  const uint16_t *w;         // bf16 [E, H]
  float *logits;             // [T, E]
  int tokens, experts, hidden;
  uint32_t *err;             // a layer's error word (the x staging wait), or null
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
  const int *seg_tok;        // [segments][kSegRows] the token of each segment row
  const int4 *segs;
  int *ctrl;
  int *flags;
  float *part;               // [grid][kPartFloats] split-K partial sums
  int *split_cnt;            // [2 x grid] split-K arrival counters (per tile and feature half)
  uint32_t *err;
  const float *clamp;        // [E] or null
  const float *shared_clamp; // [1] or null
  int hidden, inter, max_tokens, rows_cap, terms;
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

// Activation quantization into FP4 terms, one warp per 32 fp32 values, lane i
// holding value i. Term t quantizes the residual r left by terms 0..t-1:
//  * MXFP4 (one block of 32): E8M0 code c = mx4_scale_code(amax), codes
//    e2m1(r * 2^(127-c)) RN saturating, r -= e2m1 * 2^(c-127); 16 bytes of
//    codes per term at q + t * q_stride, the code at s + t * s_stride;
//  * NVFP4 under the global scale gs (lanes 0-15 and 16-31 are two blocks of
//    16): E4M3 scale sf = nv4_scale_code(amax, gs), codes e2m1(r * gs / sf) RN
//    saturating, r -= (e2m1 * sf) * inv_gs; 8 bytes of codes per block and
//    term, the two scale bytes at s + t * s_stride + {0, 1}.
// amax is the (half-)warp maximum of |r|, NaN counted as 0 (the value of an
// fmaxf chain from 0).
__device__ __forceinline__ uint32_t amax_key(float r) {
  const float a = fabsf(r);
  return a != a ? 0u : __float_as_uint(a);
}

__device__ __forceinline__ void quantize_block32_fp4_warp(float r, int terms, uint8_t *q, size_t q_stride,
                                                          uint8_t *s, size_t s_stride) {
  const int lane = threadIdx.x & 31;
  for (int t = 0; t < terms; ++t) {
    const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, amax_key(r)));
    const uint32_t c = mx4_scale_code(amax);
    const uint32_t nib = e2m1x2(__fmul_rn(r, mx_inverse(c)), 0.0f) & 15u;
    r = __fsub_rn(r, __fmul_rn(e2m1_value(nib), mx_scale_value(c)));
    const uint32_t hi = __shfl_down_sync(0xffffffffu, nib, 1);
    if ((lane & 1) == 0) q[t * q_stride + (lane >> 1)] = static_cast<uint8_t>(nib | (hi << 4));
    if (lane == 0) s[t * s_stride] = static_cast<uint8_t>(c);
  }
}

__device__ __forceinline__ void quantize_block16x2_nvfp4_warp(float r, int terms, float gs, float inv_gs,
                                                              uint8_t *q, size_t q_stride, uint8_t *s,
                                                              size_t s_stride) {
  const int lane = threadIdx.x & 31;
  for (int t = 0; t < terms; ++t) {
    uint32_t m = amax_key(r);
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {
      const uint32_t o = __shfl_xor_sync(0xffffffffu, m, off);
      m = o > m ? o : m;
    }
    const uint32_t c = nv4_scale_code(__uint_as_float(m), gs);
    const float sv = e4m3_value(static_cast<uint8_t>(c));
    const uint32_t nib = e2m1x2(__fmul_rn(r, nv4_multiplier(sv, gs)), 0.0f) & 15u;
    r = __fsub_rn(r, __fmul_rn(__fmul_rn(e2m1_value(nib), sv), inv_gs));
    const uint32_t hi = __shfl_down_sync(0xffffffffu, nib, 1);
    if ((lane & 1) == 0) q[t * q_stride + (lane >> 1)] = static_cast<uint8_t>(nib | (hi << 4));
    if ((lane & 15) == 0) s[t * s_stride + (lane >> 4)] = static_cast<uint8_t>(c);
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
__global__ void router_kernel(RouterArgs a);
__global__ void gate_topk_kernel(GateArgs g);
__global__ void route_kernel(RouteArgs r);
__global__ void front_kernel(FrontArgs f);
// the same two launches with the DeepSeek-V4.1 gate's numerics (mm_gate_dsv41.cu)
__global__ void gate_topk_dsv41_kernel(GateArgs g);
__global__ void front_dsv41_kernel(FrontArgs f);
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
