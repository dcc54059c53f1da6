// Front of the routed-MoE chain: router GEMV (K0), top-k with bias (K1a), the
// route record and slot -> row map (K1b), the MXFP4-terms quantization of the
// routed input, and the segment / work tables of the expert kernel. The top-k
// and the route build are in mm_gate.cuh; this file instantiates them with this
// library's routing numerics (IeeeRouting below).
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>

#include "megamoe.h"
#include "mm_gate.cuh"
#include "mm_kernels.cuh"
#include "mm_layout.cuh"
#include "mm_numerics.cuh"
#include "mm_ptx.cuh"

namespace mm {

// ============================================================================
// K0: router GEMV.
//
// Grid (ceil(E / 4), ceil(T / 8)): logits[t, e] = sum_h x[t, h] w[e, h] (fp32) for
// experts [4 blockIdx.x, +4) and the 8 tokens of chunk blockIdx.y. Summation
// order (the CPU oracle replays it): H is cut in parts of 1024; lane l of a
// part accumulates, for j = 0..3 and i = 0..7, the element
// h = 1024 p + 8 (l + 32 j) + i with acc = fma(x, w, acc) from acc = 0; the 32
// lane sums are combined pairwise by lane bit 4, then 3, 2, 1, 0 (the pairing
// of the butterfly acc += shfl_xor(acc, 16, 8, 4, 2, 1), computed here as a
// reduce-scatter over a warp's 4 experts x 8 tokens); the part sums in part
// order, s = ((p0 + p1) + p2) + ... bf16 x bf16 products
// are exact in fp32. The weight rows are static, so the first part's loads
// are issued before the grid-dependency wait. Dynamic shared memory:
// router_smem_bytes(H).
// ============================================================================
__global__ void __launch_bounds__(256) router_kernel(RouterArgs a) {
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // GEMV tile: experts [4 blockIdx.x, +4) x tokens [8 blockIdx.y, +8). The 8
  // token rows of x are staged once in shared memory, one bulk copy per row
  // completing on one mbarrier (a few instructions where 16-byte copies took
  // thousands). Warp w takes
  // the 1024-wide K parts w, w + 8 for all four experts, so each x load feeds
  // four experts; lane l sums elements 8 (l + 32 j) .. + 8 of the part for every
  // (expert, token), and a reduce-scatter butterfly over the 32 (expert, token)
  // sums leaves lane l with the part sum of expert l / 8, token l % 8 (the same
  // pairing of lanes as an xor all-reduce: 16, 8, 4, 2, 1). One thread per
  // (expert, token) then adds the parts in part order.
  extern __shared__ __align__(16) unsigned char router_smem[];
  uint16_t *xs = reinterpret_cast<uint16_t *>(router_smem);                  // [8][H] bf16
  float *part_val = reinterpret_cast<float *>(router_smem + 8 * a.hidden * 2);  // [4][kMaxRouterParts][8]
  const int t0 = blockIdx.y * 8;
  const int nt = min(8, a.tokens - t0);
  const int parts = a.hidden >> 10;
  const int e0 = blockIdx.x * 4;
  // the warp's first part's weights (4 experts x 32 elements per lane) are
  // loaded before the grid-dependency wait; a second part (H > 8192) when reached
  auto load_w = [&](int part, uint4 (&wv)[4][4]) {
#pragma unroll
    for (int es = 0; es < 4; ++es)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        wv[es][j] = e0 + es < a.experts && part < parts
                        ? __ldg(reinterpret_cast<const uint4 *>(a.w + static_cast<size_t>(e0 + es) * a.hidden +
                                                                1024 * part) +
                                lane + 32 * j)
                        : make_uint4(0u, 0u, 0u, 0u);
  };
  __shared__ __align__(8) uint64_t x_full;
  const uint32_t xbar = static_cast<uint32_t>(__cvta_generic_to_shared(&x_full));
  if (threadIdx.x == 0) {
    mbar_init(xbar, 1);
    fence_barrier_init();
  }
  uint4 wv[4][4];
  load_w(warp, wv);
  __syncthreads();
  pdl_wait();
  if (threadIdx.x == 0) {
    // rows of H bf16 (a multiple of 1024 elements) from 16-byte aligned x
    const uint32_t row_bytes = static_cast<uint32_t>(a.hidden) * 2u;
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(xs));
    const uint64_t keep = policy_evict_last();  // every expert tile's CTA reads these rows
    mbar_expect_tx(xbar, static_cast<uint32_t>(nt) * row_bytes);
    for (int t = 0; t < nt; ++t)
      bulk_load(sbase + static_cast<uint32_t>(t) * row_bytes, a.x + static_cast<size_t>(t0 + t) * a.hidden,
                row_bytes, xbar, keep);
  }
  {
    // bounded wait (the copies read caller-checked memory; the bound only
    // guarantees that the launch ends): on expiry the layer's error word says
    // so and no logits are written
    bool landed = false;
#pragma unroll 1
    for (int i = 0; i < 256 && !landed; ++i) landed = mbar_try_wait(xbar, 0);
    if (!landed) {
      const uint64_t w0 = globaltimer();
#pragma unroll 1
      while (!(landed = mbar_try_wait(xbar, 0)) && globaltimer() - w0 < kWaitBudgetNs) {
      }
    }
    if (__syncthreads_or(landed ? 0 : 1)) {
      if (threadIdx.x == 0 && a.err != nullptr) error_raise(a.err, kErrTimeoutFull);
      return;
    }
  }
#pragma unroll 1
  for (int part = warp; part < parts; part += 8) {
    if (part != warp) load_w(part, wv);
    // per lane: 4 experts x 8 tokens chains, each in the element order above;
    // rows t >= nt (a tile of fewer tokens: decode) run no chain and are never
    // stored
    const uint4 *xr = reinterpret_cast<const uint4 *>(xs + 1024 * part);
    const int row_u4 = a.hidden >> 3;
    float v[32];  // v[8 es + t]
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        if (t >= nt) break;
        const uint4 xv = xr[t * row_u4 + lane + 32 * j];
        const uint32_t xq[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int es = 0; es < 4; ++es) {
          const uint32_t wq[4] = {wv[es][j].x, wv[es][j].y, wv[es][j].z, wv[es][j].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            v[8 * es + t] = __fmaf_rn(__uint_as_float(xq[q] << 16), __uint_as_float(wq[q] << 16), v[8 * es + t]);
            v[8 * es + t] =
                __fmaf_rn(__uint_as_float(xq[q] & 0xffff0000u), __uint_as_float(wq[q] & 0xffff0000u), v[8 * es + t]);
          }
        }
      }
    }
    // reduce-scatter: at offset o a lane keeps the half of its current window
    // selected by its lane bit o and adds its partner's copy of that half
#pragma unroll
    for (int lvl = 0; lvl < 5; ++lvl) {
      const int off = 16 >> lvl;
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < off; ++i) {
        const float send = upper ? v[i] : v[i + off];
        const float keep = upper ? v[i + off] : v[i];
        v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, off));
      }
    }
    const int es = lane >> 3, t = lane & 7;
    if (t < nt && e0 + es < a.experts) part_val[(es * kMaxRouterParts + part) * 8 + t] = v[0];
  }
  __syncthreads();
  if (static_cast<int>(threadIdx.x) < 4 * nt) {
    const int es2 = threadIdx.x / nt, tt = threadIdx.x - es2 * nt;
    const int e2 = blockIdx.x * 4 + es2;
    if (e2 < a.experts) {
      float sum = part_val[(es2 * kMaxRouterParts) * 8 + tt];
      for (int p2 = 1; p2 < parts; ++p2) sum = __fadd_rn(sum, part_val[(es2 * kMaxRouterParts + p2) * 8 + tt]);
      a.logits[static_cast<size_t>(t0 + tt) * a.experts + e2] = sum;
    }
  }
}

// ============================================================================
// K1a numerics: sigmoid / softmax / sqrt(softplus) scores as fixed sequences of
// IEEE fp32 operations (mm_numerics.cuh; the CPU oracle replays them), keys by
// routing_key (NaN ranks last), and the weight rules: softmax over the top-k
// logits, score / sum (or sum + eps, or the guarded sum) times the routed
// scale, or GLM-5.3's bf16(scale * s / (sum + eps)).
// ============================================================================
struct IeeeRouting {
  static __device__ __forceinline__ float score(const GateArgs &g, float l) {
    if (g.score_func == MM_SCORE_SIGMOID) return det_sigmoid(l);
    if (g.score_func == MM_SCORE_SQRTSOFTPLUS) return det_sqrtsoftplus(l);
    return l;  // softmax: rank the (biased) logits
  }
  static __device__ __forceinline__ uint32_t key(float s, float b) { return routing_key(__fadd_rn(s, b)); }
  // the weight of selected slot k; the row's sum is evaluated the same way, in
  // the same order, by every lane that calls this
  static __device__ __forceinline__ float weight(const GateArgs &g, const GateSmem &sm, int k) {
    const int K = g.top_k;
    if (g.score_func == MM_SCORE_SOFTMAX) {
      float m = sm.logit[sm.sel[0]];
      for (int i = 1; i < K; ++i) m = fmaxf(m, sm.logit[sm.sel[i]]);
      float sum = 0.0f, mine = 0.0f;
      for (int i = 0; i < K; ++i) {
        const float e = det_exp(__fsub_rn(sm.logit[sm.sel[i]], m));
        sum = __fadd_rn(sum, e);
        if (i == k) mine = e;
      }
      return __fmul_rn(__fdiv_rn(mine, sum), g.routed_scaling);
    }
    const float mine = sm.score[sm.sel[k]];
    if (g.renormalize == MM_RENORM_SCALED_BF16) {
      // GLM-5.3's rule (glm5_3/sm103/moe/routing.py:3-11, ptx_tc.py routing_weight):
      // the selected scores summed in the order of a warp xor-butterfly whose
      // lane k holds slot k (the halving [i] += [i + off], off = 8, 4, 2, 1, is
      // lane 0's order), then w = bf16(scale * s / (sum + eps)), scale first;
      // IEEE division where the reference divides approximately
      float t[kMaxTopK];
#pragma unroll
      for (int i = 0; i < kMaxTopK; ++i) t[i] = i < K ? sm.score[sm.sel[i]] : 0.0f;
#pragma unroll
      for (int off = kMaxTopK / 2; off >= 1; off >>= 1)
#pragma unroll
        for (int i = 0; i < off; ++i) t[i] = __fadd_rn(t[i], t[i + off]);
      const float d = __fadd_rn(t[0], g.renorm_eps);
      return bf16_bits_to_float(float_to_bf16_bits(__fdiv_rn(__fmul_rn(g.routed_scaling, mine), d)));
    }
    if (g.renormalize) {
      float sum = 0.0f;
      for (int i = 0; i < K; ++i) sum = __fadd_rn(sum, sm.score[sm.sel[i]]);
      const float norm = g.renorm_eps > 0.0f ? __fadd_rn(sum, g.renorm_eps) : (sum > 0.0f ? sum : 1.0f);
      return __fmul_rn(__fdiv_rn(mine, norm), g.routed_scaling);
    }
    return __fmul_rn(mine, g.routed_scaling);
  }
};

__global__ void __launch_bounds__(512) gate_topk_kernel(GateArgs g) {
  pdl_launch_dependents();
  __shared__ GateSmem sm;
  pdl_wait();
  const int valid = g.num_valid != nullptr ? *g.num_valid : static_cast<int>(gridDim.x);
  gate_row<IeeeRouting>(g, blockIdx.x, valid, sm);
}

__global__ void __launch_bounds__(512) route_kernel(RouteArgs r) {
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char route_smem[];
  pdl_wait();
  build_route(r, route_smem);
}

// ============================================================================
// The front kernel: grid = T row CTAs + the routed input's quantization CTAs,
// block 512 (front_body in mm_gate.cuh).
// ============================================================================
__global__ void __launch_bounds__(512) front_kernel(FrontArgs f) {
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char front_smem[];
  front_body<IeeeRouting, true>(f, front_smem);
}


// ============================================================================
// Router top-k + route record in one launch that allocates nothing.
//
// For callers that cannot call cudaMalloc: a serving runtime that reserves the
// GPU's memory for its own caching pool at start-up, or plugin code that is
// handed only its input and output pointers and has no allocator. The
// fused launch (one CTA per row, the last CTA builds the record) needs scratch
// that outlives a CTA (the last-CTA ticket and the top-k ids of every row);
// mm_layer_create provides it with cudaMalloc, this variant keeps it in the
// file-scope array below instead: 8.25 KB of static device memory that every
// GPU which loads libmegamoe holds until the process exits.
//   words [0, kNoAllocIdsWord): the ticket (word 0; zero between launches)
//   words [kNoAllocIdsWord, + kNoAllocMaxSlots): the staged top-k ids
// ============================================================================
constexpr int kNoAllocMaxSlots = 2048;  // tokens * top_k
constexpr int kNoAllocIdsWord = 64;
constexpr int kNoAllocWords = kNoAllocIdsWord + kNoAllocMaxSlots;
static __device__ __align__(256) int g_noalloc_scratch[kNoAllocWords];

__global__ void __launch_bounds__(512) gate_route_noalloc_kernel(GateArgs g, RouteArgs r, int *scratch,
                                                                  int *ids_out) {
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char na_smem[];
  __shared__ GateSmem gsm;
  __shared__ int is_last;
  pdl_wait();  // the previous launch on this stream (same scratch) has completed
  const int valid = g.num_valid != nullptr ? *g.num_valid : r.tokens;
  gate_row<IeeeRouting>(g, blockIdx.x, valid, gsm);  // g.ids_out points into the scratch
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(&scratch[0], 1);
    is_last = ticket == static_cast<int>(gridDim.x) - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  build_route(r, na_smem);
  if (ids_out != nullptr) {
    const int slots = r.tokens * r.top_k;
    for (int i = threadIdx.x; i < slots; i += blockDim.x) ids_out[i] = __ldcg(r.ids + i);
  }
  __syncthreads();
  if (threadIdx.x == 0) scratch[0] = 0;  // re-arm the ticket for the next launch
}

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
int *g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Once per device, with that device current: the device address of the scratch
// array (in host code its name is only a stand-in) and the kernel's shared-memory
// limit raised. Runs on the first call on a device. The ticket needs no clearing
// here: a static device array is zero when the module loads, and every launch
// re-arms the ticket before it ends (a memset here would also be unordered with
// a launch on a non-blocking stream).
int noalloc_setup(int device, int **out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[device] == nullptr) {
    int *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void **>(&ptr), g_noalloc_scratch);
    if (e != cudaSuccess)
      return set_error(MM_ERR_CUDA, "mm_gate_route_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    e = cudaFuncSetAttribute(gate_route_noalloc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(route_smem_size(kMaxTokens, kMaxRouterExperts)));
    if (e != cudaSuccess)
      return set_error(MM_ERR_CUDA, "mm_gate_route_noalloc: set-up failed: %s", cudaGetErrorString(e));
    g_noalloc_ptr[device] = ptr;
  }
  *out = g_noalloc_ptr[device];
  return MM_OK;
}
}  // namespace

}  // namespace mm

extern "C" int mm_gate_route_noalloc(const mm_gate_args *gate, int32_t tokens, int32_t router_experts,
                                     int32_t top_k, int32_t experts, int32_t expert_offset, int32_t *permuted,
                                     int32_t *record, void *stream) {
  using namespace mm;
  if (!gate || !gate->logits || !gate->weights || !permuted || !record)
    return set_error(MM_ERR_INVALID, "mm_gate_route_noalloc: null pointer");
  if (tokens < 1 || tokens > kMaxTokens || router_experts < 1 || router_experts > kMaxRouterExperts ||
      top_k < 1 || top_k > kMaxTopK || top_k > router_experts)
    return set_error(MM_ERR_INVALID, "mm_gate_route_noalloc: tokens %d, router_experts %d, top_k %d out of range",
                     tokens, router_experts, top_k);
  if (tokens * top_k > kNoAllocMaxSlots)
    return set_error(MM_ERR_INVALID,
                     "mm_gate_route_noalloc: tokens * top_k = %d exceeds the static scratch (%d slots)",
                     tokens * top_k, kNoAllocMaxSlots);
  if (experts < 1 || experts > kMaxRouterExperts || expert_offset < 0 || expert_offset + experts > router_experts)
    return set_error(MM_ERR_INVALID, "mm_gate_route_noalloc: local experts [%d, %d) outside the router's %d",
                     expert_offset, expert_offset + experts, router_experts);
  if (gate->score_func != MM_SCORE_SIGMOID && gate->score_func != MM_SCORE_SOFTMAX &&
      gate->score_func != MM_SCORE_SQRTSOFTPLUS)
    return set_error(MM_ERR_UNSUPPORTED, "mm_gate_route_noalloc: score function %d is not built", gate->score_func);
  if (gate->renormalize < 0 || gate->renormalize > MM_RENORM_SCALED_BF16 ||
      (gate->renormalize == MM_RENORM_SCALED_BF16 && gate->score_func == MM_SCORE_SOFTMAX))
    return set_error(MM_ERR_INVALID, "mm_gate_route_noalloc: renormalize %d with score function %d",
                     gate->renormalize, gate->score_func);
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess || device < 0 || device >= kNoAllocMaxDevices)
    return set_error(MM_ERR_CUDA, "mm_gate_route_noalloc: no usable current device");
  int *scratch = nullptr;
  int rc = noalloc_setup(device, &scratch);
  if (rc) return rc;
  GateArgs g;
  g.logits = gate->logits;
  g.bias = gate->bias;
  g.num_valid = gate->num_valid;
  g.score_func = gate->score_func;
  g.renormalize = gate->renormalize;
  g.routed_scaling = gate->routed_scaling;
  g.renorm_eps = gate->renorm_eps;
  g.router_experts = router_experts;
  g.top_k = top_k;
  g.weights_out = gate->weights;
  g.ids_out = scratch + kNoAllocIdsWord;
  g.bias_alt = gate->bias_alt;
  g.input_ids = gate->input_ids;
  g.input_ids64 = gate->input_ids64;
  g.alt_token_id = gate->alt_token_id;
  RouteArgs r = {};
  r.ids = scratch + kNoAllocIdsWord;
  r.permuted = permuted;
  r.record = record;
  r.tokens = tokens;
  r.top_k = top_k;
  r.experts = experts;
  r.expert_offset = expert_offset;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tokens);
  cfg.blockDim = dim3(512);
  cfg.dynamicSmemBytes = route_smem_size(tokens, experts);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, gate_route_noalloc_kernel, g, r, scratch, gate->ids);
  if (e != cudaSuccess)
    return set_error(MM_ERR_CUDA, "mm_gate_route_noalloc: launch failed: %s", cudaGetErrorString(e));
  return MM_OK;
}
