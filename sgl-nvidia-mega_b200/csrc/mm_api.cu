// The C ABI of libmegamoe (include/megamoe.h): validation, layer creation
// (scale repack, TMA tensor maps, scratch), and the programmatic-dependent-launch
// chains of the routed-MoE step. Nothing here allocates after mm_layer_create.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <string>

#include <cuda.h>
#include <cuda_runtime.h>

#include "megamoe.h"
#include "mm_kernels.cuh"
#include "mm_layout.cuh"
#include "mm_ptx.cuh"

using namespace mm;

namespace {

thread_local std::string g_error;

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

#define MM_CUDA(call)                                                                      \
  do {                                                                                     \
    cudaError_t e_ = (call);                                                               \
    if (e_ != cudaSuccess)                                                                 \
      return fail(MM_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, \
                  __LINE__);                                                               \
  } while (0)

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode(EncodeTiledFn *fn) {
  static EncodeTiledFn cached = nullptr;
  if (cached == nullptr) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    MM_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (p == nullptr || q != cudaDriverEntryPointSuccess)
      return fail(MM_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cached = reinterpret_cast<EncodeTiledFn>(p);
  }
  *fn = cached;
  return MM_OK;
}

// 3-D map of packed E2M1 codes [n][rows][k/2] u8 as bytes {k/2, rows, n}, box
// {128 bytes (256 codes), box_rows, 1}, 128-byte swizzle: one box lands a
// K = 256 slice of box_rows weight rows as the K-major layout tcgen05 reads.
int encode_fp4_map(CUtensorMap *map, const void *base, int k, int rows, int n, int box_rows) {
  EncodeTiledFn enc;
  int rc = get_encode(&enc);
  if (rc) return rc;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(k) / 2, static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(n)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(k) / 2,
                                 static_cast<cuuint64_t>(k) / 2 * static_cast<cuuint64_t>(rows)};
  const cuuint32_t box[3] = {128u, static_cast<cuuint32_t>(box_rows), 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return MM_OK;
}

}  // namespace

namespace mm {
int set_error(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}
}  // namespace mm

struct mm_layer {
  mm_layer_desc d;
  int H, I, E, R, offset, K, Tmax, terms;
  int m1, m2, ks1, ks2, tg2, u2;
  int max_ctas, rows_cap, shared_row_base, route_words_max, max_segs;
  int has_shared;
  int num_sms;
  int fmt;        // kFmtMx or kFmtNv
  int block;      // elements per weight / activation scale: 32 or 16
  int sf_stage;   // scale-chunk bytes of one pipeline stage (Fmt<fmt>::kSfStageBytes)
  float gs1 = 1.0f, gs2 = 1.0f;  // NVFP4: 1 / input_scale[0], 1 / input_scale[1]
  uint8_t *sfa13 = nullptr, *sfa2 = nullptr, *ssfa13 = nullptr, *ssfa2 = nullptr;
  float *alpha = nullptr;  // NVFP4: [alpha13 E][alpha2 E][shared alpha13][shared alpha2]
  uint8_t *xq = nullptr, *xs = nullptr, *hq = nullptr, *hs = nullptr;
  int4 *segs = nullptr;
  int *ctrl = nullptr, *flags = nullptr;
  int *seg_tok = nullptr;    // [max_segs][kSegRows] segment row -> token
  float *part = nullptr;     // split-K partial sums [grid][kPartFloats]
  int *split_cnt = nullptr;  // split-K arrival counters [2 x grid]
  uint32_t *err = nullptr;
  float *logits = nullptr, *weights = nullptr;
  int *ids = nullptr, *permuted = nullptr, *record = nullptr;
  ExpertArgs ea;
};

extern "C" {

const char *mm_last_error(void) { return g_error.c_str(); }
int mm_version(void) { return 1; }

int64_t mm_route_words(int32_t tokens, int32_t top_k, int32_t experts) {
  if (tokens < 1 || top_k < 1 || experts < 1) return 0;
  return route_words(tokens, top_k, experts);
}

// The router launch's shared memory reaches 8 x H bf16 rows of x: raise the
// kernel's dynamic shared memory limit once per device.
static cudaError_t router_smem_attr() {
  static bool done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) return e;
  if (done[dev]) return cudaSuccess;
  e = cudaFuncSetAttribute(router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(router_smem_bytes(kMaxRouterHidden)));
  if (e == cudaSuccess) done[dev] = true;
  return e;
}

int mm_router_gemv(const uint16_t *x, const uint16_t *w, float *logits, int32_t tokens,
                   int32_t experts, int32_t hidden, void *stream) {
  if (!x || !w || !logits) return fail(MM_ERR_INVALID, "mm_router_gemv: null pointer");
  if (tokens < 1 || experts < 1 || hidden < 1024 || hidden % 1024 || hidden > kMaxRouterHidden)
    return fail(MM_ERR_INVALID, "mm_router_gemv: tokens %d experts %d hidden %d (hidden %% 1024 == 0, <= %d)",
                tokens, experts, hidden, kMaxRouterHidden);
  if (!aligned(x, 16) || !aligned(w, 16)) return fail(MM_ERR_INVALID, "mm_router_gemv: x and w must be 16-byte aligned");
  RouterArgs a = {};
  a.x = x;
  a.w = w;
  a.logits = logits;
  a.tokens = tokens;
  a.experts = experts;
  a.hidden = hidden;
  MM_CUDA(router_smem_attr());
  dim3 grid((experts + 3) / 4, (tokens + 7) / 8);
  MM_CUDA(launch(router_kernel, grid, dim3(256), router_smem_bytes(hidden), stream, a));
  return MM_OK;
}

static int check_gate(const mm_gate_args *a, int tokens, int E, int K) {
  if (!a || !a->logits || !a->weights || !a->ids) return fail(MM_ERR_INVALID, "gate: null pointer");
  if (tokens < 1 || tokens > kMaxTokens) return fail(MM_ERR_INVALID, "gate: tokens %d outside 1..%d", tokens, kMaxTokens);
  if (E < 1 || E > kMaxRouterExperts) return fail(MM_ERR_INVALID, "gate: %d experts outside 1..%d", E, kMaxRouterExperts);
  if (K < 1 || K > kMaxTopK || K > E) return fail(MM_ERR_INVALID, "gate: top_k %d outside 1..min(16, experts)", K);
  if (a->score_func != MM_SCORE_SIGMOID && a->score_func != MM_SCORE_SOFTMAX &&
      a->score_func != MM_SCORE_SQRTSOFTPLUS && a->score_func != MM_SCORE_SQRTSOFTPLUS_DSV41)
    return fail(MM_ERR_UNSUPPORTED,
                "gate: score function %d is not built (sigmoid, softmax, sqrtsoftplus, sqrtsoftplus_dsv41)",
                a->score_func);
  if (a->score_func == MM_SCORE_SQRTSOFTPLUS_DSV41 &&
      ((K != 3 && K != 6) || a->renormalize != MM_RENORM_SUM))
    return fail(MM_ERR_UNSUPPORTED,
                "gate: the DeepSeek-V4.1 gate numerics serve top-3 or top-6 with the sum rule (top_k %d, "
                "renormalize %d)", K, a->renormalize);
  if (a->renormalize < 0 || a->renormalize > MM_RENORM_SCALED_BF16)
    return fail(MM_ERR_INVALID, "gate: renormalize %d (0, 1 or MM_RENORM_SCALED_BF16)", a->renormalize);
  if (a->renormalize == MM_RENORM_SCALED_BF16 && a->score_func == MM_SCORE_SOFTMAX)
    return fail(MM_ERR_UNSUPPORTED, "gate: the scaled-bf16 rule takes sigmoid or sqrtsoftplus scores");
  return MM_OK;
}

static GateArgs gate_args(const mm_gate_args *a, int E, int K) {
  GateArgs g;
  g.logits = a->logits;
  g.bias = a->bias;
  g.num_valid = a->num_valid;
  g.score_func = a->score_func;
  g.renormalize = a->renormalize;
  g.routed_scaling = a->routed_scaling;
  g.renorm_eps = a->renorm_eps;
  g.router_experts = E;
  g.top_k = K;
  g.weights_out = a->weights;
  g.ids_out = a->ids;
  g.bias_alt = a->bias_alt;
  g.input_ids = a->input_ids;
  g.input_ids64 = a->input_ids64;
  g.alt_token_id = a->alt_token_id;
  return g;
}

int mm_gate_topk(const mm_gate_args *args, int32_t tokens, int32_t router_experts, int32_t top_k,
                 void *stream) {
  int rc = check_gate(args, tokens, router_experts, top_k);
  if (rc) return rc;
  MM_CUDA(launch(args->score_func == MM_SCORE_SQRTSOFTPLUS_DSV41 ? gate_topk_dsv41_kernel : gate_topk_kernel,
                 dim3(tokens), dim3(512), 0, stream, gate_args(args, router_experts, top_k)));
  return MM_OK;
}

static size_t route_smem_bytes(int tokens, int experts) {
  const int words = (tokens + 31) / 32;
  return static_cast<size_t>(experts) * words * 4 + static_cast<size_t>(experts) * 4 * 3 + 32 * 4;
}

int mm_route(const int32_t *ids, int32_t *permuted, int32_t *record, int32_t tokens, int32_t top_k,
             int32_t experts, int32_t expert_offset, void *stream) {
  if (!ids || !permuted || !record) return fail(MM_ERR_INVALID, "mm_route: null pointer");
  if (tokens < 1 || tokens > kMaxTokens) return fail(MM_ERR_INVALID, "mm_route: tokens %d outside 1..%d", tokens, kMaxTokens);
  if (top_k < 1 || top_k > kMaxTopK) return fail(MM_ERR_INVALID, "mm_route: top_k %d outside 1..%d", top_k, kMaxTopK);
  if (experts < 1 || experts > kMaxRouterExperts) return fail(MM_ERR_INVALID, "mm_route: %d experts outside 1..%d", experts, kMaxRouterExperts);
  if (expert_offset < -2)
    return fail(MM_ERR_INVALID, "mm_route: expert_offset %d (balanced dealing: -1 or -2)", expert_offset);
  RouteArgs r = {};
  r.ids = ids;
  r.permuted = permuted;
  r.record = record;
  r.tokens = tokens;
  r.top_k = top_k;
  r.experts = experts;
  r.expert_offset = expert_offset;
  const size_t smem = route_smem_bytes(tokens, experts);
  MM_CUDA(cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  MM_CUDA(launch(route_kernel, dim3(1), dim3(512), smem, stream, r));
  return MM_OK;
}

int mm_finalize(const uint16_t *rows, const float *weights, const int32_t *permuted,
                const uint16_t *shared_rows, uint16_t *out, float *partial, int32_t tokens,
                int32_t top_k, int32_t hidden, void *stream) {
  if (!rows || !weights || !permuted || (!out && !partial)) return fail(MM_ERR_INVALID, "mm_finalize: null pointer");
  if (tokens < 1 || top_k < 1 || hidden < 8 || hidden % 8) return fail(MM_ERR_INVALID, "mm_finalize: bad sizes");
  if (!aligned(rows, 16) || (shared_rows && !aligned(shared_rows, 16)) || (out && !aligned(out, 16)) ||
      (partial && !aligned(partial, 16)))
    return fail(MM_ERR_INVALID, "mm_finalize: buffers must be 16-byte aligned");
  FinalizeArgs a = {rows, weights, permuted, shared_rows, out, partial, tokens, top_k, hidden};
  dim3 grid(tokens, (hidden + 2047) / 2048);
  MM_CUDA(launch(finalize_kernel, grid, dim3(256), 0, stream, a));
  return MM_OK;
}

int mm_finalize_partial(const float *partial, uint16_t *out, int32_t tokens, int32_t hidden, void *stream) {
  if (!partial || !out || tokens < 1 || hidden < 1) return fail(MM_ERR_INVALID, "mm_finalize_partial: bad arguments");
  const size_t n = static_cast<size_t>(tokens) * hidden;
  const int blocks = static_cast<int>((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
  MM_CUDA(launch(finalize_partial_kernel, dim3(blocks), dim3(256), 0, stream, partial, out, tokens, hidden));
  return MM_OK;
}

// ---------------------------------------------------------------------------
static void free_layer(mm_layer *L) {
  if (!L) return;
  void *ptrs[] = {L->sfa13, L->sfa2, L->ssfa13, L->ssfa2, L->xq, L->xs, L->hq, L->hs, L->segs,
                  L->ctrl, L->flags, L->seg_tok, L->part, L->split_cnt, L->err, L->logits, L->weights, L->ids,
                  L->permuted, L->record, L->alpha};
  for (void *p : ptrs)
    if (p) cudaFree(p);
  delete L;
}

static int check_weights(const mm_expert_weights &w, const char *what, bool nv) {
  if (!w.w13 || !w.w13_scale || !w.w2 || !w.w2_scale) return fail(MM_ERR_INVALID, "%s: null weight pointer", what);
  if (nv && (!w.w13_scale_2 || !w.w2_scale_2))
    return fail(MM_ERR_INVALID, "%s: NVFP4 weights need w13_scale_2 and w2_scale_2", what);
  if (!aligned(w.w13, 16) || !aligned(w.w2, 16))
    return fail(MM_ERR_INVALID, "%s: packed weights must be 16-byte aligned", what);
  return MM_OK;
}

int mm_layer_create(const mm_layer_desc *desc, mm_layer **out) {
  if (!desc || !out) return fail(MM_ERR_INVALID, "mm_layer_create: null pointer");
  *out = nullptr;
  const mm_layer_desc &d = *desc;
  if (d.hidden < 256 || d.hidden % 256) return fail(MM_ERR_INVALID, "hidden %d must be a positive multiple of 256", d.hidden);
  if (d.intermediate < 64 || d.intermediate % 64)
    return fail(MM_ERR_INVALID, "intermediate %d must be a positive multiple of 64", d.intermediate);
  if (d.experts < 1 || d.experts > kMaxRouterExperts) return fail(MM_ERR_INVALID, "experts %d outside 1..%d", d.experts, kMaxRouterExperts);
  if (d.router_experts < d.experts || d.router_experts > kMaxRouterExperts)
    return fail(MM_ERR_INVALID, "router_experts %d outside experts..%d", d.router_experts, kMaxRouterExperts);
  if (d.expert_offset < 0) {  // balanced dealing: the rank holds every expert
    if (d.expert_offset < -2 || d.experts != d.router_experts)
      return fail(MM_ERR_INVALID, "balanced dealing (expert_offset %d) needs group -1 or -2 and all %d experts",
                  d.expert_offset, d.router_experts);
  } else if (d.expert_offset + d.experts > d.router_experts) {
    return fail(MM_ERR_INVALID, "local experts [%d, %d) outside the router's %d", d.expert_offset,
                d.expert_offset + d.experts, d.router_experts);
  }
  if (d.top_k < 1 || d.top_k > kMaxTopK) return fail(MM_ERR_INVALID, "top_k %d outside 1..%d", d.top_k, kMaxTopK);
  if (d.max_tokens < 1 || d.max_tokens > kMaxTokens) return fail(MM_ERR_INVALID, "max_tokens %d outside 1..%d", d.max_tokens, kMaxTokens);
  if (d.weight_format != MM_WEIGHT_MXFP4 && d.weight_format != MM_WEIGHT_NVFP4)
    return fail(MM_ERR_UNSUPPORTED, "weight format %d is not built (MXFP4, NVFP4)", d.weight_format);
  const bool nv = d.weight_format == MM_WEIGHT_NVFP4;
  if (nv && !(d.input_scale[0] > 0.0f && d.input_scale[1] > 0.0f && d.input_scale[0] < INFINITY &&
              d.input_scale[1] < INFINITY))
    return fail(MM_ERR_INVALID, "NVFP4 input scales must be positive and finite (%g, %g)", d.input_scale[0],
                d.input_scale[1]);
  if (d.act_terms < 1 || d.act_terms > kMaxTerms)
    return fail(MM_ERR_INVALID, "act_terms %d outside 1..%d", d.act_terms, kMaxTerms);
  int rc = check_weights(d.routed, "routed", nv);
  if (rc) return rc;
  const int has_shared = d.shared.w13 != nullptr;
  if (has_shared && (rc = check_weights(d.shared, "shared", nv))) return rc;

  MM_CUDA(cudaSetDevice(d.device));
  mm_layer *L = new mm_layer();
  L->d = d;
  L->H = d.hidden;
  L->I = d.intermediate;
  L->E = d.experts;
  L->R = d.router_experts;
  L->offset = d.expert_offset;
  L->K = d.top_k;
  L->Tmax = d.max_tokens;
  L->terms = d.act_terms;
  L->has_shared = has_shared;
  L->fmt = nv ? kFmtNv : kFmtMx;
  L->block = nv ? 16 : 32;
  L->sf_stage = nv ? Fmt<kFmtNv>::kSfStageBytes : Fmt<kFmtMx>::kSfStageBytes;
  if (nv) {
    L->gs1 = 1.0f / d.input_scale[0];
    L->gs2 = 1.0f / d.input_scale[1];
  }
  L->m1 = L->I / 64;
  L->m2 = L->H / 128;
  L->ks1 = L->H / kStageK;
  L->ks2 = (L->I + kStageK - 1) / kStageK;  // the down GEMM's last stage may be partial
  // short down units (one to three K stages: narrow tensor-parallel slices, DSV4.1's
  // 576-wide slice) take two 128-row tiles each, so one accumulator hand-off serves
  // two tiles; MXFP4 only (NVFP4's scale columns leave TMEM room for one tile per
  // accumulator)
  L->tg2 = (!nv && L->ks2 <= 3) ? 2 : 1;
  static_assert(Fmt<kFmtMx>::kAccCols == 2 * kBRows && Fmt<kFmtNv>::kAccCols == kBRows,
                "two-tile down units need MXFP4's double-width accumulator buffers");
  L->u2 = (L->m2 + L->tg2 - 1) / L->tg2;
  L->max_ctas = route_max_ctas(L->Tmax, L->K, L->E);
  L->shared_row_base = kTile * L->max_ctas;
  L->rows_cap = L->shared_row_base + L->Tmax;
  L->route_words_max = route_words(L->Tmax, L->K, L->E);
  L->max_segs = L->max_ctas + (L->Tmax + kSegRows - 1) / kSegRows + 1;
  int dev_sms = 0;
  cudaError_t ce = cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, d.device);
  if (ce != cudaSuccess) {
    free_layer(L);
    return fail(MM_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(ce));
  }
  L->num_sms = dev_sms;

#define ALLOC(ptr, bytes)                                                                \
  do {                                                                                   \
    cudaError_t e_ = cudaMalloc(reinterpret_cast<void **>(&(ptr)), (bytes));             \
    if (e_ != cudaSuccess) {                                                             \
      free_layer(L);                                                                     \
      return fail(MM_ERR_CUDA, "cudaMalloc(%zu): %s", static_cast<size_t>(bytes), cudaGetErrorString(e_)); \
    }                                                                                    \
  } while (0)

  const size_t E = L->E, H = L->H;
  const size_t sfs = static_cast<size_t>(L->sf_stage);
  const size_t sfa13_bytes = E * L->m1 * L->ks1 * sfs;
  const size_t sfa2_bytes = E * L->m2 * L->ks2 * sfs;
  ALLOC(L->sfa13, sfa13_bytes);
  ALLOC(L->sfa2, sfa2_bytes);
  if (has_shared) {
    ALLOC(L->ssfa13, static_cast<size_t>(L->m1) * L->ks1 * sfs);
    ALLOC(L->ssfa2, static_cast<size_t>(L->m2) * L->ks2 * sfs);
  }
  if (nv) ALLOC(L->alpha, sizeof(float) * (2 * E + 2));
  const size_t xq_bytes = kMaxTerms * static_cast<size_t>(L->Tmax) * H / 2;
  // h rows are padded to whole K stages (256 features): the pad is zeroed here and never
  // written, so the down GEMM's partial last stage (I % 256 != 0) reads zero codes and
  // scales and its loader needs no K bound
  const int hq_row = L->ks2 * (kStageK / 2);
  const int hs_row = L->ks2 * (kStageK / L->block);
  const size_t hq_bytes = kMaxTerms * static_cast<size_t>(L->rows_cap) * hq_row;
  const size_t xs_bytes = xq_bytes * 2 / L->block;
  const size_t hs_bytes = kMaxTerms * static_cast<size_t>(L->rows_cap) * hs_row;
  ALLOC(L->xq, xq_bytes);
  ALLOC(L->xs, xs_bytes);
  ALLOC(L->hq, hq_bytes);
  ALLOC(L->hs, hs_bytes);
  ALLOC(L->segs, sizeof(int4) * L->max_segs);
  ALLOC(L->ctrl, sizeof(int) * kCtrlWords);
  ALLOC(L->flags, sizeof(int) * L->max_segs);
  ALLOC(L->seg_tok, sizeof(int) * kSegRows * L->max_segs);
  const size_t grid = static_cast<size_t>(kCtasPerSm) * L->num_sms;
  ALLOC(L->part, sizeof(float) * kPartFloats * grid);
  ALLOC(L->split_cnt, sizeof(int) * 2 * grid);
  ALLOC(L->err, sizeof(uint32_t));
  ALLOC(L->logits, sizeof(float) * L->Tmax * L->R);
  ALLOC(L->weights, sizeof(float) * L->Tmax * L->K);
  ALLOC(L->ids, sizeof(int) * L->Tmax * L->K);
  ALLOC(L->permuted, sizeof(int) * L->Tmax * L->K);
  ALLOC(L->record, sizeof(int) * L->route_words_max);
#undef ALLOC
  ce = cudaMemset(L->ctrl, 0, sizeof(int) * kCtrlWords);
  if (ce == cudaSuccess) ce = cudaMemset(L->split_cnt, 0, sizeof(int) * 2 * grid);
  if (ce == cudaSuccess) ce = cudaMemset(L->err, 0, sizeof(uint32_t));
  if (ce == cudaSuccess) ce = cudaMemset(L->hq, 0, hq_bytes);
  if (ce == cudaSuccess) ce = cudaMemset(L->hs, 0, hs_bytes);
  if (ce == cudaSuccess) ce = cudaMemset(L->xq, 0, xq_bytes);
  if (ce == cudaSuccess) ce = cudaMemset(L->xs, 0, xs_bytes);
  if (ce != cudaSuccess) {
    free_layer(L);
    return fail(MM_ERR_CUDA, "cudaMemset: %s", cudaGetErrorString(ce));
  }

  // scale repack (once): canonical scales -> UMMA scale chunks
  auto repack = [&](const void *src, uint8_t *dst, int n, int rows, int k, int gate_up) -> int {
    const size_t total = static_cast<size_t>(n) * (rows / 128) * ((k + kStageK - 1) / kStageK) * sfs;
    const int blocks = static_cast<int>(total / 256 < 65536 ? (total + 255) / 256 : 65536);
    repack_scales_kernel<<<blocks, 256>>>(static_cast<const uint8_t *>(src), dst, n, rows, k, gate_up, L->I,
                                          L->block);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MM_ERR_CUDA, "repack_scales_kernel: %s", cudaGetErrorString(e));
    return MM_OK;
  };
  if ((rc = repack(d.routed.w13_scale, L->sfa13, L->E, 2 * L->I, L->H, 1)) ||
      (rc = repack(d.routed.w2_scale, L->sfa2, L->E, L->H, L->I, 0)) ||
      (has_shared && (rc = repack(d.shared.w13_scale, L->ssfa13, 1, 2 * L->I, L->H, 1))) ||
      (has_shared && (rc = repack(d.shared.w2_scale, L->ssfa2, 1, L->H, L->I, 0)))) {
    free_layer(L);
    return rc;
  }
  if (nv) {  // accumulator multipliers: scale_2 x the GEMM's input scale
    const int eb = (L->E + 255) / 256;
    nv_alpha_kernel<<<eb, 256>>>(d.routed.w13_scale_2, d.input_scale[0], L->alpha, L->E);
    nv_alpha_kernel<<<eb, 256>>>(d.routed.w2_scale_2, d.input_scale[1], L->alpha + L->E, L->E);
    if (has_shared) {
      nv_alpha_kernel<<<1, 32>>>(d.shared.w13_scale_2, d.input_scale[0], L->alpha + 2 * L->E, 1);
      nv_alpha_kernel<<<1, 32>>>(d.shared.w2_scale_2, d.input_scale[1], L->alpha + 2 * L->E + 1, 1);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      free_layer(L);
      return fail(MM_ERR_CUDA, "nv_alpha_kernel: %s", cudaGetErrorString(e));
    }
  }
  ce = cudaDeviceSynchronize();
  if (ce != cudaSuccess) {
    free_layer(L);
    return fail(MM_ERR_CUDA, "scale repack: %s", cudaGetErrorString(ce));
  }

  ExpertArgs &ea = L->ea;
  memset(&ea, 0, sizeof(ea));
  const mm_expert_weights &sw = has_shared ? d.shared : d.routed;  // placeholder maps when no shared
  if ((rc = encode_fp4_map(&ea.w13_map, d.routed.w13, L->H, 2 * L->I, L->E, 64)) ||
      (rc = encode_fp4_map(&ea.w2_map, d.routed.w2, L->I, L->H, L->E, 128)) ||
      (rc = encode_fp4_map(&ea.sw13_map, sw.w13, L->H, 2 * L->I, 1, 64)) ||
      (rc = encode_fp4_map(&ea.sw2_map, sw.w2, L->I, L->H, 1, 128))) {
    free_layer(L);
    return rc;
  }
  ea.sfa13 = L->sfa13;
  ea.sfa2 = L->sfa2;
  ea.ssfa13 = has_shared ? L->ssfa13 : L->sfa13;
  ea.ssfa2 = has_shared ? L->ssfa2 : L->sfa2;
  ea.xq = L->xq;
  ea.xs = L->xs;
  ea.hq = L->hq;
  ea.hs = L->hs;
  ea.hq_row = hq_row;
  ea.hs_row = hs_row;
  ea.segs = L->segs;
  ea.ctrl = L->ctrl;
  ea.flags = L->flags;
  ea.seg_tok = L->seg_tok;
  ea.part = L->part;
  ea.split_cnt = L->split_cnt;
  ea.err = L->err;
  ea.clamp = d.clamp;
  ea.shared_clamp = d.shared_clamp;
  if (nv) {
    ea.alpha13 = L->alpha;
    ea.alpha2 = L->alpha + L->E;
    ea.salpha13 = has_shared ? L->alpha + 2 * L->E : L->alpha;
    ea.salpha2 = has_shared ? L->alpha + 2 * L->E + 1 : L->alpha + L->E;
    ea.gs2 = L->gs2;
    ea.inv_gs2 = d.input_scale[1];
  }
  ea.hidden = L->H;
  ea.inter = L->I;
  ea.max_tokens = L->Tmax;
  ea.rows_cap = L->rows_cap;
  ea.terms = L->terms;
  ea.m1 = L->m1;
  ea.m2 = L->m2;
  ea.ks1 = L->ks1;
  ea.ks2 = L->ks2;
  ea.tg2 = L->tg2;
  ea.u2 = L->u2;
  ea.wait_ns = kWaitBudgetNs;

  ce = expert_kernel_configure(L->fmt);
  if (ce == cudaSuccess)
    ce = cudaFuncSetAttribute(front_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(route_smem_bytes(kMaxTokens, kMaxRouterExperts)));
  if (ce == cudaSuccess)
    ce = cudaFuncSetAttribute(front_dsv41_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(route_smem_bytes(kMaxTokens, kMaxRouterExperts)));
  if (ce != cudaSuccess) {
    free_layer(L);
    return fail(MM_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(ce));
  }
  *out = L;
  return MM_OK;
}

int mm_layer_destroy(mm_layer *layer) {
  if (!layer) return MM_OK;
  cudaSetDevice(layer->d.device);
  free_layer(layer);
  return MM_OK;
}

int mm_layer_get_info(const mm_layer *L, mm_layer_info *info) {
  if (!L || !info) return fail(MM_ERR_INVALID, "mm_layer_get_info: null pointer");
  info->hidden = L->H;
  info->intermediate = L->I;
  info->experts = L->E;
  info->router_experts = L->R;
  info->expert_offset = L->offset;
  info->top_k = L->K;
  info->max_tokens = L->Tmax;
  info->has_shared = L->has_shared;
  info->rows_capacity = L->rows_cap;
  info->shared_row_base = L->shared_row_base;
  info->route_words = L->route_words_max;
  info->weight_bytes = 3LL * L->H * L->I / 2 + 3LL * L->H * L->I / L->block;
  info->act_terms = L->terms;
  info->h_row_bytes = L->ea.hq_row;
  info->h_scale_row_bytes = L->ea.hs_row;
  return MM_OK;
}

static cudaError_t launch_experts(mm_layer *L, const ExpertArgs &ea, void *stream) {
  return expert_kernel_launch(L->fmt, kCtasPerSm * L->num_sms, ea, stream);
}

// The router GEMV of a layer step: logits = x w^T (fp32).
static int launch_router(mm_layer *L, const uint16_t *x, const uint16_t *w, float *logits, int tokens,
                         void *stream) {
  if (L->H % 1024 || L->H > kMaxRouterHidden)
    return fail(MM_ERR_INVALID, "router GEMV: hidden %d must be a multiple of 1024, <= %d", L->H, kMaxRouterHidden);
  if (!aligned(w, 16) || !aligned(x, 16))
    return fail(MM_ERR_INVALID, "router GEMV: x and the router weight must be 16-byte aligned");
  RouterArgs a = {};
  a.x = x;
  a.w = w;
  a.logits = logits;
  a.tokens = tokens;
  a.experts = L->R;
  a.hidden = L->H;
  a.err = L->err;
  MM_CUDA(router_smem_attr());
  MM_CUDA(launch(router_kernel, dim3((L->R + 3) / 4, (tokens + 7) / 8), dim3(256), router_smem_bytes(L->H), stream, a));
  return MM_OK;
}

// Front (gate or given ids, route, and the routed input's quantization) +
// experts. The routed input is bf16 x, or MXFP8 (x8 codes [T, H], s8 E8M0
// scales [T, H/32]) when x is null.
static int run_front_and_experts(mm_layer *L, const uint16_t *x, const mm_gate_args *gate,
                                 const int32_t *ids, int tokens, int32_t *permuted, int32_t *record,
                                 uint16_t *rows, void *stream, const uint8_t *x8 = nullptr,
                                 const uint8_t *s8 = nullptr) {
  if ((!x && !(x8 && s8)) || !permuted || !record || !rows) return fail(MM_ERR_INVALID, "layer call: null pointer");
  if (tokens < 1 || tokens > L->Tmax) return fail(MM_ERR_INVALID, "tokens %d outside 1..%d", tokens, L->Tmax);
  if ((x && !aligned(x, 16)) || (x8 && !aligned(x8, 16)) || !aligned(rows, 16))
    return fail(MM_ERR_INVALID, "x (or x_quant) and rows must be 16-byte aligned");
  FrontArgs f = {};
  if (gate) {
    int rc = check_gate(gate, tokens, L->R, L->K);
    if (rc) return rc;
    f.gate = gate_args(gate, L->R, L->K);
    f.route.ids = gate->ids;
  } else {
    if (!ids) return fail(MM_ERR_INVALID, "layer call: null ids");
    f.gate.logits = nullptr;
    f.route.ids = ids;
  }
  f.route.permuted = permuted;
  f.route.record = record;
  f.route.tokens = tokens;
  f.route.top_k = L->K;
  f.route.experts = L->E;
  f.route.expert_offset = L->offset;
  f.route.segs = L->segs;
  f.route.ctrl = L->ctrl;
  f.route.flags = L->flags;
  f.route.has_shared = L->has_shared;
  f.route.shared_row_base = L->shared_row_base;
  f.route.m1 = L->m1;
  f.route.m2 = L->u2;
  f.route.ks1 = L->ks1;
  f.route.grid = kCtasPerSm * L->num_sms;
  f.route.split_cnt = L->split_cnt;
  f.route.seg_tok = L->seg_tok;
  // the routed input's FP4 terms: one 32-element chunk per warp and pass, at most
  // two quantization CTAs per SM
  QuantArgs &q = f.quant;
  q.x = x;
  q.x8 = x ? nullptr : x8;
  q.s8 = x ? nullptr : s8;
  q.xq = L->xq;
  q.xs = L->xs;
  q.tokens = tokens;
  q.hidden = L->H;
  q.max_tokens = L->Tmax;
  q.terms = L->terms;
  q.fmt = L->fmt;
  q.gs = L->gs1;
  q.inv_gs = L->fmt == kFmtNv ? L->d.input_scale[0] : 1.0f;
  q.ctas = std::min((tokens * (L->H / 32) + 15) / 16, 2 * L->num_sms);
  f.row_ctas = gate ? tokens : 1;
  MM_CUDA(cudaSetDevice(L->d.device));
  if (gate != nullptr && gate->score_func == MM_SCORE_SQRTSOFTPLUS_DSV41) {
    // the DeepSeek-V4.1 gate's launch is compiled with flush-to-zero: the routed
    // input's quantization runs in a front_kernel launch of its own (no rows) first
    FrontArgs qf = {};
    qf.quant = q;
    qf.row_ctas = 0;
    MM_CUDA(launch(front_kernel, dim3(q.ctas), dim3(512), 0, stream, qf));
    f.quant.ctas = 0;
    MM_CUDA(launch(front_dsv41_kernel, dim3(f.row_ctas), dim3(512), route_smem_bytes(tokens, L->E), stream, f));
  } else {
    MM_CUDA(launch(front_kernel, dim3(f.row_ctas + q.ctas), dim3(512), route_smem_bytes(tokens, L->E), stream, f));
  }
  ExpertArgs ea = L->ea;
  ea.rows_out = rows;
  MM_CUDA(launch_experts(L, ea, stream));
  return MM_OK;
}

int mm_layer_rearm_experts(mm_layer *L, void *stream) {
  if (!L) return fail(MM_ERR_INVALID, "mm_layer_rearm_experts: null layer");
  MM_CUDA(cudaSetDevice(L->d.device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  MM_CUDA(cudaMemsetAsync(L->flags, 0, sizeof(int) * L->max_segs, s));
  MM_CUDA(cudaMemsetAsync(L->ctrl + kCtrlClaim, 0, sizeof(int), s));
  MM_CUDA(cudaMemsetAsync(L->split_cnt, 0, sizeof(int) * 2 * kCtasPerSm * L->num_sms, s));
  return MM_OK;
}

int mm_layer_block_downs(mm_layer *L, void *stream) {
  if (!L) return fail(MM_ERR_INVALID, "mm_layer_block_downs: null layer");
  MM_CUDA(cudaSetDevice(L->d.device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // every mailbox starts near INT_MIN: the gate_up units' increments never bring it
  // to the down units' target, so their bounded waits run out
  MM_CUDA(cudaMemsetAsync(L->flags, 0xc0, sizeof(int) * L->max_segs, s));
  MM_CUDA(cudaMemsetAsync(L->ctrl + kCtrlClaim, 0, sizeof(int), s));
  MM_CUDA(cudaMemsetAsync(L->split_cnt, 0, sizeof(int) * 2 * kCtasPerSm * L->num_sms, s));
  return MM_OK;
}

int mm_layer_set_wait_budget(mm_layer *L, int64_t microseconds) {
  if (!L) return fail(MM_ERR_INVALID, "mm_layer_set_wait_budget: null layer");
  if (microseconds < 1 || microseconds > 60000000)
    return fail(MM_ERR_INVALID, "mm_layer_set_wait_budget: %lld us outside 1..60000000",
                static_cast<long long>(microseconds));
  L->ea.wait_ns = static_cast<unsigned long long>(microseconds) * 1000ull;
  return MM_OK;
}

int mm_layer_rerun_experts(mm_layer *L, int32_t tokens, const int32_t *record, uint16_t *rows, void *stream) {
  if (!L || !record || !rows) return fail(MM_ERR_INVALID, "mm_layer_rerun_experts: null pointer");
  if (tokens < 1 || tokens > L->Tmax) return fail(MM_ERR_INVALID, "tokens %d outside 1..%d", tokens, L->Tmax);
  MM_CUDA(cudaSetDevice(L->d.device));
  ExpertArgs ea = L->ea;
  ea.rows_out = rows;
  MM_CUDA(launch_experts(L, ea, stream));
  return MM_OK;
}

int mm_layer_experts(mm_layer *L, const uint16_t *x, const int32_t *ids, int32_t tokens,
                     int32_t *permuted, int32_t *record, uint16_t *rows, void *stream) {
  if (!L) return fail(MM_ERR_INVALID, "null layer");
  return run_front_and_experts(L, x, nullptr, ids, tokens, permuted, record, rows, stream);
}

int mm_layer_gate_experts(mm_layer *L, const uint16_t *x, const mm_gate_args *gate, int32_t tokens,
                          int32_t *permuted, int32_t *record, uint16_t *rows, void *stream) {
  if (!L || !gate) return fail(MM_ERR_INVALID, "null layer or gate arguments");
  if (!x) return fail(MM_ERR_INVALID, "mm_layer_gate_experts: null x");
  return run_front_and_experts(L, x, gate, nullptr, tokens, permuted, record, rows, stream);
}

int mm_layer_experts_mxfp8(mm_layer *L, const uint8_t *x_quant, const uint8_t *x_scale, const int32_t *ids,
                           int32_t tokens, int32_t *permuted, int32_t *record, uint16_t *rows, void *stream) {
  if (!L) return fail(MM_ERR_INVALID, "null layer");
  if (!x_quant || !x_scale) return fail(MM_ERR_INVALID, "mm_layer_experts_mxfp8: null x_quant or x_scale");
  return run_front_and_experts(L, nullptr, nullptr, ids, tokens, permuted, record, rows, stream, x_quant,
                               x_scale);
}

int mm_layer_gate_experts_mxfp8(mm_layer *L, const uint8_t *x_quant, const uint8_t *x_scale,
                                const mm_gate_args *gate, int32_t tokens, int32_t *permuted, int32_t *record,
                                uint16_t *rows, void *stream) {
  if (!L || !gate) return fail(MM_ERR_INVALID, "null layer or gate arguments");
  if (!x_quant || !x_scale) return fail(MM_ERR_INVALID, "mm_layer_gate_experts_mxfp8: null x_quant or x_scale");
  return run_front_and_experts(L, nullptr, gate, nullptr, tokens, permuted, record, rows, stream, x_quant,
                               x_scale);
}

int64_t mm_layer_scratch_bytes(const mm_layer *L, int32_t which) {
  if (!L) return -1;
  const int64_t terms = kMaxTerms;
  switch (which) {
    case MM_SCRATCH_X_CODES: return terms * L->Tmax * (L->H / 2);
    case MM_SCRATCH_X_SCALES: return terms * L->Tmax * (L->H / L->block);
    case MM_SCRATCH_H_CODES: return terms * L->rows_cap * static_cast<int64_t>(L->ea.hq_row);
    case MM_SCRATCH_H_SCALES: return terms * L->rows_cap * static_cast<int64_t>(L->ea.hs_row);
    default: return -1;
  }
}

int mm_layer_read_scratch(const mm_layer *L, int32_t which, void *dst, int64_t bytes, void *stream) {
  if (!L || !dst) return fail(MM_ERR_INVALID, "mm_layer_read_scratch: null pointer");
  const int64_t size = mm_layer_scratch_bytes(L, which);
  if (size < 0) return fail(MM_ERR_INVALID, "mm_layer_read_scratch: unknown buffer %d", which);
  if (bytes != size)
    return fail(MM_ERR_INVALID, "mm_layer_read_scratch: buffer %d holds %lld bytes, not %lld", which,
                static_cast<long long>(size), static_cast<long long>(bytes));
  const void *src = which == MM_SCRATCH_X_CODES ? static_cast<const void *>(L->xq)
                    : which == MM_SCRATCH_X_SCALES ? static_cast<const void *>(L->xs)
                    : which == MM_SCRATCH_H_CODES ? static_cast<const void *>(L->hq)
                                                  : static_cast<const void *>(L->hs);
  MM_CUDA(cudaSetDevice(L->d.device));
  MM_CUDA(cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDeviceToDevice,
                          static_cast<cudaStream_t>(stream)));
  return MM_OK;
}

int mm_layer_forward(mm_layer *L, const mm_forward_args *a, void *stream) {
  if (!L || !a) return fail(MM_ERR_INVALID, "mm_layer_forward: null pointer");
  const int T = a->tokens;
  if (T < 1 || T > L->Tmax) return fail(MM_ERR_INVALID, "tokens %d outside 1..%d", T, L->Tmax);
  const float *logits = a->logits;
  if (!a->x || !aligned(a->x, 16)) return fail(MM_ERR_INVALID, "mm_layer_forward: x must be a 16-byte aligned pointer");
  MM_CUDA(cudaSetDevice(L->d.device));
  if (a->router_w) {
    float *lo = a->logits_out ? a->logits_out : L->logits;
    int rc = launch_router(L, a->x, a->router_w, lo, T, stream);
    if (rc) return rc;
    logits = lo;
  }
  if (!logits) return fail(MM_ERR_INVALID, "mm_layer_forward: neither router_w nor logits");
  mm_gate_args g = {};
  g.logits = logits;
  g.bias = a->bias;
  g.num_valid = a->num_valid;
  g.score_func = a->score_func;
  g.renormalize = a->renormalize;
  g.routed_scaling = a->routed_scaling;
  g.renorm_eps = a->renorm_eps;
  g.bias_alt = a->bias_alt;
  g.input_ids = a->input_ids;
  g.input_ids64 = a->input_ids64;
  g.alt_token_id = a->alt_token_id;
  g.weights = a->weights ? a->weights : L->weights;
  g.ids = a->ids ? a->ids : L->ids;
  int32_t *perm = a->permuted ? a->permuted : L->permuted;
  int32_t *rec = a->record ? a->record : L->record;
  if (!a->rows) return fail(MM_ERR_INVALID, "mm_layer_forward: null rows buffer");
  int rc = run_front_and_experts(L, a->x, &g, nullptr, T, perm, rec, a->rows, stream);
  if (rc) return rc;
  const uint16_t *shared = L->has_shared ? a->rows + static_cast<size_t>(L->shared_row_base) * L->H : nullptr;
  if (a->residual) {
    if (!a->comm || a->partial) return fail(MM_ERR_INVALID, "mm_layer_forward: residual needs comm and no partial");
    return mm_finalize_allreduce_norm(a->comm, a->rows, g.weights, perm, shared, a->residual, a->gamma, a->norm_eps,
                                      a->residual_out, a->out, T, L->K, L->H, stream);
  }
  if (a->comm) {
    if (!a->out || a->partial) return fail(MM_ERR_INVALID, "mm_layer_forward: comm needs out and no partial");
    return mm_finalize_allreduce(a->comm, a->rows, g.weights, perm, shared, a->out, T, L->K, L->H, stream);
  }
  if (a->out || a->partial) {
    rc = mm_finalize(a->rows, g.weights, perm, shared, a->out, a->partial, T, L->K, L->H, stream);
    if (rc) return rc;
  }
  return MM_OK;
}

int mm_stack_forward(const mm_stack_layer *layers, int32_t n, void *stream) {
  if (!layers || n < 0) return fail(MM_ERR_INVALID, "mm_stack_forward: %d layers", n);
  for (int i = 0; i < n; ++i) {
    const int rc = mm_layer_forward(layers[i].layer, &layers[i].args, stream);
    if (rc) return rc;
  }
  return MM_OK;
}

int mm_layer_check(mm_layer *L) {
  if (!L) return fail(MM_ERR_INVALID, "null layer");
  MM_CUDA(cudaSetDevice(L->d.device));
  MM_CUDA(cudaDeviceSynchronize());
  uint32_t word = 0;
  MM_CUDA(cudaMemcpy(&word, L->err, sizeof(word), cudaMemcpyDeviceToHost));
  if (word == 0) return MM_OK;
  MM_CUDA(cudaMemset(L->err, 0, sizeof(uint32_t)));
  if (word & kErrTimeoutMask) return fail(MM_ERR_DEVICE_TIMEOUT, "device wait timed out (error word 0x%x)", word);
  return fail(MM_ERR_DEVICE, "device check failed (error word 0x%x)", word);
}

}  // extern "C"
