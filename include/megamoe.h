/*
 * megamoe: B200-native (sm_100a) routed-MoE chain behind a C ABI.
 *
 * The chain: router GEMV -> sigmoid/softmax top-k with bias -> token-to-expert
 * permutation (route record) -> MXFP4 block-scaled grouped gate_up GEMM ->
 * SwiGLU + MXFP8 requant -> grouped down GEMM -> slot-order weighted combine.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), returns an int status (MM_OK = 0) and never throws.
 * Nothing here allocates or synchronizes inside a step: scratch is owned by
 * the layer handle and allocated in mm_layer_create. Launches go to the given
 * stream with programmatic dependent launch, so the calls are graph-capturable.
 * The message of the last failure on the calling thread is mm_last_error().
 *
 * Reference interfaces replaced (paths within sgl-project/sgl-nvidia-mega):
 *   mm_router_gemv       sgl_nvidia_mega/deepseek_v41/sm103/moe/src/router_mma.cu:101
 *                        (host: deepseek_v41/sm103/moe/router_mma.py:64-80)
 *   mm_gate_topk         sgl_nvidia_mega/deepseek_v41/sm103/moe/src/gate_topk.cuh:296
 *                        (host: routed_expert_gemm.py:776, launch at :867);
 *                        glm5_3/sm103/moe/routing.py:73 (MoeRouteTop8)
 *   mm_route             deepseek_v41/sm103/moe/src/route.cu:23 and route_wide.cu:62
 *                        (record layout route.cuh:6-46; host routed_expert_gemm.py:916)
 *   mm_route_words       routed_expert_gemm.py:107-120 (max_ctas / cta_words / route_words)
 *   mm_layer_create      RoutedExpertGemm.__init__, routed_expert_gemm.py:537-657
 *   mm_layer_experts     RoutedExpertGemm.__call__, routed_expert_gemm.py:703-774
 *   mm_layer_gate_experts RoutedExpertGemm.gate_topk_and_gemms, routed_expert_gemm.py:776-870
 *   mm_finalize          deepseek_v41/sm103/all_reduce_mhc.py:402-662 (finalize arithmetic);
 *                        glm5_3/sm103/moe/finalize.py:1-27
 *   mm_layer_forward     deepseek_v41/moe/step.py:101 (one MoE step: router -> combine)
 *   mm_comm_*, mm_finalize_allreduce
 *                        deepseek_v41/sm103/all_reduce_mhc.py:402-662 (per-rank publish)
 *                        and :665-1190 (rank-order reduce); AllReduceMHC.finalize :1484
 */
#ifndef MEGAMOE_H
#define MEGAMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define MM_OK 0
#define MM_ERR_INVALID 1        /* bad shape, pointer, alignment or argument   */
#define MM_ERR_UNSUPPORTED 2    /* a valid request this build does not serve  */
#define MM_ERR_CUDA 3           /* a CUDA runtime / driver call failed         */
#define MM_ERR_DEVICE_TIMEOUT 4 /* a bounded device wait gave up (error word)  */
#define MM_ERR_DEVICE 5         /* another device-side check failed            */

/* ---- routing score functions ------------------------------------------- */
#define MM_SCORE_SIGMOID 0      /* s = 1/(1+exp(-x)), key = s + bias            */
#define MM_SCORE_SOFTMAX 1      /* key = x + bias, w = softmax over the top-k   */
#define MM_SCORE_SQRTSOFTPLUS 2 /* s = sqrt(log1p(exp(x))) (x above 20: sqrt x),
                                   key = s + bias, w = s / sum (DeepSeek-V4.1) */
#define MM_SCORE_SQRTSOFTPLUS_DSV41 3 /* the same with the DeepSeek-V4.1 gate's own
                                   numerics (gate_topk.cuh:99-198 built for
                                   SGLang's Triton router): CUDA's expf / log1pf /
                                   sqrtf under flush-to-zero and approximate sqrt,
                                   NaN ranked first, the Triton reduction's sum
                                   order, div.full; ids and weights equal the
                                   reference kernel's bit for bit. top_k 3 or 6,
                                   renormalize MM_RENORM_SUM only               */

/* ---- routing weight rules (mm_gate_args.renormalize) ------------------- */
#define MM_RENORM_NONE 0        /* w = s * scale                                  */
#define MM_RENORM_SUM 1         /* w = (s / sum) * scale (sum + eps when eps > 0;
                                   a zero sum counts as 1); the sum in slot order */
#define MM_RENORM_SCALED_BF16 2 /* GLM-5.3 (glm5_3/sm103/moe/routing.py:3-11):
                                   w = bf16(scale * s / (sum + eps)), the sum in
                                   the order of a warp xor-butterfly over the
                                   slots; sigmoid or sqrtsoftplus scores        */

/* ---- expert weight formats ---------------------------------------------- */
#define MM_WEIGHT_MXFP4 0 /* E2M1 codes + one E8M0 scale per 32 along K      */
#define MM_WEIGHT_NVFP4 1 /* E2M1 codes + one E4M3 scale per 16 along K and
                             an fp32 second-level scale per expert (ModelOpt
                             NVFP4; glm5_3/sm103/moe/api.py:39-53)            */

/* One group of experts in the canonical layout (SGLang FusedMoE w13/w2):
 *   w13       u8 [n, 2*I, H/2]  E2M1 pairs, low nibble = even element;
 *                               rows [0, I) are gate (w1), rows [I, 2I) up (w3)
 *   w13_scale u8 [n, 2*I, H/32] E8M0 (value 2^(byte-127)) per 32 elements
 *             (NVFP4: [n, 2*I, H/16] E4M3 per 16 elements)
 *   w2        u8 [n, H, I/2]
 *   w2_scale  u8 [n, H, I/32]   (NVFP4: [n, H, I/16] E4M3)
 *   w13_scale_2, w2_scale_2     NVFP4 only: fp32 [n] per-expert second-level
 *             scales (weight = e2m1 * e4m3 * scale_2); NULL for MXFP4
 * w13 and w2 must be 16-byte aligned (TMA tensor maps). */
typedef struct mm_expert_weights {
  const void *w13;
  const void *w13_scale;
  const void *w2;
  const void *w2_scale;
  const float *w13_scale_2;
  const float *w2_scale_2;
} mm_expert_weights;

typedef struct mm_layer_desc {
  int32_t hidden;         /* H: multiple of 256 (router GEMV: multiple of 1024)    */
  int32_t intermediate;   /* I (this rank's slice): multiple of 256                */
  int32_t experts;        /* local routed experts (this rank's window)             */
  int32_t router_experts; /* experts the router scores (>= expert_offset+experts)  */
  int32_t expert_offset;  /* router id of local expert 0 (expert parallelism);
                             -1 - g (g = 0, 1): balanced dealing to group g of two
                             (the rank holds every expert; route.cuh:39-46)       */
  int32_t top_k;          /* 1..16                                                 */
  int32_t max_tokens;     /* largest T a call may pass: 1..256                     */
  int32_t weight_format;  /* MM_WEIGHT_MXFP4 or MM_WEIGHT_NVFP4                   */
  int32_t act_terms;      /* FP4 terms carrying each activation into the GEMMs (in
                             the weights' format): x ~ t0 + t1 + t2, t_i the FP4
                             quantization of the residual of the earlier terms.
                             1..3; 3 is the default numerics (about 1e-3 relative),
                             1 is plain MXFP4 / NVFP4.                              */
  int32_t device;         /* CUDA device ordinal the weights live on               */
  mm_expert_weights routed; /* n = experts                                         */
  mm_expert_weights shared; /* n = 1; shared.w13 == NULL: no shared expert          */
  const float *clamp;       /* [experts] SwiGLU clamp limit or NULL (no clamp)      */
  const float *shared_clamp;/* [1] or NULL                                          */
  float input_scale[2];     /* NVFP4: the static input scales of the gate_up and
                               down GEMMs (activation = e2m1 * e4m3 * input_scale;
                               the reference's FC1 / FC2 input scales, gs = 1 /
                               input_scale); ignored for MXFP4                     */
} mm_layer_desc;

typedef struct mm_layer mm_layer; /* opaque handle */

/* Routing arguments of one call (gate_topk_and_gemms / moe_fused_gate). */
typedef struct mm_gate_args {
  const float *logits;       /* [T, router_experts] fp32                          */
  const float *bias;         /* [router_experts] fp32 or NULL                     */
  const int32_t *num_valid;  /* device int32 [1] or NULL: rows >= *num_valid get
                                id -1 and weight 0 (padded graph rows)            */
  int32_t score_func;        /* MM_SCORE_*                                        */
  int32_t renormalize;       /* MM_RENORM_* (softmax always renormalizes)         */
  float routed_scaling;      /* multiplies every weight                           */
  float renorm_eps;          /* > 0: divide by sum + eps; else by the guarded sum */
  float *weights;            /* out [T, top_k] fp32                               */
  int32_t *ids;              /* out [T, top_k] int32 (router ids)                 */
  /* vision routing (gate_topk.cuh:290-346): a valid row whose input token is
   * alt_token_id ranks with bias_alt (NULL: bias) instead of bias */
  const float *bias_alt;     /* [router_experts] fp32 or NULL                     */
  const void *input_ids;     /* [T] int32 (int64 when input_ids64) or NULL        */
  int32_t input_ids64;
  int64_t alt_token_id;
} mm_gate_args;

/* Sizes of the caller-owned buffers of a layer call. */
typedef struct mm_layer_info {
  int32_t hidden, intermediate, experts, router_experts, expert_offset, top_k;
  int32_t max_tokens;
  int32_t has_shared;
  int64_t rows_capacity;   /* rows of the rows_out buffer (bf16 [rows, H])       */
  int64_t shared_row_base; /* first rows_out row of the shared expert's T rows    */
  int64_t route_words;     /* int32 words of the route record at max_tokens       */
  int64_t weight_bytes;    /* algorithmic FP4 + scale bytes of one expert         */
  int32_t act_terms;       /* FP4 terms per activation                            */
  int32_t h_row_bytes;     /* bytes of one h code row (I padded to 256 features)  */
  int64_t h_scale_row_bytes; /* bytes of one h scale row                          */
} mm_layer_info;

/* The layer's quantized activations (mm_layer_read_scratch): the routed input
 * as FP4 terms, codes [3][max_tokens][H/2] (two E2M1 per byte, low nibble =
 * even element) and scales [3][max_tokens][H/block] (E8M0 per 32, or E4M3 per
 * 16 for NVFP4), rows = tokens; the SwiGLU output h likewise, codes
 * [3][rows_capacity][h_row_bytes] and scales [3][rows_capacity]
 * [h_scale_row_bytes], rows in the permuted order of the deferred rows. Terms
 * past act_terms are unused. */
#define MM_SCRATCH_X_CODES 0
#define MM_SCRATCH_X_SCALES 1
#define MM_SCRATCH_H_CODES 2
#define MM_SCRATCH_H_SCALES 3

/* Whole-step arguments (mm_layer_forward). */
typedef struct mm_comm mm_comm; /* opaque handle: see mm_comm_create */

typedef struct mm_forward_args {
  const uint16_t *x;        /* bf16 [T, H]                                       */
  const uint16_t *router_w; /* bf16 [router_experts, H] or NULL (then logits)    */
  const float *logits;      /* fp32 [T, router_experts] when router_w is NULL    */
  float *logits_out;        /* fp32 [T, router_experts] scratch/out (router_w)   */
  const float *bias;        /* [router_experts] or NULL                          */
  const int32_t *num_valid; /* device [1] or NULL                                */
  int32_t score_func, renormalize;
  float routed_scaling, renorm_eps;
  int32_t tokens;           /* T */
  float *weights;           /* out [T, top_k]                                    */
  int32_t *ids;             /* out [T, top_k]                                    */
  int32_t *permuted;        /* out [T, top_k]                                    */
  int32_t *record;          /* out route record (mm_route_words words)           */
  uint16_t *rows;           /* out bf16 [rows_capacity, H] (deferred rows)       */
  uint16_t *out;            /* out bf16 [T, H] combined, or NULL                 */
  float *partial;           /* out fp32 [2, T, H] (routed, shared) un-rounded
                               partial sums for a cross-rank all-reduce, or NULL */
  mm_comm *comm;            /* non-NULL: out receives the group's all-reduced
                               output (mm_finalize_allreduce) instead of this
                               rank's own combine; partial must then be NULL   */
  const float *bias_alt;    /* vision routing, as in mm_gate_args              */
  const void *input_ids;
  int32_t input_ids64;
  int64_t alt_token_id;
  const uint16_t *residual; /* non-NULL (needs comm): the hop epilogue of
                               mm_finalize_allreduce_norm; out receives the
                               normalized output (NULL: none)                  */
  const uint16_t *gamma;    /* bf16 [H] RMSNorm weight (with out)              */
  float norm_eps;
  uint16_t *residual_out;   /* bf16 [T, H] new residual (may alias residual)   */
} mm_forward_args;

/* ---- library ------------------------------------------------------------ */
const char *mm_last_error(void);
int mm_version(void);

/* ---- stateless kernels ---------------------------------------------------- */
/* logits[t, e] = sum_h x[t, h] * w[e, h] in a fixed summation order
 * (replicated bit for bit by the CPU oracle). H % 1024 == 0. */
int mm_router_gemv(const uint16_t *x, const uint16_t *w, float *logits, int32_t tokens,
                   int32_t experts, int32_t hidden, void *stream);

/* Router top-k of T rows (one CTA per row). E <= 1024, 1 <= top_k <= 16. */
int mm_gate_topk(const mm_gate_args *args, int32_t tokens, int32_t router_experts,
                 int32_t top_k, void *stream);

/* int32 words of the route record for (T, top_k, local experts). */
int64_t mm_route_words(int32_t tokens, int32_t top_k, int32_t experts);

/* Route record + slot -> row map from top-k ids, bit for bit the reference's
 * (route.cuh:6-46, route_wide.cu:1-14). expert_offset >= 0: the router id of
 * local expert 0; -1 / -2: balanced dealing to group 0 / 1 (experts = all the
 * router's experts). T <= 256. */
int mm_route(const int32_t *ids, int32_t *permuted, int32_t *record, int32_t tokens,
             int32_t top_k, int32_t experts, int32_t expert_offset, void *stream);

/* The router top-k and the route record in ONE launch that allocates nothing.
 * No counterpart in the reference. For callers that cannot call cudaMalloc: a
 * serving runtime that reserves the GPU's memory for its own caching pool at
 * start-up (an allocation outside the pool fails or fragments it), or plugin
 * code that is handed only its input and output pointers and has no allocator
 * (the same fused launch inside mm_layer_* uses scratch that mm_layer_create
 * allocates).
 * Outputs equal mm_gate_topk followed by mm_route. gate->ids may be NULL (ids
 * not returned). Scratch: 8.25 KB of the library's static device memory per
 * GPU, held until exit; tokens * top_k <= 2048, larger requests are rejected
 * with MM_ERR_INVALID. The first call on a device sets the scratch up (the symbol's
 * device address, the kernel's shared-memory limit) and should come before any
 * stream capture. All
 * calls on a device share the scratch: calls that overlap on the GPU (other
 * streams) race; consecutive calls on one stream do not. */
int mm_gate_route_noalloc(const mm_gate_args *gate, int32_t tokens, int32_t router_experts,
                          int32_t top_k, int32_t experts, int32_t expert_offset,
                          int32_t *permuted, int32_t *record, void *stream);

/* out[t] = bf16(bf16(sum_k w[t,k] * rows[perm[t,k]]) + shared[t]) in slot order
 * (rows with perm -1 are skipped); shared_rows may be NULL. partial (fp32
 * [2, T, H]) receives the un-rounded routed sum and the shared row instead
 * when non-NULL (out may then be NULL). */
int mm_finalize(const uint16_t *rows, const float *weights, const int32_t *permuted,
                const uint16_t *shared_rows, uint16_t *out, float *partial,
                int32_t tokens, int32_t top_k, int32_t hidden, void *stream);

/* out = bf16(bf16(sum_r routed_r) + sum_r shared_r) from an all-reduced partial. */
int mm_finalize_partial(const float *partial, uint16_t *out, int32_t tokens,
                        int32_t hidden, void *stream);

/* ---- combine + all-reduce over NVLink peer memory ------------------------ */
/* One rank's view of a TP/EP group whose ranks exchange their partial outputs
 * by plain P2P stores into each other's buffers (CUDA IPC; no multicast). */
#define MM_IPC_HANDLE_BYTES 64

/* Allocates this rank's tile counters and mailbox (2 generations x world x
 * max_tokens x hidden bf16, every value the empty sentinel -0) on `device`. */
int mm_comm_create(int32_t rank, int32_t world, int32_t max_tokens, int32_t hidden,
                   int32_t device, mm_comm **out);
/* Writes this rank's IPC handle (MM_IPC_HANDLE_BYTES bytes) to `handle`. */
int mm_comm_handle(const mm_comm *comm, void *handle);
/* Opens the peers' buffers from all ranks' handles (world x MM_IPC_HANDLE_BYTES,
 * rank order; this rank's own entry is ignored). Once per comm. */
int mm_comm_open(mm_comm *comm, const void *handles);
int mm_comm_destroy(mm_comm *comm);
/* Opens a group whose members all live in this process (one process driving
 * several GPUs, or several ranks of one GPU): members[q] is rank q's comm
 * (members[rank] == comm), every member of the same world, max_tokens and
 * hidden. Peer access is enabled from this comm's device to each member's.
 * Instead of mm_comm_open; once per comm. No reference counterpart (the
 * reference's groups are one process per GPU, all_reduce_mhc.py:1194). */
int mm_comm_open_local(mm_comm *comm, mm_comm *const *members);
/* Synchronizes and reads (then clears) the comm's device error word:
 * MM_OK or MM_ERR_DEVICE_TIMEOUT (a peer's partial never arrived within the
 * wait budget; the group's comms must then be rebuilt). */
int mm_comm_check(mm_comm *comm);
/* The budget of the mailbox poll of this comm's launches, 1 us .. 60 s
 * (default 1.5 s). A poll that runs out sets the comm's error word and the
 * launch ends. The reference's remote waits carry deadlines too
 * (common/sync.py:157-185, all_reduce_mhc.py:917-924); there they trap. */
int mm_comm_set_wait_budget(mm_comm *comm, int64_t microseconds);

/* out[t] = bf16( sum_{r = 0..world-1} y_r[t] ) in fp32, rank order, where
 * y_r = bf16(bf16(sum_k w * rows_r[perm_r]) + shared_r) is rank r's partial
 * (mm_finalize's arithmetic on rank r's rows). One launch per rank; every rank
 * of the group must call it with the same tokens, in the same order. */
int mm_finalize_allreduce(mm_comm *comm, const uint16_t *rows, const float *weights,
                          const int32_t *permuted, const uint16_t *shared_rows,
                          uint16_t *out, int32_t tokens, int32_t top_k, int32_t hidden,
                          void *stream);

/* The same combine + all-reduce with the residual + RMSNorm epilogue of a
 * decoder hop (qwen3_5/sm103/hop/__init__.py:431 moe_finalize_all_reduce_rms_norm;
 * arithmetic hop.cu:119-139, q35_hop.cuh:258-336): per token,
 *   pre = bf16(sum_r y_r + residual)   (fp32 rank-order sum, one rounding)
 *   residual_out = pre
 *   norm_out = bf16((pre * inv) * gamma), inv = 1 / sqrt(sum(pre^2) / H + eps)
 * with sqrt and divisions IEEE-rounded and the sum of squares in a fixed fold
 * (8 features per thread in order, warp xor butterfly 16..1, 8 warps in order,
 * the row's ceil(H / 2048) CTAs in order). norm_out may be NULL (then gamma
 * too). H <= 16384. residual may alias residual_out. */
int mm_finalize_allreduce_norm(mm_comm *comm, const uint16_t *rows, const float *weights,
                               const int32_t *permuted, const uint16_t *shared_rows,
                               const uint16_t *residual, const uint16_t *gamma, float eps,
                               uint16_t *residual_out, uint16_t *norm_out, int32_t tokens,
                               int32_t top_k, int32_t hidden, void *stream);

/* ---- layer ---------------------------------------------------------------- */
int mm_layer_create(const mm_layer_desc *desc, mm_layer **out);
int mm_layer_destroy(mm_layer *layer);
int mm_layer_get_info(const mm_layer *layer, mm_layer_info *info);

/* Route + gate_up + down from given top-k ids (RoutedExpertGemm.__call__):
 * rows[permuted[t, k]] is slot (t, k)'s expert output (bf16 [rows_capacity, H]);
 * the shared expert's rows start at info.shared_row_base. */
int mm_layer_experts(mm_layer *layer, const uint16_t *x, const int32_t *ids,
                     int32_t tokens, int32_t *permuted, int32_t *record,
                     uint16_t *rows, void *stream);

/* Top-k from router logits + route + gate_up + down (gate_topk_and_gemms). */
int mm_layer_gate_experts(mm_layer *layer, const uint16_t *x, const mm_gate_args *gate,
                          int32_t tokens, int32_t *permuted, int32_t *record,
                          uint16_t *rows, void *stream);

/* mm_layer_experts and mm_layer_gate_experts with the routed input already
 * MXFP8-quantized, as SGLang hands it to the reference
 * (Mxfp4FlashinferTrtllmMoEMethod.quantize_routed_input; the reference's
 * RoutedExpertGemm.__call__(x_quant, x_scale, topk_ids, topk_weights),
 * routed_expert_gemm.py:703, and gate_topk_and_gemms(x_quant, x_scale, ...),
 * :776): x_quant u8 [T, H] E4M3 codes, x_scale u8 [T, H/32] E8M0 scales
 * (row-major, unswizzled), both 16-byte aligned. Each element enters the
 * chain as e4m3 * 2^(scale - 127) (exact, one fp32 rounding for subnormal
 * results), then as the layer's FP4 terms. */
int mm_layer_experts_mxfp8(mm_layer *layer, const uint8_t *x_quant, const uint8_t *x_scale,
                           const int32_t *ids, int32_t tokens, int32_t *permuted,
                           int32_t *record, uint16_t *rows, void *stream);
int mm_layer_gate_experts_mxfp8(mm_layer *layer, const uint8_t *x_quant, const uint8_t *x_scale,
                                const mm_gate_args *gate, int32_t tokens, int32_t *permuted,
                                int32_t *record, uint16_t *rows, void *stream);

/* Bytes of one of the layer's activation buffers (MM_SCRATCH_*), -1 for an
 * unknown one; and a stream-ordered device-to-device copy of it into dst
 * (exactly that many bytes). For inspecting the quantization bytes the chain
 * multiplies; no reference counterpart. */
int64_t mm_layer_scratch_bytes(const mm_layer *layer, int32_t which);
int mm_layer_read_scratch(const mm_layer *layer, int32_t which, void *dst, int64_t bytes,
                          void *stream);

/* Launches the expert kernel again on the work tables of this layer's last
 * front pass (same tokens, routing and input): re-computes the same rows. The
 * tables must be re-armed first (mm_layer_rearm_experts) each time: a launch
 * consumes them. A benchmark hook that times the dominant kernel alone; no
 * reference counterpart (the reference launches its GEMM pair once per route
 * record, routed_expert_gemm.py:964-999). */
int mm_layer_rerun_experts(mm_layer *layer, int32_t tokens, const int32_t *record,
                           uint16_t *rows, void *stream);

/* Re-arms the expert kernel's work tables of the last front pass (zeroes the
 * segment mailboxes and the claim counter, stream-ordered) so that
 * mm_layer_rerun_experts can launch on them again. */
int mm_layer_rearm_experts(mm_layer *layer, void *stream);

/* Re-arms the work tables like mm_layer_rearm_experts, but with every segment's
 * gate_up -> down mailbox set far below reach, so that the next
 * mm_layer_rerun_experts cannot finish: its down units' bounded waits run out,
 * the launch ends and mm_layer_check reports MM_ERR_DEVICE_TIMEOUT. A test
 * hook for the timeout path (a flag that nothing sets); the next front pass
 * (any layer call) re-arms the tables normally. No reference counterpart. */
int mm_layer_block_downs(mm_layer *layer, void *stream);

/* The budget of every bounded device wait of this layer's expert launches,
 * 1 us .. 60 s (default 1.5 s). A wait that runs out sets the layer's error
 * word, every later wait of the launch gives up at once, and the launch ends
 * (its copies and MMAs in flight drained first). */
int mm_layer_set_wait_budget(mm_layer *layer, int64_t microseconds);

/* The whole MoE step: [router GEMV] -> top-k -> route -> experts -> combine. */
int mm_layer_forward(mm_layer *layer, const mm_forward_args *args, void *stream);

/* Synchronizes the layer's device and reads (then clears) its device error
 * word: MM_OK, MM_ERR_DEVICE_TIMEOUT or MM_ERR_DEVICE. */
int mm_layer_check(mm_layer *layer);

/* ---- stack ------------------------------------------------------------------ */
/* One step of n MoE layers: mm_layer_forward(layers[i].layer, &layers[i].args)
 * for i = 0..n-1 on one stream, with no host synchronization, so the launches
 * of all layers chain by PDL (a layer's hop output is the next layer's input).
 * The host side of the reference's layer loop (deepseek_v41/moe/step.py:101,
 * called once per MoE layer by the megakernel's forward); stops at the first
 * failing layer and returns its status. */
typedef struct mm_stack_layer {
  mm_layer *layer;
  mm_forward_args args;
} mm_stack_layer;

int mm_stack_forward(const mm_stack_layer *layers, int32_t n, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* MEGAMOE_H */
