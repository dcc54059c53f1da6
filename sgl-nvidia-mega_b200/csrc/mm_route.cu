// Front of the routed-MoE chain: router GEMV (K0), top-k with bias (K1a), the
// route record and slot -> row map (K1b), the MXFP4-terms quantization of the
// routed input, and the segment / work tables of the expert kernel.
//
// The route record is bit for bit the reference's (route.cuh:6-46,94-161 for
// up to 8 rows, route_wide.cu:1-14,62-163 beyond): local experts in ascending
// id order, each one's rows in ascending token order, every expert's segment
// padded to 8-row tiles, an expert chosen by more than 8 rows owning
// consecutive tiles. The construction here is our own (multi-word row masks in
// shared memory and one block scan, for up to 256 rows).
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>

#include "megamoe.h"
#include "mm_kernels.cuh"
#include "mm_layout.cuh"
#include "mm_numerics.cuh"
#include "mm_ptx.cuh"

namespace mm {

// ============================================================================
// K0: router GEMV + routed-input quantization in one launch.
//
// CTAs [0, gemv_ctas) x grid.y: logits[t, e] = sum_h x[t, h] w[e, h] (fp32) for
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
//
// CTAs [gemv_ctas, ...) (blockIdx.y == 0): the FP4 terms of x, one 32-element
// chunk of one token per thread (one MXFP4 block or two NVFP4 blocks;
// independent of the routing). x is bf16, or MXFP8 (x8 / s8: E4M3 codes and an
// E8M0 scale per 32, the reference's pre-quantized routed input).
// ============================================================================
__global__ void __launch_bounds__(256) router_quant_kernel(RouterArgs a) {
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (static_cast<int>(blockIdx.x) >= a.gemv_ctas) {
    pdl_wait();
    if (blockIdx.y != 0 || a.xq == nullptr) return;
    const int blocks = a.hidden >> 5;
    const int idx = (blockIdx.x - a.gemv_ctas) * blockDim.x + threadIdx.x;
    if (idx >= a.tokens * blocks) return;
    const int t = idx / blocks, b = idx - t * blocks;
    float v[32];
    if (a.x8 != nullptr) {
      // MXFP8 input (the reference's x_quant / x_scale): the exact value of each
      // E4M3 code times the block's E8M0 scale, one fp32 rounding (subnormals kept)
      const uint4 *src = reinterpret_cast<const uint4 *>(a.x8 + static_cast<size_t>(t) * a.hidden + 32 * b);
      const float sv = mx_scale_value(a.s8[static_cast<size_t>(t) * blocks + b]);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint4 u = src[i];
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 16; ++j)
          v[16 * i + j] = __fmul_rn(e4m3_value(static_cast<uint8_t>(w4[j >> 2] >> (8 * (j & 3)))), sv);
      }
    } else {
      const uint4 *src = reinterpret_cast<const uint4 *>(a.x + static_cast<size_t>(t) * a.hidden + 32 * b);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 u = src[i];
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[8 * i + 2 * j] = __uint_as_float(w4[j] << 16);
          v[8 * i + 2 * j + 1] = __uint_as_float(w4[j] & 0xffff0000u);
        }
      }
    }
    const size_t q_stride = static_cast<size_t>(a.max_tokens) * (a.hidden >> 1);
    uint8_t *q = a.xq + static_cast<size_t>(t) * (a.hidden >> 1) + 16 * b;
    if (a.fmt == kFmtNv) {  // two NVFP4 blocks of 16
      const size_t s_stride = static_cast<size_t>(a.max_tokens) * 2 * blocks;
      uint8_t *sc = a.xs + static_cast<size_t>(t) * 2 * blocks + 2 * b;
      quantize_block16_nvfp4(v, a.terms, a.gs, a.inv_gs, q, q_stride, sc, s_stride);
      quantize_block16_nvfp4(v + 16, a.terms, a.gs, a.inv_gs, q + 8, q_stride, sc + 1, s_stride);
    } else {
      const size_t s_stride = static_cast<size_t>(a.max_tokens) * blocks;
      quantize_block32_fp4(v, a.terms, q, q_stride, a.xs + static_cast<size_t>(t) * blocks + b, s_stride);
    }
    return;
  }
  // GEMV tile: experts [4 blockIdx.x, +4) x tokens [8 blockIdx.y, +8). The 8
  // token rows of x are staged once in shared memory (cp.async). Warp w takes
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
  uint4 wv[4][4];
  load_w(warp, wv);
  pdl_wait();
  {
    const int per_row = a.hidden >> 3;  // uint4 per token row
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(xs));
    for (int i = threadIdx.x; i < nt * per_row; i += blockDim.x) {
      const int t = i / per_row, c = i - t * per_row;
      cp_async_16(sbase + 16u * static_cast<uint32_t>(i),
                  reinterpret_cast<const uint4 *>(a.x + static_cast<size_t>(t0 + t) * a.hidden) + c, 16u);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
  }
#pragma unroll 1
  for (int part = warp; part < parts; part += 8) {
    if (part != warp) load_w(part, wv);
    // per lane: 4 experts x 8 tokens chains, each in the element order above;
    // rows t >= nt are stale smem and never stored
    const uint4 *xr = reinterpret_cast<const uint4 *>(xs + 1024 * part);
    const int row_u4 = a.hidden >> 3;
    float v[32];  // v[8 es + t]
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int t = 0; t < 8; ++t) {
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
// K1a: one row's top-k (block of 512 threads, experts e = tid and tid + 512).
// ============================================================================
struct GateSmem {
  float score[kMaxRouterExperts];
  float logit[kMaxRouterExperts];
  unsigned long long cand[16][kMaxTopK];
  int sel[kMaxTopK];
};

__device__ __forceinline__ unsigned long long pack_key(uint32_t key, int e) {
  return (static_cast<unsigned long long>(key) << 32) | static_cast<uint32_t>(0xffffffffu - e);
}

// Computes ids/weights of row `row` and writes them to ids_out/weights_out.
__device__ void gate_row(const GateArgs &g, int row, int valid_rows, GateSmem &sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int E = g.router_experts, K = g.top_k;
  const float *lrow = g.logits + static_cast<size_t>(row) * E;
  // a valid row whose input token is alt_token_id ranks with bias_alt
  bool alt = false;
  if (g.input_ids != nullptr && row < valid_rows) {
    const long long token = g.input_ids64 ? static_cast<const long long *>(g.input_ids)[row]
                                          : static_cast<long long>(static_cast<const int *>(g.input_ids)[row]);
    alt = token == g.alt_token_id;
  }
  const float *bias = alt && g.bias_alt != nullptr ? g.bias_alt : g.bias;
  uint32_t kv[2];  // routing key + 1 of experts tid, tid + 512; 0: none or taken
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int e = tid + 512 * h;
    kv[h] = 0u;
    if (e < E) {
      const float l = lrow[e];
      const float b = bias != nullptr ? bias[e] : 0.0f;
      float s;
      if (g.score_func == 0) s = det_sigmoid(l);
      else if (g.score_func == 2) s = det_sqrtsoftplus(l);
      else s = l;  // softmax: rank the (biased) logits
      sm.score[e] = s;
      sm.logit[e] = l;
      kv[h] = routing_key(__fadd_rn(s, b)) + 1u;  // keys of real scores stay below 0xff800001
    }
  }
  // per-warp top-K candidates (every global winner is in its warp's top-K): the
  // largest key by a warp reduction, the lowest expert id among its holders by
  // ballot (experts tid < 512 precede tid + 512, and lanes ascend within each)
  for (int k = 0; k < K; ++k) {
    const uint32_t m = __reduce_max_sync(0xffffffffu, kv[0] > kv[1] ? kv[0] : kv[1]);
    unsigned long long top = 0ull;
    if (m != 0u) {
      const uint32_t b0 = __ballot_sync(0xffffffffu, kv[0] == m);
      int win;
      if (b0 != 0u) {
        const int l = __ffs(b0) - 1;
        win = warp * 32 + l;
        if (lane == l) kv[0] = 0u;
      } else {
        const int l = __ffs(__ballot_sync(0xffffffffu, kv[1] == m)) - 1;
        win = 512 + warp * 32 + l;
        if (lane == l) kv[1] = 0u;
      }
      top = pack_key(m - 1u, win);
    }
    if (lane == 0) sm.cand[warp][k] = top;
  }
  __syncthreads();
  if (warp == 0) {
    // merge 16 warps x K candidates: lane l holds warps' entries l, l+32, ...
    // (a candidate is key + 1 and expert id; key 0: empty or taken). Each
    // round: the largest key by a warp reduction, then the lowest expert id
    // among its holders by a second one -- the same pick as the largest
    // packed (key, ~id).
    constexpr int kPer = 16 * kMaxTopK / 32;
    uint32_t ckey[kPer], cid[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int idx = lane + 32 * j;  // idx = warp_id * kMaxTopK + k
      const int cw = idx / kMaxTopK, ck = idx % kMaxTopK;
      const unsigned long long c = (ck < K) ? sm.cand[cw][ck] : 0ull;
      ckey[j] = c == 0ull ? 0u : static_cast<uint32_t>(c >> 32) + 1u;
      cid[j] = 0xffffffffu - static_cast<uint32_t>(c);
    }
    for (int k = 0; k < K; ++k) {
      uint32_t lm = 0u;
#pragma unroll
      for (int j = 0; j < kPer; ++j) lm = ckey[j] > lm ? ckey[j] : lm;
      const uint32_t m = __reduce_max_sync(0xffffffffu, lm);
      uint32_t lid = 0xffffffffu;
#pragma unroll
      for (int j = 0; j < kPer; ++j) lid = (m != 0u && ckey[j] == m && cid[j] < lid) ? cid[j] : lid;
      const uint32_t wid = __reduce_min_sync(0xffffffffu, lid);
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (ckey[j] == m && cid[j] == wid) ckey[j] = 0u;
      if (lane == 0) sm.sel[k] = static_cast<int>(wid);  // 0xffffffff (-1) when nothing is left
    }
    __syncwarp();
    if (lane == 0) {
      const bool valid = row < valid_rows;
      float w[kMaxTopK];
      if (g.score_func == 1) {
        float m = sm.logit[sm.sel[0]];
        for (int k = 1; k < K; ++k) m = fmaxf(m, sm.logit[sm.sel[k]]);
        float sum = 0.0f;
        for (int k = 0; k < K; ++k) {
          w[k] = det_exp(__fsub_rn(sm.logit[sm.sel[k]], m));
          sum = __fadd_rn(sum, w[k]);
        }
        for (int k = 0; k < K; ++k) w[k] = __fmul_rn(__fdiv_rn(w[k], sum), g.routed_scaling);
      } else {
        float sum = 0.0f;
        for (int k = 0; k < K; ++k) {
          w[k] = sm.score[sm.sel[k]];
          sum = __fadd_rn(sum, w[k]);
        }
        if (g.renormalize == 2) {
          // GLM-5.3's rule (glm5_3/sm103/moe/routing.py:3-11, ptx_tc.py routing_weight):
          // the selected scores summed in the order of a warp xor-butterfly whose
          // lane k holds slot k (the halving [i] += [i + off], off = 8, 4, 2, 1, is
          // lane 0's order), then w = bf16(scale * s / (sum + eps)), scale first;
          // IEEE division where the reference divides approximately
          float t[kMaxTopK];
#pragma unroll
          for (int k = 0; k < kMaxTopK; ++k) t[k] = k < K ? w[k] : 0.0f;
#pragma unroll
          for (int off = kMaxTopK / 2; off >= 1; off >>= 1)
#pragma unroll
            for (int i = 0; i < off; ++i) t[i] = __fadd_rn(t[i], t[i + off]);
          const float d = __fadd_rn(t[0], g.renorm_eps);
          for (int k = 0; k < K; ++k)
            w[k] = bf16_bits_to_float(float_to_bf16_bits(__fdiv_rn(__fmul_rn(g.routed_scaling, w[k]), d)));
        } else if (g.renormalize) {
          const float norm = g.renorm_eps > 0.0f ? __fadd_rn(sum, g.renorm_eps)
                                                 : (sum > 0.0f ? sum : 1.0f);
          for (int k = 0; k < K; ++k) w[k] = __fmul_rn(__fdiv_rn(w[k], norm), g.routed_scaling);
        } else {
          for (int k = 0; k < K; ++k) w[k] = __fmul_rn(w[k], g.routed_scaling);
        }
      }
      for (int k = 0; k < K; ++k) {
        g.ids_out[static_cast<size_t>(row) * K + k] = valid ? sm.sel[k] : -1;
        g.weights_out[static_cast<size_t>(row) * K + k] = valid ? w[k] : 0.0f;
      }
    }
  }
}

__global__ void __launch_bounds__(512) gate_topk_kernel(GateArgs g) {
  pdl_launch_dependents();
  __shared__ GateSmem sm;
  pdl_wait();
  const int valid = g.num_valid != nullptr ? *g.num_valid : static_cast<int>(gridDim.x);
  gate_row(g, blockIdx.x, valid, sm);
}

// ============================================================================
// K1b: the route record (block of 512 threads). Dynamic shared memory:
// rowmask[experts][words] u32, first_cta[experts] int, warp totals.
// ============================================================================
__device__ void block_exclusive_scan_512(int *vals /*[1024] pairs*/, int n, int *warp_tot,
                                         int &total) {
  // vals[0..n) in place -> exclusive prefix; n <= 1024; each thread two entries
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int a = 2 * tid < n ? vals[2 * tid] : 0;
  const int b = 2 * tid + 1 < n ? vals[2 * tid + 1] : 0;
  const int local = a + b;
  int inc = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int up = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += up;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int t = lane < 16 ? warp_tot[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int up = __shfl_up_sync(0xffffffffu, t, off);
      if (lane >= off) t += up;
    }
    if (lane < 16) warp_tot[lane] = t;
  }
  __syncthreads();
  const int base = inc - local + (warp > 0 ? warp_tot[warp - 1] : 0);
  total = warp_tot[15];
  if (2 * tid < n) vals[2 * tid] = base;
  if (2 * tid + 1 < n) vals[2 * tid + 1] = base + a;
  __syncthreads();
}

__device__ void build_route(const RouteArgs &r, unsigned char *smem_raw) {
  const int tid = threadIdx.x;
  const int T = r.tokens, K = r.top_k, E = r.experts;
  const int words = (T + 31) >> 5;
  uint32_t *rowmask = reinterpret_cast<uint32_t *>(smem_raw);
  int *first = reinterpret_cast<int *>(rowmask + E * words);
  int *seg_first = first + E;
  int *warp_tot = seg_first + E;
  int *counts = warp_tot + 32;
  const int slots = T * K;
  const int max_ctas = route_max_ctas(T, K, E);
  const int cw = route_cta_words(max_ctas);
  const int limit_off = 4 + cw, token_off = 4 + 2 * cw;
  const int rec_words = token_off + kTile * max_ctas;
  for (int i = tid; i < E * words; i += blockDim.x) rowmask[i] = 0u;
  for (int i = tid; i < rec_words; i += blockDim.x) r.record[i] = 0;
  // balanced dealing (route.cuh:39-46): a negative offset selects group
  // -1 - offset of two; ids are global, and of the step's distinct experts in
  // id order the k-th belongs to group k % 2
  const bool deal = r.expert_offset < 0;
  const int group = deal ? -1 - r.expert_offset : 0;
  const int offset = deal ? 0 : r.expert_offset;
  __syncthreads();
  for (int s = tid; s < slots; s += blockDim.x) {
    const int t = s / K;
    const int e = __ldcg(r.ids + s) - offset;  // written by other CTAs: L2
    if (e >= 0 && e < E) atomicOr(&rowmask[e * words + (t >> 5)], 1u << (t & 31));
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    int c = 0;
    for (int wd = 0; wd < words; ++wd) c += __popc(rowmask[e * words + wd]);
    counts[e] = c;
    first[e] = c > 0 ? 1 : 0;  // presence, ranked below when dealing
  }
  __syncthreads();
  if (deal) {
    int present = 0;
    block_exclusive_scan_512(first, E, warp_tot, present);
    for (int e = tid; e < E; e += blockDim.x)
      if (counts[e] > 0 && (first[e] & 1) != group) counts[e] = 0;
    __syncthreads();
  }
  for (int e = tid; e < E; e += blockDim.x) {
    const int c = counts[e];
    first[e] = (c + kTile - 1) / kTile;               // tiles
    seg_first[e] = (c + kSegRows - 1) / kSegRows;     // segments
  }
  __syncthreads();
  int total_ctas = 0, total_segs = 0;
  block_exclusive_scan_512(first, E, warp_tot, total_ctas);
  block_exclusive_scan_512(seg_first, E, warp_tot, total_segs);
  if (tid == 0) {
    r.record[0] = total_ctas * kTile;
    r.record[1] = total_ctas;
  }
  for (int s = tid; s < slots; s += blockDim.x) {
    const int t = s / K;
    const int e = __ldcg(r.ids + s) - offset;  // written by other CTAs: L2
    if (e < 0 || e >= E || counts[e] == 0) {  // not held, or dealt to the other group
      r.permuted[s] = -1;
      continue;
    }
    int rank = 0;
    const uint32_t *m = rowmask + e * words;
    for (int wd = 0; wd < (t >> 5); ++wd) rank += __popc(m[wd]);
    rank += __popc(m[t >> 5] & ((1u << (t & 31)) - 1u));
    const int base_row = first[e] * kTile;
    r.permuted[s] = base_row + rank;
    r.record[token_off + base_row + rank] = t;
    if (rank % kTile == 0) {
      const int cta = first[e] + rank / kTile;
      r.record[4 + cta] = e;
      r.record[limit_off + cta] = min((cta + 1) * kTile, base_row + counts[e]);
    }
  }
  // expert-kernel work tables (shared expert's segments first)
  if (r.segs != nullptr) {
    const int shared_segs = r.has_shared ? (T + kSegRows - 1) / kSegRows : 0;
    for (int j = tid; j < shared_segs; j += blockDim.x) {
      const int rows = min(kSegRows, T - j * kSegRows);
      r.segs[j] = make_int4(-1, r.shared_row_base + j * kSegRows, rows, j * kSegRows);
    }
    for (int e = tid; e < E; e += blockDim.x) {
      const int c = counts[e];
      const int nseg = (c + kSegRows - 1) / kSegRows;
      for (int j = 0; j < nseg; ++j) {
        const int rows = min(kSegRows, c - j * kSegRows);
        r.segs[shared_segs + seg_first[e] + j] =
            make_int4(e, first[e] * kTile + j * kSegRows, rows, -1);
      }
    }
    const int nseg = shared_segs + total_segs;
    for (int j = tid; j < nseg; j += blockDim.x) r.flags[j] = 0;
    if (tid == 0) {
      r.ctrl[kCtrlSegments] = nseg;
      r.ctrl[kCtrlUnits] = nseg * (r.m1 + r.m2);
      r.ctrl[kCtrlClaim] = 0;
    }
  }
}

__global__ void __launch_bounds__(512) route_kernel(RouteArgs r) {
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char route_smem[];
  pdl_wait();
  build_route(r, route_smem);
}

// ============================================================================
// The front kernel: grid = T rows, block 512. Each CTA ranks its row (or takes
// given ids); the last CTA to finish builds the route record and the work
// tables.
// ============================================================================
__global__ void __launch_bounds__(512) front_kernel(FrontArgs f) {
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char front_smem[];
  __shared__ GateSmem gsm;
  __shared__ int is_last;
  pdl_wait();
  const int row = blockIdx.x;
  if (f.gate.logits != nullptr) {
    const int valid = f.gate.num_valid != nullptr ? *f.gate.num_valid : f.route.tokens;
    gate_row(f.gate, row, valid, gsm);
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // thread 0 (warp 0, lane 0) wrote the row's ids and weights
    __threadfence();
    const int ticket = atomicAdd(&f.route.ctrl[kCtrlTicket], 1);
    is_last = ticket == static_cast<int>(gridDim.x) - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  build_route(f.route, front_smem);
  if (threadIdx.x == 0) f.route.ctrl[kCtrlTicket] = 0;
}

// ============================================================================
// Router top-k + route record in one launch that allocates nothing.
//
// For callers that cannot call cudaMalloc: code that runs while a CUDA graph is
// being captured or inside a serving runtime that owns all device memory through
// its own pool, and that has only its input and output buffers at hand. The
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
  gate_row(g, blockIdx.x, valid, gsm);  // g.ids_out points into the scratch
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
