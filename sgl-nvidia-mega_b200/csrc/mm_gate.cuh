// Router top-k (one CTA of 512 threads per token row) and the route record /
// expert work tables (one CTA), shared by the launches of mm_route.cu (this
// library's IEEE routing numerics) and mm_gate_dsv41.cu (the DeepSeek-V4.1
// gate's numerics, a translation unit of its own because it is compiled with
// that gate's flush-to-zero and approximate square root and division).
//
// The route record is bit for bit the reference's (route.cuh:6-46,94-161 for
// up to 8 rows, route_wide.cu:1-14,62-163 beyond): local experts in ascending
// id order, each one's rows in ascending token order, every expert's segment
// padded to 8-row tiles, an expert chosen by more than 8 rows owning
// consecutive tiles. The construction here is our own (multi-word row masks in
// shared memory and one block scan, for up to 256 rows).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "mm_kernels.cuh"
#include "mm_layout.cuh"
#include "mm_ptx.cuh"

namespace mm {

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

// The merge of warp 0: the 16 warps' K candidates each, packed densely (flat
// index w K + k; lane l holds l, l + 32, ...; a candidate is key + 1 and
// expert id, key 0: empty or taken). Each round takes the largest key by a
// warp reduction, then the lowest expert id among its holders by a second one
// -- the same pick as the largest packed (key, ~id) -- into sm.sel[k].
template <int kPer>
__device__ __forceinline__ void merge_candidates(GateSmem &sm, int K, int lane) {
  uint32_t ckey[kPer], cid[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int f = lane + 32 * j;
    const unsigned long long c = f < 16 * K ? sm.cand[f / K][f % K] : 0ull;
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
}

// Computes ids/weights of row `row` and writes them to ids_out/weights_out.
// N is the routing numerics: N::score(g, logit) the unbiased score,
// N::key(score, bias) its order-preserving ranking key (larger ranks first; at
// most 0xff800000), N::weight(g, sm, k) the routing weight of the k-th selected
// expert sm.sel[k] from sm.score / sm.logit (lane k of warp 0 computes it; every
// lane evaluates the row's sum in the same order). Selection is the same for
// all: the K largest keys, the lowest expert id winning a tie.
template <class N>
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
      const float s = N::score(g, l);
      sm.score[e] = s;
      sm.logit[e] = l;
      kv[h] = N::key(s, b) + 1u;  // keys stay at or below 0xff800001
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
    if (K <= 8) merge_candidates<4>(sm, K, lane);
    else merge_candidates<8>(sm, K, lane);
    __syncwarp();
    if (lane < K) {  // lane k: slot k's id and weight
      const bool valid = row < valid_rows;
      const float wk = N::weight(g, sm, lane);
      g.ids_out[static_cast<size_t>(row) * K + lane] = valid ? sm.sel[lane] : -1;
      g.weights_out[static_cast<size_t>(row) * K + lane] = valid ? wk : 0.0f;
    }
  }
}

// ============================================================================
// K1b: the route record (block of 512 threads). Dynamic shared memory:
// rowmask[experts][words] u32, first_cta[experts] int, warp totals.
// ============================================================================
inline __device__ void block_exclusive_scan_512(int *vals /*[1024] pairs*/, int n, int *warp_tot,
                                         int &total) {
  // vals[0..n) in place -> exclusive prefix; n <= 1024; each thread two entries;
  // every thread adds the warp totals before its warp itself (16 broadcast reads)
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
  int before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    const int t = warp_tot[w];
    before += w < warp ? t : 0;
    all += t;
  }
  const int base = inc - local + before;
  total = all;
  if (2 * tid < n) vals[2 * tid] = base;
  if (2 * tid + 1 < n) vals[2 * tid + 1] = base + a;
  __syncthreads();
}

inline __device__ void build_route(const RouteArgs &r, unsigned char *smem_raw) {
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
  // balanced dealing (route.cuh:39-46): a negative offset selects group
  // -1 - offset of two; ids are global, and of the step's distinct experts in
  // id order the k-th belongs to group k % 2
  const bool deal = r.expert_offset < 0;
  const int group = deal ? -1 - r.expert_offset : 0;
  const int offset = deal ? 0 : r.expert_offset;
  // this thread's slots s = tid + 512 i (the ids were written by other CTAs:
  // L2, loaded before the zeroing below); the local experts of the first two are
  // kept for the second pass
  const int e0 = tid < slots ? __ldcg(r.ids + tid) - offset : -1;
  const int e1 = tid + 512 < slots ? __ldcg(r.ids + tid + 512) - offset : -1;
  auto slot_expert = [&](int s) { return s == tid ? e0 : (s == tid + 512 ? e1 : __ldcg(r.ids + s) - offset); };
  for (int i = tid; i < E * words; i += blockDim.x) rowmask[i] = 0u;
  for (int i = tid; i < rec_words; i += blockDim.x) r.record[i] = 0;
  __syncthreads();
  for (int s = tid; s < slots; s += blockDim.x) {
    const int t = s / K;
    const int e = slot_expert(s);
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
  // tiles and segments of every expert, scanned together: tiles in the low 16
  // bits, segments above (both totals stay below 2^16)
  for (int e = tid; e < E; e += blockDim.x) {
    const int c = counts[e];
    first[e] = (c + kTile - 1) / kTile + (((c + kSegRows - 1) / kSegRows) << 16);
  }
  __syncthreads();
  int packed_total = 0;
  block_exclusive_scan_512(first, E, warp_tot, packed_total);
  for (int e = tid; e < E; e += blockDim.x) {
    seg_first[e] = first[e] >> 16;
    first[e] &= 0xffff;
  }
  __syncthreads();
  const int total_ctas = packed_total & 0xffff, total_segs = packed_total >> 16;
  // the expert kernel's segment table lists the shared expert's segments first
  const int shared_segs = r.segs != nullptr && r.has_shared ? (T + kSegRows - 1) / kSegRows : 0;
  if (tid == 0) {
    r.record[0] = total_ctas * kTile;
    r.record[1] = total_ctas;
  }
  for (int s = tid; s < slots; s += blockDim.x) {
    const int t = s / K;
    const int e = slot_expert(s);
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
    if (r.segs != nullptr)  // the token of the row in its segment's list
      r.seg_tok[(shared_segs + seg_first[e] + rank / kSegRows) * kSegRows + rank % kSegRows] = t;
    if (rank % kTile == 0) {
      const int cta = first[e] + rank / kTile;
      r.record[4 + cta] = e;
      r.record[limit_off + cta] = min((cta + 1) * kTile, base_row + counts[e]);
    }
  }
  // expert-kernel work tables (shared expert's segments first)
  if (r.segs != nullptr) {
    for (int j = tid; j < shared_segs; j += blockDim.x) {
      const int rows = min(kSegRows, T - j * kSegRows);
      r.segs[j] = make_int4(-1, r.shared_row_base + j * kSegRows, rows, j * kSegRows);
    }
    for (int i = tid; i < shared_segs * kSegRows; i += blockDim.x) r.seg_tok[i] = i;  // the shared expert's rows: tokens in order
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
    // split-K of the gate_up tiles when they are fewer than the expert grid
    // (kMaxSplit in mm_layout.cuh): as many chunks as leave every down unit a
    // CTA of the first wave too (their weights stream while the gate_up chunks
    // run), else as many as fill the grid
    const int tiles1 = nseg * r.m1;
    const int units2 = nseg * r.m2;
    int split = 1;
    if (r.split_cnt != nullptr && tiles1 > 0 && tiles1 < r.grid) {
      split = (r.grid - units2) / tiles1;
      if (split < 2) split = r.grid / tiles1;
      split = max(1, min(min(kMaxSplit, split), r.ks1 / 2));
    }
    if (split > 1)
      for (int j = tid; j < 2 * tiles1; j += blockDim.x) r.split_cnt[j] = 0;
    if (tid == 0) {
      r.ctrl[kCtrlSegments] = nseg;
      r.ctrl[kCtrlSplit] = split;
      r.ctrl[kCtrlUnits] = nseg * (r.m1 * split + r.m2);
      r.ctrl[kCtrlClaim] = 0;
    }
  }
}

// The routed input's FP4 terms: 32-element chunks of x (one MXFP4 block or two
// NVFP4 blocks each), one chunk per warp and pass over the quantization CTAs
// (lane i: element i). x is bf16, or MXFP8 (x8 / s8: the reference's
// pre-quantized routed input, each value the exact E4M3 code times the block's
// E8M0 scale, one fp32 rounding).
__device__ __forceinline__ void quantize_x(const QuantArgs &a, int cta) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int blocks = a.hidden >> 5;
  const int chunks = a.tokens * blocks;
  const size_t q_stride = static_cast<size_t>(a.max_tokens) * (a.hidden >> 1);
#pragma unroll 1
  for (int idx = cta * warps + warp; idx < chunks; idx += a.ctas * warps) {
    const int t = idx / blocks, b = idx - t * blocks;
    const size_t e = static_cast<size_t>(idx) * 32 + lane;  // = t H + 32 b + lane
    const float v = a.x8 != nullptr ? __fmul_rn(e4m3_value(a.x8[e]), mx_scale_value(a.s8[idx]))
                                    : bf16_bits_to_float(a.x[e]);
    uint8_t *q = a.xq + static_cast<size_t>(t) * (a.hidden >> 1) + 16 * b;
    if (a.fmt == kFmtNv) {
      const size_t s_stride = static_cast<size_t>(a.max_tokens) * 2 * blocks;
      quantize_block16x2_nvfp4_warp(v, a.terms, a.gs, a.inv_gs, q, q_stride,
                                    a.xs + static_cast<size_t>(t) * 2 * blocks + 2 * b, s_stride);
    } else {
      const size_t s_stride = static_cast<size_t>(a.max_tokens) * blocks;
      quantize_block32_fp4_warp(v, a.terms, q, q_stride, a.xs + static_cast<size_t>(t) * blocks + b, s_stride);
    }
  }
}

// The front launch's body: grid = f.row_ctas row CTAs + f.quant.ctas, block
// 512. With a gate each of the T row CTAs ranks its row and the last to finish
// builds the route record and the work tables; with given ids (or one row) one
// row CTA builds them at once. The quantization CTAs (kQuant only) write the
// routed input's FP4 terms meanwhile, after the grid-dependency wait (the
// previous step's expert launch reads the same buffers); with no row CTAs the
// launch only quantizes. Dynamic shared memory: route_smem_size(T, experts).
template <class N, bool kQuant>
__device__ __forceinline__ void front_body(const FrontArgs &f, unsigned char *front_smem) {
  __shared__ GateSmem gsm;
  __shared__ int is_last;
  pdl_wait();
  if constexpr (kQuant) {
    if (static_cast<int>(blockIdx.x) >= f.row_ctas) {
      quantize_x(f.quant, blockIdx.x - f.row_ctas);
      return;
    }
  }
  const int row = blockIdx.x;
  if (f.gate.logits != nullptr) {
    const int valid = f.gate.num_valid != nullptr ? *f.gate.num_valid : f.route.tokens;
    gate_row<N>(f.gate, row, valid, gsm);
  }
  if (f.row_ctas == 1) {  // one row, or given ids: this CTA builds the route, no ticket
    __syncthreads();
    build_route(f.route, front_smem);
    return;
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // thread 0 (warp 0, lane 0) wrote the row's ids and weights
    __threadfence();
    const int ticket = atomicAdd(&f.route.ctrl[kCtrlTicket], 1);
    is_last = ticket == f.row_ctas - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  build_route(f.route, front_smem);
  if (threadIdx.x == 0) f.route.ctrl[kCtrlTicket] = 0;
}

}  // namespace mm
