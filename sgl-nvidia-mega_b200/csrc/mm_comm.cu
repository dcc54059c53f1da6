// K4 across GPUs: the weighted combine fused with the all-reduce of the ranks'
// partial outputs, over NVLink peer memory (plain P2P stores, no multicast).
//
// Every rank runs the same grid (T, ceil(H / 2048)); a CTA owns one tile of
// 8 x 256 features of one token. A thread computes its rank's partial of its 8
// features with the reference's per-rank rule (slot-order fp32 combine, round,
// + shared, round: all_reduce_mhc.py:528-640), stores it as one 16-byte store
// into its slot of the tile's mailbox on every peer, then polls its own
// mailbox until every peer's 8 values have landed and sums the world's
// partials in rank order in fp32 -> bf16 (the reference's reduce order,
// all_reduce_mhc.py:955-977). One launch replaces combine + all-reduce + round.
//
// Lamport mailbox (the reference's transport idea, all_reduce_mhc.py:11):
// an empty bf16 holds the sentinel -0 (0x8000), so the data is its own flag
// and no fence or separate signal is needed. Partials are sent with -0
// replaced by +0 (invisible in the rank-order sum, which starts at +0). A
// reader clears each value back to -0 right after reading it.
//
// Buffers (one cudaMalloc per rank, opened by the peers through CUDA IPC):
//   counters u32 [max_tokens * ceil(H / 2048)]  touches per tile slot
//   err      u32                                device error word
//   mbox     bf16 [2][world][max_tokens][hidden], two generations: touch n of
//            a tile slot uses generation n & 1. A peer writes touch n + 2 only
//            after it has read this rank's touch n + 1 partial, which this rank
//            sends after finishing touch n (its read and clear of that
//            generation). Both ranks see the same touches (every call has the
//            same token count on every rank), so the generations agree.
// After a timeout (error word set) mailboxes may hold stale values: rebuild
// the group's comms before the next call.
#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>

#include "megamoe.h"
#include "mm_kernels.cuh"
#include "mm_layout.cuh"
#include "mm_numerics.cuh"
#include "mm_ptx.cuh"

namespace mm {

constexpr int kMaxWorld = 16;
constexpr uint32_t kEmpty2 = 0x80008000u;  // two bf16 sentinels (-0, -0)

struct CommArgs {
  FinalizeArgs a;
  char *const *peers;   // device array [world]: every rank's buffer base (own included)
  uint32_t *counters;
  uint32_t *err;
  size_t off_mbox;
  int rank, world, max_tokens;
  // residual + RMSNorm epilogue (finalize_allreduce_kernel<true>)
  const uint16_t *residual, *gamma;
  uint16_t *residual_out, *norm_out;
  float eps;
  unsigned long long wait_ns;  // budget of the mailbox poll (mm_comm_set_wait_budget)
};

namespace {

__device__ __forceinline__ uint4 ld_volatile_v4(const void *p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_volatile_v4(void *p, const uint4 &v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__device__ __forceinline__ bool has_empty(uint32_t w) {
  return (w & 0xffffu) == 0x8000u || (w >> 16) == 0x8000u;
}

__device__ __forceinline__ uint32_t no_negative_zero(uint32_t w) {
  if ((w & 0xffffu) == 0x8000u) w &= 0xffff0000u;
  if ((w >> 16) == 0x8000u) w &= 0x0000ffffu;
  return w;
}

__device__ __forceinline__ void add_bf16x8(float acc[8], const uint4 &v) {
  const uint32_t q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc[2 * j] = __fadd_rn(acc[2 * j], __uint_as_float(q[j] << 16));
    acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], __uint_as_float(q[j] & 0xffff0000u));
  }
}

}  // namespace

// This rank's partial of 8 features (the per-rank combine rule), pushed to
// every peer's mailbox; then the rank-order fp32 sum of the world's partials.
__device__ __forceinline__ void combine_exchange(const CommArgs &c, int t, int h0, uint32_t gen, float sum[8]) {
  const FinalizeArgs &a = c.a;
  int perm[kMaxTopK];
  float wt[kMaxTopK];
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k) {
    perm[k] = k < a.top_k ? a.permuted[t * a.top_k + k] : -1;
    wt[k] = k < a.top_k ? a.weights[t * a.top_k + k] : 0.0f;
  }
  uint4 row[kMaxTopK];
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k)
    row[k] = perm[k] >= 0 ? *reinterpret_cast<const uint4 *>(a.rows + static_cast<size_t>(perm[k]) * a.hidden + h0)
                          : make_uint4(0u, 0u, 0u, 0u);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k) {
    if (perm[k] < 0) continue;
    const uint32_t q[4] = {row[k].x, row[k].y, row[k].z, row[k].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[2 * j] = __fmaf_rn(wt[k], __uint_as_float(q[j] << 16), acc[2 * j]);
      acc[2 * j + 1] = __fmaf_rn(wt[k], __uint_as_float(q[j] & 0xffff0000u), acc[2 * j + 1]);
    }
  }
  float sh[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) sh[i] = 0.0f;
  if (a.shared_rows != nullptr) {
    const uint4 v = *reinterpret_cast<const uint4 *>(a.shared_rows + static_cast<size_t>(t) * a.hidden + h0);
    const uint32_t q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sh[2 * j] = __uint_as_float(q[j] << 16);
      sh[2 * j + 1] = __uint_as_float(q[j] & 0xffff0000u);
    }
  }
  uint32_t packed[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float lo = __fadd_rn(bf16_bits_to_float(float_to_bf16_bits(acc[2 * j])), sh[2 * j]);
    const float hi = __fadd_rn(bf16_bits_to_float(float_to_bf16_bits(acc[2 * j + 1])), sh[2 * j + 1]);
    packed[j] = no_negative_zero(static_cast<uint32_t>(float_to_bf16_bits(lo)) |
                                 (static_cast<uint32_t>(float_to_bf16_bits(hi)) << 16));
  }
  const uint4 mine = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  const size_t gen_base = static_cast<size_t>(gen) * c.world;
  const size_t my_slot = ((gen_base + c.rank) * c.max_tokens + t) * a.hidden + h0;
  for (int q = 0; q < c.world; ++q) {
    if (q == c.rank) continue;
    uint16_t *dst = reinterpret_cast<uint16_t *>(c.peers[q] + c.off_mbox) + my_slot;
    st_volatile_v4(dst, mine);
  }
  uint16_t *mbox = reinterpret_cast<uint16_t *>(c.peers[c.rank] + c.off_mbox);
#pragma unroll
  for (int i = 0; i < 8; ++i) sum[i] = 0.0f;
  const uint64_t t0 = globaltimer();
  for (int s = 0; s < c.world; ++s) {
    if (s == c.rank) {
      add_bf16x8(sum, mine);
      continue;
    }
    uint16_t *src = mbox + ((gen_base + s) * c.max_tokens + t) * a.hidden + h0;
    uint4 v = ld_volatile_v4(src);
#pragma unroll 1
    for (uint32_t i = 0; has_empty(v.x) || has_empty(v.y) || has_empty(v.z) || has_empty(v.w); ++i) {
      if ((i & 31u) == 31u && (error_set(c.err) || globaltimer() - t0 > c.wait_ns)) {
        error_raise(c.err, kErrTimeoutFlag);
        break;
      }
      v = ld_volatile_v4(src);
    }
    add_bf16x8(sum, v);
    st_volatile_v4(src, make_uint4(kEmpty2, kEmpty2, kEmpty2, kEmpty2));
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float v[8]) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    w[j] = static_cast<uint32_t>(float_to_bf16_bits(v[2 * j])) |
           (static_cast<uint32_t>(float_to_bf16_bits(v[2 * j + 1])) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void unpack_bf16x8(const uint4 &v, float f[8]) {
  const uint32_t q[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(q[j] << 16);
    f[2 * j + 1] = __uint_as_float(q[j] & 0xffff0000u);
  }
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float ld_cluster_f32(const float *local, uint32_t cta) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(local));
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(cta));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
  return v;
}

// grid (T, Y = ceil(H / 2048)), 256 threads; kNorm: launched as clusters of
// (1, Y, 1), one cluster per token row, whose CTAs fold the row's sum of
// squares through distributed shared memory.
template <bool kNorm>
__global__ void __launch_bounds__(256) finalize_allreduce_kernel(CommArgs c) {
  pdl_launch_dependents();
  const int t = blockIdx.x;
  const int h0 = (blockIdx.y * 256 + threadIdx.x) * 8;
  const bool active = h0 < c.a.hidden;
  uint4 gam_bits = make_uint4(0u, 0u, 0u, 0u);
  if (kNorm && active && c.gamma != nullptr)  // a weight: read before the wait
    gam_bits = *reinterpret_cast<const uint4 *>(c.gamma + h0);
  pdl_wait();
  // a tile is keyed by its slot (token, feature block), not by the launch's
  // shape, so every slot's generations alternate across calls of any token count
  const int bid = blockIdx.x + c.max_tokens * blockIdx.y;
  __shared__ uint32_t s_cnt;
  if (threadIdx.x == 0) s_cnt = c.counters[bid];
  __syncthreads();
  const uint32_t gen = s_cnt & 1u;
  if (threadIdx.x == 0) c.counters[bid] = s_cnt + 1u;
  float sum[8];
  if (active) combine_exchange(c, t, h0, gen, sum);
  const size_t o = static_cast<size_t>(t) * c.a.hidden + h0;
  if constexpr (!kNorm) {
    if (active) *reinterpret_cast<uint4 *>(c.a.out + o) = pack_bf16x8(sum);
  } else {
    // pre = bf16(sum + residual); the row's sum of squares in the fixed fold:
    // thread (8 features in order), warp (xor butterfly 16..1), CTA (warps in
    // order), row (CTAs in order)
    float pre[8];
    float sq = 0.0f;
    if (active) {
      float res[8];
      unpack_bf16x8(*reinterpret_cast<const uint4 *>(c.residual + o), res);
#pragma unroll
      for (int e = 0; e < 8; ++e) pre[e] = __fadd_rn(sum[e], res[e]);
      const uint4 p = pack_bf16x8(pre);
      *reinterpret_cast<uint4 *>(c.residual_out + o) = p;
      unpack_bf16x8(p, pre);
#pragma unroll
      for (int e = 0; e < 8; ++e) sq = __fadd_rn(sq, __fmul_rn(pre[e], pre[e]));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, off));
    __shared__ float s_warp[8];
    __shared__ float s_cta;
    if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
      float v = 0.0f;
#pragma unroll
      for (int w = 0; w < 8; ++w) v = __fadd_rn(v, s_warp[w]);
      s_cta = v;
    }
    cluster_sync_all();
    float total = 0.0f;
    for (uint32_t y = 0; y < gridDim.y; ++y) total = __fadd_rn(total, ld_cluster_f32(&s_cta, y));
    cluster_sync_all();  // no CTA leaves while a peer may still read its s_cta
    if (active && c.norm_out != nullptr) {
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(c.a.hidden)), c.eps)));
      float gam[8], nv[8];
      unpack_bf16x8(gam_bits, gam);
#pragma unroll
      for (int e = 0; e < 8; ++e) nv[e] = __fmul_rn(__fmul_rn(pre[e], inv), gam[e]);
      *reinterpret_cast<uint4 *>(c.norm_out + o) = pack_bf16x8(nv);
    }
  }
}

__global__ void fill_u32_kernel(uint32_t *p, size_t n, uint32_t v) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    p[i] = v;
}

}  // namespace mm

using namespace mm;

struct mm_comm {
  int rank, world, max_tokens, hidden, device, max_blocks;
  unsigned long long wait_ns = kWaitBudgetNs;
  bool ipc_opened = false;  // the peers' buffers are CUDA IPC mappings (closed at destroy)
  char *base = nullptr;
  size_t bytes = 0, off_counters = 0, off_err = 0, off_mbox = 0;
  char *peer[kMaxWorld] = {};
  char **peer_table = nullptr;  // device copy of peer[]
  bool opened = false;
};

static_assert(sizeof(cudaIpcMemHandle_t) == MM_IPC_HANDLE_BYTES, "IPC handle size");

static int launch_comm(mm_comm *c, const char *what, const uint16_t *rows, const float *weights,
                       const int32_t *permuted, const uint16_t *shared_rows, uint16_t *out, const uint16_t *residual,
                       const uint16_t *gamma, float eps, uint16_t *residual_out, uint16_t *norm_out, int tokens,
                       int top_k, int hidden, void *stream) {
  const bool norm = residual != nullptr;
  if (!c || !rows || !weights || !permuted) return set_error(MM_ERR_INVALID, "%s: null pointer", what);
  if (!c->opened) return set_error(MM_ERR_INVALID, "%s: peers not opened (mm_comm_open)", what);
  if (tokens < 1 || tokens > c->max_tokens || hidden != c->hidden || top_k < 1 || top_k > kMaxTopK)
    return set_error(MM_ERR_INVALID, "%s: tokens %d (<= %d), hidden %d (== %d), top_k %d", what, tokens,
                     c->max_tokens, hidden, c->hidden, top_k);
  const int ctas = (hidden + 2047) / 2048;
  if (norm && ctas > 8) return set_error(MM_ERR_UNSUPPORTED, "%s: hidden %d > 16384", what, hidden);
  const uintptr_t bits = reinterpret_cast<uintptr_t>(rows) | reinterpret_cast<uintptr_t>(out) |
                         reinterpret_cast<uintptr_t>(shared_rows) | reinterpret_cast<uintptr_t>(residual) |
                         reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(residual_out) |
                         reinterpret_cast<uintptr_t>(norm_out);
  if (bits % 16) return set_error(MM_ERR_INVALID, "%s: buffers must be 16-byte aligned", what);
  CommArgs a;
  a.a = FinalizeArgs{rows, weights, permuted, shared_rows, out, nullptr, tokens, top_k, hidden};
  a.peers = c->peer_table;
  a.counters = reinterpret_cast<uint32_t *>(c->base + c->off_counters);
  a.err = reinterpret_cast<uint32_t *>(c->base + c->off_err);
  a.off_mbox = c->off_mbox;
  a.rank = c->rank;
  a.world = c->world;
  a.max_tokens = c->max_tokens;
  a.residual = residual;
  a.gamma = gamma;
  a.residual_out = residual_out;
  a.norm_out = norm_out;
  a.eps = eps;
  a.wait_ns = c->wait_ns;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tokens, ctas);
  cfg.blockDim = dim3(256);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = ctas;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = norm ? 2 : 1;
  cudaError_t e = cudaSetDevice(c->device);
  if (e == cudaSuccess)
    e = norm ? cudaLaunchKernelEx(&cfg, finalize_allreduce_kernel<true>, a)
             : cudaLaunchKernelEx(&cfg, finalize_allreduce_kernel<false>, a);
  if (e != cudaSuccess) return set_error(MM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return MM_OK;
}

extern "C" {

int mm_comm_create(int32_t rank, int32_t world, int32_t max_tokens, int32_t hidden, int32_t device,
                   mm_comm **out) {
  if (!out) return set_error(MM_ERR_INVALID, "mm_comm_create: null pointer");
  *out = nullptr;
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world)
    return set_error(MM_ERR_INVALID, "mm_comm_create: rank %d of world %d (world <= %d)", rank, world, kMaxWorld);
  if (max_tokens < 1 || max_tokens > kMaxTokens || hidden < 8 || hidden % 8)
    return set_error(MM_ERR_INVALID, "mm_comm_create: max_tokens %d, hidden %d", max_tokens, hidden);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return set_error(MM_ERR_CUDA, "mm_comm_create: cudaSetDevice: %s", cudaGetErrorString(e));
  mm_comm *c = new mm_comm();
  c->rank = rank;
  c->world = world;
  c->max_tokens = max_tokens;
  c->hidden = hidden;
  c->device = device;
  c->max_blocks = max_tokens * ((hidden + 2047) / 2048);
  auto align = [](size_t v) { return (v + 255) & ~static_cast<size_t>(255); };
  c->off_counters = 0;
  c->off_err = align(c->off_counters + sizeof(uint32_t) * c->max_blocks);
  c->off_mbox = align(c->off_err + sizeof(uint32_t));
  const size_t mbox_words = static_cast<size_t>(world) * max_tokens * hidden;  // 2 generations x 2 B
  c->bytes = align(c->off_mbox + sizeof(uint32_t) * mbox_words);
  e = cudaMalloc(reinterpret_cast<void **>(&c->base), c->bytes);
  if (e == cudaSuccess) e = cudaMemset(c->base, 0, c->off_mbox);
  if (e == cudaSuccess) {
    fill_u32_kernel<<<296, 256>>>(reinterpret_cast<uint32_t *>(c->base + c->off_mbox), mbox_words, kEmpty2);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&c->peer_table), sizeof(char *) * world);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->base) cudaFree(c->base);
    if (c->peer_table) cudaFree(c->peer_table);
    delete c;
    return set_error(MM_ERR_CUDA, "mm_comm_create: %s", cudaGetErrorString(e));
  }
  c->peer[rank] = c->base;
  *out = c;
  return MM_OK;
}

int mm_comm_handle(const mm_comm *c, void *handle) {
  if (!c || !handle) return set_error(MM_ERR_INVALID, "mm_comm_handle: null pointer");
  cudaError_t e = cudaSetDevice(c->device);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->base);
  if (e != cudaSuccess) return set_error(MM_ERR_CUDA, "mm_comm_handle: %s", cudaGetErrorString(e));
  memcpy(handle, &h, sizeof(h));
  return MM_OK;
}

int mm_comm_open(mm_comm *c, const void *handles) {
  if (!c || !handles) return set_error(MM_ERR_INVALID, "mm_comm_open: null pointer");
  if (c->opened) return set_error(MM_ERR_INVALID, "mm_comm_open: already open");
  cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return set_error(MM_ERR_CUDA, "mm_comm_open: %s", cudaGetErrorString(e));
  for (int q = 0; q < c->world; ++q) {
    if (q == c->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const char *>(handles) + static_cast<size_t>(q) * MM_IPC_HANDLE_BYTES, sizeof(h));
    void *p = nullptr;
    e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int r = 0; r < q; ++r)
        if (r != c->rank && c->peer[r]) {
          cudaIpcCloseMemHandle(c->peer[r]);
          c->peer[r] = nullptr;
        }
      return set_error(MM_ERR_CUDA, "mm_comm_open: rank %d's buffer: %s", q, cudaGetErrorString(e));
    }
    c->peer[q] = static_cast<char *>(p);
  }
  c->ipc_opened = true;
  e = cudaMemcpy(c->peer_table, c->peer, sizeof(char *) * c->world, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return set_error(MM_ERR_CUDA, "mm_comm_open: %s", cudaGetErrorString(e));
  c->opened = true;
  return MM_OK;
}

int mm_comm_open_local(mm_comm *c, mm_comm *const *members) {
  if (!c || !members) return set_error(MM_ERR_INVALID, "mm_comm_open_local: null pointer");
  if (c->opened) return set_error(MM_ERR_INVALID, "mm_comm_open_local: already open");
  for (int q = 0; q < c->world; ++q) {
    const mm_comm *m = members[q];
    if (!m || m->rank != q || m->world != c->world || m->max_tokens != c->max_tokens || m->hidden != c->hidden)
      return set_error(MM_ERR_INVALID, "mm_comm_open_local: member %d does not belong to this group", q);
    if (q == c->rank && m != c) return set_error(MM_ERR_INVALID, "mm_comm_open_local: member %d is not this comm", q);
  }
  cudaError_t e = cudaSetDevice(c->device);
  for (int q = 0; q < c->world && e == cudaSuccess; ++q) {
    const int dev = members[q]->device;
    if (dev == c->device) continue;
    int can = 0;
    e = cudaDeviceCanAccessPeer(&can, c->device, dev);
    if (e == cudaSuccess && !can)
      return set_error(MM_ERR_UNSUPPORTED, "mm_comm_open_local: device %d cannot reach device %d", c->device, dev);
    if (e == cudaSuccess) {
      e = cudaDeviceEnablePeerAccess(dev, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        e = cudaSuccess;
      }
    }
  }
  if (e != cudaSuccess) return set_error(MM_ERR_CUDA, "mm_comm_open_local: %s", cudaGetErrorString(e));
  for (int q = 0; q < c->world; ++q) c->peer[q] = members[q]->base;
  e = cudaMemcpy(c->peer_table, c->peer, sizeof(char *) * c->world, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return set_error(MM_ERR_CUDA, "mm_comm_open_local: %s", cudaGetErrorString(e));
  c->opened = true;
  return MM_OK;
}

int mm_comm_set_wait_budget(mm_comm *c, int64_t microseconds) {
  if (!c) return set_error(MM_ERR_INVALID, "mm_comm_set_wait_budget: null comm");
  if (microseconds < 1 || microseconds > 60000000)
    return set_error(MM_ERR_INVALID, "mm_comm_set_wait_budget: %lld us outside 1..60000000",
                     static_cast<long long>(microseconds));
  c->wait_ns = static_cast<unsigned long long>(microseconds) * 1000ull;
  return MM_OK;
}

int mm_comm_destroy(mm_comm *c) {
  if (!c) return MM_OK;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int q = 0; q < c->world; ++q)
    if (c->ipc_opened && q != c->rank && c->peer[q]) cudaIpcCloseMemHandle(c->peer[q]);
  if (c->peer_table) cudaFree(c->peer_table);
  if (c->base) cudaFree(c->base);
  delete c;
  return MM_OK;
}

int mm_comm_check(mm_comm *c) {
  if (!c) return set_error(MM_ERR_INVALID, "mm_comm_check: null pointer");
  cudaError_t e = cudaSetDevice(c->device);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  uint32_t word = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&word, c->base + c->off_err, sizeof(word), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_error(MM_ERR_CUDA, "mm_comm_check: %s", cudaGetErrorString(e));
  if (word == 0) return MM_OK;
  cudaMemset(c->base + c->off_err, 0, sizeof(uint32_t));
  return set_error(MM_ERR_DEVICE_TIMEOUT, "a peer's partial never arrived (error word 0x%x); rebuild the group's comms", word);
}

int mm_finalize_allreduce(mm_comm *c, const uint16_t *rows, const float *weights, const int32_t *permuted,
                          const uint16_t *shared_rows, uint16_t *out, int32_t tokens, int32_t top_k,
                          int32_t hidden, void *stream) {
  if (!out) return set_error(MM_ERR_INVALID, "mm_finalize_allreduce: null out");
  return launch_comm(c, "mm_finalize_allreduce", rows, weights, permuted, shared_rows, out, nullptr, nullptr, 0.0f,
                     nullptr, nullptr, tokens, top_k, hidden, stream);
}

int mm_finalize_allreduce_norm(mm_comm *c, const uint16_t *rows, const float *weights, const int32_t *permuted,
                               const uint16_t *shared_rows, const uint16_t *residual, const uint16_t *gamma,
                               float eps, uint16_t *residual_out, uint16_t *norm_out, int32_t tokens,
                               int32_t top_k, int32_t hidden, void *stream) {
  if (!residual || !residual_out) return set_error(MM_ERR_INVALID, "mm_finalize_allreduce_norm: null residual");
  if (norm_out && !gamma) return set_error(MM_ERR_INVALID, "mm_finalize_allreduce_norm: norm_out needs gamma");
  if (!(eps >= 0.0f)) return set_error(MM_ERR_INVALID, "mm_finalize_allreduce_norm: eps %g", eps);
  return launch_comm(c, "mm_finalize_allreduce_norm", rows, weights, permuted, shared_rows, nullptr, residual, gamma,
                     eps, residual_out, norm_out, tokens, top_k, hidden, stream);
}

}  // extern "C"
