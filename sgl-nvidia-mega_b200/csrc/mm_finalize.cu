// K4: the weighted combine (deferred finalize).
//   out[t] = bf16( bf16( sum_k w[t,k] * rows[perm[t,k]] ) + shared[t] )
// accumulated in fp32 in slot order k = 0, 1, ... (acc = fma(w, row, acc) from
// acc = 0), slots with perm = -1 (experts another rank holds) skipped.
// Reference: deepseek_v41/sm103/all_reduce_mhc.py:528-640 (slot-order fp32 sum,
// round_routed, + shared, round) and glm5_3/sm103/moe/finalize.py:1-27.
// The reference's -0 -> +0 sanitizing belongs to its Lamport mailbox transport
// and is not part of the arithmetic here.
#include <cstdint>
#include <cuda_runtime.h>

#include "mm_kernels.cuh"
#include "mm_layout.cuh"
#include "mm_numerics.cuh"
#include "mm_ptx.cuh"

namespace mm {

// grid (T, ceil(H / 2048)), block 256; a thread owns 8 consecutive features.
__global__ void __launch_bounds__(256) finalize_kernel(FinalizeArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  const int h0 = (blockIdx.y * 256 + threadIdx.x) * 8;
  if (h0 >= a.hidden) return;
  // every slot's row index and weight first, then every row load, then the
  // slot-order accumulation (the loads are independent; the order is not)
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
  const size_t o = static_cast<size_t>(t) * a.hidden + h0;
  if (a.partial != nullptr) {
    float4 *r = reinterpret_cast<float4 *>(a.partial + o);
    float4 *s = reinterpret_cast<float4 *>(a.partial + static_cast<size_t>(a.tokens) * a.hidden + o);
    r[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    r[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    s[0] = make_float4(sh[0], sh[1], sh[2], sh[3]);
    s[1] = make_float4(sh[4], sh[5], sh[6], sh[7]);
  }
  if (a.out != nullptr) {
    uint32_t packed[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = __fadd_rn(bf16_bits_to_float(float_to_bf16_bits(acc[2 * j])), sh[2 * j]);
      const float hi = __fadd_rn(bf16_bits_to_float(float_to_bf16_bits(acc[2 * j + 1])), sh[2 * j + 1]);
      packed[j] = static_cast<uint32_t>(float_to_bf16_bits(lo)) |
                  (static_cast<uint32_t>(float_to_bf16_bits(hi)) << 16);
    }
    *reinterpret_cast<uint4 *>(a.out + o) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
}

// out = bf16(bf16(partial[0]) + partial[1]) after a cross-rank sum of the partials.
__global__ void __launch_bounds__(256) finalize_partial_kernel(const float *__restrict__ partial,
                                                               uint16_t *__restrict__ out, int tokens,
                                                               int hidden) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t n = static_cast<size_t>(tokens) * hidden;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float r = bf16_bits_to_float(float_to_bf16_bits(partial[i]));
    out[i] = float_to_bf16_bits(__fadd_rn(r, partial[n + i]));
  }
}

}  // namespace mm
