// CPU execution shim for the reference's route kernels (TEST INFRASTRUCTURE).
//
// Lets the reference's own CUDA source (route.cuh, route_wide.cu) compile with
// g++ and run one thread block as std::threads: threadIdx is thread-local,
// __shared__ variables become function-local statics shared by the block,
// __syncthreads is a block-wide std::barrier and __shfl_up_sync exchanges
// through a per-warp buffer between two warp-wide barriers.
#pragma once
#include <algorithm>
#include <barrier>
#include <cstdint>

#define __device__
#define __forceinline__ inline
#define __global__
#define __launch_bounds__(x)
#define __shared__ static
#define __restrict__ __restrict

struct ShimDim3 {
  unsigned x, y, z;
};
extern thread_local ShimDim3 threadIdx;

void __syncthreads();
int __shfl_up_sync(unsigned mask, int value, unsigned offset);

inline int __popc(unsigned v) { return __builtin_popcount(v); }
inline int __popcll(unsigned long long v) { return __builtin_popcountll(v); }
inline unsigned atomicOr(unsigned *p, unsigned v) { return __atomic_fetch_or(p, v, __ATOMIC_SEQ_CST); }
inline unsigned long long atomicOr(unsigned long long *p, unsigned long long v) {
  return __atomic_fetch_or(p, v, __ATOMIC_SEQ_CST);
}
inline unsigned atomicXor(unsigned *p, unsigned v) { return __atomic_fetch_xor(p, v, __ATOMIC_SEQ_CST); }
using std::min;
