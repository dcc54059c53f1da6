// Runs the reference's route kernels on the CPU (TEST INFRASTRUCTURE; see
// ref_route_shim.h). ref_route() replays route.cu:23-37 (Clear, block sync,
// Zero, Build of route.cuh) with 64 threads; ref_route_wide() runs
// route_wide.cu's kernel with 512 threads. Built by `make -C oracle ref` from
// the reference tree in place; the result is the pin of the oracle's or_route.
#include <barrier>
#include <thread>
#include <vector>

#include "ref_route_shim.h"
#include "route.cuh"

thread_local ShimDim3 threadIdx;
static std::barrier<> *g_block = nullptr;
static std::barrier<> *g_warp[16] = {};
static int g_xchg[16][32];

void __syncthreads() { g_block->arrive_and_wait(); }

int __shfl_up_sync(unsigned, int value, unsigned offset) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  g_xchg[warp][lane] = value;
  g_warp[warp]->arrive_and_wait();
  const int r = lane >= static_cast<int>(offset) ? g_xchg[warp][lane - offset] : value;
  g_warp[warp]->arrive_and_wait();
  return r;
}

extern "C" void dsv41_routed_expert_route_wide(const int *ids, int *permuted, int *record, int rows,
                                               int top_k, int experts, int expert_offset);

template <typename F>
static void run_block(int threads, F body) {
  std::barrier<> block(threads);
  std::vector<std::barrier<> *> warps;
  for (int w = 0; w < threads / 32; ++w) warps.push_back(new std::barrier<>(32));
  g_block = &block;
  for (int w = 0; w < threads / 32; ++w) g_warp[w] = warps[w];
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t)
    pool.emplace_back([t, &body] {
      threadIdx = ShimDim3{static_cast<unsigned>(t), 0u, 0u};
      body(t);
    });
  for (auto &th : pool) th.join();
  for (auto *b : warps) delete b;
  g_block = nullptr;
}

extern "C" void ref_route(const int *ids, int *permuted, int *record, unsigned *barrier, int rows,
                          int top_k, int experts, int expert_offset) {
  constexpr int kThreads = 64;  // route.cu:18
  static route::Scratch scratch;
  run_block(kThreads, [&](int thread) {
    route::Clear(scratch, thread, kThreads);
    __syncthreads();
    route::Zero(record, rows, top_k, experts, thread, kThreads);
    route::Build(scratch, ids, permuted, record, barrier, rows, top_k, experts, expert_offset, thread);
  });
}

extern "C" void ref_route_wide(const int *ids, int *permuted, int *record, int rows, int top_k,
                               int experts, int expert_offset) {
  run_block(512, [&](int) {
    dsv41_routed_expert_route_wide(ids, permuted, record, rows, top_k, experts, expert_offset);
  });
}
