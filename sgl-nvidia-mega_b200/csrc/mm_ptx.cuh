// Thin inline-PTX wrappers for sm_100a: programmatic dependent launch, mbarriers
// with bounded waits, TMA / bulk / cp.async copies, and the tcgen05 family
// (TMEM allocation, smem->TMEM copies, block-scaled MMA, commits, TMEM loads).
//
// Every wait here is bounded by the %globaltimer: on expiry it ORs a code into
// the layer's device error word and returns false, and every later wait of the
// launch sees the word set and gives up at once, so a launch that meets a
// missing producer ends with an error status instead of hanging the GPU.
#pragma once
#include <cstdint>

namespace mm {

// ---- error word codes (the host maps them to MM_ERR_DEVICE_TIMEOUT) -------
constexpr uint32_t kErrTimeoutFull = 1u << 0;    // smem stage never filled
constexpr uint32_t kErrTimeoutEmpty = 1u << 1;   // smem stage never released
constexpr uint32_t kErrTimeoutAcc = 1u << 2;     // accumulator hand-off stalled
constexpr uint32_t kErrTimeoutWork = 1u << 3;    // work ring hand-off stalled
constexpr uint32_t kErrTimeoutFlag = 1u << 4;    // gate_up segment never finished
constexpr uint32_t kErrBadUnit = 1u << 8;        // a work item failed its checks
constexpr uint32_t kErrTimeoutMask = 0xffu;

// The default budget of one bounded wait, 1.5 s: far above any legitimate wait
// of one launch, far below any watchdog. Layers and comms carry their own budget
// (mm_layer_set_wait_budget / mm_comm_set_wait_budget), passed to every wait.
constexpr uint64_t kWaitBudgetNs = 1500000000ull;
// The limit of a teardown drain (copies and MMAs this CTA issued, which complete
// in microseconds); a drain ignores the error word, so a launch that gave up
// still lets its own in-flight work land before it frees shared memory and TMEM.
constexpr uint64_t kDrainBudgetNs = 20000000ull;

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- programmatic dependent launch ---------------------------------------
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---- error word -------------------------------------------------------------
__device__ __forceinline__ bool error_set(const uint32_t *err) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(err) : "memory");
  return v != 0u;
}
__device__ __forceinline__ void error_raise(uint32_t *err, uint32_t code) {
  atomicOr(err, code);
}

// ---- mbarriers ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0u;
}
// Wait for the phase with this parity to complete; false (and the error word
// set) when `budget_ns` runs out or another wait of the launch already failed.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t *err,
                                          uint32_t code, uint64_t budget_ns = kWaitBudgetNs) {
#pragma unroll 1
  for (int i = 0; i < 256; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
#pragma unroll 1
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u) {
      if (error_set(err)) return false;
      if (globaltimer() - t0 > budget_ns) {
        error_raise(err, code);
        return false;
      }
    }
  }
}
// A teardown drain: wait for the phase regardless of the error word, at most
// kDrainBudgetNs; false when the limit ran out.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
#pragma unroll 1
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u && globaltimer() - t0 > kDrainBudgetNs) return false;
  }
}

// ---- L2 cache policies ----------------------------------------------------
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- TMA / bulk copies (no multicast anywhere in this library) -------------
__device__ __forceinline__ void tma_prefetch_desc(const void *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
// 3-D tiled load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void *map, int32_t c0, int32_t c1,
                                            int32_t c2, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(bar), "l"(policy)
      : "memory");
}
// Untiled bulk load (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                          uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}
// Ampere-style asynchronous copies; `src_bytes` 0 fills the destination with zeros.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
// Arrive on `bar` once this thread's earlier cp.async copies have landed; the
// barrier's expected count includes this arrival (noinc).
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 -----------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// 32 TMEM lanes x 128 bits, broadcast to the four lane quadrants (scale factors).
__device__ __forceinline__ void tc_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}
// D (+)= A * B with per-32 E8M0 scales for A (FP4/FP6/FP8) and B; one thread issues.
__device__ __forceinline__ void tc_mma_mxf8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                uint32_t idesc, uint32_t sfa_tmem,
                                                uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::
          "r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05 operation this thread issued has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}
// Warp-collective load of 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tc_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05 format, version 1).
//  bits [0,14) start >> 4, [16,30) leading byte offset >> 4,
//  [32,46) stride byte offset >> 4, [46,48) version = 1, [49,52) base offset,
//  [61,64) layout: 0 none (interleaved core matrices), 2 = 128-byte swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3fffu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}
constexpr uint32_t kLayoutNone = 0;
constexpr uint32_t kLayoutSw128 = 2;

// Instruction descriptor of kind::mxf8f6f4.block_scale: A E2M1 (5), B E4M3 (0),
// both K-major, E8M0 scales, M = 128, N = n; scale-factor byte ids per MMA.
__device__ __forceinline__ uint32_t idesc_mxf4_e4m3(uint32_t n, uint32_t a_sf_id,
                                                    uint32_t b_sf_id) {
  uint32_t d = 0;
  d |= (b_sf_id & 3u) << 4;
  d |= 5u << 7;             // A format E2M1
  d |= 0u << 10;            // B format E4M3
  d |= ((n >> 3) & 0x3fu) << 17;
  d |= 1u << 23;            // scale format E8M0
  d |= (128u >> 4) << 24;   // M = 128
  d |= (a_sf_id & 3u) << 29;
  return d;
}

// ---- small integer helpers ---------------------------------------------------
__host__ __device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace mm
