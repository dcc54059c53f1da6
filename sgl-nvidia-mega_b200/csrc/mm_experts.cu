// The persistent expert kernel (K2 + K3): every routed expert's gate_up GEMM
// with the SwiGLU (+ clamp) and MXFP4-terms requant epilogue, then every
// expert's down GEMM, in one launch of two CTAs per SM (kCtasPerSm).
//
// Work: a segment is up to 16 consecutive permuted rows of one expert (the
// shared expert's tokens form segments too). A gate_up unit streams one 128-row
// tile of w13 (64 gate rows + the 64 matching up rows) through all of H, or
// through one of `split` K chunks of H when the step has fewer gate_up tiles
// than the grid (split-K, mm_layout.cuh), and multiplies it with the segment's
// rows; a down unit streams one 128-row tile of w2 (or two, for narrow MXFP4
// slices) through all of I. Units are numbered [all gate_up units][all down units];
// CTA b runs unit b first and then claims units from a global counter, so
// every gate_up unit is taken before any later down unit; a down unit's
// activations wait on its segment's mailbox (the number of finished gate_up
// warps), while its weights stream before that wait.
// Reference semantics: gemm1.cu:6-7 (h = MX(clamped SwiGLU(x W13^T))),
// gemm2.cu:6-7 (rows = h W2^T in bf16, deferred-finalize rows).
//
// Arithmetic: tcgen05.mma kind::mxf4 block32 (E2M1 x E2M1, an E8M0 scale per 32
// along K for both operands), M = 128 weight rows, N = terms * n activation
// rows, K = 64 per instruction, fp32 accumulators in TMEM. The activations are
// carried as MXFP4 terms (see quantize_block32_fp4_warp), each term in its own
// accumulator columns; the epilogue adds the terms.
//
// Warp roles (224 threads):
//   warp 0    producer: claims units, TMA-loads packed weight tiles (128-byte rows,
//             128-byte swizzle) and bulk-loads the pre-laid scale chunks;
//   warp 1    MMA: TMEM owner; copies scale chunks to TMEM (tcgen05.cp) and issues
//             the MMAs, one thread;
//   warp 2    B loader: gathers the segment's activation terms with cp.async into
//             the 128-byte-swizzled K-major layout;
//   warps 3-6 epilogue: TMEM -> registers; SwiGLU + requant (gate_up) or bf16 rows
//             (down).
// No TMA multicast is used anywhere (one CTA per cluster).
#include <cstdint>
#include <cuda_runtime.h>

#include "mm_kernels.cuh"
#include "mm_layout.cuh"
#include "mm_numerics.cuh"
#include "mm_ptx.cuh"

namespace mm {

namespace {

constexpr uint32_t kATxBytes = kAStageBytes;  // packed codes land as they are

// Unit u: gate_up units [0, nseg m1 split) (segment, 128-row gate_up tile m, K
// chunk c), then down units (segment, down unit m covering w2 tiles
// [m tg2, m tg2 + tg2); c = 0).
__device__ __forceinline__ void decode_unit(int u, int nseg, int m1, int split, int m2, bool &g2, int &seg,
                                            int &m, int &c) {
  const int per1 = m1 * split;
  const int n1 = nseg * per1;
  if (u < n1) {
    g2 = false;
    seg = u / per1;
    const int r = u - seg * per1;
    m = r / split;
    c = r - m * split;
  } else {
    g2 = true;
    c = 0;
    const int v = u - n1;
    seg = v / m2;
    m = v - seg * m2;
  }
}

// The K stages of a unit: [k0, k0 + n) of ks_u for gate_up chunk c of `split`;
// a down unit's tiles one after the other (tiles x ks_u stages from 0).
__device__ __forceinline__ void unit_stages(bool g2, int c, int split, int ks_u, int tiles, int &k0, int &n) {
  if (g2) {
    k0 = 0;
    n = tiles * ks_u;
  } else {
    k0 = c * ks_u / split;
    n = (c + 1) * ks_u / split - k0;
  }
}

__device__ __forceinline__ int ld_acquire(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Split-K count-in of a one- or two-row segment: one acquire-release atomic on
// lane 0, between two warp barriers. The warp barrier before it orders the
// other lanes' partial-sum stores before lane 0's release (release is
// cumulative); the one after it orders their loads of the other chunks'
// partials after lane 0's acquire.
__device__ __forceinline__ int atom_add_acq_rel(int *p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Mailbox increments that complete one gate_up tile of a segment: one per half
// of the tile's features (its SwiGLU warp, or a split-K tile's last warp of
// the half when the segment has one or two rows), or one per epilogue warp of
// every chunk when a split-K tile's rows are shared out.
__device__ __forceinline__ int tile_publishes(int split, int rows) { return split > 1 && rows > 2 ? 4 * split : 2; }

__device__ __forceinline__ int ld_shared_volatile(const int *p) {
  return *reinterpret_cast<const volatile int *>(p);
}

// The segment descriptor of unit work, cached across a role's consecutive units
// of the same segment (a run of short units would otherwise wait on one L2
// round trip per unit for it).
struct SegCache {
  int seg = -1;
  int4 sg;
  __device__ __forceinline__ const int4 &get(const int4 *segs, int s) {
    if (s != seg) {
      sg = segs[s];
      seg = s;
    }
    return sg;
  }
};

// Wait until `flag` >= target; false (and the error word set) when `budget_ns`
// runs out or another wait of the launch already failed.
__device__ bool wait_flag(const int *flag, int target, uint32_t *err, uint64_t budget_ns) {
  if (ld_acquire(flag) >= target) return true;
  const uint64_t t0 = globaltimer();
#pragma unroll 1
  for (uint32_t i = 0;; ++i) {  // each poll is an L2 round trip: no sleep between them
    if (ld_acquire(flag) >= target) return true;
    if ((i & 15u) == 0u) {
      if (error_set(err)) return false;
      if (globaltimer() - t0 > budget_ns) {
        error_raise(err, kErrTimeoutFlag);
        return false;
      }
    }
  }
}

// Instruction descriptor of kind::mxf4 block32: A and B E2M1 (format 1), both
// K-major, E8M0 scales, M = 128, N = n, K = 64; scale-factor byte id 0 or 2
// (each MMA consumes two consecutive scale bytes per row).
__device__ __forceinline__ uint32_t idesc_mxf4(uint32_t n, uint32_t sf_id) {
  uint32_t d = 0;
  d |= (sf_id & 3u) << 4;   // B scale-factor id
  d |= 1u << 7;             // A format E2M1
  d |= 1u << 10;            // B format E2M1
  d |= ((n >> 3) & 0x3fu) << 17;
  d |= 1u << 23;            // scale format E8M0
  d |= (128u >> 4) << 24;   // M = 128
  d |= (sf_id & 3u) << 29;  // A scale-factor id
  return d;
}

__device__ __forceinline__ void mma_mxf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::
          "r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}

// Instruction descriptor of kind::mxf4nvf4 block16: A and B E2M1 (format 1),
// both K-major, E4M3 scales (scale format 0), M = 128, N = n, K = 64; each MMA
// consumes four scale bytes per row (scale-factor id 0).
__device__ __forceinline__ uint32_t idesc_nvf4(uint32_t n) {
  uint32_t d = 0;
  d |= 1u << 7;             // A format E2M1
  d |= 1u << 10;            // B format E2M1
  d |= ((n >> 3) & 0x3fu) << 17;
  d |= (128u >> 4) << 24;   // M = 128
  return d;
}

__device__ __forceinline__ void mma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::
          "r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}

}  // namespace

// kTg2: down tiles per down unit (p.tg2; 2 only for MXFP4 layers with one or two K
// stages per down tile), a template argument so single-tile layers run the plain loop.
template <int F, int kTg2>
__global__ void __launch_bounds__(kExpertThreads, kCtasPerSm) expert_kernel(const __grid_constant__ ExpertArgs p) {
  using L = Fmt<F>;
  static_assert(kTg2 == 1 || (kTg2 == 2 && L::kAccCols >= 2 * kBRows), "two-tile units need double-width accumulators");
  constexpr bool kNv = F == kFmtNv;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char *sbase = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t bars = base + L::kSmemBar;
  auto bar = [&](int i) -> uint32_t { return bars + 8u * static_cast<uint32_t>(i); };
  int *work_ids = reinterpret_cast<int *>(sbase + L::kSmemWorkIds);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sbase + L::kSmemTmemBase);
  uint32_t *err = p.err;
  const uint64_t wb = p.wait_ns;  // budget of every bounded wait below

  pdl_launch_dependents();

  // ---- set-up ----------------------------------------------------------------
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarFull + s), 1 + 32);  // producer's expect_tx + 32 loader lanes
      mbar_init(bar(kBarEmpty + s), 1);      // MMA commit
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar(kBarAccFull + a), 1);
      mbar_init(bar(kBarAccEmpty + a), 4);
    }
    for (int w = 0; w < kWorkSlots; ++w) {
      mbar_init(bar(kBarWorkFull + w), 1);
      mbar_init(bar(kBarWorkEmpty + w), 6);
    }
    mbar_init(bar(kBarDrain), 1);
    mbar_init(bar(kBarExFull), 2);  // the two up-row warps
    mbar_init(bar(kBarExFree), 2);  // the two gate-row warps
    fence_barrier_init();
  }
  {  // zero the activation and scale areas once: rows a unit does not load stay finite
    uint4 *z = reinterpret_cast<uint4 *>(sbase + L::kSmemB);
    const int n16 = (L::kSmemEpi - L::kSmemB) / 16;
    for (int i = threadIdx.x; i < n16; i += blockDim.x) z[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *reinterpret_cast<volatile uint32_t *>(tmem_slot);

  if (warp == 0) {
    // =========================== producer ===================================
    if (lane == 0) {
      tma_prefetch_desc(&p.w13_map);
      tma_prefetch_desc(&p.w2_map);
      tma_prefetch_desc(&p.sw13_map);
      tma_prefetch_desc(&p.sw2_map);
      pdl_wait();
      const int nseg = p.ctrl[kCtrlSegments];
      const int total = p.ctrl[kCtrlUnits];
      const int split = p.ctrl[kCtrlSplit];
      const uint64_t policy = policy_evict_first();
      uint32_t stage = 0, phase = 0, ws = 0, wphase = 0;
      // CTA b's first unit is unit b, unclaimed: the first wave gives every CTA
      // exactly one unit (with claims, a CTA could take two long gate_up units
      // while another took two short down units). Later units come from the
      // counter, offset by the grid, in batches of max(1, 8 / stages)
      // consecutive units: one claim per about eight stages of loads, so a run
      // of one-stage down units (narrow tensor-parallel slices) does not wait on
      // a claim's round trip per unit. The next batch is claimed three stages
      // before the last load of the current batch's last-but-one unit, so the
      // round trip hides behind the stages in flight, and a CTA takes units
      // only shortly before it runs them.
      SegCache seg_cache;
      int cur = static_cast<int>(blockIdx.x);
      int a_next = total, a_end = total;  // the current batch's units not yet started
      int b_next = total, b_end = total;  // the next batch, once claimed
      bool b_claimed = false;
      bool ok = true;
      int filled = 0;  // stages filled (the drain waits for the last ring's copies to land)
#pragma unroll 1
      while (ok) {
        const int u = cur;
        const bool have = u < total;
        cur = total;
        if (!mbar_wait(bar(kBarWorkEmpty + ws), wphase ^ 1u, err, kErrTimeoutWork, wb)) break;
        work_ids[ws] = have ? u : -1;
        mbar_arrive(bar(kBarWorkFull + ws));
        if (++ws == kWorkSlots) { ws = 0; wphase ^= 1u; }
        if (!have) break;
        bool g2;
        int seg, m, c;
        decode_unit(u, nseg, p.m1, split, p.u2, g2, seg, m, c);
        const int4 sg = seg_cache.get(p.segs, seg);
        const int e = sg.x < 0 ? 0 : sg.x;
        const bool sh = sg.x < 0;
        const CUtensorMap *map = g2 ? (sh ? &p.sw2_map : &p.w2_map) : (sh ? &p.sw13_map : &p.w13_map);
        // a down unit's stages run over its tiles, K stages within a tile; the
        // tiles' scale chunks are consecutive ([expert][tile][K stage]); a
        // gate_up chunk's stages are [k0, k0 + ks_n) of its tile
        const int ks_u = g2 ? p.ks2 : p.ks1;
        const int t0 = g2 ? m * kTg2 : m;
        int k0, ks_n;
        unit_stages(g2, c, split, ks_u, kTg2 == 1 ? 1 : min(kTg2, p.m2 - t0), k0, ks_n);
        const uint8_t *sfa = g2 ? (sh ? p.ssfa2 : p.sfa2) : (sh ? p.ssfa13 : p.sfa13);
        sfa += ((static_cast<size_t>(e) * (g2 ? p.m2 : p.m1) + t0) * static_cast<size_t>(ks_u) + k0) *
               L::kSfStageBytes;
        const int claim_at = ks_n > 3 ? ks_n - 3 : 0;
        const bool refill = !b_claimed && a_end - a_next <= 1;
        int tt = 0, kq = k0;  // tile of the unit (down units) and K stage within it
#pragma unroll 1
        for (int ks = 0; ks < ks_n; ++ks) {
          if (refill && ks == claim_at) {
            const int batch = ks_n >= 8 ? 1 : 8 / ks_n;
            b_next = static_cast<int>(gridDim.x) + atomicAdd(&p.ctrl[kCtrlClaim], batch);
            b_end = b_next + batch;
            b_claimed = true;
          }
          if (filled >= kStages && !mbar_wait(bar(kBarEmpty + stage), phase ^ 1u, err, kErrTimeoutEmpty, wb)) {
            ok = false;
            break;
          }
          const uint32_t full = bar(kBarFull + stage);
          mbar_expect_tx(full, kATxBytes + L::kSfStageBytes);
          const uint32_t sa = base + L::kSmemA + stage * kAStageBytes;
          const int x = kq * kRowBytes;  // byte offset along K
          if (!g2) {
            tma_load_3d(sa, map, x, 64 * m, e, full, policy);
            tma_load_3d(sa + 64 * kRowBytes, map, x, p.inter + 64 * m, e, full, policy);
          } else {
            tma_load_3d(sa, map, x, 128 * (t0 + tt), e, full, policy);
          }
          bulk_load(base + L::kSmemSfa + stage * L::kSfStageBytes,
                    sfa + static_cast<size_t>(ks) * L::kSfStageBytes, L::kSfStageBytes, full, policy);
          ++filled;
          if (++kq == ks_u) { kq = 0; ++tt; }
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (a_next >= a_end && b_claimed) {
          a_next = b_next;
          a_end = b_end;
          b_claimed = false;
        }
        if (a_next < a_end) cur = a_next++;
      }
      // drain: the copies of the last ring's fills have landed (their full
      // barriers completed), so no copy is in flight when the CTA exits. After a
      // failed wait too (the drain ignores the error word, with its own limit:
      // a stage whose activation rows never arrived waits out the limit)
      for (int i = 0; i < kStages && i < filled; ++i) {
        if (stage == 0) {
          stage = kStages - 1;
          phase ^= 1u;
        } else {
          --stage;
        }
        mbar_wait_drain(bar(kBarFull + stage), phase);
      }
    }
  } else if (warp == 1) {
    // ============================== MMA =====================================
    if (lane == 0) {
      pdl_wait();
      const int nseg = p.ctrl[kCtrlSegments];
      const int split = p.ctrl[kCtrlSplit];
      uint32_t stage = 0, phase = 0, ws = 0, wphase = 0, acc = 0, acc_phase = 0;
      // descriptor words that never change: A/B 128-byte-swizzled K-major with
      // 1 KB between 8-row groups; scale chunks: 32 rows x 16 B, 128 B apart
      const uint64_t sw_hi = smem_desc(0, 0, 1024, kLayoutSw128);
      const uint64_t sf_hi = smem_desc(0, 0, 128, kLayoutNone);
      const uint32_t idesc_base = kNv ? idesc_nvf4(0) : idesc_mxf4(0, 0);
      SegCache seg_cache;
#pragma unroll 1
      while (true) {
        if (!mbar_wait(bar(kBarWorkFull + ws), wphase, err, kErrTimeoutWork, wb)) break;
        const int u = ld_shared_volatile(work_ids + ws);
        mbar_arrive(bar(kBarWorkEmpty + ws));
        if (++ws == kWorkSlots) { ws = 0; wphase ^= 1u; }
        if (u < 0) break;
        bool g2;
        int seg, m, c;
        decode_unit(u, nseg, p.m1, split, p.u2, g2, seg, m, c);
        const int4 sg = seg_cache.get(p.segs, seg);
        const uint32_t n = static_cast<uint32_t>((sg.z + 7) & ~7);
        const uint32_t nmma = n * static_cast<uint32_t>(p.terms);  // term 0 rows, term 1 rows, ...
        const uint32_t id0 = idesc_base | ((nmma >> 3) << 17);
        const uint32_t id2 = id0 | (2u << 4) | (2u << 29);  // MXFP4: the chunk's second byte pair
        const int ks_u = g2 ? p.ks2 : p.ks1;
        int k0, ks_n;
        unit_stages(g2, c, split, ks_u, kTg2 == 1 ? 1 : min(kTg2, p.m2 - m * kTg2), k0, ks_n);
        if (!mbar_wait(bar(kBarAccEmpty + acc), acc_phase ^ 1u, err, kErrTimeoutAcc, wb)) break;
        tc_fence_after();
        // accumulator buffers tg2 x kBRows columns apart (single-tile layers keep them adjacent)
        const uint32_t acc_tmem = tbase + L::kTmemAcc + acc * static_cast<uint32_t>(kTg2 * kBRows);
        bool ok = true;
        uint32_t d_tmem = acc_tmem;  // the unit's current tile: its accumulator kBRows columns further
        int kq = 0;                  // K stage within the tile (within the chunk: the first accumulates from 0)
        // a down unit of two one-stage tiles: both tiles multiply the activation
        // rows (and B scales) of its first stage; that slot is released after the
        // second tile's MMAs, and the loader copies the rows once
        const bool share_b = kTg2 == 2 && g2 && ks_u == 1 && ks_n == 2;
        uint32_t keep_stage = 0;
#pragma unroll 1
        for (int ks = 0; ks < ks_n; ++ks) {
          if (!mbar_wait(bar(kBarFull + stage), phase, err, kErrTimeoutFull, wb)) {
            ok = false;
            break;
          }
          tc_fence_after();
          fence_proxy_async_smem();  // activation rows and B scales arrived via cp.async
          const bool reuse = share_b && ks == 1;  // the second tile: B of the first stage
          const uint32_t b_stage = reuse ? keep_stage : stage;
          const uint32_t sfa_t = tbase + L::kTmemSfa + stage * L::kTmemSfCols;
          const uint32_t sfb_t = tbase + L::kTmemSfb + b_stage * L::kTmemSfCols;
          const uint64_t sfa_d = sf_hi | ((base + L::kSmemSfa + stage * L::kSfStageBytes) >> 4);
          const uint64_t sfb_d = sf_hi | ((base + L::kSmemSfb + stage * L::kSfStageBytes) >> 4);
#pragma unroll
          for (int c = 0; c < L::kChunks; ++c) {
            tc_cp_32x128b_warpx4(sfa_t + 4 * c, sfa_d + ((512 * c) >> 4));
            if (!reuse) tc_cp_32x128b_warpx4(sfb_t + 4 * c, sfb_d + ((512 * c) >> 4));
          }
          const uint64_t a_d = sw_hi | ((base + L::kSmemA + stage * kAStageBytes) >> 4);
          const uint64_t b_d = sw_hi | ((base + L::kSmemB + b_stage * kBStageBytes) >> 4);
          // four K = 64 steps of 32 bytes along the 128-byte swizzled row.
          // MXFP4: scale chunk k / 2 holds the k-blocks of steps 2j, 2j + 1 at
          // byte pairs 0 and 2; NVFP4: chunk k holds step k's four k-blocks
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if constexpr (kNv)
              mma_nvf4(d_tmem, a_d + 2 * k, b_d + 2 * k, id0, sfa_t + 4 * k, sfb_t + 4 * k, (kq | k) != 0 ? 1u : 0u);
            else
              mma_mxf4(d_tmem, a_d + 2 * k, b_d + 2 * k, (k & 1) ? id2 : id0, sfa_t + 4 * (k >> 1),
                       sfb_t + 4 * (k >> 1), (kq | k) != 0 ? 1u : 0u);
          }
          if (share_b && ks == 0) {
            keep_stage = stage;  // released with the second tile's stage
          } else {
            if (reuse) tc_commit(bar(kBarEmpty + keep_stage));
            tc_commit(bar(kBarEmpty + stage));
          }
          if (++kq == ks_u) { kq = 0; d_tmem += kBRows; }
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        tc_commit(bar(kBarAccFull + acc));
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
      // every tcgen05 operation issued above has completed before teardown (also
      // after a failed wait: the drain ignores the error word)
      tc_commit(bar(kBarDrain));
      mbar_wait_drain(bar(kBarDrain), 0);
    }
  } else if (warp == 2) {
    // ============================ B loader ===================================
    // Per unit, every lane fixes its share of a stage once: 16-byte piece
    // pc = lane % 8 of B rows rr = lane / 8 + 4 i (term t rows at [t n, (t+1) n));
    // per stage it only issues the copies at the stage's K offset. The shares
    // depend only on the unit's segment and kind (gate_up or down), not on its
    // weight tile, so they are kept while consecutive units share both: a run
    // of short down units of one segment pays the set-up once.
    pdl_wait();
    const int nseg = p.ctrl[kCtrlSegments];
    const int split = p.ctrl[kCtrlSplit];
    uint32_t stage = 0, phase = 0, ws = 0, wphase = 0;
    SegCache seg_cache;
    int ready_seg = -1;                 // a segment whose mailbox is known complete
    int share_seg = -1;                 // the segment / kind the shares below belong to
    bool share_g2 = false;
    const int pc = lane & 7;            // 16-byte piece of the 128-byte stage row
    const int quarter = lane >> 3;
    constexpr int kPieces = kBRows / 4;  // rows per lane
    constexpr int kC = L::kChunks;
    uint32_t soff[kPieces], doff[kPieces];
    uint32_t s_base[2];  // scale bytes of B rows lane and lane + 32 at stage 0 (chunk c: + 4 c)
    uint32_t pmask = 0, smask = 0;  // bit i: piece i / scale row half i holds a segment row (else zero-fill)
    int nb = 0;
    int fills = 0;  // stages filled, counted up to kStages
    const uint8_t *dq = nullptr, *dsc = nullptr;
#pragma unroll 1
    while (true) {
      int u = -1, okw = 1;
      if (lane == 0) {
        okw = mbar_wait(bar(kBarWorkFull + ws), wphase, err, kErrTimeoutWork, wb) ? 1 : 0;
        if (okw) {
          u = ld_shared_volatile(work_ids + ws);
          mbar_arrive(bar(kBarWorkEmpty + ws));
        }
      }
      u = __shfl_sync(0xffffffffu, u, 0);
      okw = __shfl_sync(0xffffffffu, okw, 0);
      if (++ws == kWorkSlots) { ws = 0; wphase ^= 1u; }
      if (!okw || u < 0) break;
      bool g2;
      int seg, m, c;
      decode_unit(u, nseg, p.m1, split, p.u2, g2, seg, m, c);
      if (seg != share_seg || g2 != share_g2) {
        share_seg = seg;
        share_g2 = g2;
        // a gate_up unit's x rows are its segment's tokens: the list is loaded
        // beside the segment descriptor (one L2 round trip for both)
        const int tok = !g2 && lane < kSegRows ? __ldcg(p.seg_tok + seg * kSegRows + lane) : 0;
        const int4 sg = seg_cache.get(p.segs, seg);
        const int rows = sg.z;
        const int n = (rows + 7) & ~7;  // 8 or 16 (rows <= kSegRows)
        const int nsh = n == 8 ? 3 : 4;
        nb = n * p.terms;  // B rows of this unit
        // source row of segment row `lane` (lanes >= rows: row 0, never read)
        int src = 0;
        if (lane < rows) src = g2 ? sg.y + lane : tok;
        const int K = g2 ? p.inter : p.hidden;
        dq = g2 ? p.hq : p.xq;
        dsc = g2 ? p.hs : p.xs;
        // packed bytes and scale bytes per row: x's rows are exactly H (a multiple of 256);
        // h's are padded to whole stages and zero past I
        const uint32_t rowb = g2 ? static_cast<uint32_t>(p.hq_row) : static_cast<uint32_t>(K) >> 1;
        const uint32_t term_q = static_cast<uint32_t>(g2 ? p.rows_cap : p.max_tokens) * rowb;
        const uint32_t srow = g2 ? static_cast<uint32_t>(p.hs_row) : static_cast<uint32_t>(K / L::kBlock);
        const uint32_t term_s = static_cast<uint32_t>(g2 ? p.rows_cap : p.max_tokens) * srow;
        // piece i's segment row (quarter + 4 i) & (n - 1) is quarter + 4 (i % (n / 4)):
        // a lane reads two source rows (n = 8) or four (n = 16)
        int src_q[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) src_q[j] = __shfl_sync(0xffffffffu, src, quarter + 4 * j);
#pragma unroll
        for (int i = 0; i < kPieces; ++i) {
          const int rr = quarter + 4 * i;
          const int t = rr >> nsh;
          const int r = rr & (n - 1);
          const int sr = n == 8 ? src_q[i & 1] : src_q[i & 3];
          soff[i] = static_cast<uint32_t>(t) * term_q + static_cast<uint32_t>(sr) * rowb + pc * 16;
          doff[i] = (rr >> 3) * 1024 + (rr & 7) * 128 + ((pc ^ (rr & 7)) << 4);
          pmask = (rr < nb && r < rows) ? (pmask | (1u << i)) : (pmask & ~(1u << i));
        }
        // scale pieces: B rows rr = lane and lane + 32 (segment row lane % n for
        // both), every chunk of the stage
        const int s_src = __shfl_sync(0xffffffffu, src, lane & (n - 1));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int rr = lane + 32 * h;
          const int t = rr >> nsh;
          const int r = rr & (n - 1);
          const int sr = s_src;
          s_base[h] = static_cast<uint32_t>(t) * term_s + static_cast<uint32_t>(sr) * srow;
          smask = (rr < nb && r < rows) ? (smask | (1u << h)) : (smask & ~(1u << h));
        }
      }
      // a down unit's rows are its segment's h rows: the shares above depend
      // only on the segment descriptor, so they are ready when the mailbox
      // completes (once complete, a mailbox stays complete in this launch)
      if (g2 && seg != ready_seg) {
        int okf = 1;
        const int target = p.m1 * tile_publishes(split, seg_cache.get(p.segs, seg).z);
        if (lane == 0) okf = wait_flag(p.flags + seg, target, err, wb) ? 1 : 0;
        okf = __shfl_sync(0xffffffffu, okf, 0);
        if (!okf) break;
        ready_seg = seg;
      }
      // a down unit's tiles share their B: stage ks loads K stage ks % ks_u; a
      // gate_up chunk loads K stages [k0, k0 + ks_n)
      const int ks_u = g2 ? p.ks2 : p.ks1;
      int k0, ks_n;
      unit_stages(g2, c, split, ks_u, kTg2 == 1 ? 1 : min(kTg2, p.m2 - m * kTg2), k0, ks_n);
      const bool share_b = kTg2 == 2 && g2 && ks_u == 1 && ks_n == 2;  // as the MMA warp decides
#pragma unroll 1
      for (int ks = 0, kq = k0; ks < ks_n; ++ks, kq = (kq + 1 == ks_u) ? 0 : kq + 1) {
        if (fills < kStages) {
          ++fills;  // the ring's first pass: every slot is still empty
        } else {
          int oke = 1;
          if (lane == 0) oke = mbar_wait(bar(kBarEmpty + stage), phase ^ 1u, err, kErrTimeoutEmpty, wb) ? 1 : 0;
          oke = __shfl_sync(0xffffffffu, oke, 0);
          if (!oke) break;
        }
        // a down unit of two one-stage tiles: the second tile's MMA reads the
        // first stage's rows, so its stage only gets this loader's arrival (after
        // the first stage's copies land: the arrival follows all prior copies)
        if (!(share_b && ks == 1)) {
          const uint32_t sb = base + L::kSmemB + stage * kBStageBytes;
          const uint8_t *gq = dq + kq * kRowBytes;
#pragma unroll
          for (int i = 0; i < kPieces; ++i) {
            if (quarter + 4 * i < nb) cp_async_16(sb + doff[i], gq + soff[i], ((pmask >> i) & 1u) * 16u);
          }
          const uint32_t ssb = base + L::kSmemSfb + stage * L::kSfStageBytes;
          const uint8_t *gs = dsc + kq * L::kSfRow;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (lane + 32 * h < nb) {
#pragma unroll
              for (int c = 0; c < kC; ++c)  // chunk c, row lane + 32 h: byte 16 (row % 32) + 4 (row / 32)
                cp_async_4(ssb + c * 512 + lane * 16 + h * 4, gs + s_base[h] + c * 4, ((smask >> h) & 1u) * 4u);
            }
          }
        }
        cp_async_arrive_noinc(bar(kBarFull + stage));
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else {
    // ============================ epilogue ===================================
    // No block-level barrier here: the gate_up hand-off between the up-row and
    // gate-row warps goes through two mbarriers with bounded waits, and each
    // gate-row warp publishes its own h rows to the segment mailbox. Split-K
    // chunks hand off through global memory instead (mm_layout.cuh).
    pdl_wait();
    const int nseg = p.ctrl[kCtrlSegments];
    const int split = p.ctrl[kCtrlSplit];
    const int q = warp & 3;             // TMEM lane quadrant of this warp
    const int row = 32 * q + lane;      // accumulator row (weight-tile row)
    float *ex = reinterpret_cast<float *>(sbase + L::kSmemEpi);
    uint32_t ws = 0, wphase = 0, acc = 0, acc_phase = 0, ex_phase = 0;
    SegCache seg_cache;
    // SwiGLU (+ clamp) of the 32 features f = 64 m + 32 fq + lane of `rows` token
    // rows of segment sg from row j_base on (gate gv[i], up uv[i] for row
    // j_base + i), requantized into h's FP4 terms, then this warp's increment of
    // the segment's mailbox (two per whole gate_up tile, four per split-K chunk).
    // One call site: the split-K and the whole-tile paths both end here.
    auto swiglu_publish = [&](const int4 &sg, int seg, int m, int fq, const float (&gv)[kSegRows],
                              const float (&uv)[kSegRows], int j_base, int rows) {
      const float *lim = sg.x < 0 ? p.shared_clamp : p.clamp;
      const bool clamped = lim != nullptr;
      const float limit = clamped ? lim[sg.x < 0 ? 0 : sg.x] : 0.0f;
      const int f = 64 * m + 32 * fq + lane;  // feature (column of h)
      const size_t rowb = static_cast<size_t>(p.hq_row);
      const size_t tq = static_cast<size_t>(p.rows_cap) * rowb;      // term stride of hq
      const size_t ts = static_cast<size_t>(p.rows_cap) * p.hs_row;  // term stride of hs
      // one row's SwiGLU and FP4 terms (the token row sg.y + j): h = up *
      // silu(gate), then one MXFP4 block of 32 or two NVFP4 blocks of 16 (lane
      // halves) per term, each term quantizing the previous terms' remainder
      auto silu_row = [&](float g, float up) {
        if (clamped) {
          up = fminf(fmaxf(up, -limit), limit);
          g = fminf(g, limit);
        }
        return __fmul_rn(up, __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))));
      };
      auto quant_term = [&](float &r, uint32_t &nib, uint32_t &code) {
        if constexpr (kNv) {
          float amax = fabsf(r);
#pragma unroll
          for (int off = 8; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
          code = nv4_scale_code(amax, p.gs2);
          const float sv = e4m3_value(static_cast<uint8_t>(code));
          nib = e2m1x2(__fmul_rn(r, nv4_multiplier(sv, p.gs2)), 0.0f) & 15u;
          r = __fsub_rn(r, __fmul_rn(__fmul_rn(e2m1_value(nib), sv), p.inv_gs2));
        } else {
          const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(r))));
          code = mx4_scale_code(amax);
          nib = e2m1x2(__fmul_rn(r, mx_inverse(code)), 0.0f) & 15u;
          r = __fsub_rn(r, __fmul_rn(e2m1_value(nib), mx_scale_value(code)));
        }
      };
      auto store_term = [&](int t, int j, uint32_t nib, uint32_t code) {
        const uint32_t up_nib = __shfl_down_sync(0xffffffffu, nib, 1);
        const size_t prow = static_cast<size_t>(sg.y + j_base + j);
        if (j < rows) {
          if ((lane & 1) == 0) p.hq[t * tq + prow * rowb + (f >> 1)] = static_cast<uint8_t>(nib | (up_nib << 4));
          if ((lane & (L::kBlock - 1)) == 0)
            p.hs[t * ts + prow * p.hs_row + f / L::kBlock] = static_cast<uint8_t>(code);
        }
      };
      bool staged = false;
      if constexpr (!kNv) staged = rows > 4;
      if (staged) {
        // MXFP4, more than 4 rows (a whole tile: a split-K warp has at most 4):
        // the SwiGLU with lane = feature, then through this gate warp's part of
        // the exchange (its up sums already in registers; released once read
        // back) each token row's block of 32 features goes to two lanes (lane
        // 2 r + hh: features 16 hh .. 16 hh + 15 of row r). A term's block amax
        // is a 16-element local maximum and one shuffle (of the magnitudes'
        // bits, as a warp reduction of them), and two features convert per
        // instruction; each element's arithmetic is the one-lane-per-feature
        // form's, so the bytes are the same. (Up to 4 rows the
        // lane-per-feature forms below are shorter.)
        float *qx = ex + 32 * fq * kSegRows;  // this gate warp's rows of the exchange
        {
          // one row per pass of a compact loop, the rows rotating down
          float gq[kSegRows], uq[kSegRows];
#pragma unroll
          for (int j = 0; j < kSegRows; ++j) {
            gq[j] = gv[j];
            uq[j] = uv[j];
          }
#pragma unroll 1
          for (int j = 0; j < rows; ++j) {
            qx[j * 32 + lane] = silu_row(gq[0], uq[0]);
#pragma unroll
            for (int i = 0; i + 1 < kSegRows; ++i) {
              gq[i] = gq[i + 1];
              uq[i] = uq[i + 1];
            }
          }
        }
        __syncwarp();
        const int jr = lane >> 1, hh = lane & 1;
        const bool live = jr < rows;
        float x[16];
        const float4 *src = reinterpret_cast<const float4 *>(qx + (live ? jr : 0) * 32 + 16 * hh);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float4 w = src[k];
          x[4 * k] = live ? w.x : 0.0f;
          x[4 * k + 1] = live ? w.y : 0.0f;
          x[4 * k + 2] = live ? w.z : 0.0f;
          x[4 * k + 3] = live ? w.w : 0.0f;
        }
        __syncwarp();  // the tile is read: the exchange is free for the next unit's up rows
        if (lane == 0) mbar_arrive(bar(kBarExFree));
        const size_t prow = static_cast<size_t>(sg.y + j_base + (live ? jr : 0));
        const int f0 = 64 * m + 32 * fq;  // the block's first feature
        for (int t = 0; t < p.terms; ++t) {
          uint32_t abits = 0u;
#pragma unroll
          for (int i = 0; i < 16; ++i) abits = max(abits, __float_as_uint(fabsf(x[i])));
          abits = max(abits, __shfl_xor_sync(0xffffffffu, abits, 1));
          const uint32_t code = mx4_scale_code(__uint_as_float(abits));
          const float inv = mx_inverse(code), sv = mx_scale_value(code);
          uint32_t w[2] = {0u, 0u};
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t b = e2m1x2(__fmul_rn(x[2 * k], inv), __fmul_rn(x[2 * k + 1], inv));
            w[k >> 2] |= b << (8 * (k & 3));
            x[2 * k] = __fsub_rn(x[2 * k], __fmul_rn(e2m1_value(b), sv));
            x[2 * k + 1] = __fsub_rn(x[2 * k + 1], __fmul_rn(e2m1_value(b >> 4), sv));
          }
          if (live) {
            *reinterpret_cast<uint2 *>(p.hq + t * tq + prow * rowb + (f0 >> 1) + 8 * hh) = make_uint2(w[0], w[1]);
            if (hh == 0) p.hs[t * ts + prow * p.hs_row + f0 / L::kBlock] = static_cast<uint8_t>(code);
          }
        }
      } else {
        if (rows <= 2) {
          // a row or two (small batches): one row at a time, the shortest code
  #pragma unroll
          for (int j = 0; j < 2; ++j) {
            if (j >= rows) break;
            float r = silu_row(gv[j], uv[j]);
            for (int t = 0; t < p.terms; ++t) {
              uint32_t nib, code;
              quant_term(r, nib, code);
              store_term(t, j, nib, code);
            }
          }
        } else {
          // rows in groups of kG, one group per pass of a compact loop: each row's
          // quantization is a chain of warp reductions and conversions, so
          // independent rows in flight hide its latency; the rows' values rotate
          // down by a group after each pass (register indices stay fixed), and
          // rows past `rows` run on zeros and are not stored
          constexpr int kG = 4;
          float gq[kSegRows], uq[kSegRows];
  #pragma unroll
          for (int j = 0; j < kSegRows; ++j) {
            gq[j] = gv[j];
            uq[j] = uv[j];
          }
  #pragma unroll 1
          for (int j0 = 0; j0 < rows; j0 += kG) {
            float r[kG];
  #pragma unroll
            for (int i = 0; i < kG; ++i) {
              const bool live = j0 + i < rows;
              r[i] = silu_row(live ? gq[i] : 0.0f, live ? uq[i] : 0.0f);
            }
  #pragma unroll 1
            for (int t = 0; t < p.terms; ++t) {
              uint32_t nib[kG], code[kG];
  #pragma unroll
              for (int i = 0; i < kG; ++i) quant_term(r[i], nib[i], code[i]);
  #pragma unroll
              for (int i = 0; i < kG; ++i) store_term(t, j0 + i, nib[i], code[i]);
            }
  #pragma unroll
            for (int i = 0; i + kG < kSegRows; ++i) {
              gq[i] = gq[i + kG];
              uq[i] = uq[i + kG];
            }
          }
        }
      }
      // every lane's h bytes, then lane 0's release increment (cumulative over
      // the warp barrier) publishes them
      __syncwarp();
      if (lane == 0) asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(p.flags + seg) : "memory");
    };
#pragma unroll 1
    while (true) {
      int u = -1, okw = 1;
      if (lane == 0) {
        okw = mbar_wait(bar(kBarWorkFull + ws), wphase, err, kErrTimeoutWork, wb) ? 1 : 0;
        if (okw) {
          u = ld_shared_volatile(work_ids + ws);
          mbar_arrive(bar(kBarWorkEmpty + ws));
        }
      }
      u = __shfl_sync(0xffffffffu, u, 0);
      okw = __shfl_sync(0xffffffffu, okw, 0);
      if (++ws == kWorkSlots) { ws = 0; wphase ^= 1u; }
      if (!okw || u < 0) break;
      bool g2;
      int seg, m, c;
      decode_unit(u, nseg, p.m1, split, p.u2, g2, seg, m, c);
      const int4 sg = seg_cache.get(p.segs, seg);
      const int rows = sg.z;
      const int n = (rows + 7) & ~7;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(bar(kBarAccFull + acc), acc_phase, err, kErrTimeoutAcc, wb) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      // a down unit holds tg2 tiles: tile tt's accumulator at tt x kBRows columns
      const int tiles = g2 ? (kTg2 == 1 ? 1 : min(kTg2, p.m2 - m * kTg2)) : 1;
      const uint32_t acc_addr =
          tbase + (static_cast<uint32_t>(32 * q) << 16) + L::kTmemAcc + acc * static_cast<uint32_t>(kTg2 * kBRows);
      const bool chunked = !g2 && split > 1;
#pragma unroll 1
      for (int tt = 0; tt < tiles; ++tt) {
        uint32_t ra[32], rb[16];
        const uint32_t taddr = acc_addr + static_cast<uint32_t>(tt * kBRows);
        tc_ld_32x32b_x32(taddr, ra);
        tc_ld_32x32b_x16(taddr + 32, rb);
        tc_wait_ld();
        if (tt == tiles - 1) {  // every tile read: the accumulator buffer is free
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kBarAccEmpty + acc));
          if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
        // columns [t n, (t+1) n) hold term t's products; row j's value = sum of terms
        float v[kSegRows];
#pragma unroll
        for (int j = 0; j < kSegRows; ++j) {
          float a = __uint_as_float(ra[j]);
          if (p.terms > 1) a = __fadd_rn(a, __uint_as_float(n == 8 ? ra[8 + j] : ra[16 + j]));
          if (p.terms > 2) a = __fadd_rn(a, __uint_as_float(n == 8 ? ra[16 + j] : rb[j]));
          v[j] = a;
        }
        float al = 1.0f;  // NVFP4: the product of the two second-level scales (a split
        if constexpr (kNv) {  // tile applies it once, to the sum of its chunks)
          al = sg.x < 0 ? (g2 ? p.salpha2[0] : p.salpha13[0]) : (g2 ? p.alpha2[sg.x] : p.alpha13[sg.x]);
          if (!chunked) {
#pragma unroll
            for (int j = 0; j < kSegRows; ++j) v[j] = __fmul_rn(v[j], al);
          }
        }
        if (!g2) {
          // gate_up: v becomes the gate and upv the up sums of features
          // 64 m + 32 fq + lane, for the warp that runs the SwiGLU (fq its half)
          float upv[kSegRows];
          int fq = -1;
          int j_base = 0, nj = rows;
          if (chunked) {
            // split-K chunk: this warp's rows of the chunk's partial sums go to
            // the chunk's slot, then the tile's chunks are added in chunk order
            const int tile = u / split;
            const int chunk = u - tile * split;
            float *mine = p.part + static_cast<size_t>(u) * kPartFloats + row;
#pragma unroll
            for (int j = 0; j < kSegRows; ++j)
              if (j < rows) mine[j * 128] = v[j];
            __syncwarp();
            if (rows <= 2) {
              // a row or two: the warp counts in for its half of the features
              // (gate rows 32 fq + lane, up rows 64 + 32 fq + lane); the half's
              // last warp adds every chunk, each row's chunks all in flight
              int last = 0;
              if (lane == 0) last = atom_add_acq_rel(p.split_cnt + 2 * tile + (q & 1), 1) == 2 * split - 1 ? 1 : 0;
              last = __shfl_sync(0xffffffffu, last, 0);
              __syncwarp();
              if (last) {
                fq = q & 1;
                const float *base = p.part + static_cast<size_t>(tile) * split * kPartFloats + 32 * fq + lane;
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                  float g = 0.0f, up = 0.0f;
                  if (j < rows) {
                    float gp[kMaxSplit], upp[kMaxSplit];
#pragma unroll
                    for (int cc = 0; cc < kMaxSplit; ++cc) {
                      if (cc < split) {
                        gp[cc] = __ldcg(base + cc * kPartFloats + j * 128);
                        upp[cc] = __ldcg(base + cc * kPartFloats + j * 128 + 64);
                      }
                    }
                    g = gp[0];
                    up = upp[0];
#pragma unroll
                    for (int cc = 1; cc < kMaxSplit; ++cc) {
                      if (cc < split) {
                        g = __fadd_rn(g, gp[cc]);
                        up = __fadd_rn(up, upp[cc]);
                      }
                    }
                  }
                  v[j] = g;
                  upv[j] = up;
                }
              }
            } else {
              // more rows: every warp of the tile's chunks counts in (4 per
              // chunk) and waits for all of them (the chunks are first-wave
              // units, resident together); the 2 x split warps of each half of
              // the features then each finish a block of the token rows
              int okc = 1;
              if (lane == 0) {
                asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(p.split_cnt + 2 * tile) : "memory");
                okc = wait_flag(p.split_cnt + 2 * tile, 4 * split, err, wb) ? 1 : 0;
              }
              okc = __shfl_sync(0xffffffffu, okc, 0);
              __syncwarp();  // lane 0's acquire orders the warp's loads below
              if (!okc) {
                ok = 0;
                break;
              }
              fq = q & 1;
              const int nw = 2 * split;  // >= 4: at most 4 rows per warp
              const int per = (rows + nw - 1) / nw;
              j_base = min(rows, (2 * chunk + (q >> 1)) * per);
              nj = min(rows - j_base, per);
              // the warp's rows, chunk by chunk, added in chunk order (rows past
              // nj read an in-slot row and are never stored)
              const float *base = p.part + static_cast<size_t>(tile) * split * kPartFloats + 32 * fq + lane;
              int ro[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) ro[i] = min(j_base + i, kSegRows - 1) * 128;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                v[i] = __ldcg(base + ro[i]);
                upv[i] = __ldcg(base + ro[i] + 64);
              }
#pragma unroll 1
              for (int cc = 1; cc < split; ++cc) {
                float gp[4], upp[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  gp[i] = __ldcg(base + cc * kPartFloats + ro[i]);
                  upp[i] = __ldcg(base + cc * kPartFloats + ro[i] + 64);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  v[i] = __fadd_rn(v[i], gp[i]);
                  upv[i] = __fadd_rn(upv[i], upp[i]);
                }
              }
            }
            if constexpr (kNv) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                v[i] = __fmul_rn(v[i], al);
                upv[i] = __fmul_rn(upv[i], al);
              }
            }
          } else if (q >= 2) {
            // rows 64..127 (up of features 64m + row - 64): to the gate-row warp
            if (lane == 0) ok = mbar_wait(bar(kBarExFree), ex_phase ^ 1u, err, kErrTimeoutAcc, wb) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
#pragma unroll
            for (int j = 0; j < kSegRows; ++j) ex[(row - 64) * kSegRows + j] = v[j];
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarExFull));
            ex_phase ^= 1u;
          } else {
            // rows 0..63: gate of features 64m + row, the up sums from the exchange
            if (lane == 0) ok = mbar_wait(bar(kBarExFull), ex_phase, err, kErrTimeoutAcc, wb) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
#pragma unroll
            for (int j = 0; j < kSegRows; ++j) upv[j] = ex[row * kSegRows + j];
            __syncwarp();
            // MXFP4 with more than 4 rows stages its requantization in this
            // warp's part of the exchange and releases it there
            if (kNv || rows <= 4)
              if (lane == 0) mbar_arrive(bar(kBarExFree));
            ex_phase ^= 1u;
            fq = q;
          }
          if (fq >= 0) swiglu_publish(sg, seg, m, fq, v, upv, j_base, nj);
        } else {
          // features 128 (m tg2 + tt) + row of the segment's rows, bf16
          const size_t col = static_cast<size_t>(128 * (m * kTg2 + tt) + row);
#pragma unroll
          for (int j = 0; j < kSegRows; ++j) {
            if (j >= rows) break;
            p.rows_out[static_cast<size_t>(sg.y + j) * p.hidden + col] = float_to_bf16_bits(v[j]);
          }
        }
      }
      if (!ok) break;
    }
  }

  // ---- teardown --------------------------------------------------------------
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
  // The work tables (claim counter, mailboxes) are re-armed by the next front
  // pass (build_route), or by mm_layer_rearm_experts before a relaunch on the
  // same tables: no end-of-kernel fence and ticket.
}

// ============================================================================
// Scale repack (layer creation): canonical scales [n][rows][K/block] -> UMMA
// scale chunks [n][tile][K/256][chunks][32 m0][4 m1][4 kk], chunks = 256 /
// block / 4 (2 for MXFP4's E8M0 per 32, 4 for NVFP4's E4M3 per 16); chunk c
// byte kk of row r holds k-block 4c + kk of the stage. gate_up tiles take gate
// rows 64t + r (r < 64) and up rows I + 64t + r - 64; down tiles rows 128t + r.
// ============================================================================
__global__ void repack_scales_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
                                     int n, int rows, int k, int gate_up, int inter, int block) {
  const int ks_n = (k + kStageK - 1) / kStageK;  // a partial last stage gets zero scales past k
  const int tiles = rows / 128;
  const int per_row = kStageK / block;          // scale bytes of a row per stage
  const int cols = k / block;                   // scale columns of a row
  const int stage_bytes = per_row * 128;        // = chunks * 512
  const size_t total = static_cast<size_t>(n) * tiles * ks_n * stage_bytes;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(idx % stage_bytes);
    size_t rest = idx / stage_bytes;
    const int ks = static_cast<int>(rest % ks_n);
    rest /= ks_n;
    const int t = static_cast<int>(rest % tiles);
    const int e = static_cast<int>(rest / tiles);
    const int c = b >> 9, w = b & 511;
    const int m0 = w >> 4, m1 = (w >> 2) & 3, kk = w & 3;
    const int r = m0 + 32 * m1;
    const int kb = ks * per_row + 4 * c + kk;
    const int srow = gate_up ? (r < 64 ? 64 * t + r : inter + 64 * t + (r - 64)) : 128 * t + r;
    dst[idx] = kb < cols ? src[(static_cast<size_t>(e) * rows + srow) * cols + kb] : static_cast<uint8_t>(0);
  }
}

// NVFP4 accumulator multipliers: alpha[e] = scale_2[e] * input_scale (the
// reference's g1_alpha / g2_alpha, glm5_3/sm103/moe/api.py:49-50).
__global__ void nv_alpha_kernel(const float *__restrict__ scale_2, float input_scale, float *__restrict__ alpha,
                                int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) alpha[i] = __fmul_rn(scale_2[i], input_scale);
}

cudaError_t expert_kernel_configure(int fmt) {
  if (fmt == kFmtNv)
    return cudaFuncSetAttribute(expert_kernel<kFmtNv, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                Fmt<kFmtNv>::kSmemAlloc);
  cudaError_t e = cudaFuncSetAttribute(expert_kernel<kFmtMx, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Fmt<kFmtMx>::kSmemAlloc);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(expert_kernel<kFmtMx, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Fmt<kFmtMx>::kSmemAlloc);
  return e;
}

cudaError_t expert_kernel_launch(int fmt, int ctas, const ExpertArgs &ea, void *stream) {
  const dim3 grid(ctas), block(kExpertThreads);
  if (fmt == kFmtNv) {
    if (ea.tg2 != 1) return cudaErrorInvalidValue;
    return launch(expert_kernel<kFmtNv, 1>, grid, block, Fmt<kFmtNv>::kSmemAlloc, stream, ea);
  }
  if (ea.tg2 == 2) return launch(expert_kernel<kFmtMx, 2>, grid, block, Fmt<kFmtMx>::kSmemAlloc, stream, ea);
  if (ea.tg2 != 1) return cudaErrorInvalidValue;
  return launch(expert_kernel<kFmtMx, 1>, grid, block, Fmt<kFmtMx>::kSmemAlloc, stream, ea);
}

}  // namespace mm
