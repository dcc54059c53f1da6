// Data layouts shared by the host side and the kernels of the routed-MoE chain.
//
// HBM, per layer (all device memory, allocated once at layer creation):
//   weights     caller-owned canonical MXFP4 (E2M1 codes, [n, rows, K/2] u8) read
//               in place by TMA (128-byte rows, 128-byte swizzle);
//   sfa13/sfa2  the weight scales re-laid once as UMMA scale chunks:
//               [n][m_tile][k_stage][chunks][32 m0][4 m1][4 kk] bytes (2 chunks
//               for MXFP4, 4 for NVFP4), so one bulk copy per pipeline stage
//               lands them ready for tcgen05.cp;
//   xq/xs       the routed input as FP4 terms: [term][T][H/2] packed E2M1 and
//               [term][T][H/block] scales, written by the router launch;
//   hq/hs       the SwiGLU output of gate_up, [term][rows][I/2] and
//               [term][rows][I/block], rows in the reference's padded permuted order;
//   segs/ctrl   work tables built by the front kernel (below);
//   err         the device error word.
#pragma once
#include <cstdint>

namespace mm {

// ---- route record (bit for bit the reference's, route.cuh:6-46) ---------------
constexpr int kTile = 8;
__host__ __device__ inline int route_max_ctas(int rows, int top_k, int experts) {
  const int slots = rows * top_k;
  const int filled = experts < slots ? experts : slots;
  return filled + (slots - filled) / kTile;
}
__host__ __device__ inline int route_cta_words(int max_ctas) { return (max_ctas + 3) / 4 * 4; }
__host__ __device__ inline int route_words(int rows, int top_k, int experts) {
  const int m = route_max_ctas(rows, top_k, experts);
  return 4 + 2 * route_cta_words(m) + kTile * m;
}

// ---- expert work -----------------------------------------------------------------
// A segment is up to kSegRows consecutive permuted rows of one expert; one work
// unit streams one 128-row weight tile of that expert through the whole K and
// multiplies it with all the segment's rows (N = rows rounded up to 8).
constexpr int kSegRows = 16;
constexpr int kMaxTokens = 256;
constexpr int kMaxTopK = 16;
constexpr int kMaxRouterExperts = 1024;

struct Segment {   // int4 in memory
  int expert;      // local expert index, -1 for the shared expert
  int row_base;    // first permuted row (rows_out / hq row)
  int rows;        // 1..kSegRows
  int token_base;  // shared expert: token of row_base; routed: -1 (each row's token: the segment's token list)
};

// ctrl words
constexpr int kCtrlSegments = 0;  // number of segments
constexpr int kCtrlUnits = 1;     // gate_up units + down units
constexpr int kCtrlClaim = 2;     // units claimed after the first wave (reset to 0 by the front kernel)
constexpr int kCtrlTicket = 3;    // front kernel's last-CTA ticket (reset by the last CTA)
constexpr int kCtrlSplit = 4;     // K chunks per gate_up tile (split-K), chosen by the front kernel
constexpr int kCtrlWords = 8;

// Split-K of the gate_up units. When a step's gate_up tiles (segments x I/64)
// number fewer than the expert grid, each tile's K (H) is cut into `split`
// chunks of at least two stages, one unit each, so that every CTA streams
// weights from the first wave: split = min(kMaxSplit, grid / tiles, ks1 / 2).
// A chunk's epilogue warps store their fp32 partial sums (terms added) to a
// slot of their own, kPartFloats per chunk ([segment row j][tile row]); the last
// of the 2 x split warps covering one half of the tile's features (its gate
// rows and the matching up rows), counted per (tile, half), adds the chunks'
// partials in chunk order and runs the SwiGLU epilogue. Chunk units number at
// most the grid, so the partial slots are indexed by the unit id.
constexpr int kMaxSplit = 8;
constexpr int kPartFloats = kSegRows * 128;

// ---- the persistent expert kernel's shared memory -----------------------------------
// Weights and activations are both packed E2M1 (two codes per byte) with a block
// scale along K (format below), multiplied by tcgen05.mma with K = 64.
// The activations are carried as up to kMaxTerms FP4 terms (x ~ t0 + t1 + t2,
// each term the FP4 quantization of the previous residual); a stage's B rows
// hold term 0 of the segment's n rows at [0, n), term 1 at [n, 2n), term 2 at
// [2n, 3n) (n = rows rounded up to 8), so one MMA with N = terms * n multiplies
// every term, each into its own accumulator columns.
constexpr int kMaxTerms = 3;
// Two CTAs share each SM (kCtasPerSm), each with its own 4-stage ring: two
// independent producer -> MMA -> release loops per SM hide each other's
// per-stage hand-off latency, which one deeper ring cannot.
constexpr int kCtasPerSm = 2;
constexpr int kStages = 4;
constexpr int kStageK = 256;                    // K elements per pipeline stage
constexpr int kRowBytes = kStageK / 2;          // 128: one 128-byte swizzle row
constexpr int kAStageBytes = 128 * kRowBytes;   // 16 KB: 128 weight rows
constexpr int kBRows = kMaxTerms * kSegRows;    // 48
constexpr int kBStageBytes = kBRows * kRowBytes;  // 6 KB
constexpr int kEpiBytes = 64 * kSegRows * 4;    // gate_up epilogue exchange
constexpr int kWorkSlots = 4;

// barriers: full[S], empty[S], acc_full[2], acc_empty[2], work_full[W], work_empty[W], drain,
// epilogue staging full / free
constexpr int kBarFull = 0;
constexpr int kBarEmpty = kStages;
constexpr int kBarAccFull = 2 * kStages;
constexpr int kBarAccEmpty = 2 * kStages + 2;
constexpr int kBarWorkFull = 2 * kStages + 4;
constexpr int kBarWorkEmpty = 2 * kStages + 4 + kWorkSlots;
constexpr int kBarDrain = 2 * kStages + 4 + 2 * kWorkSlots;
constexpr int kBarExFull = kBarDrain + 1;   // gate_up epilogue: up rows staged
constexpr int kBarExFree = kBarDrain + 2;   // gate_up epilogue: staging consumed
constexpr int kNumBars = kBarDrain + 3;

// ---- block-scaled FP4 formats ----------------------------------------------------
// kFmtMx (MXFP4): an E8M0 scale per 32 elements along K, tcgen05.mma
//   kind::mxf4 block32 (two scale bytes of a row per K = 64 instruction);
// kFmtNv (NVFP4): an E4M3 scale per 16 elements along K (and an fp32
//   second-level scale per expert, applied in the epilogue), tcgen05.mma
//   kind::mxf4nvf4 block16 (four scale bytes of a row per instruction).
// A stage's scales travel as 512-byte chunks (128 rows x 4 bytes: byte
// 16 m0 + 4 m1 + kk holds row m0 + 32 m1's k-block kk), copied to TMEM by
// tcgen05.cp 32x128b.warpx4 into 4 columns each.
constexpr int kFmtMx = 0;
constexpr int kFmtNv = 1;
template <int F>
struct Fmt {
  static constexpr int kBlock = F == kFmtNv ? 16 : 32;     // elements per scale
  static constexpr int kSfRow = kStageK / kBlock;          // scale bytes per row per stage
  static constexpr int kChunks = kSfRow / 4;               // 512-byte chunks per stage
  static constexpr int kSfStageBytes = kChunks * 512;      // 1 KB or 2 KB
  // shared memory (offsets from the 1 KB-aligned base)
  static constexpr int kSmemA = 0;
  static constexpr int kSmemB = kSmemA + kStages * kAStageBytes;
  static constexpr int kSmemSfa = kSmemB + kStages * kBStageBytes;
  static constexpr int kSmemSfb = kSmemSfa + kStages * kSfStageBytes;
  static constexpr int kSmemEpi = kSmemSfb + kStages * kSfStageBytes;
  static constexpr int kSmemBar = kSmemEpi + kEpiBytes;
  static constexpr int kSmemWorkIds = kSmemBar + 8 * kNumBars;
  static constexpr int kSmemTmemBase = kSmemWorkIds + 4 * kWorkSlots;
  static constexpr int kSmemTotal = kSmemTmemBase + 16;
  static constexpr int kSmemAlloc = kSmemTotal + 1024;  // room to align the base to 1 KB
  // TMEM columns: 2 accumulator buffers of kAccCols fp32 columns, then per stage
  // the A scale chunks and the B scale chunks (4 columns per chunk). An MXFP4
  // buffer holds two weight tiles' accumulators (2 x kBRows: two-tile down
  // units, 2 x 96 + 2 x 4 x 8 = 256 columns); NVFP4's larger scale chunks leave
  // room for one (2 x 48 + 2 x 4 x 16 = 224)
  static constexpr int kAccCols = F == kFmtNv ? kBRows : 2 * kBRows;
  static constexpr int kTmemAcc = 0;
  static constexpr int kTmemSfCols = 4 * kChunks;
  static constexpr int kTmemSfa = 2 * kAccCols;
  static constexpr int kTmemSfb = kTmemSfa + kStages * kTmemSfCols;
  static constexpr int kTmemEnd = kTmemSfb + kStages * kTmemSfCols;
  static_assert(kSmemAlloc <= 232448, "expert kernel shared memory over the 227 KB limit");
  static_assert(kCtasPerSm * (kSmemAlloc + 1024) <= 233472, "two CTAs must fit one SM's 228 KB");
  static_assert(kSmemB % 1024 == 0 && kBStageBytes % 1024 == 0 && kSmemSfa % 128 == 0 && kSmemSfb % 128 == 0,
                "alignment");
};
constexpr int kTmemCols = 256;  // x kCtasPerSm = the SM's 512 columns
static_assert(Fmt<kFmtMx>::kTmemEnd <= kTmemCols && Fmt<kFmtNv>::kTmemEnd <= kTmemCols, "TMEM columns");
static_assert(kCtasPerSm * kTmemCols <= 512, "TMEM columns per SM");

constexpr int kExpertThreads = 224;  // 7 warps: producer, MMA, B loader, 4 epilogue

}  // namespace mm
