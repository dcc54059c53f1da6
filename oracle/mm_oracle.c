/*
 * CPU oracle of the routed-MoE chain: the bit-exact parts (TEST INFRASTRUCTURE).
 *
 * This file is the checker, never the product: only tests/, the smoke() entry
 * and bench.py's CPU-baseline leg load it. It restates the reference's
 * algorithm for each step in plain C99 with IEEE-754 binary32 arithmetic
 * (compiled with -ffp-contract=off, fmaf from libm), so that the CUDA kernels'
 * routing, permutation, quantization and combine can be compared bit for bit.
 *
 * Parity pins: or_route is checked against the reference's own route.cuh /
 * route_wide.cu compiled for the CPU (oracle/ref_route_shim.h, oracle/Makefile,
 * tests/test_oracle.py); the fixtures under tests/golden/ were generated
 * from it (tests/golden/make_golden.py).
 */
#include <math.h>
#include <stdlib.h>
#include <stdint.h>
#include <string.h>

static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bf16_to_f(uint16_t b) { return u2f((uint32_t)b << 16); }
/* round-to-nearest-even fp32 -> bf16 (NaN kept quiet) */
static inline uint16_t f_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* ---------------------------------------------------------------------------
 * Router GEMV in the kernel's fixed order: H in parts of 1024; in part p, lane l
 * (0..31) accumulates h = 1024 p + 8 (l + 32 j) + i for j = 0..3, i = 0..7, with
 * acc = fma(x, w, acc) from 0; lanes combine by the xor butterfly 16, 8, 4, 2, 1;
 * parts in order, s = ((p0 + p1) + p2) + ... Reference operation:
 * router_mma.cu:101 (logits = x . W^T in fp32 from bf16 operands); the
 * summation order is the kernel's own.
 * ------------------------------------------------------------------------- */
void or_router_gemv(const uint16_t *x, const uint16_t *w, float *logits, int T, int E, int H) {
  const int parts = H / 1024;
  for (int t = 0; t < T; ++t)
    for (int e = 0; e < E; ++e) {
      float s = 0.0f;
      for (int p = 0; p < parts; ++p) {
        float lane[32];
        for (int l = 0; l < 32; ++l) {
          float acc = 0.0f;
          for (int j = 0; j < 4; ++j)
            for (int i = 0; i < 8; ++i) {
              const int h = 1024 * p + 8 * (l + 32 * j) + i;
              acc = fmaf(bf16_to_f(x[(size_t)t * H + h]), bf16_to_f(w[(size_t)e * H + h]), acc);
            }
          lane[l] = acc;
        }
        for (int off = 16; off >= 1; off >>= 1) {
          float nxt[32];
          for (int l = 0; l < 32; ++l) nxt[l] = lane[l] + lane[l ^ off];
          memcpy(lane, nxt, sizeof(lane));
        }
        s = p == 0 ? lane[0] : s + lane[0];
      }
      logits[(size_t)t * E + e] = s;
    }
}

/* ---------------------------------------------------------------------------
 * exp(x): Cody-Waite reduction with n = rint(x log2e) (via the 1.5*2^23 add),
 * r = x - n ln2_hi - n ln2_lo, e^r by the degree-7 Taylor polynomial (Horner,
 * fma), scaled exactly by 2^n. The same operation sequence as the kernel's, so
 * the two agree bit for bit; accuracy is about 1 ulp.
 * ------------------------------------------------------------------------- */
float or_det_exp(float x) {
  if (x != x) return x;
  if (x > 0x1.62e430p+6f) return u2f(0x7f800000u);
  if (x < -0x1.a00000p+6f) return 0.0f;
  const float t = fmaf(x, 0x1.715476p+0f, 0x1.8p+23f);
  const float n = t - 0x1.8p+23f;
  float r = fmaf(-n, 0x1.62e400p-1f, x);
  r = fmaf(-n, 0x1.7f7d1cp-20f, r);
  float p = 0x1.a01a02p-13f;
  p = fmaf(p, r, 0x1.6c16c2p-10f);
  p = fmaf(p, r, 0x1.111112p-7f);
  p = fmaf(p, r, 0x1.555556p-5f);
  p = fmaf(p, r, 0x1.555556p-3f);
  p = fmaf(p, r, 0x1.000000p-1f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ni = (int)n;
  if (ni > 127) return (p * u2f((uint32_t)(ni - 1 + 127) << 23)) * 2.0f;
  if (ni < -126) return (p * u2f((uint32_t)(ni + 100 + 127) << 23)) * u2f((uint32_t)(-100 + 127) << 23);
  return p * u2f((uint32_t)(ni + 127) << 23);
}

float or_sigmoid(float x) { return 1.0f / (1.0f + or_det_exp(-x)); }

/* log(u), u >= 1 finite: u = m 2^k, m in [sqrt(1/2), sqrt(2)), log u = k ln2 +
 * 2 atanh(f / (2 + f)), f = m - 1, atanh by its odd series to s^11 (Horner in
 * z = s^2, fma); the kernel's sequence (mm_numerics.cuh det_log). */
float or_det_log(float u) {
  const uint32_t bits = f2u(u);
  int k = (int)((bits >> 23) & 0xffu) - 127;
  float m = u2f((bits & 0x7fffffu) | 0x3f800000u);
  if (m > 0x1.6a09e6p+0f) { m = m * 0.5f; k += 1; }
  const float f = m - 1.0f;
  const float s = f / (2.0f + f);
  const float z = s * s;
  float q = 0x1.745d18p-4f;
  q = fmaf(q, z, 0x1.c71c72p-4f);
  q = fmaf(q, z, 0x1.24924ap-3f);
  q = fmaf(q, z, 0x1.99999ap-3f);
  q = fmaf(q, z, 0x1.555556p-2f);
  q = fmaf(q, z, 1.0f);
  const float lm = (s + s) * q;
  const float kf = (float)k;
  return fmaf(kf, 0x1.62e400p-1f, fmaf(kf, 0x1.7f7d1cp-20f, lm));
}

/* log1p(y), y >= 0: Goldberg's log(1 + y) * y / ((1 + y) - 1). */
float or_det_log1p(float y) {
  const float u = 1.0f + y;
  if (u == 1.0f) return y;
  return or_det_log(u) * (y / (u - 1.0f));
}

/* sqrt(softplus(x)) (deepseek_v41/sm103/moe/src/gate_topk.cuh:99-104): x above
 * 20, else log1p(exp(x)); IEEE square root. */
float or_sqrtsoftplus(float x) {
  if (x != x) return x;
  const float sp = x > 20.0f ? x : or_det_log1p(or_det_exp(x));
  return sqrtf(sp);
}

static float or_score(int score_func, float l) {
  return score_func == 0 ? or_sigmoid(l) : score_func == 2 ? or_sqrtsoftplus(l) : l;
}

/* Order-preserving key of score + bias: -0 as +0 (gate_topk.cuh:129-145), NaN
 * below every number (glm5_3/sm103/primitives/ptx_tc.py:393-402). */
uint32_t or_routing_key(float v) {
  if (v != v) return 0u;
  const uint32_t b = f2u(v + 0.0f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

/* ---------------------------------------------------------------------------
 * Router top-k of every row (reference: gate_topk.cuh:101-303 and
 * glm5_3/sm103/moe/routing.py:3-11,32-70; softmax over the selected logits as
 * qwen3_5/sm103/moe/src/route_topk.cu:1-6). score_func 0: s = sigmoid(logit),
 * key = s + bias; 2: s = sqrt(softplus(logit)), key = s + bias (DeepSeek-V4.1,
 * gate_topk.cuh:99-104); 1: s = logit, key = logit + bias, weights = softmax
 * over the k selected logits. Selection: k times the largest key, the lowest expert id on
 * ties; slot order = selection order. Weights: s / (sum + eps) when eps > 0,
 * else s / (sum > 0 ? sum : 1), sum in slot order, times the routed scale;
 * renormalize 0: s * scale. Rows >= num_valid: id -1, weight 0.
 * ------------------------------------------------------------------------- */
void or_gate_topk(const float *logits, const float *bias_main, int num_valid, int score_func,
                  int renormalize, float scale, float eps, int T, int E, int K, float *weights,
                  int *ids, const float *bias_alt, const int64_t *input_ids, int64_t alt_token_id) {
  for (int t = 0; t < T; ++t) {
    const float *l = logits + (size_t)t * E;
    /* vision routing (gate_topk.cuh:290-346): a valid row whose token is
     * alt_token_id ranks with bias_alt (bias when bias_alt is NULL) */
    const int alt = input_ids && t < num_valid && input_ids[t] == alt_token_id;
    const float *bias = alt && bias_alt ? bias_alt : bias_main;
    int sel[64];
    unsigned char taken[4096];
    memset(taken, 0, (size_t)E);
    for (int k = 0; k < K; ++k) {
      int best = -1;
      uint32_t bkey = 0;
      for (int e = 0; e < E; ++e) {
        if (taken[e]) continue;
        const float s = or_score(score_func, l[e]);
        const uint32_t key = or_routing_key(s + (bias ? bias[e] : 0.0f));
        if (best < 0 || key > bkey) { best = e; bkey = key; }
      }
      sel[k] = best;
      taken[best] = 1;
    }
    float w[64];
    if (score_func == 1) {
      float m = l[sel[0]];
      for (int k = 1; k < K; ++k) m = fmaxf(m, l[sel[k]]);
      float sum = 0.0f;
      for (int k = 0; k < K; ++k) { w[k] = or_det_exp(l[sel[k]] - m); sum = sum + w[k]; }
      for (int k = 0; k < K; ++k) w[k] = (w[k] / sum) * scale;
    } else {
      float sum = 0.0f;
      for (int k = 0; k < K; ++k) { w[k] = or_score(score_func, l[sel[k]]); sum = sum + w[k]; }
      if (renormalize == 2) {
        /* GLM-5.3 (glm5_3/sm103/moe/routing.py:3-11; routing_weight in
         * glm5_3/sm103/primitives/ptx_tc.py): the selected scores summed in the
         * order of a warp xor-butterfly with slot k in lane k (lane 0's order is
         * the halving t[i] += t[i + off], off = 8, 4, 2, 1), then
         * w = bf16(scale * s / (sum + eps)) with the scale multiplied first */
        float t[16];
        for (int k = 0; k < 16; ++k) t[k] = k < K ? w[k] : 0.0f;
        for (int off = 8; off >= 1; off >>= 1)
          for (int i = 0; i < off; ++i) t[i] = t[i] + t[i + off];
        const float d = t[0] + eps;
        for (int k = 0; k < K; ++k) w[k] = bf16_to_f(f_to_bf16((scale * w[k]) / d));
      } else if (renormalize) {
        const float norm = eps > 0.0f ? sum + eps : (sum > 0.0f ? sum : 1.0f);
        for (int k = 0; k < K; ++k) w[k] = (w[k] / norm) * scale;
      } else {
        for (int k = 0; k < K; ++k) w[k] = w[k] * scale;
      }
    }
    const int valid = t < num_valid;
    for (int k = 0; k < K; ++k) {
      ids[(size_t)t * K + k] = valid ? sel[k] : -1;
      weights[(size_t)t * K + k] = valid ? w[k] : 0.0f;
    }
  }
}

/* ---------------------------------------------------------------------------
 * Route record (route.cuh:6-46 layout; route.cuh:94-161 and route_wide.cu:62-163
 * rules): local experts e = id - offset in [0, experts) ascending; an expert's
 * rows ascending; each expert owns ceil(count/8) consecutive 8-row tiles starting
 * at the exclusive prefix sum of the tiles of the experts below it;
 * permuted[t,k] = first_tile*8 + rank (rank = earlier rows choosing e), -1 for a
 * non-local id. record: [0] = 8*tiles, [1] = tiles, [2,4) = 0,
 * [4, 4+C) tile -> expert, [4+C, 4+2C) tile -> row limit
 * min((tile+1)*8, first*8 + count), [4+2C, 4+2C+8M) padded row -> token, the
 * rest zero; M = max_ctas, C = M rounded up to 4.
 * ------------------------------------------------------------------------- */
int or_route_words(int T, int K, int experts) {
  const int slots = T * K, filled = experts < slots ? experts : slots;
  const int m = filled + (slots - filled) / 8;
  return 4 + 2 * ((m + 3) / 4 * 4) + 8 * m;
}

void or_route(const int *ids, int *permuted, int *record, int T, int K, int experts, int offset) {
  const int slots = T * K, filled = experts < slots ? experts : slots;
  const int m = filled + (slots - filled) / 8;
  const int cw = (m + 3) / 4 * 4, limit_off = 4 + cw, token_off = 4 + 2 * cw;
  memset(record, 0, sizeof(int) * (size_t)or_route_words(T, K, experts));
  static int count[4096], first[4096];
  for (int e = 0; e < experts; ++e) count[e] = 0;
  /* balanced dealing (route.cuh:39-46, route_wide.cu:87-110): a negative
   * offset selects group -1 - offset of two; ids are global, and of the step's
   * distinct experts in id order the k-th belongs to group k % 2 */
  const int deal = offset < 0, group = deal ? -1 - offset : 0;
  if (deal) offset = 0;
  for (int s = 0; s < slots; ++s) {
    const int e = ids[s] - offset;
    if (e >= 0 && e < experts) count[e]++;
  }
  if (deal) {
    int rank = 0;
    for (int e = 0; e < experts; ++e) {
      if (!count[e]) continue;
      if ((rank & 1) != group) count[e] = 0;
      rank++;
    }
  }
  int tiles = 0;
  for (int e = 0; e < experts; ++e) { first[e] = tiles; tiles += (count[e] + 7) / 8; }
  record[0] = 8 * tiles;
  record[1] = tiles;
  for (int s = 0; s < slots; ++s) {
    const int t = s / K, e = ids[s] - offset;
    if (e < 0 || e >= experts || count[e] == 0) { permuted[s] = -1; continue; }
    int rank = 0;  /* earlier rows that chose e (top-k ids of a row are distinct) */
    for (int s2 = 0; s2 < slots; ++s2)
      if (s2 / K < t && ids[s2] - offset == e) rank++;
    const int p = first[e] * 8 + rank;
    permuted[s] = p;
    record[token_off + p] = t;
    if (rank % 8 == 0) {
      const int tile = first[e] + rank / 8;
      const int lim = first[e] * 8 + count[e];
      record[4 + tile] = e;
      record[limit_off + tile] = (tile + 1) * 8 < lim ? (tile + 1) * 8 : lim;
    }
  }
}

/* ---------------------------------------------------------------------------
 * MXFP8 (E4M3 codes + E8M0 scale per 32), route_quant.cuh:1-15 and
 * gemm1.cu:905-1000: amax of the block (448 when zero) times fp32(1/448); the
 * E8M0 code is that product's exponent, rounded up when its mantissa is not
 * zero; codes are e4m3(v * 2^(127-code)), round to nearest even, saturating.
 * The second term (this build's default numerics) quantizes the residual
 * v - e4m3 * 2^(code-127) the same way.
 * ------------------------------------------------------------------------- */
uint32_t or_mx_scale_code(float amax) {
  const float num = amax == 0.0f ? 448.0f : amax;
  const uint32_t b = f2u(num * 0x1.24924ap-9f);
  const uint32_t ex = (b >> 23) & 0xffu, ma = b & 0x7fffffu;
  uint32_t code = ex;
  if (ma != 0u && ex != 254u) {
    if (ex != 0u) code = ex + 1u;
    else if (ma > 0x400000u) code = 1u;
  }
  if (ex == 255u) code = 255u;
  return code;
}
static float mx_inverse(uint32_t c) { return c == 254u ? u2f(0x400000u) : u2f((254u - c) << 23); }
static float mx_scale_value(uint32_t c) { return c == 0u ? u2f(0x400000u) : u2f(c << 23); }

/* e4m3 (fn) encoding, round to nearest even, finite overflow saturating to 448 */
uint8_t or_e4m3(float v) {
  if (v != v) return 0x7f;
  const uint8_t sign = (f2u(v) >> 31) ? 0x80 : 0x00;
  double a = fabs((double)v);
  if (a >= 448.0) return sign | 0x7e;
  int code;
  if (a < 0x1p-6) {  /* subnormal grid: m * 2^-9 */
    const double q = nearbyint(a * 512.0);
    code = (int)q;  /* q == 8 is the smallest normal: exponent field 1, mantissa 0 */
  } else {
    int e;
    frexp(a, &e);   /* a = f * 2^e, f in [0.5, 1) */
    e -= 1;         /* a in [2^e, 2^(e+1)) */
    double q = nearbyint(a * ldexp(1.0, 3 - e));  /* 8..16 */
    if (q >= 16.0) { q = 8.0; e += 1; }
    if (e > 8) return sign | 0x7e;
    code = ((e + 7) << 3) | ((int)q - 8);
    if (code > 0x7e) code = 0x7e;
  }
  return sign | (uint8_t)code;
}
float or_e4m3_value(uint8_t c) {
  const uint32_t s = c >> 7, e = (c >> 3) & 15u, m = c & 7u;
  float v;
  if (e == 0u) v = (float)m * 0x1p-9f;
  else if (e == 15u && m == 7u) v = u2f(0x7fc00000u);
  else v = u2f(((e + 120u) << 23) | (m << 20));
  return s ? -v : v;
}

/* blocks of 32 values -> codes/scales of `terms` terms */
void or_mxfp8_quant(const float *v, int nblocks, int terms, uint8_t *q_hi, uint8_t *q_lo,
                    uint8_t *s_hi, uint8_t *s_lo) {
  for (int b = 0; b < nblocks; ++b) {
    const float *x = v + (size_t)b * 32;
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    const uint32_t c = or_mx_scale_code(amax);
    const float inv = mx_inverse(c), sv = mx_scale_value(c);
    float r[32], amax2 = 0.0f;
    for (int i = 0; i < 32; ++i) {
      const uint8_t q = or_e4m3(x[i] * inv);
      q_hi[(size_t)b * 32 + i] = q;
      r[i] = x[i] - or_e4m3_value(q) * sv;
      amax2 = fmaxf(amax2, fabsf(r[i]));
    }
    s_hi[b] = (uint8_t)c;
    if (terms < 2) continue;
    const uint32_t c2 = or_mx_scale_code(amax2);
    const float inv2 = mx_inverse(c2);
    for (int i = 0; i < 32; ++i) q_lo[(size_t)b * 32 + i] = or_e4m3(r[i] * inv2);
    s_lo[b] = (uint8_t)c2;
  }
}

/* ---------------------------------------------------------------------------
 * MXFP4 terms of the activations (the kernels' numerics: E2M1 codes, E8M0 scale
 * per 32): per block, term t quantizes the residual r left by the earlier terms:
 * amax of |r| (6 when zero) times fp32(1/6), E8M0 code = that product's
 * exponent, rounded up when its mantissa is not zero (the MX rule above with
 * E2M1's largest magnitude 6); codes e2m1(r * 2^(127-code)), round to nearest
 * even, saturating at 6; r -= value(code) * 2^(code-127). Two codes per byte,
 * the even element in the low nibble.
 * ------------------------------------------------------------------------- */
uint32_t or_mx4_scale_code(float amax) {
  const float num = amax == 0.0f ? 6.0f : amax;
  const uint32_t b = f2u(num * 0x1.555556p-3f);
  const uint32_t ex = (b >> 23) & 0xffu, ma = b & 0x7fffffu;
  uint32_t code = ex;
  if (ma != 0u && ex != 254u) {
    if (ex != 0u) code = ex + 1u;
    else if (ma > 0x400000u) code = 1u;
  }
  if (ex == 255u) code = 255u;
  return code;
}

/* E2M1 code (bits 0-3) of v: round to nearest, ties to the even code, |v| > 6 -> 6 */
uint8_t or_e2m1(float v) {
  const uint8_t sign = (f2u(v) >> 31) ? 8u : 0u;
  const float a = fabsf(v);
  uint8_t m;
  if (a != a) m = 7;
  else if (a <= 0.25f) m = 0;
  else if (a < 0.75f) m = 1;
  else if (a <= 1.25f) m = 2;
  else if (a < 1.75f) m = 3;
  else if (a <= 2.5f) m = 4;
  else if (a < 3.5f) m = 5;
  else if (a <= 5.0f) m = 6;
  else m = 7;
  return sign | m;
}

float or_e2m1_value(uint8_t c) {
  static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  const float v = mag[c & 7u];
  return (c & 8u) ? -v : v;
}

/* v: nblocks x 32 values; q: [terms][nblocks * 16] bytes; s: [terms][nblocks] */
void or_fp4_quant(const float *v, int nblocks, int terms, uint8_t *q, uint8_t *s) {
  for (int b = 0; b < nblocks; ++b) {
    float r[32];
    for (int i = 0; i < 32; ++i) r[i] = v[(size_t)b * 32 + i];
    for (int t = 0; t < terms; ++t) {
      float amax = 0.0f;
      for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(r[i]));
      const uint32_t c = or_mx4_scale_code(amax);
      const float inv = mx_inverse(c), sv = mx_scale_value(c);
      for (int i = 0; i < 32; i += 2) {
        const uint8_t lo = or_e2m1(r[i] * inv), hi = or_e2m1(r[i + 1] * inv);
        q[(size_t)t * nblocks * 16 + (size_t)b * 16 + i / 2] = (uint8_t)(lo | (hi << 4));
        r[i] = r[i] - or_e2m1_value(lo) * sv;
        r[i + 1] = r[i + 1] - or_e2m1_value(hi) * sv;
      }
      s[(size_t)t * nblocks + b] = (uint8_t)c;
    }
  }
}

/* ---------------------------------------------------------------------------
 * Weighted combine (all_reduce_mhc.py:528-640; glm5_3/sm103/moe/finalize.py):
 * acc = fma(w, row, acc) over k in slot order from 0 (perm -1 skipped), routed =
 * bf16(acc), out = bf16(routed + shared).
 * ------------------------------------------------------------------------- */
void or_finalize(const uint16_t *rows, const float *w, const int *perm, const uint16_t *shared,
                 uint16_t *out, int T, int K, int H) {
  for (int t = 0; t < T; ++t)
    for (int h = 0; h < H; ++h) {
      float acc = 0.0f;
      for (int k = 0; k < K; ++k) {
        const int p = perm[t * K + k];
        if (p < 0) continue;
        acc = fmaf(w[t * K + k], bf16_to_f(rows[(size_t)p * H + h]), acc);
      }
      const float routed = bf16_to_f(f_to_bf16(acc));
      const float s = shared ? bf16_to_f(shared[(size_t)t * H + h]) : 0.0f;
      out[(size_t)t * H + h] = f_to_bf16(routed + s);
    }
}

/* ---------------------------------------------------------------------------
 * Cross-rank sum of the ranks' finalized partials (all_reduce_mhc.py:955-977,
 * rank_lanes = 1): acc = 0; acc += bf16 partial of rank r for r = 0..world-1
 * in fp32; out = bf16(acc). y holds world arrays of n values, rank-major.
 * ------------------------------------------------------------------------- */
void or_allreduce_ranks(const uint16_t *y, uint16_t *out, int world, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    float acc = 0.0f;
    for (int r = 0; r < world; ++r) acc += bf16_to_f(y[(size_t)r * n + i]);
    out[i] = f_to_bf16(acc);
  }
}

/* ---------------------------------------------------------------------------
 * All-reduce + residual + RMSNorm epilogue of the combine (the hop of
 * qwen3_5/sm103/hop/src/hop.cu:119-139, q35_hop.cuh:258-336: pre =
 * bf16(rank-order fp32 sum + residual); inv = 1/sqrt(sum(pre^2)/H + eps);
 * norm = bf16((pre * inv) * gamma)). The sum of squares follows the kernel's
 * fixed fold: a thread owns 8 consecutive features (feature 8 * (256 * c + 32 *
 * w + l) for CTA c, warp w, lane l), sums x*x over them in order from 0; a
 * warp folds its lanes by xor butterfly 16, 8, 4, 2, 1; a CTA adds its 8 warp
 * sums in order from 0; the row adds its CTA sums in order from 0. sqrt and
 * the divisions are IEEE (correctly rounded). y: world arrays of T x H bf16,
 * rank-major. gamma NULL: norm_out is not written.
 * ------------------------------------------------------------------------- */
void or_allreduce_norm(const uint16_t *y, const uint16_t *residual, const uint16_t *gamma, float eps,
                       uint16_t *residual_out, uint16_t *norm_out, int world, int T, int H) {
  const size_t n = (size_t)T * H;
  const int ctas = (H + 2047) / 2048;
  float *pre = (float *)malloc(sizeof(float) * (size_t)H);
  for (int t = 0; t < T; ++t) {
    for (int h = 0; h < H; ++h) {
      const size_t i = (size_t)t * H + h;
      float acc = 0.0f;
      for (int r = 0; r < world; ++r) acc += bf16_to_f(y[(size_t)r * n + i]);
      const uint16_t p = f_to_bf16(acc + bf16_to_f(residual[i]));
      residual_out[i] = p;
      pre[h] = bf16_to_f(p);
    }
    float total = 0.0f;
    for (int c = 0; c < ctas; ++c) {
      float cta = 0.0f;
      for (int w = 0; w < 8; ++w) {
        float lane[32];
        for (int l = 0; l < 32; ++l) {
          const int h0 = 8 * (256 * c + 32 * w + l);
          float s = 0.0f;
          if (h0 < H)
            for (int e = 0; e < 8; ++e) s += pre[h0 + e] * pre[h0 + e];
          lane[l] = s;
        }
        for (int off = 16; off >= 1; off >>= 1) {
          float nxt[32];
          for (int l = 0; l < 32; ++l) nxt[l] = lane[l] + lane[l ^ off];
          memcpy(lane, nxt, sizeof(lane));
        }
        cta += lane[0];
      }
      total += cta;
    }
    const float inv = 1.0f / sqrtf(total / (float)H + eps);
    if (gamma && norm_out)
      for (int h = 0; h < H; ++h)
        norm_out[(size_t)t * H + h] = f_to_bf16((pre[h] * inv) * bf16_to_f(gamma[h]));
  }
  free(pre);
}

/* ---------------------------------------------------------------------------
 * NVFP4 terms (E2M1 codes, an E4M3 scale per 16 under a global scale gs; the
 * reference's rule glm5_3/sm103/primitives/ptx_tc.py:320-337 written with IEEE
 * operations): per block of 16, term t quantizes the residual r left by the
 * earlier terms: sf = e4m3(gs * (amax(|r|) * fp32(1/6))) RN saturating, the
 * multiplier f = gs / value(sf) (0 when sf is 0), codes e2m1(r * f) RN
 * saturating, r -= (e2m1 * value(sf)) * inv_gs. q: [terms][nblocks * 8] bytes
 * (element 2j in the low nibble), s: [terms][nblocks].
 * ------------------------------------------------------------------------- */
uint8_t or_nv4_scale_code(float amax, float gs) { return or_e4m3(gs * (amax * 0x1.555556p-3f)); }

void or_nvfp4_quant(const float *v, int nblocks, int terms, float gs, float inv_gs, uint8_t *q, uint8_t *s) {
  for (int b = 0; b < nblocks; ++b) {
    float r[16];
    for (int i = 0; i < 16; ++i) r[i] = v[(size_t)b * 16 + i];
    for (int t = 0; t < terms; ++t) {
      float amax = 0.0f;
      for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(r[i]));
      const uint8_t c = or_nv4_scale_code(amax, gs);
      const float sv = or_e4m3_value(c);
      const float f = sv == 0.0f ? 0.0f : gs / sv;
      for (int i = 0; i < 16; i += 2) {
        const uint8_t lo = or_e2m1(r[i] * f), hi = or_e2m1(r[i + 1] * f);
        q[(size_t)t * nblocks * 8 + (size_t)b * 8 + i / 2] = (uint8_t)(lo | (hi << 4));
        r[i] = r[i] - (or_e2m1_value(lo) * sv) * inv_gs;
        r[i + 1] = r[i + 1] - (or_e2m1_value(hi) * sv) * inv_gs;
      }
      s[(size_t)t * nblocks + b] = c;
    }
  }
}
