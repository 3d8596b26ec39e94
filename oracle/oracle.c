/*
 * CPU oracle — TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may load this library, and only as the
 * checker; the product path (moe_serving_profile_b200) never does.
 *
 * Plain-C restatement of the exact (integer / bit-level) stages of the
 * reference MoE expert layer (luoshuqing2001/MoE_Serving_Profile):
 *   - bf16 round-to-nearest-even, e4m3 and e2m1/ue8m0 decoding
 *   - block-scaled FP8 dequantisation     moe_serving/qwen3_parallel.py:48-53
 *   - MXFP4 decoding (transformers' _convert_moe_packed_tensors, called at
 *     moe_serving/gpt_oss_parallel.py:183-193; transformers 5.5.0
 *     integrations/mxfp4.py:279-330 is the readable proxy)
 *   - router logits in the library's documented fixed fp32 order, and the
 *     top-k selection of torch.topk on CUDA (k <= 32) with its slot order
 *     for equal values, the selection the reference's routers run
 *     (transformers qwen3_moe/modeling_qwen3_moe.py:266 and
 *     gpt_oss/modeling_gpt_oss.py:129 call torch.topk; moe_serving/moe.py:104)
 *   - the expert-contiguous permutation in (slot, token) order
 *     (moe_serving/parallel_numerics.py:21-26)
 *   - the ordered bf16 combine (parallel_numerics.py:26-35; moe.py:123-136)
 *   - e4m3 encoding and the W8A8 per-(row, 128-column) activation
 *     quantisation (efficient_kernels.py:243-274)
 * Compile with -ffp-contract=off so every float operation rounds as written.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

/* float -> bf16 bits, round to nearest even; NaN stays a quiet NaN */
uint16_t oracle_f32_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}
float oracle_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }
static float bf16r(float f) { return oracle_bf16_to_f32(oracle_f32_to_bf16(f)); }

/* e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa; 0x7f/0xff are NaN, no inf */
float oracle_e4m3_to_f32(uint8_t v) {
  const uint32_t s = v >> 7, e = (v >> 3) & 15u, m = v & 7u;
  float mag;
  if (e == 15u && m == 7u) return NAN;
  if (e == 0u)
    mag = ldexpf((float)m, -9); /* subnormal: m/8 * 2^-6 */
  else
    mag = ldexpf(1.0f + (float)m / 8.0f, (int)e - 7);
  return s ? -mag : mag;
}

/* bf16(fp32(w) * scale[r/br][c/bc]) for w e4m3 [rows, cols] */
void oracle_dequant_fp8(const uint8_t* w, const float* scales, int rows, int cols, int br,
                        int bc, uint16_t* out) {
  const int nbc = (cols + bc - 1) / bc;
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < cols; ++c) {
      const float s = scales[(r / br) * nbc + c / bc];
      out[(long)r * cols + c] = oracle_f32_to_bf16(oracle_e4m3_to_f32(w[(long)r * cols + c]) * s);
    }
}

static const float kE2M1[16] = {0.0f,  0.5f,  1.0f,  1.5f,  2.0f,  3.0f,  4.0f,  6.0f,
                                -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

/* 2^(s - 127) as an fp32 value (s = 0 is the subnormal 2^-127, s = 255 +inf) */
static float ue8m0(uint8_t s) {
  if (s == 0) return u2f(0x00400000u);
  if (s == 255) return u2f(0x7f800000u);
  return u2f((uint32_t)s << 23);
}

/* blocks [rows, G, 16] bytes (low nibble = even element), scales [rows, G]
   -> bf16 [rows, G * 32] (row-major, before the reference's transpose) */
void oracle_decode_mxfp4(const uint8_t* blocks, const uint8_t* scales, int rows, int G,
                         uint16_t* out) {
  for (long r = 0; r < rows; ++r)
    for (int g = 0; g < G; ++g) {
      const float sc = ue8m0(scales[r * G + g]);
      for (int b = 0; b < 16; ++b) {
        const uint8_t byte = blocks[(r * G + g) * 16 + b];
        const long o = r * (long)G * 32 + g * 32 + 2 * b;
        out[o] = oracle_f32_to_bf16(kE2M1[byte & 15] * sc);
        out[o + 1] = oracle_f32_to_bf16(kE2M1[byte >> 4] * sc);
      }
    }
}

/* Fixed-order fp32 dot product of two bf16 vectors of length H (H % 8 == 0):
   segment s covers h in [64 s, min(64 s + 64, H)) and is one fmaf chain in
   increasing h starting from 0; the segments are then added in increasing s
   (dot = ((seg0 + seg1) + seg2) + ...). The same order as the router kernels
   (moe_serving_profile_b200/csrc/router.cu), independent of T and of the
   launch shape. */
float oracle_dot_bf16(const uint16_t* x, const uint16_t* w, int H) {
  float dot = 0.0f;
  for (int s0 = 0; s0 < H; s0 += 64) {
    const int s1 = s0 + 64 < H ? s0 + 64 : H;
    float seg = 0.0f;
    for (int h = s0; h < s1; ++h) seg = fmaf(oracle_bf16_to_f32(x[h]), oracle_bf16_to_f32(w[h]), seg);
    dot = s0 == 0 ? seg : dot + seg;
  }
  return dot;
}

/* mode 0: bf16 logits, mode 1: bf16 logits with bias (bf16 [E]), mode 2: fp32.
   Output as float (holding the bf16 value for modes 0, 1). */
void oracle_router_logits(const uint16_t* x, long ldx, const uint16_t* w, const uint16_t* bias,
                          int T, int H, int E, int mode, float* logits) {
  for (int t = 0; t < T; ++t)
    for (int e = 0; e < E; ++e) {
      float acc = oracle_dot_bf16(x + (long)t * ldx, w + (long)e * H, H);
      if (mode == 2) {
        logits[(long)t * E + e] = acc;
      } else {
        if (mode == 1) acc += oracle_bf16_to_f32(bias[e]);
        logits[(long)t * E + e] = bf16r(acc);
      }
    }
}

static int greater(float a, int ia, float b, int ib) {
  /* NaN sorts above every number; equal values by ascending index */
  const int na = a != a, nb = b != b;
  if (na || nb) {
    if (na && nb) return ia < ib;
    return na;
  }
  if (a != b) return a > b;
  return ia < ib;
}

/* torch's descending comparator: a NaN is larger than any number */
static int key_gt(float a, float b) { return (a != a && b == b) || a > b; }

/* top-k of each row of values [T, E] in the slot order torch.topk gives on
   CUDA for k <= 32 (pinned against torch's outputs by the fixtures of
   tests/golden/make_router_golden.py):
     1. the selected set: keys above the k-th largest key, then the
        lowest-index keys equal to it;
     2. laid out in index order, keys above the k-th first, in 32 slots
        (slots k..31 invalid);
     3. sorted by a 32-slot bitonic network whose comparator (a at the lower
        slot, b at the upper) exchanges the pair when
        ((a valid and a > b) or b invalid) equals the stage's direction
        (direction = bit `size` of the slot in the building stages, 0 in the
        final merge), so equal keys trade places on every ascending stage. */
void oracle_topk(const float* values, int T, int E, int K, int64_t* indices) {
  char* taken = (char*)malloc((size_t)E);
  int sel[32];
  for (int t = 0; t < T; ++t) {
    memset(taken, 0, (size_t)E);
    const float* row = values + (long)t * E;
    for (int k = 0; k < K; ++k) {
      int best = -1;
      for (int e = 0; e < E; ++e) {
        if (taken[e]) continue;
        if (best < 0 || greater(row[e], e, row[best], best)) best = e;
      }
      taken[best] = 1;
      sel[k] = best;
    }
    const float kth = row[sel[K - 1]];
    float key[32];
    int idx[32], valid[32];
    int n = 0;
    for (int pass = 0; pass < 2; ++pass)          /* above the k-th, then equal to it */
      for (int e = 0; e < E; ++e) {
        if (!taken[e]) continue;
        const int above = key_gt(row[e], kth) || (row[e] != row[e] && kth == kth);
        if (above == (pass == 0)) {
          key[n] = row[e];
          idx[n] = e;
          valid[n] = 1;
          ++n;
        }
      }
    for (int i = n; i < 32; ++i) {
      key[i] = 0.f;
      idx[i] = -1;
      valid[i] = 0;
    }
    for (int size = 2; size <= 32; size <<= 1)
      for (int stride = size >> 1; stride > 0; stride >>= 1)
        for (int a = 0; a < 32; ++a) {
          if (a & stride) continue;
          const int b = a + stride;
          const int dir = size < 32 ? (a & size) != 0 : 0;
          const int swap = (key_gt(key[a], key[b]) && valid[a]) || !valid[b];
          if (swap == dir) {
            const float tk = key[a];
            const int ti = idx[a], tv = valid[a];
            key[a] = key[b], idx[a] = idx[b], valid[a] = valid[b];
            key[b] = tk, idx[b] = ti, valid[b] = tv;
          }
        }
    for (int k = 0; k < K; ++k) indices[(long)t * K + k] = idx[k];
  }
  free(taken);
}

/* Stable counting sort of the assignments in slot-major order. Ids outside
   [0, E) are dropped (inverse = -1). Returns the number of placed rows. */
int oracle_permute(const int64_t* idx, int T, int K, int E, int32_t* counts, int32_t* offsets,
                   int32_t* perm_src, int32_t* inverse) {
  memset(counts, 0, sizeof(int32_t) * (size_t)E);
  for (long j = 0; j < (long)T * K; ++j) {
    const int64_t e = idx[j];
    if (e >= 0 && e < E) counts[e]++;
  }
  offsets[0] = 0;
  for (int e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
  int32_t* run = (int32_t*)malloc(sizeof(int32_t) * (size_t)E);
  memcpy(run, offsets, sizeof(int32_t) * (size_t)E);
  for (int k = 0; k < K; ++k)
    for (int t = 0; t < T; ++t) {
      const long src = (long)t * K + k;
      const int64_t e = idx[src];
      if (e < 0 || e >= E) {
        inverse[src] = -1;
        continue;
      }
      const int pos = run[e]++;
      perm_src[pos] = (int32_t)src;
      inverse[src] = pos;
    }
  free(run);
  return offsets[E];
}

/* Ordered combine; order 0: ascending expert id, order 1: ascending
   (expert / epr, slot). scale: contribution = bf16(f32(row) * w). */
void oracle_combine(const uint16_t* rows, long ld_rows, const int32_t* inverse,
                    const int64_t* idx, int T, int K, int H, int order, int epr, int64_t lo,
                    int64_t hi, int scale, const float* weights, uint16_t* out) {
  int* sel = (int*)malloc(sizeof(int) * (size_t)K);
  int64_t* key = (int64_t*)malloc(sizeof(int64_t) * (size_t)K);
  float* acc = (float*)malloc(sizeof(float) * (size_t)H);
  for (int t = 0; t < T; ++t) {
    int n = 0;
    for (int k = 0; k < K; ++k) {
      const int64_t e = idx[(long)t * K + k];
      const int r = inverse[(long)t * K + k];
      if (r < 0 || e < lo || e >= hi) continue;
      const int64_t kk = order == 0 ? e * 64 + k : (e / epr) * 64 + k;
      int p = n++;
      while (p > 0 && key[p - 1] > kk) {
        key[p] = key[p - 1];
        sel[p] = sel[p - 1];
        --p;
      }
      key[p] = kk;
      sel[p] = k;
    }
    for (int h = 0; h < H; ++h) acc[h] = 0.0f;
    for (int i = 0; i < n; ++i) {
      const int k = sel[i];
      const int r = inverse[(long)t * K + k];
      const float wv = scale ? weights[(long)t * K + k] : 1.0f;
      for (int h = 0; h < H; ++h) {
        float c = oracle_bf16_to_f32(rows[(long)r * ld_rows + h]);
        if (scale) c = bf16r(c * wv);
        acc[h] = bf16r(acc[h] + c);
      }
    }
    for (int h = 0; h < H; ++h) out[(long)t * H + h] = oracle_f32_to_bf16(acc[h]);
  }
  free(sel);
  free(key);
  free(acc);
}

/* fp32 -> e4m3fn code, round to nearest even, saturating to +-448 (the
   largest finite value); NaN -> 0x7f. From the format: normal values
   2^(e-7) * (1 + m/8) for exponent field e = 1..15 (e = 15, m = 7 is NaN),
   subnormals 2^-6 * m/8. In each binade [2^p, 2^(p+1)) (p >= -6) the
   representable values are 2^(p-3) apart, below 2^-6 they are 2^-9 apart, so
   a value rounds to the nearest multiple of that quantum (ties to even). */
uint8_t oracle_f32_to_e4m3(float f) {
  const uint8_t sign = (f2u(f) >> 31) ? 0x80 : 0x00;
  const float a = fabsf(f);
  if (a != a) return 0x7f;
  if (a >= 448.0f) return sign | 0x7e;
  if (a == 0.0f) return sign;
  int ex;
  frexpf(a, &ex);                       /* a in [2^(ex-1), 2^ex) */
  int p = ex - 1;
  if (p < -6) p = -6;
  const float step = ldexpf(1.0f, p - 3);
  const float v = rintf(a / step) * step; /* exact scaling; rintf rounds half to even */
  if (v == 0.0f) return sign;
  frexpf(v, &ex);
  p = ex - 1;                           /* v may have rounded up into the next binade */
  if (p < -6) return sign | (uint8_t)(v / ldexpf(1.0f, -9));      /* subnormal: m = v / 2^-9 */
  const int mant = (int)(v / ldexpf(1.0f, p - 3)) - 8;
  return sign | (uint8_t)(((p + 7) << 3) | mant);
}

/* Dynamic FP8 activation quantisation of the W8A8 path (the activation side
   of moe_serving/efficient_kernels.py:243-274): for row r and 128-column
   group g, s[r,g] = amax / 448 over the group's bf16 values (1 if all are
   zero) and q[r,c] = e4m3(x[src(r), c] / s[r,g]) for c < k_valid, 0 up to
   k_pad. src(r) = map[r] / div, or r without a map. */
void oracle_act_quant_fp8(const uint16_t* x, long ldx, const int32_t* map, int div, int rows,
                          int k_valid, int k_pad, uint8_t* q, float* s) {
  const int groups = (k_pad + 127) / 128;
  for (int r = 0; r < rows; ++r) {
    const long src = map ? map[r] / div : r;
    const uint16_t* xr = x + src * ldx;
    for (int g = 0; g < groups; ++g) {
      float amax = 0.0f;
      for (int c = g * 128; c < g * 128 + 128 && c < k_valid; ++c) {
        const float v = fabsf(oracle_bf16_to_f32(xr[c]));
        if (v > amax) amax = v;
      }
      const float sc = amax > 0.0f ? amax / 448.0f : 1.0f;
      s[(long)r * groups + g] = sc;
      for (int c = g * 128; c < g * 128 + 128 && c < k_pad; ++c)
        q[(long)r * k_pad + c] = c < k_valid ? oracle_f32_to_e4m3(oracle_bf16_to_f32(xr[c]) / sc) : 0;
    }
  }
}
