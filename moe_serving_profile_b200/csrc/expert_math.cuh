// Element arithmetic shared by the grouped expert GEMMs (tcgen05 tiles and
// the register-operand decode kernel): the packed weight blob's layout
// constants, the exact FP8 / MXFP4 weight conversions and the epilogue
// activations, each in the reference's order of bf16 roundings.
#pragma once

#include "ptx.cuh"

namespace b200 {

constexpr uint32_t kRawFp8 = 128u * 64u;    // 128 rows x 64 e4m3
constexpr uint32_t kRawMx = 128u * 32u;     // 128 rows x 64 e2m1
// scale forms of a packed blob: FP8 one fp32 per 64-row half, FP8 fp32 per
// (row, 16-column chunk), MXFP4 two ue8m0 bytes per row
enum { kScaleHalf = 0, kScaleChunk = 1, kScaleMx = 2 };
enum { kWBf16 = 0, kWFp8 = 1, kWMx = 2 };
enum { kEpiSwiglu = 0, kEpiClamp = 1, kEpiDown = 2, kEpiClampF32 = 3, kEpiDownF32 = 4 };

// 2^(s-127) as the fp32 value torch's ldexp multiplies by (exact, including
// the subnormal s = 0 and the overflow s = 255).
__device__ __forceinline__ float ue8m0_to_f32(uint32_t s) {
  if (s == 0u) return __uint_as_float(0x00400000u);
  if (s == 255u) return __uint_as_float(0x7f800000u);
  return __uint_as_float(s << 23);
}

// Two f16 (one word, element 0 low) -> two fp32 (exact).
__device__ __forceinline__ void f16x2_to_f32(uint32_t h, float& x, float& y) {
  asm("{\n\t.reg .f16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
      "cvt.f32.f16 %0, a;\n\tcvt.f32.f16 %1, b;\n\t}"
      : "=f"(x), "=f"(y) : "r"(h));
}

// 16 e4m3 -> 16 bf16 = bf16(fp32(w) * scale) through the hardware e4m3 -> f16
// conversion (exact), an exact f16 -> fp32 widening, one fp32 multiply and
// one round to bf16: the reference's arithmetic for every scale.
__device__ __forceinline__ void fp8x16_cvt(const uint4& q, float scale, uint32_t (&o)[8]) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t h01, h23;
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, lo;\n\tcvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
        : "=r"(h01), "=r"(h23) : "r"(w[i]));
    float a0, a1, a2, a3;
    f16x2_to_f32(h01, a0, a1);
    f16x2_to_f32(h23, a2, a3);
    mul2_f32(a0, a1, scale);
    mul2_f32(a2, a3, scale);
    o[2 * i] = pack_bf16x2(a0, a1);
    o[2 * i + 1] = pack_bf16x2(a2, a3);
  }
}

// 32 e2m1 (16 bytes, element 0 in the low nibble) -> 32 bf16 =
// e2m1 * 2^(S-127) through the hardware e2m1 -> f16 conversion (exact); the
// power-of-two scale and the bf16 rounding are exact too.
__device__ __forceinline__ void mx32_cvt(const uint4& q, uint32_t sexp, uint32_t (&o)[16]) {
  const float s = ue8m0_to_f32(sexp);
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t h[4];
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3]) : "r"(w[i]));
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      float lo, hi;
      f16x2_to_f32(h[b], lo, hi);
      mul2_f32(lo, hi, s);
      o[4 * i + b] = pack_bf16x2(lo, hi);
    }
  }
}

// 16 e2m1 (8 bytes, element 0 in the low nibble of q.x) -> 16 bf16 =
// e2m1 * 2^(S-127), element pairs in o[0..7]; arithmetic as mx32_cvt.
__device__ __forceinline__ void mx16_cvt(const uint2& q, uint32_t sexp, uint32_t (&o)[8]) {
  const float s = ue8m0_to_f32(sexp);
  const uint32_t w[2] = {q.x, q.y};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    uint32_t h[4];
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3]) : "r"(w[i]));
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      float lo, hi;
      f16x2_to_f32(h[b], lo, hi);
      mul2_f32(lo, hi, s);
      o[4 * i + b] = pack_bf16x2(lo, hi);
    }
  }
}

// The epilogue roundings use the hardware conversion (bf16r): these warps
// share the SM's issue slots with the converter warps, and the integer form
// takes four operations a value.
__device__ __forceinline__ float silu_bf16(float g) { return bf16r(g / (1.f + expf(-g))); }

__device__ __forceinline__ float epilogue_gated(int epi, float g, float u, float bg, float bu,
                                                float alpha, float limit) {
  if (epi == kEpiSwiglu) {
    const float gb = bf16r(g);
    const float ub = bf16r(u);
    return bf16r(silu_bf16(gb) * ub);
  }
  if (epi == kEpiClampF32) {
    // fp32 throughout, one rounding: fp32 accumulator + fp32 bias, clamp,
    // gate * sigmoid(alpha * gate) * (up + 1)
    float gf = g + bg;
    float uf = u + bu;
    gf = gf > limit ? limit : gf;
    uf = uf < -limit ? -limit : (uf > limit ? limit : uf);
    const float sg = gf / (1.f + expf(-alpha * gf));
    return bf16r(sg * (uf + 1.f));
  }
  float gb = bf16r(bf16r(g) + bg);
  float ub = bf16r(bf16r(u) + bu);
  gb = gb > limit ? limit : gb;
  ub = ub < -limit ? -limit : (ub > limit ? limit : ub);
  const float t1 = bf16r(gb * alpha);
  const float t2 = bf16r(1.f / (1.f + expf(-t1)));
  const float glu = bf16r(gb * t2);
  const float t3 = bf16r(ub + 1.f);
  return bf16r(t3 * glu);
}

}  // namespace b200
