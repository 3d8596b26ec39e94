// Grouped expert GEMM on tcgen05 tensor cores (sm_100a): a persistent,
// warp-specialised kernel.
//
// Orientation ("swap AB"): the weights are the M = 128 operand and the token
// rows of one expert the N operand (a tile of 16..256 permuted rows), so a
// decode batch with a handful of rows per expert still streams each weight
// tile once at full width instead of padding a 128-row M tile with 1-8 rows.
//   gated (gate/up): a tile is 64 features; A rows 0-63 are the gate rows and
//     64-127 the up rows of those features, so one 128 x N MMA feeds both
//     halves of SwiGLU and twice as many tiles exist for small batches.
//   down: a tile is 128 output features.
//
// One CTA per SM loops over tiles t = blockIdx.x, blockIdx.x + gridDim.x, ...
// (tile = (expert, token tile, feature tile), feature tile fastest so that
// concurrently running CTAs share token rows in L2). 16 warps:
//   warp 0      TMA: raw weight tiles (e4m3 / e2m1 bytes) into a ring of raw
//               stages, or bf16 weights straight into the A stages
//   warp 1      TMEM allocator and tcgen05.mma issuer (one thread); two
//               accumulator slots so a tile's epilogue overlaps the next
//               tile's main loop
//   warp 2      TMA for the token rows: tile::gather4 of the routed tokens'
//               rows (gate/up) or a 2D tile of contiguous rows (down)
//   warps 4-7   epilogue (TMEM lane quarters 0-3): activation / bias /
//               routing weight, bf16 stores
//   warps 8-15  dequantisers: raw stage -> bf16 A stage in the 128-byte
//               swizzled K-major layout tcgen05 reads; warp w owns A stage w
//               and converts every na-th k-block by itself
// All rings are phase-tracked mbarriers; every wait is bounded (see ptx.cuh).
#include <cuda_fp8.h>

#include "gemm_params.h"
#include "ptx.cuh"

namespace b200 {

namespace gemm {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kThreads = 512;
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpB = 2;
constexpr int kWarpEpi = 4;      // warps 4..7
constexpr int kWarpConv = 8;     // warps 8..15
constexpr int kConvWarps = 8;
constexpr int kConvThreads = kConvWarps * 32;
constexpr uint32_t kATile = 128u * 128u;    // 128 rows x 64 bf16
constexpr uint32_t kRawFp8 = 128u * 64u;    // 128 rows x 64 e4m3
constexpr uint32_t kRawMx = 128u * 32u;     // 128 rows x 64 e2m1

enum { kWBf16 = 0, kWFp8 = 1, kWMx = 2 };
enum { kEpiSwiglu = 0, kEpiClamp = 1, kEpiDown = 2 };

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

struct Tile {
  int e, ft, row0, nrows;
};

// Position in a ring of mbarrier-guarded stages, advanced without division.
struct Ring {
  int n, idx;
  uint32_t phase;
  __device__ explicit Ring(int n_) : n(n_), idx(0), phase(0u) {}
  __device__ void next() {
    if (++idx == n) {
      idx = 0;
      phase ^= 1u;
    }
  }
};

// prefix[e] = token tiles of local experts < e (prefix[n_experts] = total).
__device__ __forceinline__ Tile decode_tile(int t, const int* prefix, const GemmParams& p) {
  Tile r;
  const int u = t / p.feat_tiles;
  r.ft = t - u * p.feat_tiles;
  int lo = 0, hi = p.n_experts;  // largest lo with prefix[lo] <= u
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= u) lo = mid; else hi = mid;
  }
  r.e = lo;
  const int sub = u - prefix[lo];
  const int start = p.offsets[p.expert_begin + lo];
  const int cnt = p.offsets[p.expert_begin + lo + 1] - start;
  r.row0 = start + sub * p.bn;
  r.nrows = min(p.bn, cnt - sub * p.bn);
  return r;
}

// 16 e4m3 -> 16 bf16 holding bf16(fp32(w) * scale), the reference's dequant.
__device__ __forceinline__ void fp8x16_to_bf16(const uint4& q, float scale, uint32_t (&o)[8]) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(
        static_cast<__nv_fp8x2_storage_t>(w[i] & 0xffffu), __NV_E4M3);
    const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(
        static_cast<__nv_fp8x2_storage_t>(w[i] >> 16), __NV_E4M3);
    float a0 = __half2float(__ushort_as_half(lo.x));
    float a1 = __half2float(__ushort_as_half(lo.y));
    float a2 = __half2float(__ushort_as_half(hi.x));
    float a3 = __half2float(__ushort_as_half(hi.y));
    mul2_f32(a0, a1, scale);
    mul2_f32(a2, a3, scale);
    o[2 * i] = pack_bf16x2(a0, a1);
    o[2 * i + 1] = pack_bf16x2(a2, a3);
  }
}

// 2^(s-127) as the fp32 value torch's ldexp multiplies by (exact, including
// the subnormal s = 0 and the overflow s = 255).
__device__ __forceinline__ float ue8m0_to_f32(uint32_t s) {
  if (s == 0u) return __uint_as_float(0x00400000u);
  if (s == 255u) return __uint_as_float(0x7f800000u);
  return __uint_as_float(s << 23);
}

// 16 bytes of e2m1 pairs (low nibble first) -> 32 bf16 (exact).
__device__ __forceinline__ void mx32_to_bf16(const uint4& q, float scale, const float* lut,
                                             uint32_t (&o)[16]) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t byte = (w[i] >> (8 * b)) & 0xffu;
      float lo = lut[byte & 15u];
      float hi = lut[byte >> 4];
      mul2_f32(lo, hi, scale);
      o[4 * i + b] = pack_bf16x2(lo, hi);
    }
  }
}

// Four e4m3 codes (one word) -> four bf16 holding bf16(fp32(w) * scale).
// The fp32 bit pattern (c & 0x7f) << 20 | sign << 31 has the value
// e4m3(c) * 2^-120 for every code (normal codes give normal fp32, subnormal
// codes subnormal fp32), so multiplying it by s120 = scale * 2^120 yields the
// same real product as fp32(w) * scale and rounds once, exactly as the
// reference does; only the final bf16 pack uses the conversion pipe.
// Requires scale < 2^8 (s120 finite); the 0x7f / 0xff NaN codes are not
// propagated as NaN.
__device__ __forceinline__ void fp8x4_scaled(uint32_t w, float s120, uint32_t& o01,
                                             uint32_t& o23) {
  float f0 = __uint_as_float(((w << 20) & 0x07f00000u) | ((w << 24) & 0x80000000u));
  float f1 = __uint_as_float(((w << 12) & 0x07f00000u) | ((w << 16) & 0x80000000u));
  float f2 = __uint_as_float(((w << 4) & 0x07f00000u) | ((w << 8) & 0x80000000u));
  float f3 = __uint_as_float(((w >> 4) & 0x07f00000u) | (w & 0x80000000u));
  mul2_f32(f0, f1, s120);
  mul2_f32(f2, f3, s120);
  o01 = pack_bf16x2(f0, f1);
  o23 = pack_bf16x2(f2, f3);
}

// Eight e2m1 codes (one word, element 0 in the low nibble) -> eight bf16.
// The fp32 pattern (n & 7) << 22 | sign << 31 has the value e2m1(n) * 2^-126
// for every code; times s = 2^(S-1) it is e2m1(n) * 2^(S-127) exactly, a value
// bf16 represents, so the bf16 is the high half of the fp32 bits (no
// rounding, no conversion instruction). Requires S <= 128.
__device__ __forceinline__ void mx8_scaled(uint32_t w, float s, uint32_t (&o)[4]) {
  float f[8];
  f[0] = __uint_as_float(((w << 22) & 0x01c00000u) | ((w << 28) & 0x80000000u));
  f[1] = __uint_as_float(((w << 18) & 0x01c00000u) | ((w << 24) & 0x80000000u));
  f[2] = __uint_as_float(((w << 14) & 0x01c00000u) | ((w << 20) & 0x80000000u));
  f[3] = __uint_as_float(((w << 10) & 0x01c00000u) | ((w << 16) & 0x80000000u));
  f[4] = __uint_as_float(((w << 6) & 0x01c00000u) | ((w << 12) & 0x80000000u));
  f[5] = __uint_as_float(((w << 2) & 0x01c00000u) | ((w << 8) & 0x80000000u));
  f[6] = __uint_as_float(((w >> 2) & 0x01c00000u) | ((w << 4) & 0x80000000u));
  f[7] = __uint_as_float(((w >> 6) & 0x01c00000u) | (w & 0x80000000u));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    mul2_f32(f[2 * i], f[2 * i + 1], s);
    o[i] = __byte_perm(__float_as_uint(f[2 * i]), __float_as_uint(f[2 * i + 1]), 0x7632);
  }
}

__device__ __forceinline__ float silu_bf16(float g) { return bf16_rn(g / (1.f + expf(-g))); }

__device__ __forceinline__ float epilogue_gated(int epi, float g, float u, float bg, float bu,
                                                float alpha, float limit) {
  if (epi == kEpiSwiglu) {
    const float gb = bf16_rn(g);
    const float ub = bf16_rn(u);
    return bf16_rn(silu_bf16(gb) * ub);
  }
  float gb = bf16_rn(bf16_rn(g) + bg);
  float ub = bf16_rn(bf16_rn(u) + bu);
  gb = gb > limit ? limit : gb;
  ub = ub < -limit ? -limit : (ub > limit ? limit : ub);
  const float t1 = bf16_rn(gb * alpha);
  const float t2 = bf16_rn(1.f / (1.f + expf(-t1)));
  const float glu = bf16_rn(gb * t2);
  const float t3 = bf16_rn(ub + 1.f);
  return bf16_rn(t3 * glu);
}

__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap bmap,
                    const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ float s_lut[16];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* sbase = smem_raw + (base_u32 - raw_u32);

  // A wait already timed out on this device (status not yet cleared): do not
  // start more work that would queue behind the same fault.
  if (*reinterpret_cast<volatile int*>(p.status) & kStatusWaitTimeout) return;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(sbase + p.bar_off);
  uint64_t* raw_empty = raw_full + p.nr;
  uint64_t* a_full = raw_empty + p.nr;
  uint64_t* a_empty = a_full + p.na;
  uint64_t* b_full = a_empty + p.na;
  uint64_t* b_empty = b_full + p.nb;
  uint64_t* acc_full = b_empty + p.nb;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(mma_done + 1);
  int* s_total = reinterpret_cast<int*>(s_tmem + 1);
  int* prefix = s_total + 1;             // [n_experts + 1]

  if (warp == 0) {
    int acc = 0;
    if (lane == 0) prefix[0] = 0;
    for (int base = 0; base < p.n_experts; base += 32) {
      const int e = base + lane;
      int nt = 0;
      if (e < p.n_experts) {
        const int cnt = p.offsets[p.expert_begin + e + 1] - p.offsets[p.expert_begin + e];
        nt = (cnt + p.bn - 1) / p.bn;
      }
      int incl = nt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += v;
      }
      if (e < p.n_experts) prefix[e + 1] = acc + incl;
      acc += __shfl_sync(kFull, incl, 31);
    }
    if (lane == 0) *s_total = acc * p.feat_tiles;
  }
  if (threadIdx.x < 16) {
    const int m = threadIdx.x & 7;
    const float v = (m == 0) ? 0.f : (m == 1) ? 0.5f : (m == 2) ? 1.f : (m == 3) ? 1.5f
                  : (m == 4) ? 2.f : (m == 5) ? 3.f : (m == 6) ? 4.f : 6.f;
    s_lut[threadIdx.x] = (threadIdx.x & 8) ? -v : v;
  }
  if (threadIdx.x == 32 * kWarpTma) {
    for (int i = 0; i < p.nr; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 1);
    }
    for (int i = 0; i < p.na; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < p.nb; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
    tma_prefetch_desc(&wmap);
    tma_prefetch_desc(&bmap);
  }
  if (warp == kWarpMma) {
    tmem_alloc(s_tmem, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int total = *s_total;
  const int planes = p.gated ? 2 : 1;

  if (warp == kWarpTma) {
    // ------------------------------------------------ weight TMA producer
    if (lane == 0) {
      bool ok = true;
      const uint32_t rowbytes = p.wfmt == kWFp8 ? 64u : 32u;
      const uint32_t rpb = 128u * rowbytes;
      // raw stage s feeds A stage s (one ring): each raw stage is drained by
      // exactly one dequantiser warp, which steps through its phases in order
      Ring ring(p.na);
      uint64_t* full = p.wfmt == kWBf16 ? a_full : raw_full;
      uint64_t* empty = p.wfmt == kWBf16 ? a_empty : raw_empty;
      int issued = 0;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        const Tile tl = decode_tile(t, prefix, p);
        const int wrow = tl.e * planes * p.feat_pad + tl.ft * p.feat_tile;
        for (int kb = 0; kb < p.nkb; ++kb, ring.next(), ++issued) {
          const int s = ring.idx;
          if (!wait_bounded(&empty[s], ring.phase ^ 1u, p.status, 32)) {
            ok = false;
            break;
          }
          if (p.wfmt == kWBf16) {
            mbar_arrive_expect_tx(&full[s], kATile);
            uint8_t* dst = sbase + p.a_off + s * kATile;
            tma_load_2d(dst, &wmap, &full[s], kb * 64, wrow);
            if (p.gated) tma_load_2d(dst + 64 * 128, &wmap, &full[s], kb * 64, wrow + p.feat_pad);
          } else {
            mbar_arrive_expect_tx(&full[s], rpb);
            uint8_t* dst = sbase + p.raw_off + s * rpb;
            const int c0 = kb * static_cast<int>(rowbytes);
            tma_load_2d(dst, &wmap, &full[s], c0, wrow);
            if (p.gated) tma_load_2d(dst + 64 * rowbytes, &wmap, &full[s], c0, wrow + p.feat_pad);
          }
        }
      }
      // every issued copy has landed before the CTA may exit
      for (int i = max(0, issued - ring.n); i < issued; ++i)
        wait_bounded(&full[i % ring.n], (i / ring.n) & 1, p.status, 32);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, p.bn);
      Ring ra(p.na), rb(p.nb);
      int tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x, ++tc) {
        const int slot = tc & 1;
        if (!wait_bounded(&acc_empty[slot], ((tc >> 1) & 1) ^ 1, p.status)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(slot * p.bn);
        for (int kb = 0; kb < p.nkb; ++kb, ra.next(), rb.next()) {
          if (!wait_bounded(&a_full[ra.idx], ra.phase, p.status) ||
              !wait_bounded(&b_full[rb.idx], rb.phase, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sdesc_k_sw128(base_u32 + p.a_off + ra.idx * kATile);
          const uint64_t bdesc = sdesc_k_sw128(base_u32 + p.b_off + rb.idx * p.bn * 128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&a_empty[ra.idx]);
          umma_commit(&b_empty[rb.idx]);
        }
        umma_commit(&acc_full[slot]);
      }
      // all issued MMAs have finished before TMEM is released
      umma_commit(mma_done);
      wait_bounded(mma_done, 0, p.status);
    }
  } else if (warp == kWarpB) {
    // ------------------------------------------------ token-row TMA producer
    Ring ring(p.nb);
    int issued = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
      const Tile tl = decode_tile(t, prefix, p);
      int tok[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int q4 = (lane + 32 * j) * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = (q4 + i < tl.nrows) ? q4 + i : 0;   // padding rows repeat row 0
          tok[j][i] = (p.b_gather && q4 < p.bn) ? p.b_map[tl.row0 + r] / p.b_div : 0;
        }
      }
      for (int kb = 0; kb < p.nkb; ++kb, ring.next(), ++issued) {
        const int s = ring.idx;
        if (!wait_bounded(&b_empty[s], ring.phase ^ 1u, p.status, 32)) {
          ok = false;
          break;
        }
        uint8_t* dst = sbase + p.b_off + s * p.bn * 128;
        if (lane == 0) mbar_arrive_expect_tx(&b_full[s], p.bn * 128);
        __syncwarp();
        if (p.b_gather) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int q = lane + 32 * j;
            if (q * 4 < p.bn)
              tma_gather4(dst + q * 512, &bmap, &b_full[s], kb * 64, tok[j][0], tok[j][1], tok[j][2],
                          tok[j][3]);
          }
        } else if (lane == 0) {
          tma_load_2d(dst, &bmap, &b_full[s], kb * 64, tl.row0);
        }
      }
    }
    if (lane == 0)
      for (int i = max(0, issued - p.nb); i < issued; ++i)
        wait_bounded(&b_full[i % p.nb], (i / p.nb) & 1, p.status, 32);
  } else if (warp >= kWarpEpi && warp < kWarpEpi + 4) {
    // ------------------------------------------------ epilogue
    // TMEM lane quarter q holds 32 features x N tokens. Each 16-token chunk
    // is finished in registers, staged in shared memory as bf16 rows and
    // written out with 16-byte coalesced stores (rows beyond the tile and
    // features beyond n_feat are never written).
    const int q = warp - kWarpEpi;
    const int te = threadIdx.x - kWarpEpi * 32;
    const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16);
    float* xbuf = reinterpret_cast<float*>(sbase + p.x_off);                      // [4][16][32] f32
    uint16_t* stage = reinterpret_cast<uint16_t*>(sbase + p.x_off + 8192);        // [2][16][128] bf16
    float* rowv = reinterpret_cast<float*>(sbase + p.x_off + 16384);             // [256] f32
    int tc = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++tc) {
      const Tile tl = decode_tile(t, prefix, p);
      const int slot = tc & 1;
      // the four epilogue warps agree on success before using their barrier
      const bool ok =
          named_bar_and(1, 128, wait_bounded(&acc_full[slot], (tc >> 1) & 1, p.status, 128));
      if (!ok) break;
      tc_fence_after();
      const int ncols = (tl.nrows + 15) & ~15;
      if (p.gated) {
        const int fl = (q & 1) * 32 + lane;
        const int f = tl.ft * 64 + fl;
        const bool fvalid = f < p.n_feat;
        float bg = 0.f, bu = 0.f;
        if (p.bias != nullptr && fvalid) {
          bg = __bfloat162float(p.bias[(long long)(tl.e * 2) * p.feat_pad + f]);
          bu = __bfloat162float(p.bias[(long long)(tl.e * 2 + 1) * p.feat_pad + f]);
        }
        const int jb = (q >> 1) * 8;
        for (int c0 = 0, ci = 0; c0 < ncols; c0 += 16, ++ci) {
          uint32_t r[16];
          tmem_ld16(tq + slot * p.bn + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) xbuf[(q * 16 + j) * 32 + lane] = __uint_as_float(r[j]);
          named_bar_sync(1, 128);
          uint16_t* st = stage + (ci & 1) * 16 * 64;     // [16][64]
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int j = jb + jj;
            const float g = xbuf[((q & 1) * 16 + j) * 32 + lane];
            const float u = xbuf[((2 + (q & 1)) * 16 + j) * 32 + lane];
            const float a = epilogue_gated(p.epi, g, u, bg, bu, p.alpha, p.limit);
            st[j * 64 + fl] = static_cast<uint16_t>(__float_as_uint(a) >> 16);
          }
          named_bar_sync(1, 128);
          const int j = te >> 3;
          const int c8 = (te & 7) * 8;
          if (c0 + j < tl.nrows && tl.ft * 64 + c8 < p.n_feat)
            *reinterpret_cast<uint4*>(p.out + (long long)(tl.row0 + c0 + j) * p.ldo + tl.ft * 64 + c8) =
                *reinterpret_cast<const uint4*>(st + j * 64 + c8);
        }
      } else {
        const int fl = q * 32 + lane;
        const int f = tl.ft * 128 + fl;
        const bool fvalid = f < p.n_feat;
        float b0 = 0.f;
        if (p.bias != nullptr && fvalid) b0 = __bfloat162float(p.bias[(long long)tl.e * p.feat_pad + f]);
        const bool scaled = p.row_w != nullptr;
        if (scaled) {
          for (int i = te; i < tl.nrows; i += 128) {
            const int src = p.row_src[tl.row0 + i];
            rowv[i] = p.row_w_bf16
                          ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.row_w)[src])
                          : reinterpret_cast<const float*>(p.row_w)[src];
          }
          named_bar_sync(1, 128);
        }
        for (int c0 = 0, ci = 0; c0 < ncols; c0 += 16, ++ci) {
          uint32_t r[16];
          tmem_ld16(tq + slot * p.bn + c0, r);
          tmem_ld_wait();
          uint16_t* st = stage + (ci & 1) * 16 * 128;    // [16][128]
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float y = bf16_rn(__uint_as_float(r[j]));
            if (p.bias != nullptr) y = bf16_rn(y + b0);
            if (scaled) y = bf16_rn(y * rowv[c0 + j]);
            st[j * 128 + fl] = static_cast<uint16_t>(__float_as_uint(y) >> 16);
          }
          named_bar_sync(1, 128);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = te + 128 * h;
            const int j = c >> 4;
            const int c8 = (c & 15) * 8;
            if (c0 + j < tl.nrows && tl.ft * 128 + c8 < p.n_feat)
              *reinterpret_cast<uint4*>(p.out + (long long)(tl.row0 + c0 + j) * p.ldo + tl.ft * 128 + c8) =
                  *reinterpret_cast<const uint4*>(st + j * 128 + c8);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[slot]);
    }
  } else if (warp >= kWarpConv && warp < kWarpConv + p.na && p.wfmt != kWBf16) {
    // ------------------------------------------------ dequantisers
    // Warp w owns A stage w and converts this CTA's k-blocks w, w + na,
    // w + 2 na, ... on its own (16 fp8 chunks or 8 mxfp4 groups per lane),
    // so na k-blocks are converted concurrently with no cross-warp barrier.
    const int w = warp - kWarpConv;
    const int kb_per_sc = (p.wfmt == kWFp8 && p.sc_bc % 64 == 0) ? p.sc_bc / 64 : 0;
    int t = blockIdx.x, kb = w, it = w, uses = 0, cur_t = -1;
    Tile tl{0, 0, 0, 0};
    const float* srow[2] = {nullptr, nullptr};   // gate/first-half and up/second-half scale rows
    const uint8_t* mscale = nullptr;
    while (true) {
      while (kb >= p.nkb) {
        kb -= p.nkb;
        t += gridDim.x;
      }
      if (t >= total) break;
      if (t != cur_t) {
        cur_t = t;
        tl = decode_tile(t, prefix, p);
        if (p.wfmt == kWFp8) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            // rows 64h..64h+63: a plane of the gated tile, or half the down tile
            const int pl = p.gated ? h : 0;
            const int f = tl.ft * p.feat_tile + (p.gated ? 0 : 64 * h);
            const int sri = min(min(f, p.n_feat - 1) / p.sc_br, p.sc_nbr - 1);
            srow[h] = p.fp8_scale + ((long long)(tl.e * planes + pl) * p.sc_nbr + sri) * p.sc_nbc;
          }
        } else {
          mscale = p.mx_scale + (long long)(tl.e * planes) * p.feat_pad * p.mx_groups;
        }
      }
      // raw stage w and A stage w are used only by this warp, once per `uses`,
      // so the phase this warp waits for is never more than one ahead
      const int sr = w;
      if (!wait_bounded(&raw_full[sr], uses & 1, p.status) ||
          !wait_bounded(&a_empty[w], (uses & 1) ^ 1, p.status)) break;
      uint8_t* astage = sbase + p.a_off + w * kATile;
      if (p.wfmt == kWFp8) {
        const uint8_t* raw = sbase + p.raw_off + sr * kRawFp8;
        // uniform scale per half-tile when the scale block covers it
        const bool uni = kb_per_sc != 0 && p.sc_br % 64 == 0;
        float sh[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) sh[h] = uni ? __ldg(srow[h] + min(kb / kb_per_sc, p.sc_nbc - 1)) : 0.f;
#pragma unroll 4
        for (int j = 0; j < 16; ++j) {
          const int item = lane + 32 * j;
          const int row = item >> 2;
          const int v = item & 3;
          const uint4 qv = *reinterpret_cast<const uint4*>(raw + row * 64 + v * 16);
          float scale;
          if (uni) {
            scale = (j >> 3) ? sh[1] : sh[0];
          } else {
            const int pl = p.gated ? (row >> 6) : 0;
            const int f = tl.ft * p.feat_tile + (p.gated ? (row & 63) : row);
            const int sri = min(min(f, p.n_feat - 1) / p.sc_br, p.sc_nbr - 1);
            const int sci = min((kb * 64 + v * 16) / p.sc_bc, p.sc_nbc - 1);
            scale = __ldg(p.fp8_scale + ((long long)(tl.e * planes + pl) * p.sc_nbr + sri) * p.sc_nbc + sci);
          }
          uint32_t o[8];
          if (scale < 256.f) {
            const float s120 = scale * 0x1p120f;
            fp8x4_scaled(qv.x, s120, o[0], o[1]);
            fp8x4_scaled(qv.y, s120, o[2], o[3]);
            fp8x4_scaled(qv.z, s120, o[4], o[5]);
            fp8x4_scaled(qv.w, s120, o[6], o[7]);
          } else {
            fp8x16_to_bf16(qv, scale, o);
          }
          *reinterpret_cast<uint4*>(astage + swz(row, 2 * v)) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(astage + swz(row, 2 * v + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
      } else {
        const uint8_t* raw = sbase + p.raw_off + sr * kRawMx;
#pragma unroll 4
        for (int j = 0; j < 8; ++j) {
          const int item = lane + 32 * j;
          const int row = item >> 1;
          const int g = item & 1;
          const uint4 qv = *reinterpret_cast<const uint4*>(raw + row * 32 + g * 16);
          const int pl = p.gated ? (row >> 6) : 0;
          const int f = tl.ft * p.feat_tile + (p.gated ? (row & 63) : row);
          const uint32_t sexp =
              __ldg(mscale + ((long long)pl * p.feat_pad + f) * p.mx_groups + kb * 2 + g);
          uint32_t o[16];
          if (sexp <= 128u) {
            const float s = __uint_as_float((sexp + 126u) << 23);
            mx8_scaled(qv.x, s, *reinterpret_cast<uint32_t(*)[4]>(o));
            mx8_scaled(qv.y, s, *reinterpret_cast<uint32_t(*)[4]>(o + 4));
            mx8_scaled(qv.z, s, *reinterpret_cast<uint32_t(*)[4]>(o + 8));
            mx8_scaled(qv.w, s, *reinterpret_cast<uint32_t(*)[4]>(o + 12));
          } else {
            mx32_to_bf16(qv, ue8m0_to_f32(sexp), s_lut, o);
          }
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            *reinterpret_cast<uint4*>(astage + swz(row, 4 * g + q4)) =
                make_uint4(o[4 * q4], o[4 * q4 + 1], o[4 * q4 + 2], o[4 * q4 + 3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&raw_empty[sr]);
        mbar_arrive(&a_full[w]);
      }
      it += p.na;
      kb += p.na;
      ++uses;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

}  // namespace gemm

const void* gemm_kernel_ptr() { return reinterpret_cast<const void*>(&gemm::moe_gemm_kernel); }

}  // namespace b200
