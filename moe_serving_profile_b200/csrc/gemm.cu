// Grouped expert GEMM on tcgen05 tensor cores (sm_100a).
//
// Orientation ("swap AB"): the weights are the M = 128 operand (128 output
// features of one expert per CTA) and the token rows are the N operand (a
// tile of 16..256 permuted rows of that expert). One CTA therefore streams
// each weight tile from HBM exactly once per token tile, which is what makes
// decode batches (1..64 tokens, a handful of rows per expert) bandwidth-bound
// instead of wasting a 128-row M tile on 1-8 real rows.
//
// Per CTA (384 threads, 12 warps):
//   warp 0      TMA producer: raw weight tiles (fp8 / mxfp4 bytes) into a ring
//               of raw stages, or bf16 weights straight into the A stages
//   warp 1      TMEM allocator and tcgen05.mma issuer (one thread)
//   warps 2-3   token-row gather: cp.async 16-byte chunks into the 128-byte
//               swizzled K-major layout of the B stages
//   warps 4-11  dequantisers: raw stage -> bf16 A stage in the swizzled
//               layout; warps 4-7 also run the epilogue (TMEM lanes 0-127)
// Gated launches (gate/up) keep two accumulators, gate in TMEM columns
// [0, N) and up in [N, 2N), so the SwiGLU epilogue sees both values of a
// feature in the same thread.
//
// Split-K: when there are too few (expert, feature-tile, token-tile) work
// items to cover the GPU, `ks` CTAs of a cluster share one tile and split the
// K range; ranks 1..ks-1 push their fp32 partials into rank 0's shared memory
// (DSMEM) and rank 0 adds them in rank order. The split depends only on the
// launch arguments, never on timing, so results are deterministic.
#include <cuda_fp8.h>

#include "gemm_params.h"
#include "ptx.cuh"

namespace b200 {

namespace gemm {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kThreads = 384;
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpB = 2;        // warps 2, 3
constexpr int kWarpConv = 4;     // warps 4..11
constexpr int kConvThreads = 256;
constexpr int kBThreads = 64;
constexpr uint32_t kAPlane = 128u * 128u;    // 128 rows x 64 bf16
constexpr uint32_t kRawFp8 = 128u * 64u;     // 128 rows x 64 e4m3
constexpr uint32_t kRawMx = 128u * 32u;      // 128 rows x 64 e2m1

enum { kWBf16 = 0, kWFp8 = 1, kWMx = 2 };
enum { kEpiSwiglu = 0, kEpiClamp = 1, kEpiDown = 2 };

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// 16 e4m3 -> 16 bf16 (bf16(fp32(w) * scale), as the reference dequantises).
__device__ __forceinline__ void fp8x16_to_bf16(const uint4& q, float scale, uint32_t (&o)[8]) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(
        static_cast<__nv_fp8x2_storage_t>(w[i] & 0xffffu), __NV_E4M3);
    const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(
        static_cast<__nv_fp8x2_storage_t>(w[i] >> 16), __NV_E4M3);
    const float a0 = __half2float(__ushort_as_half(lo.x)) * scale;
    const float a1 = __half2float(__ushort_as_half(lo.y)) * scale;
    const float a2 = __half2float(__ushort_as_half(hi.x)) * scale;
    const float a3 = __half2float(__ushort_as_half(hi.y)) * scale;
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

// 16 bytes of e2m1 pairs (low nibble first) -> 32 bf16.
__device__ __forceinline__ void mx32_to_bf16(const uint4& q, float scale, const float* lut,
                                             uint32_t (&o)[16]) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t byte = (w[i] >> (8 * b)) & 0xffu;
      const float lo = lut[byte & 15u] * scale;
      const float hi = lut[byte >> 4] * scale;
      o[4 * i + b] = pack_bf16x2(lo, hi);
    }
  }
}

__device__ __forceinline__ float silu_bf16(float g) { return bf16r(g / (1.f + expf(-g))); }

__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ float s_lut[16];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* sbase = smem_raw + (base_u32 - raw_u32);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(sbase + p.bar_off);
  uint64_t* raw_empty = raw_full + p.nr;
  uint64_t* a_full = raw_empty + p.nr;
  uint64_t* a_empty = a_full + p.na;
  uint64_t* b_full = a_empty + p.na;
  uint64_t* b_empty = b_full + p.nb;
  uint64_t* acc_full = b_empty + p.nb;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(acc_full + 1);
  int* s_tile = reinterpret_cast<int*>(s_tmem + 1);

  // ---- which (expert, token tile) this CTA row owns
  if (warp == 0) {
    const int tile = blockIdx.y;
    int acc = 0;
    int fe = -1, frow = 0, fn = 0;
    for (int base = 0; base < p.n_experts; base += 32) {
      const int e = base + lane;
      int cnt = 0, start = 0;
      if (e < p.n_experts) {
        start = p.offsets[p.expert_begin + e];
        cnt = p.offsets[p.expert_begin + e + 1] - start;
      }
      const int nt = (cnt + p.bn - 1) / p.bn;
      int incl = nt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += v;
      }
      const int excl = incl - nt;
      const bool mine = nt > 0 && tile >= acc + excl && tile < acc + incl;
      const unsigned bal = __ballot_sync(kFull, mine);
      if (bal != 0u) {
        const int src = __ffs(bal) - 1;
        const int te = __shfl_sync(kFull, e, src);
        const int ts = __shfl_sync(kFull, start, src);
        const int tc = __shfl_sync(kFull, cnt, src);
        const int tx = __shfl_sync(kFull, excl, src);
        const int sub = tile - acc - tx;
        fe = te;
        frow = ts + sub * p.bn;
        fn = min(p.bn, tc - sub * p.bn);
        break;
      }
      acc += __shfl_sync(kFull, incl, 31);
    }
    if (lane == 0) {
      s_tile[0] = fe;
      s_tile[1] = frow;
      s_tile[2] = fn;
    }
  }
  if (threadIdx.x < 16) {
    // e2m1 code -> value
    const int m = threadIdx.x & 7;
    float v = (m == 0) ? 0.f : (m == 1) ? 0.5f : (m == 2) ? 1.f : (m == 3) ? 1.5f
            : (m == 4) ? 2.f : (m == 5) ? 3.f : (m == 6) ? 4.f : 6.f;
    s_lut[threadIdx.x] = (threadIdx.x & 8) ? -v : v;
  }
  __syncthreads();
  const int e_loc = s_tile[0];
  if (e_loc < 0) return;  // no such tile: uniform over the CTA and its cluster
  const int row0 = s_tile[1];
  const int nrows = s_tile[2];

  const uint32_t crank = (p.ks > 1) ? cluster_ctarank() : 0u;
  const int feat_tile = blockIdx.x / p.ks;
  // rank r of ks takes k-blocks [r*nkb/ks, (r+1)*nkb/ks): at least one each
  // because the host keeps ks <= nkb
  const int kb0 = static_cast<int>(crank) * p.nkb / p.ks;
  const int kb1 = (static_cast<int>(crank) + 1) * p.nkb / p.ks;
  const int nk = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.nr; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kConvThreads / 32);
    }
    for (int i = 0; i < p.na; ++i) {
      mbar_init(&a_full[i], p.wfmt == kWBf16 ? 1 : kConvThreads / 32);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < p.nb; ++i) {
      mbar_init(&b_full[i], kBThreads);
      mbar_init(&b_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(s_tmem, p.tmem_cols);
    tmem_relinquish();
  }
  if (warp == kWarpTma && lane == 0) tma_prefetch_desc(&wmap);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (p.ks > 1) cluster_sync();
  const uint32_t tmem = *s_tmem;
  const uint32_t a_stage_bytes = kAPlane * p.planes;

  if (warp == kWarpTma) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      const int wrow = (e_loc * p.planes) * p.feat_pad + feat_tile * 128;
      for (int i = 0; i < nk; ++i) {
        const int kb = kb0 + i;
        if (p.wfmt == kWBf16) {
          const int s = i % p.na;
          if (!wait_bounded(&a_empty[s], ((i / p.na) & 1) ^ 1, p.status)) break;
          mbar_arrive_expect_tx(&a_full[s], a_stage_bytes);
          for (int pl = 0; pl < p.planes; ++pl)
            tma_load_2d(sbase + p.a_off + s * a_stage_bytes + pl * kAPlane, &wmap, &a_full[s],
                        kb * 64, wrow + pl * p.feat_pad);
        } else {
          const int s = i % p.nr;
          const uint32_t rpb = (p.wfmt == kWFp8) ? kRawFp8 : kRawMx;
          if (!wait_bounded(&raw_empty[s], ((i / p.nr) & 1) ^ 1, p.status)) break;
          mbar_arrive_expect_tx(&raw_full[s], rpb * p.planes);
          const int c0 = (p.wfmt == kWFp8) ? kb * 64 : kb * 32;
          for (int pl = 0; pl < p.planes; ++pl)
            tma_load_2d(sbase + p.raw_off + (s * p.planes + pl) * rpb, &wmap, &raw_full[s], c0,
                        wrow + pl * p.feat_pad);
        }
      }
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, p.bn);
      for (int i = 0; i < nk; ++i) {
        const int sa = i % p.na;
        const int sb = i % p.nb;
        if (!wait_bounded(&a_full[sa], (i / p.na) & 1, p.status)) break;
        if (!wait_bounded(&b_full[sb], (i / p.nb) & 1, p.status)) break;
        tc_fence_after();
        const uint32_t a_addr = base_u32 + p.a_off + sa * a_stage_bytes;
        const uint64_t bdesc = sdesc_k_sw128(base_u32 + p.b_off + sb * p.bn * 128);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          for (int pl = 0; pl < p.planes; ++pl) {
            const uint64_t adesc = sdesc_k_sw128(a_addr + pl * kAPlane);
            umma_bf16(tmem + pl * p.bn, adesc + 2 * kk, bdesc + 2 * kk, idesc,
                      (i > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(&a_empty[sa]);
        umma_commit(&b_empty[sb]);
      }
      umma_commit(acc_full);
    }
  } else if (warp < kWarpConv) {
    // ------------------------------------------------ token-row gather
    const int tb = threadIdx.x - kWarpB * 32;
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int s = i % p.nb;
      if (!wait_bounded(&b_empty[s], ((i / p.nb) & 1) ^ 1, p.status)) {
        ok = false;
        break;
      }
      const int kb = kb0 + i;
      const uint32_t dst0 = base_u32 + p.b_off + s * p.bn * 128;
      for (int ch = tb; ch < nrows * 8; ch += kBThreads) {
        const int r = ch >> 3;
        const int c = ch & 7;
        const int grow = row0 + r;
        const long long srow = p.b_map ? static_cast<long long>(p.b_map[grow] / p.b_div) : grow;
        const int k = kb * 64 + c * 8;
        const bool valid = k < p.k_valid;
        const __nv_bfloat16* src = valid ? p.b_src + srow * p.ldb + k : p.b_src;
        cp_async_16(dst0 + swz(r, c), src, valid ? 16u : 0u);
      }
      cp_async_commit();
      if (i >= 1) {
        cp_async_wait<1>();
        fence_proxy_async_smem();
        mbar_arrive(&b_full[(i - 1) % p.nb]);
      }
    }
    if (ok && nk >= 1) {
      cp_async_wait<0>();
      fence_proxy_async_smem();
      mbar_arrive(&b_full[(nk - 1) % p.nb]);
    }
  } else if (p.wfmt != kWBf16) {
    // ------------------------------------------------ dequantisers
    const int tc = threadIdx.x - kWarpConv * 32;
    for (int i = 0; i < nk; ++i) {
      const int sr = i % p.nr;
      const int sa = i % p.na;
      if (!wait_bounded(&raw_full[sr], (i / p.nr) & 1, p.status)) break;
      if (!wait_bounded(&a_empty[sa], ((i / p.na) & 1) ^ 1, p.status)) break;
      const int kb = kb0 + i;
      uint8_t* astage = sbase + p.a_off + sa * a_stage_bytes;
      if (p.wfmt == kWFp8) {
        const uint8_t* raw = sbase + p.raw_off + sr * p.planes * kRawFp8;
        const int n_items = p.planes * 512;
        for (int it = tc; it < n_items; it += kConvThreads) {
          const int pl = it >> 9;
          const int r = (it >> 2) & 127;
          const int v = it & 3;
          const uint4 q = *reinterpret_cast<const uint4*>(raw + pl * kRawFp8 + r * 64 + v * 16);
          const int f = min(feat_tile * 128 + r, p.n_feat - 1);
          const int k = kb * 64 + v * 16;
          const int sr_i = min(f / p.sc_br, p.sc_nbr - 1);
          const int sc_i = min(k / p.sc_bc, p.sc_nbc - 1);
          const float scale =
              __ldg(p.fp8_scale + ((long long)(e_loc * p.planes + pl) * p.sc_nbr + sr_i) * p.sc_nbc + sc_i);
          uint32_t o[8];
          fp8x16_to_bf16(q, scale, o);
          uint8_t* dst = astage + pl * kAPlane;
          *reinterpret_cast<uint4*>(dst + swz(r, 2 * v)) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(dst + swz(r, 2 * v + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
      } else {
        const uint8_t* raw = sbase + p.raw_off + sr * p.planes * kRawMx;
        const int n_items = p.planes * 256;
        for (int it = tc; it < n_items; it += kConvThreads) {
          const int pl = it >> 8;
          const int r = (it >> 1) & 127;
          const int g = it & 1;
          const uint4 q = *reinterpret_cast<const uint4*>(raw + pl * kRawMx + r * 32 + g * 16);
          const int f = feat_tile * 128 + r;
          const uint32_t sexp = __ldg(
              p.mx_scale + ((long long)(e_loc * p.planes + pl) * p.feat_pad + f) * p.mx_groups + kb * 2 + g);
          uint32_t o[16];
          mx32_to_bf16(q, ue8m0_to_f32(sexp), s_lut, o);
          uint8_t* dst = astage + pl * kAPlane;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(dst + swz(r, 4 * g + j)) =
                make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&raw_empty[sr]);
        mbar_arrive(&a_full[sa]);
      }
    }
  }

  // ------------------------------------------------ epilogue
  const bool epi_warp = warp >= kWarpConv && warp < kWarpConv + 4;
  const int q = warp - kWarpConv;
  const int fl = q * 32 + lane;
  const int f = feat_tile * 128 + fl;
  const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16);
  const int ncols = (nrows + 15) & ~15;
  const int bn4 = p.bn >> 2;
  if (epi_warp) {
    wait_bounded(acc_full, 0, p.status);
    tc_fence_after();
    if (p.ks > 1 && crank != 0u) {
      const uint32_t red0 = mapa_shared(base_u32 + p.red_off, 0);
      const int slot = static_cast<int>(crank) - 1;
      for (int c0 = 0; c0 < ncols; c0 += 16) {
        for (int pl = 0; pl < p.planes; ++pl) {
          uint32_t r[16];
          tmem_ld16(tl + pl * p.bn + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4) {
            const uint32_t addr =
                red0 + static_cast<uint32_t>((((slot * p.planes + pl) * bn4 + (c0 >> 2) + j4) * 128 + fl) * 16);
            st_cluster_f32x4(addr, __uint_as_float(r[4 * j4]), __uint_as_float(r[4 * j4 + 1]),
                             __uint_as_float(r[4 * j4 + 2]), __uint_as_float(r[4 * j4 + 3]));
          }
        }
      }
    }
  }
  __syncwarp();
  if (p.ks > 1) cluster_sync();

  if (epi_warp && crank == 0u) {
    const float* red = reinterpret_cast<const float*>(sbase + p.red_off);
    float bias0 = 0.f, bias1 = 0.f;
    const bool fvalid = f < p.n_feat;
    if (p.bias != nullptr && fvalid) {
      bias0 = __bfloat162float(p.bias[(long long)(e_loc * p.planes) * p.feat_pad + f]);
      if (p.planes == 2)
        bias1 = __bfloat162float(p.bias[(long long)(e_loc * p.planes + 1) * p.feat_pad + f]);
    }
    for (int c0 = 0; c0 < ncols; c0 += 16) {
      float g[16], u[16];
      {
        uint32_t r[16];
        tmem_ld16(tl + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) g[j] = __uint_as_float(r[j]);
      }
      if (p.planes == 2) {
        uint32_t r[16];
        tmem_ld16(tl + p.bn + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) u[j] = __uint_as_float(r[j]);
      }
      for (int s = 0; s + 1 < p.ks; ++s) {
#pragma unroll
        for (int j4 = 0; j4 < 4; ++j4) {
          const float4 v = *reinterpret_cast<const float4*>(
              red + ((((s * p.planes) * bn4 + (c0 >> 2) + j4) * 128 + fl) * 4));
          g[4 * j4] += v.x;
          g[4 * j4 + 1] += v.y;
          g[4 * j4 + 2] += v.z;
          g[4 * j4 + 3] += v.w;
        }
        if (p.planes == 2) {
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4) {
            const float4 v = *reinterpret_cast<const float4*>(
                red + ((((s * p.planes + 1) * bn4 + (c0 >> 2) + j4) * 128 + fl) * 4));
            u[4 * j4] += v.x;
            u[4 * j4 + 1] += v.y;
            u[4 * j4 + 2] += v.z;
            u[4 * j4 + 3] += v.w;
          }
        }
      }
      if (!fvalid) continue;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (c0 + j >= nrows) continue;
        const long long row = row0 + c0 + j;
        float res;
        if (p.epi == kEpiSwiglu) {
          const float gb = bf16r(g[j]);
          const float ub = bf16r(u[j]);
          res = bf16r(silu_bf16(gb) * ub);
        } else if (p.epi == kEpiClamp) {
          float gb = bf16r(bf16r(g[j]) + bias0);
          float ub = bf16r(bf16r(u[j]) + bias1);
          gb = gb > p.limit ? p.limit : gb;
          ub = ub < -p.limit ? -p.limit : (ub > p.limit ? p.limit : ub);
          const float t1 = bf16r(gb * p.alpha);
          const float t2 = bf16r(1.f / (1.f + expf(-t1)));
          const float glu = bf16r(gb * t2);
          const float t3 = bf16r(ub + 1.f);
          res = bf16r(t3 * glu);
        } else {
          float y = bf16r(g[j]);
          if (p.bias != nullptr) y = bf16r(y + bias0);
          if (p.row_w != nullptr) {
            const int src = p.row_src[row];
            const float wv = p.row_w_bf16
                                 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.row_w)[src])
                                 : reinterpret_cast<const float*>(p.row_w)[src];
            y = bf16r(y * wv);
          }
          res = y;
        }
        p.out[row * p.ldo + f] = __float2bfloat16_rn(res);
      }
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
