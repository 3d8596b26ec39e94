// W8A8 ("efficient" numerics of the reference's grouped FP8 path,
// moe_serving/efficient_kernels.py:243-274): dynamic FP8 quantisation of the
// activations per (row, 128-column group) and the grouped GEMM that
// multiplies those e4m3 rows with the e4m3 block-scaled weights on the
// tensor cores (tcgen05.mma kind::f8f6f4).
//
// act_quant: q[r, c] = e4m3_rn_satfinite(x[src(r), c] / s[r, g]) for
// c < k_valid (0 beyond), s[r, g] = amax_g / 448 over the group's values
// (1 for an all-zero group), g = c / 128. One warp per (row, group), four
// values per lane; src(r) = map[r] / div (a row gather) or r.
//
// w8a8_gemm: for every (expert, feature tile of 128 weight rows, tile of BN
// permuted rows), D[f, n] = sum over 128-column groups g of
// sw[f, g] * sa[n, g] * (sum_{k in g} W[f, k] * Q[n, k]), the inner sum an
// exact-product fp32 MMA accumulation in tensor memory, the outer sum
// ("promotion") in fp32 registers of the epilogue warps. Weights come
// straight from the packed FP8 blobs (their rows already sit in the 64-byte
// swizzled operand layout), a 128-column group of token rows by one
// 128-byte-swizzled TMA box.
#include "internal.h"
#include "ptx.cuh"

namespace b200 {
namespace {

constexpr unsigned kFull = 0xffffffffu;

// Two fp32 -> two e4m3 (x0 in the low byte), round to nearest even,
// saturating to +-448.
__device__ __forceinline__ uint32_t e4m3x2(float x0, float x1) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
  return r;
}

__global__ void __launch_bounds__(256) act_quant_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                        const int* __restrict__ map, int div, int rows,
                                                        int k_valid, int k_pad, uint8_t* __restrict__ q,
                                                        float* __restrict__ s,
                                                        const int* __restrict__ range_offsets, int lo,
                                                        int hi) {
  const int groups = (k_pad + 127) / 128;
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)rows * groups) return;
  const int r = static_cast<int>(w / groups), g = static_cast<int>(w - (long long)r * groups);
  // only the rows [offsets[lo], offsets[hi]) of one rank's experts (the
  // others are never read by that rank's GEMM)
  if (range_offsets != nullptr && (r < range_offsets[lo] || r >= range_offsets[hi])) return;
  const long long src = map ? map[r] / div : r;
  const int c = g * 128 + lane * 4;
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (c < k_valid) {   // k_valid % 4 == 0: four columns are valid together
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(x + src * ldx + c));
    v[0] = __uint_as_float(u.x << 16);
    v[1] = __uint_as_float(u.x & 0xffff0000u);
    v[2] = __uint_as_float(u.y << 16);
    v[3] = __uint_as_float(u.y & 0xffff0000u);
  }
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, o));
  const float sc = amax > 0.f ? amax / 448.f : 1.f;
  if (c < k_pad) {
    const uint32_t packed = e4m3x2(v[0] / sc, v[1] / sc) | (e4m3x2(v[2] / sc, v[3] / sc) << 16);
    *reinterpret_cast<uint32_t*>(q + (long long)r * k_pad + c) = packed;
  }
  if (lane == 0) s[(long long)r * groups + g] = sc;
}

}  // namespace

cudaError_t launch_act_quant(cudaStream_t st, const void* x, long long ldx, const int* map, int div,
                             int rows, int k_valid, int k_pad, void* q, float* s, const int* range_offsets,
                             int expert_lo, int expert_hi) {
  if (rows == 0) return cudaSuccess;
  const long long warps = (long long)rows * ((k_pad + 127) / 128);
  act_quant_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, map, div, rows, k_valid, k_pad, static_cast<uint8_t*>(q), s,
      range_offsets, expert_lo, expert_hi);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ GEMM
namespace w8 {

constexpr int kThreads = kW8A8Threads;   // warp 0 copies, warp 1 MMA, warps 2-9 promotion + epilogue
constexpr int kEpi = kThreads - 64;      // promotion / epilogue threads
constexpr uint32_t kAStage = 8192;       // 128 weight rows x 64 e4m3

// Group accumulators in tensor memory: 4 (512 columns at 128-row tiles), so
// the MMAs run up to three groups ahead of the promotion.
constexpr int kTmemBufs = 4;

struct Tile {
  int e, ft, row0, nrows;
};

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

template <int BN>
__device__ __forceinline__ Tile decode_tile(int t, const int* prefix, const W8A8Params& p) {
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
  r.row0 = start + sub * BN;
  r.nrows = min(BN, cnt - sub * BN);
  return r;
}

__device__ __forceinline__ float swiglu_bf16(float g, float u) {
  const float gb = bf16_rn(g), ub = bf16_rn(u);
  return bf16_rn(bf16_rn(gb / (1.f + expf(-gb))) * ub);
}

// Promotion scales of one 128-column group, staged per thread through a
// 4-slot shared-memory ring by cp.async (issued 4 groups ahead): slot
// [0, 128) token scales qs[row0 + te, g] (0 past the tile's rows),
// [128, 384) the weight block scales of rows 0-63 and 64-127 (the blob of
// k-block 2g), two per thread.
constexpr int kScaleRing = 4;
constexpr int kRingSlot = 384;   // floats

__device__ __forceinline__ void issue_scales(const W8A8Params& p, const uint8_t* wb, const Tile& tl, int te,
                                             int g, float* ring) {
  float* slot = ring + (g % kScaleRing) * kRingSlot;
  cp_async_4(smem_u32(slot + te), p.qs + (long long)(tl.row0 + (te < tl.nrows ? te : 0)) * p.qs_groups + g,
             te < tl.nrows ? 4u : 0u);
  cp_async_8(smem_u32(slot + 128 + 2 * te), wb + (long long)(2 * g) * p.blob_bytes + kAStage, 8u);
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    w8a8_gemm_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ W8A8Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* sbase = smem_raw + (base_u32 - raw_u32);
  if (*reinterpret_cast<volatile int*>(p.status) & kStatusWaitTimeout) return;

  constexpr int NB = kTmemBufs;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(sbase + p.bar_off);
  uint64_t* empty = full + p.ns;
  uint64_t* acc_full = empty + p.ns;    // [NB]
  uint64_t* acc_empty = acc_full + NB;  // [NB]
  uint64_t* mma_done = acc_empty + NB;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(mma_done + 1);
  int* s_total = reinterpret_cast<int*>(s_tmem + 1);
  int* prefix = s_total + 1;            // [n_experts + 1]

  if (warp == 0) {
    int acc = 0;
    if (lane == 0) prefix[0] = 0;
    for (int base = 0; base < p.n_experts; base += 32) {
      const int e = base + lane;
      int nt = 0;
      if (e < p.n_experts) {
        const int cnt = p.offsets[p.expert_begin + e + 1] - p.offsets[p.expert_begin + e];
        nt = (cnt + BN - 1) / BN;
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
    if (lane == 0) {
      *s_total = acc * p.feat_tiles;
      for (int i = 0; i < p.ns; ++i) {
        mbar_init(&full[i], 1);
        mbar_init(&empty[i], 1);
      }
      for (int i = 0; i < NB; ++i) {
        mbar_init(&acc_full[i], 1);
        mbar_init(&acc_empty[i], kEpi / 32);
      }
      mbar_init(mma_done, 1);
      fence_mbar_init();
      tma_prefetch_desc(&qmap);
    }
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int total = *s_total;
  // One stage per 128-column group: the weight blobs of k-blocks 2g and
  // 2g + 1 (64-byte-swizzled rows, 8 KB each) and the group's token rows as
  // one 128-byte-swizzled TMA box of BN rows x 128 B.
  constexpr uint32_t kBStage = BN * 128;
  constexpr uint32_t kBOff = 2 * kAStage;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      Ring ring(p.ns);
      int issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        const Tile tl = decode_tile<BN>(t, prefix, p);
        const uint8_t* wb = p.wblob + (long long)(tl.e * p.feat_tiles + tl.ft) * p.nkb * p.blob_bytes;
        for (int g = 0; g < p.ngroups; ++g, ring.next(), ++issued) {
          const int s = ring.idx;
          if (!wait_bounded(&empty[s], ring.phase ^ 1u, p.status)) {
            ok = false;
            break;
          }
          const int nblobs = min(2, p.nkb - 2 * g);
          uint8_t* st = sbase + s * p.stage_bytes;
          mbar_arrive_expect_tx(&full[s], nblobs * kAStage + kBStage);
          for (int b = 0; b < nblobs; ++b)
            bulk_load(st + b * kAStage, wb + (long long)(2 * g + b) * p.blob_bytes, kAStage, &full[s]);
          tma_load_2d(st + kBOff, &qmap, &full[s], g * 128, tl.row0);
        }
      }
      // every issued copy has landed before the CTA may exit
      for (int i = max(0, issued - p.ns); i < issued; ++i)
        wait_bounded(&full[i % p.ns], (i / p.ns) & 1, p.status, 32);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    // Group g of a tile (one stage) accumulates into buffer gc % NB (gc
    // counts the CTA's groups), which the promotion warps drain.
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(128, BN);
      Ring ring(p.ns);
      int gc = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        for (int g = 0; g < p.ngroups; ++g, ++gc, ring.next()) {
          const int buf = gc % NB;
          const int s = ring.idx;
          if (!wait_bounded(&acc_empty[buf], ((gc / NB) & 1) ^ 1, p.status) ||
              !wait_bounded(&full[s], ring.phase, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + static_cast<uint32_t>(buf * BN);
          const uint32_t st = base_u32 + s * p.stage_bytes;
          const uint64_t bdesc = sdesc_k_sw128(st + kBOff);
          const int nk = 2 * min(2, p.nkb - 2 * g);   // K = 32 slices of this group
#pragma unroll 1
          for (int j = 0; j < nk; ++j)
            umma_e4m3(d, sdesc_k_sw64(st + (j >> 1) * kAStage) + 2 * (j & 1), bdesc + 2 * j, idesc,
                      j > 0 ? 1u : 0u);
          umma_commit(&empty[s]);
          umma_commit(&acc_full[buf]);
        }
      }
      // all issued MMAs have finished before TMEM is released
      umma_commit(mma_done);
      wait_bounded(mma_done, 0, p.status);
    }
  } else {
    // ------------------------------------------------ promotion + epilogue
    // Warp w reads TMEM lanes 32 (w % 4) .. + 31, so its lane i holds weight
    // row r = 32 (w % 4) + i (gated tiles: rows 0..63 gate, 64..127 up rows
    // of the same 64 features); warps 2-5 take token columns [0, BN/2),
    // warps 6-9 [BN/2, BN).
    constexpr int CB = BN / 2;
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int half = r >> 6;
    const int n0 = ((warp - 2) >> 2) * CB;
    const int te = threadIdx.x - 64;
    const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16);
    float* sc_s = reinterpret_cast<float*>(sbase + p.x_off);   // [2 slots][2 halves][128] combined scales
    float* rowv = sc_s + 512;                                   // [128] routing weights
    float* ring = rowv + 128;                                   // [kScaleRing][kRingSlot] staged scales
    uint16_t* ux16 = reinterpret_cast<uint16_t*>(ring + kScaleRing * kRingSlot);   // gated: [BN][64] bf16 up values
    const bool scaled = !p.gated && p.row_w != nullptr;
    int gc = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const Tile tl = decode_tile<BN>(t, prefix, p);
      const uint8_t* wb = p.wblob + (long long)(tl.e * p.feat_tiles + tl.ft) * p.nkb * p.blob_bytes;
      if (te < BN) {
#pragma unroll
        for (int i = 0; i < kScaleRing; ++i) {
          if (i < p.ngroups) issue_scales(p, wb, tl, te, i, ring);
          cp_async_commit();
        }
      }
      if (scaled && te < tl.nrows) {
        const int src = p.row_src[tl.row0 + te];
        rowv[te] = p.row_w_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.row_w)[src])
                                : reinterpret_cast<const float*>(p.row_w)[src];
      }
      float tot[CB];
#pragma unroll
      for (int n = 0; n < CB; ++n) tot[n] = 0.f;
      bool ok = true;
      for (int g = 0; g < p.ngroups; ++g, ++gc) {
        const int buf = gc % NB;
        float* sc = sc_s + (gc & 1) * 256;
        if (te < BN) {
          cp_async_wait<kScaleRing - 1>();   // group g's scales have landed
          const float* slot = ring + (g % kScaleRing) * kRingSlot;
          const float qv = slot[te];
          sc[te] = qv * slot[128 + 2 * te];
          sc[128 + te] = qv * slot[129 + 2 * te];
          if (g + kScaleRing < p.ngroups) issue_scales(p, wb, tl, te, g + kScaleRing, ring);
          cp_async_commit();
        }
        // publishes sc and lets the eight warps agree on success
        ok = named_bar_and(1, kEpi, wait_bounded(&acc_full[buf], (gc / NB) & 1, p.status));
        if (!ok) break;
        tc_fence_after();
        const float4* s4 = reinterpret_cast<const float4*>(sc + half * 128 + n0);
        // all of the group's TMEM loads are issued before one wait
        uint32_t v[CB];
        const uint32_t ta = tq + static_cast<uint32_t>(buf * BN + n0);
        if constexpr (CB % 16 == 0) {
#pragma unroll
          for (int c0 = 0; c0 < CB; c0 += 16)
            tmem_ld16(ta + static_cast<uint32_t>(c0), *reinterpret_cast<uint32_t(*)[16]>(&v[c0]));
        } else {
          tmem_ld8(ta, *reinterpret_cast<uint32_t(*)[8]>(&v[0]));
        }
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < CB; j += 4) {
          const float4 s = s4[j >> 2];
          tot[j] = fmaf(__uint_as_float(v[j]), s.x, tot[j]);
          tot[j + 1] = fmaf(__uint_as_float(v[j + 1]), s.y, tot[j + 1]);
          tot[j + 2] = fmaf(__uint_as_float(v[j + 2]), s.z, tot[j + 2]);
          tot[j + 3] = fmaf(__uint_as_float(v[j + 3]), s.w, tot[j + 3]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      }
      if (!ok) break;
      // Outputs go straight from registers: thread r writes feature r of its
      // token columns, a warp 32 consecutive bf16 (64 B) per token row.
      uint16_t* out16 = reinterpret_cast<uint16_t*>(p.out);
      if (p.gated) {
        // up rows (64..127) hand their bf16 values to the gate rows (0..63)
        if (half == 1) {
#pragma unroll
          for (int n = 0; n < CB; ++n)
            ux16[(n0 + n) * 64 + (r - 64)] = static_cast<uint16_t>(__float_as_uint(bf16_rn(tot[n])) >> 16);
        }
        named_bar_sync(1, kEpi);
        if (half == 0 && tl.ft * 64 + r < p.n_feat) {
#pragma unroll
          for (int n = 0; n < CB; ++n) {
            if (n0 + n < tl.nrows) {
              const float u = __uint_as_float(static_cast<uint32_t>(ux16[(n0 + n) * 64 + r]) << 16);
              out16[(long long)(tl.row0 + n0 + n) * p.ldo + tl.ft * 64 + r] =
                  static_cast<uint16_t>(__float_as_uint(swiglu_bf16(tot[n], u)) >> 16);
            }
          }
        }
        // ux16 is next written after the next tile's group barriers
      } else {
        // rowv (written before the group barriers) is visible here
        if (tl.ft * 128 + r < p.n_feat) {
#pragma unroll
          for (int n = 0; n < CB; ++n) {
            if (n0 + n < tl.nrows) {
              float y = bf16_rn(tot[n]);
              if (scaled) y = bf16_rn(y * rowv[n0 + n]);
              out16[(long long)(tl.row0 + n0 + n) * p.ldo + tl.ft * 128 + r] =
                  static_cast<uint16_t>(__float_as_uint(y) >> 16);
            }
          }
        }
        named_bar_sync(1, kEpi);   // every rowv read is done before the next tile rewrites it
      }
    }
    cp_async_wait<0>();   // no scale copy is still landing when the CTA exits
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

}  // namespace w8

// Shared memory of one CTA for token tile bn: the epilogue buffers (combined
// scales 2 KB, routing weights 512 B, the scale ring 6 KB and, for gated
// tiles, the bf16 up values).
uint32_t w8a8_epilogue_bytes(int bn, int gated) {
  return 8704u + (gated ? static_cast<uint32_t>(bn) * 128u : 0u);
}

int w8a8_tmem_buffers(int) {
  return w8::kTmemBufs;
}

const void* w8a8_kernel_ptr(int bn) {
  switch (bn) {
    case 16: return reinterpret_cast<const void*>(&w8::w8a8_gemm_kernel<16>);
    case 32: return reinterpret_cast<const void*>(&w8::w8a8_gemm_kernel<32>);
    case 64: return reinterpret_cast<const void*>(&w8::w8a8_gemm_kernel<64>);
    case 128: return reinterpret_cast<const void*>(&w8::w8a8_gemm_kernel<128>);
    default: return nullptr;
  }
}

}  // namespace b200
