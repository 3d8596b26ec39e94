// Grouped expert GEMM for short token tiles (decode batches, 16 or 32 rows
// per expert tile) with the weights converted straight into register
// operands of mma.sync (m16n8k16, bf16 x bf16 -> fp32).
//
// At a few tokens per expert the GEMM streams every weight byte once and
// does little arithmetic with it, so its bound is HBM bandwidth. The tcgen05
// kernel (gemm.cu) hands each converted k-block through tensor memory to a
// single issuing thread and back through commits; at 16-token tiles that
// round trip, not the bandwidth, set the pace (a 64-token batch's gate/up
// ran at a third of HBM bandwidth with or without the conversion work).
// Here the warps that convert a k-block also multiply it, from registers:
// no tensor-memory stage, no issuing thread, no commit.
//
// One CTA of 18 warps per SM loops over tiles t = blockIdx.x, + gridDim.x,
// ... (tile = (expert, token tile, feature tile) as in gemm.cu):
//   warp 0      one thread: per k-block, one bulk copy of the packed weight
//               blob (128 rows x 64 columns of e4m3 / e2m1 + scales) into a
//               ring of shared-memory stages
//   warp 17     one thread: per k-block, one 2D TMA box of the tile's token
//               rows (contiguous permuted rows, 64 columns, 128-byte
//               swizzle) into the stage's token box
//   warps 1-16  math: k-block i of the CTA goes to the eight warps of parity
//               i % 2; warp r of them (r = 0..7) owns 16 weight rows (one
//               m16 tile: gated, the gate and up rows of 8 features, so that
//               each thread holds both halves of its SwiGLU inputs) and all
//               token columns. At the end of a tile one warp of a pair hands
//               its partial sums to the other through shared memory, which
//               adds them and runs the epilogue from registers (the two
//               warps take the epilogues of alternate tiles). Sixteen warps
//               keep the conversion pipes busy: the exact e4m3 -> bf16
//               conversion of one k-block (8192 values) takes about 290
//               cycles with 8 warps resident and 140 with 32.
// k-slot mapping: lane (g, t) (g = lane / 4, t = lane % 4) holds physical
// columns 16 t .. 16 t + 15 of its rows, one 16-byte chunk (FP8) or 8 bytes
// (MXFP4); MMA step s (0..3) uses physical columns 16 t + 4 s .. + 3 as its
// k slots 2t, 2t+1, 2t+8, 2t+9. The token fragments follow the same mapping,
// so every column meets its own weight and each MMA sums a permutation of
// 16 columns of the k-block.
#include <algorithm>
#include <mutex>

#include "expert_math.cuh"
#include "gemm_params.h"
#include "ptx.cuh"

namespace b200 {
namespace decode {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kThreads = 576;
constexpr int kWarpW = 0;
constexpr int kWarpMath = 1;   // warps 1..16
constexpr int kWarpTok = 17;

struct Tile {
  int e, ft, row0, nrows;
};

// Ring of mbarrier-guarded stages visited with a stride (the stages of one
// parity), advanced without division.
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
__device__ __forceinline__ Tile decode_tile(int t, const int* prefix, const DecodeParams& p) {
  Tile r;
  const int u = t / p.feat_tiles;
  r.ft = t - u * p.feat_tiles;
  int lo = 0, hi = p.n_experts;   // largest lo with prefix[lo] <= u
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

// Token tiles per expert, scanned by one warp into prefix[0..n_experts];
// returns the CTA-wide tile count (feature tiles included) to lane 0.
__device__ int tile_prefix(const DecodeParams& p, int* prefix, int lane) {
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
  return acc * p.feat_tiles;
}

// Weight producer (one thread): k-block i of the CTA into stage i % nr, the
// packed blob by one bulk copy.
__device__ void produce_weights(const DecodeParams& p, uint8_t* sbase, const int* prefix, int total,
                                uint64_t* full, uint64_t* empty) {
  Ring ring(p.nr);
  int issued = 0;
  bool ok = true;
  for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
    const Tile tl = decode_tile(t, prefix, p);
    const uint8_t* src = p.wblob + (long long)(tl.e * p.feat_tiles + tl.ft) * p.nkb * p.blob_bytes;
    for (int kb = 0; kb < p.nkb; ++kb, ring.next(), ++issued) {
      if (!wait_bounded(&empty[ring.idx], ring.phase ^ 1u, p.status, 32)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&full[ring.idx], p.blob_bytes);
      bulk_load(sbase + ring.idx * p.stage_bytes, src + (long long)kb * p.blob_bytes, p.blob_bytes,
                &full[ring.idx]);
    }
  }
  // every issued copy has landed before the CTA may exit
  for (int i = max(0, issued - p.nr); i < issued; ++i)
    wait_bounded(&full[i % p.nr], (i / p.nr) & 1, p.status, 32);
}

// Token producer (one thread): the tile's bn token rows x 64 columns of
// k-block i into token box i % nr by one 2D TMA box (128-byte swizzle:
// 16-byte chunk j of row n lands at chunk j ^ (n & 7); rows past the tensor
// and columns past k_valid read as zero). A thread of its own: a tensor copy
// costs the issuing thread about as long as the weight blob's bulk copy.
__device__ void produce_tokens(const DecodeParams& p, const CUtensorMap* tmap, uint8_t* sbase,
                               const int* prefix, int total, uint64_t* full, uint64_t* empty) {
  Ring ring(p.nr);
  int issued = 0;
  bool ok = true;
  for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
    const Tile tl = decode_tile(t, prefix, p);
    for (int kb = 0; kb < p.nkb; ++kb, ring.next(), ++issued) {
      if (!wait_bounded(&empty[ring.idx], ring.phase ^ 1u, p.status, 32)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&full[ring.idx], static_cast<uint32_t>(p.bn) * 128u);
      tma_load_2d(sbase + p.tok_off + ring.idx * p.bn * 128, tmap, &full[ring.idx], kb * 64, tl.row0);
    }
  }
  for (int i = max(0, issued - p.nr); i < issued; ++i)
    wait_bounded(&full[i % p.nr], (i / p.nr) & 1, p.status, 32);
}

// Epilogue of one tile from the summed fragments: thread (g, tq) holds rows
// g and g + 8 of the warp's m16 tile for token columns 8 nt + 2 tq + {0, 1}.
// Gated: row g is the gate and row g + 8 the up projection of feature
// ft * 64 + 8 rg + g. Down: rows are output features ft * 128 + 16 rg +
// {g, g + 8}. Arithmetic as the tcgen05 kernel's.
// Per-tile epilogue inputs from global memory, loaded before the tile's
// k-blocks so that their latency overlaps them: the two bias values of the
// thread's rows and the routing weights of its token columns.
template <int NT>
struct EpiInputs {
  float b[2];
  float w[NT][2];
};

template <int NT>
__device__ __forceinline__ void load_epilogue_inputs(const DecodeParams& p, const Tile& tl, int rg, int g, int tq,
                                                     EpiInputs<NT>& in) {
  in.b[0] = in.b[1] = 0.f;
  if (p.bias != nullptr) {
    if (p.gated) {
      const int f = tl.ft * 64 + 8 * rg + g;
      if (f < p.n_feat) {
        in.b[0] = __bfloat162float(p.bias[(long long)(tl.e * 2) * p.feat_pad + f]);
        in.b[1] = __bfloat162float(p.bias[(long long)(tl.e * 2 + 1) * p.feat_pad + f]);
      }
    } else {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int h = tl.ft * 128 + 16 * rg + 8 * hh + g;
        if (h < p.n_feat) in.b[hh] = __bfloat162float(p.bias[(long long)tl.e * p.feat_pad + h]);
      }
    }
  }
  const bool scaled = !p.gated && p.row_w != nullptr;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int j = 8 * nt + 2 * tq + i;
      in.w[nt][i] = 1.f;
      if (scaled && j < tl.nrows) {
        const int src = p.row_src[tl.row0 + j];
        in.w[nt][i] = p.row_w_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.row_w)[src])
                                   : reinterpret_cast<const float*>(p.row_w)[src];
      }
    }
}

template <int NT>
__device__ void epilogue(const DecodeParams& p, const Tile& tl, const float (&acc)[NT][4], const EpiInputs<NT>& in,
                         int rg, int g, int tq) {
  if (p.gated) {
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
    const int f = tl.ft * 64 + 8 * rg + g;
    if (f >= p.n_feat) return;
    const float bg = in.b[0], bu = in.b[1];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int j = 8 * nt + 2 * tq + i;
        if (j < tl.nrows) {
          const float a = epilogue_gated(p.epi, acc[nt][i], acc[nt][2 + i], bg, bu, p.alpha, p.limit);
          out[(long long)(tl.row0 + j) * p.ldo + f] = __float2bfloat16_rn(a);
        }
      }
    return;
  }
  const bool scaled = p.row_w != nullptr;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int h = tl.ft * 128 + 16 * rg + 8 * hh + g;
    if (h >= p.n_feat) continue;
    const float b = in.b[hh];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int j = 8 * nt + 2 * tq + i;
        if (j >= tl.nrows) continue;
        const float a = acc[nt][2 * hh + i];
        const long long o = (long long)(tl.row0 + j) * p.ldo + h;
        if (p.epi == kEpiDownF32) {
          static_cast<float*>(p.out)[o] = a + b;
        } else {
          float y = bf16_rn(a);
          if (p.bias != nullptr) y = bf16_rn(y + b);
          if (scaled) y = bf16_rn(y * in.w[nt][i]);
          static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(y);
        }
      }
  }
}

// Math warp mw (0..15): k-blocks of parity mw / 8, weight rows of group
// rg = mw % 8 (one m16 tile: gated, the gate and up rows of features
// 8 rg .. + 7; down, rows 16 rg .. + 15), all NT x 8 token columns. xchg:
// per warp pair two buffers (by tile parity) of 32 lanes x 4 NT floats.
template <int NT, int WFMT>
__device__ void math_warp(const DecodeParams& p, uint8_t* sbase, const int* prefix, int total,
                          uint64_t* full, uint64_t* empty, float* xchg, int mw, int lane) {
  const int par = mw >> 3;
  const int rg = mw & 7;
  const int g = lane >> 2, tq = lane & 3;
  // fragment rows g (top) and g + 8 (bottom)
  const int rtop = p.gated ? 8 * rg + g : 16 * rg + g;
  const int rbot = p.gated ? 64 + rtop : rtop + 8;
  Ring ring(p.nr / 2);
  int tc = 0, i0 = 0;
  for (int t = blockIdx.x; t < total; t += gridDim.x, ++tc, i0 += p.nkb) {
    const Tile tl = decode_tile(t, prefix, p);
    // the pair's epilogue alternates between its warps by tile
    const bool owner = par == (tc & 1);
    EpiInputs<NT> ein;
    if (owner) load_epilogue_inputs<NT>(p, tl, rg, g, tq, ein);
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;
    bool ok = true;
    for (int kb = (par - i0) & 1; kb < p.nkb; kb += 2) {
      const int s = par + 2 * ring.idx;
      if (!wait_spin(&full[s], ring.phase, p.status)) {
        ok = false;
        break;
      }
      const uint8_t* st = sbase + s * p.stage_bytes;
      uint32_t at[8], ab[8];   // converted rows: bf16 pairs of columns 16 tq .. + 15
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = h ? rbot : rtop;
        uint32_t(&dst)[8] = h ? ab : at;
        if (WFMT == kWFp8) {
          const float* sc = reinterpret_cast<const float*>(st + kRawFp8);
          const uint4 q = *reinterpret_cast<const uint4*>(st + row * 64 + ((tq ^ ((row >> 1) & 3)) << 4));
          const float scale = p.scale_form == kScaleHalf ? sc[row >> 6] : sc[row * 4 + tq];
          fp8x16_cvt(q, scale, dst);
        } else {
          const uint2 q = *reinterpret_cast<const uint2*>(
              st + row * 32 + (((tq >> 1) ^ ((row >> 2) & 1)) << 4) + ((tq & 1) << 3));
          const uint32_t sx = *reinterpret_cast<const unsigned short*>(st + kRawMx + row * 2);
          mx16_cvt(q, (sx >> (8 * (tq >> 1))) & 0xffu, dst);
        }
      }
      uint4 bt[NT][2];   // token g + 8 nt: columns 16 tq .. + 7 and + 8 .. + 15
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int n = 8 * nt + g;
        const uint8_t* rowp = sbase + p.tok_off + (s * p.bn + n) * 128;
        bt[nt][0] = *reinterpret_cast<const uint4*>(rowp + (((2 * tq) ^ (n & 7)) << 4));
        bt[nt][1] = *reinterpret_cast<const uint4*>(rowp + (((2 * tq + 1) ^ (n & 7)) << 4));
      }
      // the stage's bytes are in registers: release it
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      ring.next();
#pragma unroll
      for (int s4 = 0; s4 < 4; ++s4) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint4& c = bt[nt][s4 >> 1];
          const uint32_t b0 = (s4 & 1) ? c.z : c.x;
          const uint32_t b1 = (s4 & 1) ? c.w : c.y;
          mma_16816_bf16(acc[nt], at[2 * s4], ab[2 * s4], at[2 * s4 + 1], ab[2 * s4 + 1], b0, b1);
        }
      }
    }
    // partial sums of the other warp to the tile's owner (the sum of two
    // values, the same in either order); both warps agree on success before
    // either goes on
    float* xb = xchg + (rg * 2 + (tc & 1)) * (32 * 4 * NT);
    if (!owner) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) xb[(nt * 4 + i) * 32 + lane] = acc[nt][i];
    }
    if (!named_bar_and(1 + rg, 64, ok)) break;
    if (!owner) continue;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[nt][i] += xb[(nt * 4 + i) * 32 + lane];
    epilogue<NT>(p, tl, acc, ein, rg, g, tq);
  }
}

template <int NT, int WFMT>
__global__ void __launch_bounds__(kThreads, 1)
    moe_decode_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  uint8_t* sbase = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
  // a wait already timed out on this device (status not yet cleared): do not
  // start more work that would queue behind the same fault
  if (*reinterpret_cast<volatile int*>(p.status) & kStatusWaitTimeout) return;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(sbase + p.bar_off);
  uint64_t* empty = full + p.nr;
  int* s_total = reinterpret_cast<int*>(empty + p.nr);
  int* prefix = s_total + 1;
  float* xchg = reinterpret_cast<float*>(sbase + p.x_off);
  if (warp == 0) {
    const int tot = tile_prefix(p, prefix, lane);
    if (lane == 0) *s_total = tot;
  }
  if (threadIdx.x == 32) {
    // full: the two producers' expect_tx arrivals; empty: the eight math
    // warps of the stage's parity
    for (int i = 0; i < p.nr; ++i) {
      mbar_init(&full[i], 2);
      mbar_init(&empty[i], 8);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmap);
  }
  __syncthreads();
  const int total = *s_total;
  if (warp == kWarpW) {
    if (lane == 0) produce_weights(p, sbase, prefix, total, full, empty);
  } else if (warp == kWarpTok) {
    if (lane == 0) produce_tokens(p, &tmap, sbase, prefix, total, full, empty);
  } else {
    math_warp<NT, WFMT>(p, sbase, prefix, total, full, empty, xchg, warp - kWarpMath, lane);
  }
}

}  // namespace decode

int launch_decode_gemm(const CUtensorMap& tmap, const DecodeParams& p, int grid, uint32_t smem,
                       cudaStream_t stream) {
  if ((p.wfmt != kWFp8 && p.wfmt != kWMx) || (p.bn != 16 && p.bn != 32) || smem > kDecodeSmemMax)
    return static_cast<int>(cudaErrorInvalidValue);
  const int ki = (p.wfmt == kWMx ? 2 : 0) + (p.bn == 32 ? 1 : 0);
  const void* kerns[4] = {reinterpret_cast<const void*>(&decode::moe_decode_kernel<2, kWFp8>),
                          reinterpret_cast<const void*>(&decode::moe_decode_kernel<4, kWFp8>),
                          reinterpret_cast<const void*>(&decode::moe_decode_kernel<2, kWMx>),
                          reinterpret_cast<const void*>(&decode::moe_decode_kernel<4, kWMx>)};
  const void* kern = kerns[ki];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  {
    // the shared-memory limit is raised once per kernel and device
    static std::mutex mu;
    static bool raised[4][kDecodeMaxDevices] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= kDecodeMaxDevices) return static_cast<int>(cudaErrorInvalidDevice);
    if (!raised[ki][dev]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kDecodeSmemMax));
      if (e != cudaSuccess) return static_cast<int>(e);
      raised[ki][dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(decode::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  void* args[] = {const_cast<CUtensorMap*>(&tmap), const_cast<DecodeParams*>(&p)};
  return static_cast<int>(cudaLaunchKernelExC(&cfg, kern, args));
}

}  // namespace b200
