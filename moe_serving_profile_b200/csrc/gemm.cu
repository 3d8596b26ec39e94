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
//   warp 0      TMA: one bulk copy per k-block of the packed weight blob
//               (e4m3 / e2m1 rows + scales) into a ring of shared-memory
//               stages, or 2D tiles of bf16 weights straight into
//               shared-memory A stages
//   warp 1      TMEM allocator and tcgen05.mma issuer (one thread); two
//               accumulator slots so a tile's epilogue overlaps the next
//               tile's main loop
//   warp 2      TMA for the token rows: tile::gather4 of the routed tokens'
//               rows (gate/up) or a 2D tile of contiguous rows (down)
//   warps 4-7   epilogue (TMEM lane quarters 0-3): activation / bias /
//               routing weight, bf16 stores
//   warps 8-15  converters (quantised weights), in one of three forms:
//               - two MMA issuers (token tiles up to 64 rows): two groups of
//                 four warps; group g converts the CTA's k-blocks g, g + 2,
//                 ..., each lane one weight row, into tensor-memory A stages
//                 (warp w owns TMEM lanes 32 (w % 4) .. + 31) that
//                 tcgen05.mma reads as its A operand; four A stages per
//                 group let a group run ahead of the MMA's consumption;
//               - one issuer (128- and 160-row tiles): all eight warps
//                 convert every k-block, half a weight row per lane, into
//                 the same tensor-memory A stages;
//               - 256-row tiles (a_smem; only when the caller asks for
//                 them): all eight warps convert every
//                 k-block into 128-byte-swizzled shared-memory A stages, so
//                 that the whole tensor memory holds two 256-column
//                 accumulator slots.
// All rings are phase-tracked mbarriers; every wait is bounded (see ptx.cuh).
#include "expert_math.cuh"
#include "gemm_params.h"
#include "ptx.cuh"

namespace b200 {

namespace gemm {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kThreads = 512;
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpMma2 = 3;     // second MMA issuer (two-issuer tiles)
constexpr int kWarpB = 2;
constexpr int kWarpEpi = 4;      // warps 4..7
constexpr int kWarpConv = 8;     // warps 8..15
constexpr uint32_t kATile = 128u * 128u;    // 128 rows x 64 bf16
constexpr uint32_t kAStageCols = 32;        // TMEM columns per A stage (64 bf16 / lane)

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

// Rows per token tile of an expert with cnt rows: bn, or (a_smem) the
// expert's ceil(cnt / bn) tiles cut evenly, rounded up to 16 rows; when the
// rounding would leave the last tile empty, bn.
__device__ __forceinline__ int chunk_rows(int cnt, const GemmParams& p) {
  if (!p.a_smem || cnt <= 0) return p.bn;
  const int nt = (cnt + p.bn - 1) / p.bn;
  const int cs = ((cnt + nt - 1) / nt + 15) & ~15;
  return (nt - 1) * cs < cnt ? cs : p.bn;
}

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
  const int cs = chunk_rows(cnt, p);
  r.row0 = start + sub * cs;
  r.nrows = min(cs, cnt - sub * cs);
  return r;
}

// MMA N of a tile: its rows rounded up to 16 (a_smem), else the launch's bn.
__device__ __forceinline__ int tile_n(const Tile& tl, const GemmParams& p) {
  return p.a_smem ? ((tl.nrows + 15) & ~15) : p.bn;
}

// 16 accumulator columns of this thread's TMEM lane summed over the banks
// the tile wrote (bank b at column offset b * stride): bank0, bank0 + 1, ...
// (mod nacc), nbanks of them, in that order.
__device__ __forceinline__ void load_acc(uint32_t taddr, int stride, int bank0, int nacc, int nbanks,
                                         float (&acc)[16]) {
  uint32_t r[16];
  tmem_ld16(taddr + static_cast<uint32_t>(bank0 * stride), r);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j] = __uint_as_float(r[j]);
  for (int k = 1; k < nbanks; ++k) {
    const int b = (bank0 + k) & (nacc - 1);
    tmem_ld16(taddr + static_cast<uint32_t>(b * stride), r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] += __uint_as_float(r[j]);
  }
}

// MMA issuer j of `step` (1 or 2). Issuer j takes the CTA's k-blocks
// i = j, j + step, ... (A / B stages j + step * r) and accumulates k-block i
// into bank i % nacc of the tile's slot (nacc = 1, 2 or 4; with two issuers
// nacc is even, so the two never share a bank). It waits once for G of its
// k-blocks' A and B stages, then issues their 4G MMAs and G stage releases
// as straight-line code, specialised at compile time on where A lives and on
// whether one commit releases both rings. Measured in isolation: a barrier
// wait and tensor fence before every k-block leave the tensor pipe idle
// about 160 of every 480 cycles at 160-token tiles, one per two k-blocks
// about 40; a conditional branch between MMAs costs the issuing thread tens
// of cycles (a loop with one runtime-conditional commit: 443 against 227
// cycles per k-block of 16-token MMAs); one thread issues a 16..64-token
// k-block in about 227 cycles, two together one per 156..192 cycles.
template <bool kTmemA, bool kJoint, int G>
__device__ void mma_issue_groups(const GemmParams& p, uint32_t tmem, uint32_t base_u32, const int* prefix,
                                int total, uint64_t* a_full, uint64_t* a_empty, uint64_t* b_full,
                                uint64_t* b_empty, uint64_t* acc_full, uint64_t* acc_empty,
                                uint64_t* mma_done, int j, int step) {
  Ring ra(p.na / step), rb(p.nb / step);
  int tc = 0;
  int i0 = 0;   // CTA-wide index of the tile's first k-block
  bool ok = true;
  auto kblock = [&](uint32_t d, int sa, int sb, uint32_t idesc, uint32_t acc) {
    const uint64_t bdesc = sdesc_k_sw128(base_u32 + p.b_off + static_cast<uint32_t>(sb * p.bn * 128));
    if (kTmemA)
      umma_kblock_tmem_a(d, tmem + p.a_col0 + static_cast<uint32_t>(sa) * kAStageCols, bdesc, idesc, acc);
    else
      umma_kblock_smem_a(d, sdesc_k_sw128(base_u32 + p.a_off + static_cast<uint32_t>(sa) * kATile), bdesc,
                         idesc, acc);
    umma_commit(&a_empty[sa]);
    if (!kJoint) umma_commit(&b_empty[sb]);
  };
  for (int t = blockIdx.x; ok && t < total; t += gridDim.x, ++tc, i0 += p.nkb) {
    const int slot = p.acc_slots == 2 ? (tc & 1) : 0;
    const uint32_t use = p.acc_slots == 2 ? static_cast<uint32_t>(tc >> 1) : static_cast<uint32_t>(tc);
    const uint32_t idesc = idesc_bf16_f32(128, tile_n(decode_tile(t, prefix, p), p));
    if (!wait_bounded(&acc_empty[slot], (use & 1u) ^ 1u, p.status)) break;
    tc_fence_after();
    const uint32_t d0 = tmem + static_cast<uint32_t>(slot * p.nacc * p.bn);
    const int kb0 = (j - i0) & (step - 1);                     // this issuer's first k-block
    const int mine = kb0 < p.nkb ? (p.nkb - kb0 + step - 1) / step : 0;
    for (int m = 0; m < mine; m += G) {
      const int n = min(G, mine - m);
      int sa[G], sb[G];
#pragma unroll
      for (int i = 0; i < G; ++i) {
        sa[i] = j + step * ra.idx;
        sb[i] = j + step * rb.idx;
        if (i < n) {
          if (ok && (!wait_bounded(&a_full[sa[i]], ra.phase, p.status) ||
                     !wait_bounded(&b_full[sb[i]], rb.phase, p.status)))
            ok = false;
          ra.next();
          rb.next();
        }
      }
      if (!ok) break;
      tc_fence_after();
      // bank and accumulate flag of each k-block: arithmetic, no branches
      uint32_t d[G], acc[G];
#pragma unroll
      for (int i = 0; i < G; ++i) {
        const int kb = kb0 + (m + i) * step;
        d[i] = d0 + static_cast<uint32_t>(((i0 + kb) & (p.nacc - 1)) * p.bn);
        acc[i] = kb >= p.nacc ? 1u : 0u;   // a bank's first k-block of the tile overwrites
      }
      if (n == G) {
#pragma unroll
        for (int i = 0; i < G; ++i) kblock(d[i], sa[i], sb[i], idesc, acc[i]);
      } else {
        for (int i = 0; i < n; ++i) kblock(d[i], sa[i], sb[i], idesc, acc[i]);
      }
    }
    if (!ok) break;
    umma_commit(&acc_full[slot]);
  }
  // all issued MMAs have finished before TMEM is released
  umma_commit(mma_done);
  wait_bounded(mma_done, 0, p.status);
}

__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap bmap,
                    const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
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
  if (threadIdx.x == 32 * kWarpTma) {
    // quantised weights: a raw stage is drained, and an A stage filled, by
    // the four warps of one converter group (a_smem: by all eight)
    const uint32_t group = p.wfmt == kWBf16 ? 1u : ((p.a_smem || p.n_issuers == 1) ? 8u : 4u);
    for (int i = 0; i < p.nr; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], group);
    }
    for (int i = 0; i < p.na; ++i) {
      mbar_init(&a_full[i], group);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < p.nb; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], static_cast<uint32_t>(p.n_issuers));
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(mma_done, static_cast<uint32_t>(p.n_issuers));
    fence_mbar_init();
    if (p.wfmt == kWBf16) tma_prefetch_desc(&wmap);   // quantised weights use bulk copies
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
      // k-block i of this CTA goes to raw stage i % nr (nr even), drained by
      // converter group i % 2, whose warps step through its phases in order.
      // BF16 tiles go straight to shared-memory A stages.
      Ring ring(p.wfmt == kWBf16 ? p.na : p.nr);
      uint64_t* full = p.wfmt == kWBf16 ? a_full : raw_full;
      uint64_t* empty = p.wfmt == kWBf16 ? a_empty : raw_empty;
      int issued = 0;
      Tile tl2{0, 0, 0, 0};
      if (blockIdx.x < total) tl2 = decode_tile(blockIdx.x, prefix, p);
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        const Tile tl = tl2;   // decoded one tile ahead
        if (t + gridDim.x < total) tl2 = decode_tile(t + gridDim.x, prefix, p);
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
            const long long blob = (long long)(tl.e * p.feat_tiles + tl.ft) * p.nkb + kb;
            mbar_arrive_expect_tx(&full[s], p.blob_bytes);
            bulk_load(sbase + p.raw_off + s * p.stage_bytes, p.wblob + blob * p.blob_bytes,
                      p.blob_bytes, &full[s]);
          }
        }
      }
      // every issued copy has landed before the CTA may exit
      for (int i = max(0, issued - ring.n); i < issued; ++i)
        wait_bounded(&full[i % ring.n], (i / ring.n) & 1, p.status, 32);
    }
  } else if (warp == kWarpMma || (warp == kWarpMma2 && p.n_issuers == 2)) {
    // ------------------------------------------------ MMA issuers
    // With two issuers, issuer j (warp 1 or 3) takes the CTA's k-blocks
    // i = j, j + 2, ... (the A stages converter group j fills) and
    // accumulates k-block i into bank i % nacc (nacc even), so the two never
    // share an accumulator; one thread issues a short-tile k-block in about
    // 227 cycles, two together one per 156..192. Both commit to acc_full.
    if (lane == 0) {
      const bool tmem_a = p.wfmt != kWBf16 && !p.a_smem;
      const int j = warp == kWarpMma ? 0 : 1;
#define B200_ISSUE(TA, J)                                                                           \
  mma_issue_groups<TA, J, 2>(p, tmem, base_u32, prefix, total, a_full, a_empty, b_full, b_empty, acc_full, \
                             acc_empty, mma_done, j, p.n_issuers)
      if (tmem_a && p.joint_ab) B200_ISSUE(true, true);
      else if (tmem_a) B200_ISSUE(true, false);
      else if (p.joint_ab) B200_ISSUE(false, true);
      else B200_ISSUE(false, false);
#undef B200_ISSUE
    }
  } else if (warp == kWarpB) {
    // ------------------------------------------------ token-row TMA producer
    // The gathered rows' token ids of the next tile are loaded while this
    // tile's k-blocks are issued.
    Ring ring(p.nb);
    int issued = 0;
    bool ok = true;
    int tok[2][4], nxt[2][4];
    auto load_tok = [&](const Tile& tl_, int (&d)[2][4]) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int q4 = (lane + 32 * j) * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = (q4 + i < tl_.nrows) ? q4 + i : 0;   // padding rows repeat row 0
          d[j][i] = (p.b_gather && q4 < p.bn) ? p.b_map[tl_.row0 + r] / p.b_div : 0;
        }
      }
    };
    int t = blockIdx.x;
    Tile tl{0, 0, 0, 0};
    if (t < total) {
      tl = decode_tile(t, prefix, p);
      load_tok(tl, tok);
    }
    for (; ok && t < total; t += gridDim.x) {
      const int t2 = t + gridDim.x;
      Tile tl2 = tl;
      if (t2 < total) {
        tl2 = decode_tile(t2, prefix, p);
        load_tok(tl2, nxt);
      }
      for (int kb = 0; kb < p.nkb; ++kb, ring.next(), ++issued) {
        const int s = ring.idx;
        if (!wait_bounded(p.joint_ab ? &a_empty[s] : &b_empty[s], ring.phase ^ 1u, p.status, 32)) {
          ok = false;
          break;
        }
        uint8_t* dst = sbase + p.b_off + s * p.bn * 128;
        if (p.a_smem) {
          // 64-row boxes covering the tile's MMA N (rows past the tile are
          // read but never stored; past the tensor they are zero-filled)
          const int nbox = (tile_n(tl, p) + 63) >> 6;
          if (lane == 0) {
            mbar_arrive_expect_tx(&b_full[s], static_cast<uint32_t>(nbox) * 64u * 128u);
            for (int j = 0; j < nbox; ++j)
              tma_load_2d(dst + j * 64 * 128, &bmap, &b_full[s], kb * 64, tl.row0 + j * 64);
          }
          __syncwarp();
          continue;
        }
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
      tl = tl2;
      if (t2 < total) {
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int i = 0; i < 4; ++i) tok[j][i] = nxt[j][i];
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
    // features beyond n_feat are never written). Gated tiles pair the gate
    // (lanes 0-63) and up (64-127) rows of a feature through a shared
    // exchange buffer; the down projection needs no exchange, so each warp
    // stages and writes its own features.
    const int q = warp - kWarpEpi;
    const int te = threadIdx.x - kWarpEpi * 32;
    const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16);
    float* xbuf = reinterpret_cast<float*>(sbase + p.x_off);                      // [4][16][32] f32
    uint16_t* stage = reinterpret_cast<uint16_t*>(sbase + p.x_off + 8192);        // [2][16][128] bf16
    float* rowv = reinterpret_cast<float*>(sbase + p.x_off + 16384);             // [256] f32
    const bool scaled = !p.gated && p.row_w != nullptr;
    int tc = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++tc) {
      // tile bookkeeping and bias first: their loads overlap the accumulator wait
      const Tile tl = decode_tile(t, prefix, p);
      const int slot = p.acc_slots == 2 ? (tc & 1) : 0;
      const uint32_t use = p.acc_slots == 2 ? static_cast<uint32_t>(tc >> 1) : static_cast<uint32_t>(tc);
      const int fl = p.gated ? (q & 1) * 32 + lane : q * 32 + lane;
      const int f = tl.ft * (p.gated ? 64 : 128) + fl;
      const bool fvalid = f < p.n_feat;
      float b0 = 0.f, b1 = 0.f;
      if (p.bias != nullptr && fvalid) {
        if (p.gated) {
          b0 = __bfloat162float(p.bias[(long long)(tl.e * 2) * p.feat_pad + f]);
          b1 = __bfloat162float(p.bias[(long long)(tl.e * 2 + 1) * p.feat_pad + f]);
        } else {
          b0 = __bfloat162float(p.bias[(long long)tl.e * p.feat_pad + f]);
        }
      }
      if (scaled) {
        // the routing weights of the tile's rows, published by the barrier below
        named_bar_sync(1, 128);   // every reader of the previous tile's weights is done
        for (int i = te; i < tl.nrows; i += 128) {
          const int src = p.row_src[tl.row0 + i];
          rowv[i] = p.row_w_bf16
                        ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.row_w)[src])
                        : reinterpret_cast<const float*>(p.row_w)[src];
        }
      }
      const int bank0 = (tc * p.nkb) & (p.nacc - 1);
      // the four epilogue warps agree on success before using their barrier
      const bool ok =
          named_bar_and(1, 128, wait_bounded(&acc_full[slot], use & 1u, p.status, 128));
      if (!ok) break;
      tc_fence_after();
      const int ncols = (tl.nrows + 15) & ~15;
      if (p.gated) {
        const float bg = b0, bu = b1;
        const int jb = (q >> 1) * 8;
        for (int c0 = 0, ci = 0; c0 < ncols; c0 += 16, ++ci) {
          float acc[16];
          load_acc(tq + slot * p.nacc * p.bn + c0, p.bn, bank0, p.nacc, p.nbanks, acc);
#pragma unroll
          for (int j = 0; j < 16; ++j) xbuf[(q * 16 + j) * 32 + lane] = acc[j];
          named_bar_sync(1, 128);
          uint16_t* st = stage + (ci & 1) * 16 * 64;     // [16][64]
          // every exchange read before any staging store: both go through
          // generic pointers, so interleaved they would serialise on the
          // compiler's aliasing assumption
          float gv[8], uv[8];
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            gv[jj] = xbuf[((q & 1) * 16 + jb + jj) * 32 + lane];
            uv[jj] = xbuf[((2 + (q & 1)) * 16 + jb + jj) * 32 + lane];
          }
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const float a = epilogue_gated(p.epi, gv[jj], uv[jj], bg, bu, p.alpha, p.limit);
            st[(jb + jj) * 64 + fl] = static_cast<uint16_t>(__float_as_uint(a) >> 16);
          }
          named_bar_sync(1, 128);
          const int j = te >> 3;
          const int c8 = (te & 7) * 8;
          if (c0 + j < tl.nrows && tl.ft * 64 + c8 < p.n_feat)
            *reinterpret_cast<uint4*>(p.out + (long long)(tl.row0 + c0 + j) * p.ldo + tl.ft * 64 + c8) =
                *reinterpret_cast<const uint4*>(st + j * 64 + c8);
        }
      } else if (p.epi == kEpiDownF32) {
        // fp32 rows acc + bias, unrounded: each warp stages its 32 features x
        // 16 tokens (2 KB, two alternating buffers in the exchange and
        // staging areas) and writes 16 rows x 128 bytes with 16-byte stores
        float* fst = reinterpret_cast<float*>(sbase + p.x_off) + q * 1024;   // [2][16][32] f32 of this warp
        float* out0 = reinterpret_cast<float*>(p.out) + (long long)tl.row0 * p.ldo;
        for (int c0 = 0, ci = 0; c0 < ncols; c0 += 16, ++ci) {
          float acc[16];
          load_acc(tq + slot * p.nacc * p.bn + c0, p.bn, bank0, p.nacc, p.nbanks, acc);
          float* st = fst + (ci & 1) * 512;
#pragma unroll
          for (int j = 0; j < 16; ++j) st[j * 32 + lane] = acc[j] + b0;
          __syncwarp();
          // lane l, pass i: token row (l + 32 i) / 8, features 4 ((l + 32 i) & 7) .. + 3
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int c = lane + 32 * i;
            const int j = c0 + (c >> 3);
            const int fo = tl.ft * 128 + 32 * q + 4 * (c & 7);
            if (j < tl.nrows && fo < p.n_feat)
              *reinterpret_cast<float4*>(out0 + (long long)j * p.ldo + fo) =
                  *reinterpret_cast<const float4*>(st + (c >> 3) * 32 + 4 * (c & 7));
          }
        }
      } else {
        // Each warp stages its 32 features x 16 tokens in its own buffer
        // (two, alternating) and writes 16 rows x 64 bytes with 16-byte
        // stores: no barrier across warps inside the tile. The routing
        // weights of the tile's rows are published once per tile.
        uint16_t* wst = stage + q * 1024;   // [2][16][32] bf16 of this warp
        uint16_t* out0 = reinterpret_cast<uint16_t*>(p.out) + (long long)tl.row0 * p.ldo;
        for (int c0 = 0, ci = 0; c0 < ncols; c0 += 16, ++ci) {
          float acc[16];
          load_acc(tq + slot * p.nacc * p.bn + c0, p.bn, bank0, p.nacc, p.nbanks, acc);
          uint16_t* st = wst + (ci & 1) * 512;
          // the chunk's routing weights read before any staging store (generic
          // pointers: interleaved, each load would wait for the last store)
          float wv[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) wv[j] = scaled ? rowv[c0 + j] : 1.f;
          // roundings by the hardware conversion: the integer form (four
          // ops a value) cost this epilogue, which shares the SM's issue slots
          // with the converter warps, 17 us of the 4096-token down GEMM
          uint32_t yb[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float y = bf16r(acc[j]);
            if (p.bias != nullptr) y = bf16r(y + b0);
            if (scaled) y = bf16r(y * wv[j]);
            yb[j] = __float_as_uint(y) >> 16;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) st[j * 32 + lane] = static_cast<uint16_t>(yb[j]);
          __syncwarp();
          // lane l, pass i: chunk row (l + 32 i) / 4, features 8 ((l + 32 i) & 3) .. + 7
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int c = lane + 32 * i;
            const int j = c0 + (c >> 2);
            const int fo = tl.ft * 128 + 32 * q + 8 * (c & 3);
            if (j < tl.nrows && fo < p.n_feat)
              *reinterpret_cast<uint4*>(out0 + (long long)j * p.ldo + fo) =
                  *reinterpret_cast<const uint4*>(st + c * 8);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[slot]);
    }
  } else if (warp >= kWarpConv && p.a_smem) {
    // ------------------------------------------------ converters (a_smem)
    // All eight warps convert every k-block: lane l of converter warp c takes
    // weight row 16 c + l / 2, half h = l & 1 (32 of its 64 values), and
    // writes the four 16-byte bf16 chunks 4h .. 4h + 3 of that row into the
    // shared-memory A stage at their 128-byte-swizzle positions (eight
    // consecutive lanes hit eight distinct 16-byte bank groups, so each
    // store is four wavefronts). Raw rows are read through the packing's
    // chunk permutation, also without conflicts.
    const int row = (warp - kWarpConv) * 16 + (lane >> 1);
    const int h = lane & 1;
    const int half = row >> 6;                           // gate/up plane or down half
    Ring rr(p.nr), ar(p.na);
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
      for (int kb = 0; kb < p.nkb; ++kb) {
        if (!wait_spin(&raw_full[rr.idx], rr.phase, p.status, 32) ||
            !wait_spin(&a_empty[ar.idx], ar.phase ^ 1u, p.status, 32)) {
          ok = false;
          break;
        }
        const uint8_t* stage = sbase + p.raw_off + rr.idx * p.stage_bytes;
        uint32_t o[16];
        if (p.wfmt == kWFp8) {
          const uint8_t* raw = stage + row * 64;
          const float* sc = reinterpret_cast<const float*>(stage + kRawFp8);
          const int sw = (row >> 1) & 3;
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int c = 2 * h + j;
            const uint4 qv = *reinterpret_cast<const uint4*>(raw + ((c ^ sw) << 4));
            const float scale = p.scale_form == kScaleHalf ? sc[half] : sc[row * 4 + c];
            fp8x16_cvt(qv, scale, *reinterpret_cast<uint32_t(*)[8]>(o + 8 * j));
          }
        } else {
          const uint8_t* raw = stage + row * 32;
          const int sw = (row >> 2) & 1;
          const uint32_t sx = *reinterpret_cast<const unsigned short*>(stage + kRawMx + row * 2);
          const uint4 qv = *reinterpret_cast<const uint4*>(raw + ((h ^ sw) << 4));
          mx32_cvt(qv, (sx >> (8 * h)) & 0xffu, o);
        }
        // the raw bytes and scales are in registers: release the stage
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rr.idx]);
        uint8_t* a = sbase + p.a_off + ar.idx * kATile;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(a + swz(row, 4 * h + j)) =
              make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[ar.idx]);
        rr.next();
        ar.next();
      }
    }
  } else if (warp >= kWarpConv && p.wfmt != kWBf16 && p.n_issuers == 1) {
    // ------------------------------------------------ converters (one issuer)
    // All eight warps convert every k-block, in order: warp w writes TMEM
    // lane quarter w % 4 (lane i: weight row 32 (w % 4) + i) and column half
    // h = (w - 8) / 4 of the A stage (k values 32 h .. 32 h + 31, TMEM
    // columns 16 h .. 16 h + 15). Half a row per lane halves the latency of a
    // k-block's conversion against one four-warp group per k-block.
    const int qw = warp & 3;
    const int h = (warp - kWarpConv) >> 2;
    const int row = qw * 32 + lane;
    const int half = row >> 6;                           // gate/up plane or down half
    const uint32_t tq = tmem + (static_cast<uint32_t>(qw * 32) << 16) + p.a_col0 + static_cast<uint32_t>(h * 16);
    Ring rr(p.nr), ar(p.na);
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
      for (int kb = 0; kb < p.nkb; ++kb) {
        if (!wait_spin(&raw_full[rr.idx], rr.phase, p.status, 32) ||
            !wait_spin(&a_empty[ar.idx], ar.phase ^ 1u, p.status, 32)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* stage = sbase + p.raw_off + rr.idx * p.stage_bytes;
        uint32_t o[16];
        if (p.wfmt == kWFp8) {
          const uint8_t* raw = stage + row * 64;
          const float* sc = reinterpret_cast<const float*>(stage + kRawFp8);
          const int sw = (row >> 1) & 3;
          uint4 qv[2];
          float scale[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int c = 2 * h + j;
            qv[j] = *reinterpret_cast<const uint4*>(raw + ((c ^ sw) << 4));
            scale[j] = p.scale_form == kScaleHalf ? sc[half] : sc[row * 4 + c];
          }
#pragma unroll
          for (int j = 0; j < 2; ++j) fp8x16_cvt(qv[j], scale[j], *reinterpret_cast<uint32_t(*)[8]>(o + 8 * j));
        } else {
          const uint8_t* raw = stage + row * 32;
          const int sw = (row >> 2) & 1;
          const uint32_t sx = *reinterpret_cast<const unsigned short*>(stage + kRawMx + row * 2);
          const uint4 qv = *reinterpret_cast<const uint4*>(raw + ((h ^ sw) << 4));
          mx32_cvt(qv, (sx >> (8 * h)) & 0xffu, o);
        }
        // the raw bytes and scales are in registers: release the stage
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rr.idx]);
        tmem_st16(tq + static_cast<uint32_t>(ar.idx) * kAStageCols, o);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[ar.idx]);
        rr.next();
        ar.next();
      }
    }
  } else if (warp >= kWarpConv && p.wfmt != kWBf16) {
    // ------------------------------------------------ converters
    // Group g = (warp - 8) / 4 converts the CTA's k-blocks g, g + 2, ...;
    // within a k-block, lane i of warp w converts weight row 32 (w % 4) + i
    // (64 values) and stores it to TMEM lane 32 (w % 4) + i of A stage
    // g + 2 j. Raw stages g + 2 j are read back conflict-free through the
    // packing's chunk permutation.
    const int g = (warp - kWarpConv) >> 2;
    const int qw = warp & 3;
    const int row = qw * 32 + lane;
    const int half = row >> 6;                           // gate/up plane or down half
    const uint32_t tq = tmem + (static_cast<uint32_t>(qw * 32) << 16) + p.a_col0;
    int t = blockIdx.x, kb = g;
    while (kb >= p.nkb) {
      kb -= p.nkb;
      t += gridDim.x;
    }
    Ring rr(p.nr / 2), ar(p.na / 2);
    while (t < total) {
      const int rs = g + 2 * rr.idx;
      const int as = g + 2 * ar.idx;
      // polls with a short sleep: prompt when the converters run level with
      // the MMA (prefill), few issue slots taken from the MMA warps otherwise
      if (!wait_spin(&raw_full[rs], rr.phase, p.status, 32) ||
          !wait_spin(&a_empty[as], ar.phase ^ 1u, p.status, 32)) break;
      tc_fence_after();
      const uint8_t* stage = sbase + p.raw_off + rs * p.stage_bytes;
      uint32_t o[32];
      if (p.wfmt == kWFp8) {
        const uint8_t* raw = stage + row * 64;
        const float* sc = reinterpret_cast<const float*>(stage + kRawFp8);
        const int sw = (row >> 1) & 3;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 qv = *reinterpret_cast<const uint4*>(raw + ((c ^ sw) << 4));
          const float scale = p.scale_form == kScaleHalf ? sc[half] : sc[row * 4 + c];
          fp8x16_cvt(qv, scale, *reinterpret_cast<uint32_t(*)[8]>(o + 8 * c));
        }
      } else {
        const uint8_t* raw = stage + row * 32;
        const int sw = (row >> 2) & 1;
        const uint32_t sx = *reinterpret_cast<const unsigned short*>(stage + kRawMx + row * 2);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint4 qv = *reinterpret_cast<const uint4*>(raw + ((c ^ sw) << 4));
          mx32_cvt(qv, (sx >> (8 * c)) & 0xffu, *reinterpret_cast<uint32_t(*)[16]>(o + 16 * c));
        }
      }
      // the raw bytes and scales are in registers: release the stage to the TMA
      __syncwarp();
      if (lane == 0) mbar_arrive(&raw_empty[rs]);
      tmem_st32(tq + static_cast<uint32_t>(as) * kAStageCols, o);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[as]);
      rr.next();
      ar.next();
      kb += 2;
      while (kb >= p.nkb) {
        kb -= p.nkb;
        t += gridDim.x;
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
