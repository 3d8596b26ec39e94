// Router: logits on CUDA cores in a fixed fp32 summation order, then a
// warp-per-token softmax / top-k / count kernel.
//
// Fixed order of every dot product x[t,:] . w[e,:] (H a multiple of 8):
//   segment s covers h in [64 s, min(64 s + 64, H)) and is one fmaf chain in
//   increasing h starting from 0 (bf16 x bf16 products are exact in fp32);
//   the segments are added in increasing s: ((seg0 + seg1) + seg2) + ...
// The order does not depend on T, the batch composition or the launch shape,
// so a token is routed identically in every batch and on every EP rank.
//   router_logits_warp_kernel   small batches: one warp per (1 token, 2
//                               experts), or (4 tokens, 8 experts) from 64
//                               tokens on; lane l runs segments l, l + 32,
//                               ..., folded in order through shared memory
//   router_logits_tile_kernel   larger batches: blocks of tokens x experts; four
//                               segments run side by side on four thread
//                               groups, their sums are folded in order
#include "internal.h"
#include "ptx.cuh"

namespace b200 {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kSeg = 64;            // elements per segment
constexpr int kMaxSegPerLane = 4;   // H <= 32 * 4 * 64 = 8192

enum RouterMode { kQwen3 = 0, kGptOss = 1, kNative = 2 };

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ void store_logit(void* logits, const __nv_bfloat16* bias, int mode, int t,
                                            int e, int E, float v) {
  if (mode == kNative) {
    reinterpret_cast<float*>(logits)[(long long)t * E + e] = v;
  } else {
    if (bias != nullptr) v += __bfloat162float(bias[e]);
    reinterpret_cast<__nv_bfloat16*>(logits)[(long long)t * E + e] = __float2bfloat16_rn(v);
  }
}

// One warp per (TT tokens, TE experts). Lane l runs segment 32 r + l of
// every output in round r; the round's sums go through shared memory and lane
// o < TT * TE folds output o's sums into its running dot in increasing order.
template <int TT, int TE>
__global__ void __launch_bounds__(256) router_logits_warp_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ bias, int T, int H, int E, int mode, void* logits) {
  constexpr int NO = TT * TE;   // outputs per warp (<= 32)
  static_assert(NO <= 32, "one output per lane");
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int n_et = (E + TE - 1) / TE;
  const int t0 = (gw / n_et) * TT;
  const int e0 = (gw % n_et) * TE;
  if (t0 >= T) return;
  const int nseg = (H + kSeg - 1) / kSeg;
  __shared__ float fold[8][NO][33];   // [warp][output][segment of the round], skewed rows
  float (*fw)[33] = fold[threadIdx.x >> 5];
  const __nv_bfloat16* xr[TT];
  const __nv_bfloat16* wr[TE];
#pragma unroll
  for (int a = 0; a < TT; ++a) xr[a] = x + min(t0 + a, T - 1) * ldx;   // rows past T / E repeat
#pragma unroll
  for (int b = 0; b < TE; ++b) wr[b] = w + (long long)min(e0 + b, E - 1) * H;   // the last (unused)
  float dot = 0.f;
  for (int r = 0; r < kMaxSegPerLane && 32 * r < nseg; ++r) {
    const int s = 32 * r + lane;
    float seg[TT][TE];
#pragma unroll
    for (int a = 0; a < TT; ++a)
#pragma unroll
      for (int b = 0; b < TE; ++b) seg[a][b] = 0.f;
    auto vec8 = [&](int h) {   // 8 columns h .. h + 7 into every chain
      float xf[TT][8];
#pragma unroll
      for (int a = 0; a < TT; ++a) bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(xr[a] + h)), xf[a]);
#pragma unroll
      for (int b = 0; b < TE; ++b) {
        float wf[8];
        bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(wr[b] + h)), wf);
#pragma unroll
        for (int a = 0; a < TT; ++a)
#pragma unroll
          for (int j = 0; j < 8; ++j) seg[a][b] = fmaf(xf[a][j], wf[j], seg[a][b]);
      }
    };
    if (s < nseg) {
      const int h0 = s * kSeg, len = min(kSeg, H - h0);
      if (len == kSeg) {
#pragma unroll(NO <= 4 ? 8 : 2)
        for (int v = 0; v < 8; ++v) vec8(h0 + 8 * v);
      } else {
        for (int v = 0; v < len / 8; ++v) vec8(h0 + 8 * v);
      }
    }
#pragma unroll
    for (int a = 0; a < TT; ++a)
#pragma unroll
      for (int b = 0; b < TE; ++b) fw[a * TE + b][lane] = seg[a][b];
    __syncwarp();
    if (lane < NO) {
      const int ns = min(32, nseg - 32 * r);
      for (int q = 0; q < ns; ++q) dot = (r == 0 && q == 0) ? fw[lane][q] : dot + fw[lane][q];
    }
    __syncwarp();
  }
  if (lane < NO) {
    const int t = t0 + lane / TE, e = e0 + lane % TE;
    if (t < T && e < E) store_logit(logits, bias, mode, t, e, E, dot);
  }
}

// Tiled logits for larger batches. A block of 512 threads computes TB = 8 TI
// tokens x EB = 16 EJ experts. H is walked in rounds of four segments
// (256 columns): thread group g = tid / 128 runs segment 4 r + g of round r
// for TI x EJ outputs (thread (tg, eg) = (tid % 128 / 16, tid % 16): tokens
// TI tg .. + TI - 1, experts eg + 16 j), the segment sums go through shared
// memory, and the owner of each output folds the round's sums into its
// running dot in increasing segment order. Each round's x columns are staged
// as fp32 in rows padded to 260 floats, so the rows a warp reads together
// fall in distinct banks.
template <int TI, int EJ>
struct TileShape {
  static constexpr int TB = 8 * TI, EB = 16 * EJ;
  static constexpr int kRow = 260;                     // fp32 row stride: 256 + 4 (bank skew)
  static constexpr int kXBytes = TB * kRow * 4;        // x: [TB][260] fp32
  static constexpr int kWBytes = EB * kRow * 4;        // w: [EB][260] fp32
  static constexpr int kFBytes = 4 * TB * EB * 4;      // segment sums: [4][TB][EB] fp32
  static constexpr int kSmem = kXBytes + kWBytes + kFBytes;
  static constexpr int XV = (TB * 32 + 511) / 512, WV = (EB * 32 + 511) / 512;   // staged vectors / thread
};

template <int TI, int EJ>
__global__ void __launch_bounds__(512, 1) router_logits_tile_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ bias, int T, int H, int E, int mode, void* logits) {
  using S = TileShape<TI, EJ>;
  constexpr int TB = S::TB, EB = S::EB;
  extern __shared__ __align__(16) uint8_t router_smem[];
  float* xs = reinterpret_cast<float*>(router_smem);
  float* ws = reinterpret_cast<float*>(router_smem + S::kXBytes);
  float* fb = reinterpret_cast<float*>(router_smem + S::kXBytes + S::kWBytes);
  const int tid = threadIdx.x;
  const int g = tid >> 7, tg = (tid & 127) >> 4, eg = tid & 15;
  const int t0 = blockIdx.x * TB, e0 = blockIdx.y * EB;
  const int nseg = (H + kSeg - 1) / kSeg;
  const int rounds = (nseg + 3) / 4;

  uint4 xq[S::XV], wq[S::WV];
  auto fetch = [&](int r) {
#pragma unroll
    for (int i = 0; i < S::XV; ++i) {
      const int vi = tid + 512 * i, row = vi >> 5, h = 256 * r + 8 * (vi & 31);
      xq[i] = make_uint4(0, 0, 0, 0);
      if (vi < TB * 32 && t0 + row < T && h < H)
        xq[i] = __ldg(reinterpret_cast<const uint4*>(x + (t0 + row) * ldx + h));
    }
#pragma unroll
    for (int i = 0; i < S::WV; ++i) {
      const int vi = tid + 512 * i, row = vi >> 5, h = 256 * r + 8 * (vi & 31);
      wq[i] = make_uint4(0, 0, 0, 0);
      if (vi < EB * 32 && e0 + row < E && h < H)
        wq[i] = __ldg(reinterpret_cast<const uint4*>(w + (long long)(e0 + row) * H + h));
    }
  };
  // rows of 256 fp32 at a stride of 260: the 4-float skew per row puts the
  // rows a warp reads together (two token rows, 16 expert rows) in distinct
  // banks, and every read is a per-thread base plus a constant offset
  auto put_row = [](float* base, int row, int v, const uint4& q) {
    float f[8];
    bf16x8_to_f32(q, f);
    float4* rr = reinterpret_cast<float4*>(base + row * S::kRow + 8 * v);
    rr[0] = make_float4(f[0], f[1], f[2], f[3]);
    rr[1] = make_float4(f[4], f[5], f[6], f[7]);
  };
  auto put = [&]() {
#pragma unroll
    for (int i = 0; i < S::XV; ++i) {
      const int vi = tid + 512 * i;
      if (vi < TB * 32) put_row(xs, vi >> 5, vi & 31, xq[i]);
    }
#pragma unroll
    for (int i = 0; i < S::WV; ++i) {
      const int vi = tid + 512 * i;
      if (vi < EB * 32) put_row(ws, vi >> 5, vi & 31, wq[i]);
    }
  };
  const float* xb = xs + (TI * tg) * S::kRow + 64 * g;   // this thread's token rows, segment g
  const float* wb = ws + eg * S::kRow + 64 * g;           // this thread's expert rows, segment g
  // one 8-column chunk c of the thread's segment into the TI x EJ chains
  auto chunk8 = [&](int c, float (&seg)[TI][EJ]) {
    float xv[TI][8];
#pragma unroll
    for (int i = 0; i < TI; ++i) {
      const float4* xr = reinterpret_cast<const float4*>(xb + i * S::kRow + 8 * c);
      const float4 lo = xr[0], hi = xr[1];
      xv[i][0] = lo.x; xv[i][1] = lo.y; xv[i][2] = lo.z; xv[i][3] = lo.w;
      xv[i][4] = hi.x; xv[i][5] = hi.y; xv[i][6] = hi.z; xv[i][7] = hi.w;
    }
#pragma unroll
    for (int j = 0; j < EJ; ++j) {
      const float4* wr = reinterpret_cast<const float4*>(wb + 16 * j * S::kRow + 8 * c);
      const float4 lo = wr[0], hi = wr[1];
      const float wf[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
      for (int i = 0; i < TI; ++i)
#pragma unroll
        for (int k = 0; k < 8; ++k) seg[i][j] = fmaf(xv[i][k], wf[k], seg[i][j]);
    }
  };

  constexpr int kOwn = (TB * EB + 511) / 512;
  float dot[kOwn];
  fetch(0);
  for (int r = 0; r < rounds; ++r) {
    put();
    __syncthreads();   // staging visible; the previous round's fold is done
    if (r + 1 < rounds) fetch(r + 1);   // in flight during this round's chains
    const int s = 4 * r + g;
    if (s < nseg) {
      const int len = min(kSeg, H - s * kSeg);
      float seg[TI][EJ];
#pragma unroll
      for (int i = 0; i < TI; ++i)
#pragma unroll
        for (int j = 0; j < EJ; ++j) seg[i][j] = 0.f;
      if (len == kSeg) {
#pragma unroll
        for (int c = 0; c < 8; ++c) chunk8(c, seg);
      } else {
        for (int c = 0; c < len / 8; ++c) chunk8(c, seg);
      }
#pragma unroll
      for (int i = 0; i < TI; ++i)
#pragma unroll
        for (int j = 0; j < EJ; ++j) fb[(g * TB + TI * tg + i) * EB + eg + 16 * j] = seg[i][j];
    }
    __syncthreads();
    // fold this round's segments, in increasing order, into the owned outputs
    const int ns = min(4, nseg - 4 * r);
#pragma unroll
    for (int k = 0; k < kOwn; ++k) {
      const int o = tid + 512 * k;
      if (o >= TB * EB) continue;
      for (int q = 0; q < ns; ++q) {
        const float v = fb[q * TB * EB + o];
        dot[k] = (r == 0 && q == 0) ? v : dot[k] + v;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kOwn; ++k) {
    const int o = tid + 512 * k;
    const int t = t0 + o / EB, e = e0 + o % EB;
    if (o < TB * EB && t < T && e < E) store_logit(logits, bias, mode, t, e, E, dot[k]);
  }
}

template <int TI, int EJ>
cudaError_t launch_tile(cudaStream_t st, const __nv_bfloat16* x, long long ldx, const __nv_bfloat16* w,
                        const __nv_bfloat16* b, int T, int H, int E, int mode, void* logits) {
  using S = TileShape<TI, EJ>;
  // the shared-memory opt-in is per device; callers set the same value, so a
  // race between two threads only repeats the call
  static bool attr[64] = {};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    err = cudaFuncSetAttribute(router_logits_tile_kernel<TI, EJ>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem);
    if (err != cudaSuccess) return err;
    attr[dev] = true;
  }
  const dim3 grid((T + S::TB - 1) / S::TB, (E + S::EB - 1) / S::EB);
  router_logits_tile_kernel<TI, EJ><<<grid, 512, S::kSmem, st>>>(x, ldx, w, b, T, H, E, mode, logits);
  return cudaGetLastError();
}

// Monotone map float -> uint32 (NaN sorts above everything, as torch.topk).
__device__ __forceinline__ uint32_t order_key(float f) {
  if (f != f) return 0xffffffffu;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// torch's descending comparator: a NaN is larger than any number.
__device__ __forceinline__ bool gt_nan(float a, float b) {
  return (a != a && b == b) || a > b;
}

constexpr int kMaxPerLane = 16;  // E <= 512

// Sum over lanes 0 .. K-1 (lanes K .. P-1 contribute 0, P = the power of two
// >= K) by xor-butterfly: lane 0 gets ((v0 + v4) + (v2 + v6)) + ((v1 + v5) +
// (v3 + v7)) at K = 8. This is the order of torch's CUDA sum over a row of K
// values and of the warp reduction of its softmax over K values.
__device__ __forceinline__ float butterfly_sum(float v, int K) {
  int p = 1;
  while (p < K) p <<= 1;
  for (int o = p >> 1; o >= 1; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// One warp per token. The selection reproduces torch.topk on CUDA for
// k <= 32 bit for bit, including the slot order of equal values:
//   1. the k selected experts are those with a key above the k-th largest
//      key, plus the lowest-index experts whose key equals it;
//   2. they are laid out in index order, the above-the-k-th ones first, in
//      32 slots (slots k .. 31 invalid);
//   3. a 32-slot bitonic sorting network orders them: comparator (a, b) with
//      a at the lower slot swaps when "not (a valid and a > b) and b valid"
//      equals the stage's direction, so equal keys are exchanged whenever the
//      direction is ascending (the final merge is descending throughout).
// Keys: the fp32 softmax probabilities (QWEN3, NATIVE; the softmax is
// torch's warp softmax: lane-sequential sums over e = lane + 32 i, then a
// xor-butterfly across lanes, probs = exp(x - max) / sum) or the bf16 logits
// (GPT_OSS). Sums over the k selected values use butterfly_sum.
// NL: keys per lane (experts e = lane + 32 i, i < NL), the smallest of 1, 4, 8,
// 16 that covers E: entries past E are -inf and change no sum or selection,
// so every NL gives the same result; with 16 for every E, the loops of a
// 128-expert router ran four times the entries they needed.
template <int NL>
__global__ void __launch_bounds__(256) router_select_kernel(const void* __restrict__ logits,
                                                             int T, int E, int K, int mode,
                                                             int normalize, float* probs,
                                                             void* scores,
                                                             long long* __restrict__ indices,
                                                             int* counts) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;

  float key[NL];
#pragma unroll
  for (int i = 0; i < NL; ++i) {
    const int e = lane + 32 * i;
    float v = -INFINITY;
    if (e < E) {
      if (mode == kNative)
        v = reinterpret_cast<const float*>(logits)[(long long)t * E + e];
      else
        v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(logits)[(long long)t * E + e]);
    }
    key[i] = v;
  }

  if (mode != kGptOss) {
    // ---- softmax over all E (fp32): the keys become the probabilities
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < NL; ++i) mx = fmaxf(mx, key[i]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
    float lsum = 0.f;
#pragma unroll
    for (int i = 0; i < NL; ++i) {
      key[i] = (lane + 32 * i < E) ? expf(key[i] - mx) : 0.f;
      lsum += key[i];
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) lsum += __shfl_xor_sync(kFull, lsum, o);
#pragma unroll
    for (int i = 0; i < NL; ++i) {
      const int e = lane + 32 * i;
      key[i] = key[i] / lsum;
      if (mode == kQwen3 && probs != nullptr && e < E) probs[(long long)t * E + e] = key[i];
    }
  }

  // ---- 1. the selected set: K rounds of (key descending, index ascending)
  uint32_t taken = 0;
  int sidx = -1;        // lane k < K: the k-th selected expert
  float skey = 0.f;
  for (int k = 0; k < K; ++k) {
    unsigned long long best = 0ull;
#pragma unroll
    for (int i = 0; i < NL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !((taken >> i) & 1u)) {
        const unsigned long long c =
            (static_cast<unsigned long long>(order_key(key[i])) << 32) | (0xffffffffu - e);
        best = c > best ? c : best;
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(kFull, best, o);
      best = other > best ? other : best;
    }
    const int e_sel = static_cast<int>(0xffffffffu - static_cast<uint32_t>(best));
    if ((e_sel & 31) == lane) taken |= 1u << (e_sel >> 5);
    float vsel = 0.f;
#pragma unroll
    for (int i = 0; i < NL; ++i)
      if (lane + 32 * i == e_sel) vsel = key[i];
    vsel = __shfl_sync(kFull, vsel, e_sel & 31);
    if (lane == k) {
      sidx = e_sel;
      skey = vsel;
    }
  }

  // ---- 2. index order, keys above the k-th first
  const float kth = __shfl_sync(kFull, skey, K - 1);
  const int grp = lane < K ? (order_key(skey) > order_key(kth) ? 0 : 1) : 2;
  int pos = 0;
  for (int j = 0; j < K; ++j) {
    const int gj = __shfl_sync(kFull, grp, j);
    const int ij = __shfl_sync(kFull, sidx, j);
    if (lane < K && (gj < grp || (gj == grp && ij < sidx))) ++pos;
  }
  float okey = 0.f;
  int oidx = -1;
  for (int j = 0; j < K; ++j) {
    const int pj = __shfl_sync(kFull, pos, j);
    const float kj = __shfl_sync(kFull, skey, j);
    const int ij = __shfl_sync(kFull, sidx, j);
    if (lane == pj) {
      okey = kj;
      oidx = ij;
    }
  }
  bool valid = lane < K;

  // ---- 3. the 32-slot bitonic network (lane = slot)
  auto step = [&](int stride, bool dir) {
    const float pk = __shfl_xor_sync(kFull, okey, stride);
    const int pi = __shfl_xor_sync(kFull, oidx, stride);
    const bool pv = __shfl_xor_sync(kFull, valid ? 1 : 0, stride) != 0;
    const bool is_a = (lane & stride) == 0;
    const float ka = is_a ? okey : pk, kb = is_a ? pk : okey;
    const bool va = is_a ? valid : pv, vb = is_a ? pv : valid;
    const bool swap = (gt_nan(ka, kb) && va) || !vb;
    if (swap == dir) {
      okey = pk;
      oidx = pi;
      valid = pv;
    }
  };
#pragma unroll
  for (int size = 2; size < 32; size <<= 1)
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) step(stride, (lane & size) != 0);
#pragma unroll
  for (int stride = 16; stride > 0; stride >>= 1) step(stride, false);

  // lanes 0 .. K-1 now hold the slots in torch's order
  const bool mine = lane < K;
  if (mode == kGptOss) {
    // softmax over the k selected bf16 logits (fp32 arithmetic, bf16 result)
    const float top = __shfl_sync(kFull, okey, 0);
    const float ex = mine ? expf(okey - top) : 0.f;
    const float s = __shfl_sync(kFull, butterfly_sum(ex, K), 0);
    if (mine) reinterpret_cast<__nv_bfloat16*>(scores)[(long long)t * K + lane] = __float2bfloat16_rn(ex / s);
  } else {
    const float p = mine ? okey : 0.f;
    float wv = p;
    if (normalize) {
      float s = __shfl_sync(kFull, butterfly_sum(p, K), 0);
      if (mode == kNative) s = fmaxf(s, 1e-20f);
      wv = p / s;
    }
    if (mine) {
      if (mode == kQwen3)
        reinterpret_cast<float*>(scores)[(long long)t * K + lane] = wv;
      else
        reinterpret_cast<__nv_bfloat16*>(scores)[(long long)t * K + lane] = __float2bfloat16_rn(wv);
    }
  }
  if (mine) {
    indices[(long long)t * K + lane] = oidx;
    if (counts && oidx >= 0 && oidx < E) atomicAdd(&counts[oidx], 1);
  }
}

// Compact routing record: int64 expert ids -> int16, fp32 / bf16 weights ->
// fp16 (round to nearest even), 4 assignments per thread.
__global__ void __launch_bounds__(256) route_record_kernel(const long long* __restrict__ indices,
                                                           const void* __restrict__ scores,
                                                           int scores_bf16, long long n,
                                                           int16_t* __restrict__ out_idx,
                                                           __half* __restrict__ out_scores) {
  const long long i0 = 4ll * ((long long)blockIdx.x * blockDim.x + threadIdx.x);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const long long i = i0 + u;
    if (i >= n) return;
    out_idx[i] = static_cast<int16_t>(indices[i]);
    const float w = scores_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(scores)[i])
                                : reinterpret_cast<const float*>(scores)[i];
    out_scores[i] = __float2half_rn(w);
  }
}

}  // namespace

cudaError_t launch_router_logits(cudaStream_t st, int mode, const void* hidden, long long ldx,
                                 const void* weight, const void* bias, int T, int H, int E,
                                 void* logits) {
  if (T == 0) return cudaSuccess;
  const auto* x = static_cast<const __nv_bfloat16*>(hidden);
  const auto* w = static_cast<const __nv_bfloat16*>(weight);
  const auto* b = static_cast<const __nv_bfloat16*>(bias);
  // launch shapes measured on B200 (qwen3: E = 128, H = 2048; gpt-oss:
  // E = 32, H = 2880); every shape computes the same fixed order
  if (E > 32) {
    if (T >= 2048) return launch_tile<4, 4>(st, x, ldx, w, b, T, H, E, mode, logits);
    if (T >= 1024) return launch_tile<2, 4>(st, x, ldx, w, b, T, H, E, mode, logits);
    if (T >= 256) return launch_tile<2, 2>(st, x, ldx, w, b, T, H, E, mode, logits);
  } else {
    if (T >= 4096) return launch_tile<4, 2>(st, x, ldx, w, b, T, H, E, mode, logits);
    if (T >= 1536) return launch_tile<2, 2>(st, x, ldx, w, b, T, H, E, mode, logits);
  }
  if (T >= 64) {
    constexpr int TT = 4, TE = 8;   // the router weight is read once per 4 tokens
    const long long warps = (long long)((T + TT - 1) / TT) * ((E + TE - 1) / TE);
    router_logits_warp_kernel<TT, TE><<<static_cast<int>((warps + 7) / 8), 256, 0, st>>>(
        x, ldx, w, b, T, H, E, mode, logits);
  } else {
    // two warps per block spread a handful of tokens over many SMs
    constexpr int TT = 1, TE = 2;
    const long long warps = (long long)T * ((E + TE - 1) / TE);
    router_logits_warp_kernel<TT, TE><<<static_cast<int>((warps + 1) / 2), 64, 0, st>>>(
        x, ldx, w, b, T, H, E, mode, logits);
  }
  return cudaGetLastError();
}

cudaError_t launch_router_select(cudaStream_t st, int mode, const void* logits, int T, int E,
                                 int K, int normalize, void* probs, void* scores,
                                 long long* indices, int* counts) {
  if (T == 0) return cudaSuccess;
  const int blocks = (T + 7) / 8;
#define B200_SELECT(NL_)                                                                           \
  router_select_kernel<NL_><<<blocks, 256, 0, st>>>(logits, T, E, K, mode, normalize,           \
                                                    static_cast<float*>(probs), scores, indices, counts)
  if (E <= 32) B200_SELECT(1);
  else if (E <= 128) B200_SELECT(4);
  else if (E <= 256) B200_SELECT(8);
  else B200_SELECT(kMaxPerLane);
#undef B200_SELECT
  return cudaGetLastError();
}

cudaError_t launch_route_record(cudaStream_t st, const long long* indices, const void* scores,
                                int scores_bf16, long long n, void* out_idx, void* out_scores) {
  if (n == 0) return cudaSuccess;
  const long long threads = (n + 3) / 4;
  route_record_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, st>>>(
      indices, scores, scores_bf16, n, static_cast<int16_t*>(out_idx), static_cast<__half*>(out_scores));
  return cudaGetLastError();
}

}  // namespace b200
