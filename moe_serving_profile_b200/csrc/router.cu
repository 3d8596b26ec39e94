// Router: logits GEMV/GEMM on CUDA cores in a fixed fp32 summation order,
// then a warp-per-token softmax / top-k / count kernel.
//
// Fixed order of every dot product x[t,:] . w[e,:] (H a multiple of 8):
//   vector v = h / 8 belongs to partial p = v % 32; each partial accumulates
//   its vectors in increasing v, and inside a vector its 8 products in
//   increasing h, with fmaf (bf16 x bf16 products are exact in fp32);
//   the 32 partials are then combined pairwise: p[i] += p[i ^ o] for
//   o = 16, 8, 4, 2, 1 (all lanes end with the same value).
// The order does not depend on T, the batch composition or the launch shape,
// so a token is routed identically in every batch and on every EP rank.
#include "internal.h"
#include "ptx.cuh"

namespace b200 {
namespace {

constexpr unsigned kFull = 0xffffffffu;

enum RouterMode { kQwen3 = 0, kGptOss = 1, kNative = 2 };

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// One warp computes TT tokens x TE experts.
template <int TT, int TE>
__global__ void __launch_bounds__(256) router_logits_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ bias, int T, int H, int E, int mode, void* logits) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int n_et = (E + TE - 1) / TE;
  const int t0 = (gw / n_et) * TT;
  const int e0 = (gw % n_et) * TE;
  if (t0 >= T) return;

  float acc[TT][TE];
#pragma unroll
  for (int a = 0; a < TT; ++a)
#pragma unroll
    for (int b = 0; b < TE; ++b) acc[a][b] = 0.f;

  const int nvec = H >> 3;
  for (int v = lane; v < nvec; v += 32) {
    float xf[TT][8];
#pragma unroll
    for (int a = 0; a < TT; ++a) {
      uint4 q = make_uint4(0, 0, 0, 0);
      if (t0 + a < T) q = __ldg(reinterpret_cast<const uint4*>(x + (t0 + a) * ldx) + v);
      bf16x8_to_f32(q, xf[a]);
    }
#pragma unroll
    for (int b = 0; b < TE; ++b) {
      uint4 q = make_uint4(0, 0, 0, 0);
      if (e0 + b < E) q = __ldg(reinterpret_cast<const uint4*>(w + (long long)(e0 + b) * H) + v);
      float wf[8];
      bf16x8_to_f32(q, wf);
#pragma unroll
      for (int a = 0; a < TT; ++a)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[a][b] = fmaf(xf[a][j], wf[j], acc[a][b]);
    }
  }
#pragma unroll
  for (int a = 0; a < TT; ++a)
#pragma unroll
    for (int b = 0; b < TE; ++b)
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) acc[a][b] += __shfl_xor_sync(kFull, acc[a][b], o);

  // Lane l writes output l (TT * TE <= 32).
#pragma unroll
  for (int a = 0; a < TT; ++a)
#pragma unroll
    for (int b = 0; b < TE; ++b) {
      if (lane != a * TE + b) continue;
      const int t = t0 + a, e = e0 + b;
      if (t >= T || e >= E) continue;
      float vsum = acc[a][b];
      if (mode == kNative) {
        reinterpret_cast<float*>(logits)[(long long)t * E + e] = vsum;
      } else {
        if (bias != nullptr) vsum += __bfloat162float(bias[e]);
        reinterpret_cast<__nv_bfloat16*>(logits)[(long long)t * E + e] = __float2bfloat16_rn(vsum);
      }
    }
}

// Monotone map float -> uint32 (NaN sorts above everything, as torch.topk).
__device__ __forceinline__ uint32_t order_key(float f) {
  if (f != f) return 0xffffffffu;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

constexpr int kMaxPerLane = 16;  // E <= 512

// One warp per token.
__global__ void __launch_bounds__(256) router_select_kernel(const void* __restrict__ logits,
                                                             int T, int E, int K, int mode,
                                                             int normalize, float* probs,
                                                             void* scores,
                                                             long long* __restrict__ indices,
                                                             int* counts) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;

  float val[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int e = lane + 32 * i;
    float v = -INFINITY;
    if (e < E) {
      if (mode == kNative)
        v = reinterpret_cast<const float*>(logits)[(long long)t * E + e];
      else
        v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(logits)[(long long)t * E + e]);
    }
    val[i] = v;
  }

  // ---- top-k on the logits: value descending, ties by ascending expert id.
  uint32_t taken = 0;
  int my_idx = -1;      // lane k < K holds slot k
  float my_val = 0.f;
  for (int k = 0; k < K; ++k) {
    unsigned long long best = 0ull;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !((taken >> i) & 1u)) {
        const unsigned long long c =
            (static_cast<unsigned long long>(order_key(val[i])) << 32) | (0xffffffffu - e);
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
    // the selected value, recovered from the winning lane
    float vsel = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i)
      if (lane + 32 * i == e_sel) vsel = val[i];
    vsel = __shfl_sync(kFull, vsel, e_sel & 31);
    if (lane == k) {
      my_idx = e_sel;
      my_val = vsel;
    }
  }
  const float top = __shfl_sync(kFull, my_val, 0);

  if (mode == kGptOss) {
    // softmax over the k selected bf16 logits, result rounded to bf16
    const float ex = (lane < K) ? expf(my_val - top) : 0.f;
    float s = 0.f;
    for (int k = 0; k < K; ++k) s += __shfl_sync(kFull, ex, k);
    if (lane < K) {
      reinterpret_cast<__nv_bfloat16*>(scores)[(long long)t * K + lane] = __float2bfloat16_rn(ex / s);
      indices[(long long)t * K + lane] = my_idx;
      if (counts) atomicAdd(&counts[my_idx], 1);
    }
    return;
  }

  // ---- softmax over all E (fp32); QWEN3 writes the probabilities
  float lsum = 0.f;
  float ex[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    ex[i] = (lane + 32 * i < E) ? expf(val[i] - top) : 0.f;
    lsum += ex[i];
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) lsum += __shfl_xor_sync(kFull, lsum, o);
  if (mode == kQwen3 && probs != nullptr) {
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int e = lane + 32 * i;
      if (e < E) probs[(long long)t * E + e] = ex[i] / lsum;
    }
  }
  // probability of my slot
  float psel = 0.f;
  for (int k = 0; k < K; ++k) {
    const int e = __shfl_sync(kFull, my_idx, k);
    float pe = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i)
      if (lane + 32 * i == e) pe = ex[i] / lsum;
    pe = __shfl_sync(kFull, pe, e & 31);
    if (lane == k) psel = pe;
  }
  float denom = 1.f;
  if (normalize) {
    float s = 0.f;
    for (int k = 0; k < K; ++k) s += __shfl_sync(kFull, psel, k);
    denom = (mode == kNative) ? fmaxf(s, 1e-20f) : s;
  }
  if (lane < K) {
    const float wv = normalize ? psel / denom : psel;
    if (mode == kQwen3)
      reinterpret_cast<float*>(scores)[(long long)t * K + lane] = wv;
    else
      reinterpret_cast<__nv_bfloat16*>(scores)[(long long)t * K + lane] = __float2bfloat16_rn(wv);
    indices[(long long)t * K + lane] = my_idx;
    if (counts) atomicAdd(&counts[my_idx], 1);
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
  if (T >= 64) {
    constexpr int TT = 4, TE = 8;
    const long long warps = (long long)((T + TT - 1) / TT) * ((E + TE - 1) / TE);
    const int blocks = static_cast<int>((warps + 7) / 8);
    router_logits_kernel<TT, TE><<<blocks, 256, 0, st>>>(x, ldx, w, b, T, H, E, mode, logits);
  } else {
    constexpr int TT = 1, TE = 4;
    const long long warps = (long long)T * ((E + TE - 1) / TE);
    const int blocks = static_cast<int>((warps + 7) / 8);
    router_logits_kernel<TT, TE><<<blocks, 256, 0, st>>>(x, ldx, w, b, T, H, E, mode, logits);
  }
  return cudaGetLastError();
}

cudaError_t launch_router_select(cudaStream_t st, int mode, const void* logits, int T, int E,
                                 int K, int normalize, void* probs, void* scores,
                                 long long* indices, int* counts) {
  if (T == 0) return cudaSuccess;
  const int blocks = (T + 7) / 8;
  router_select_kernel<<<blocks, 256, 0, st>>>(logits, T, E, K, mode, normalize,
                                               static_cast<float*>(probs), scores, indices,
                                               counts);
  return cudaGetLastError();
}

}  // namespace b200
