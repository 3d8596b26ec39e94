// Ordered combine: out[t] = bf16 running sum of the token's contribution rows
// in a fixed expert order, rounding to bf16 after every add (the arithmetic
// of index_add_ on a bf16 tensor, one expert at a time). Deterministic, no
// atomics: one CTA per token, 16-byte vectors per thread.
#include "internal.h"
#include "ptx.cuh"

namespace b200 {
namespace {

constexpr int kMaxK = 32;

__global__ void __launch_bounds__(128) combine_kernel(
    const __nv_bfloat16* __restrict__ rows, long long ld_rows, const int* __restrict__ inverse,
    const long long* __restrict__ indices, int T, int K, int H, int order, int epr, int lo,
    int hi, int scale_rows, const void* __restrict__ weights, int weights_bf16,
    __nv_bfloat16* __restrict__ out, long long ld_out) {
  const int t = blockIdx.x;
  // The token's contributions in order: lane k of warp 0 reads slot k, its
  // rank among the valid slots (keys are distinct) is its position, and the
  // sorted rows and weights go to shared memory for the whole block.
  __shared__ int s_row[kMaxK];
  __shared__ float s_w[kMaxK];
  __shared__ int s_n;
  if (threadIdx.x < 32) {
    const int k = threadIdx.x;
    bool valid = false;
    long long kk = 0;
    int r = -1;
    float wv = 1.f;
    if (k < K) {
      const long long e = indices[(long long)t * K + k];
      r = inverse[(long long)t * K + k];
      valid = !(r < 0 || e < lo || e >= hi);
      kk = (order == 0) ? e * kMaxK + k : (e / epr) * kMaxK + k;
      if (valid && scale_rows)
        wv = weights_bf16
                 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(weights)[(long long)t * K + k])
                 : reinterpret_cast<const float*>(weights)[(long long)t * K + k];
    }
    const unsigned vmask = __ballot_sync(0xffffffffu, valid);
    int pos = 0;
    for (int j = 0; j < K; ++j) {
      const long long kj = __shfl_sync(0xffffffffu, kk, j);
      if (((vmask >> j) & 1u) && kj < kk) ++pos;
    }
    if (valid) {
      s_row[pos] = r;
      s_w[pos] = wv;
    }
    if (k == 0) s_n = __popc(vmask);
  }
  __syncthreads();
  const int n = s_n;
  const int nvec = H >> 3;
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    // up to 8 rows' vectors are loaded before any is added, then added in
    // the sorted order (the loads overlap; the arithmetic order is unchanged)
    for (int i0 = 0; i0 < n; i0 += 8) {
      uint4 q[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (i0 + u < n) q[u] = __ldg(reinterpret_cast<const uint4*>(rows + s_row[i0 + u] * ld_rows) + v);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (i0 + u >= n) break;
        const uint32_t wd[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float c0 = __uint_as_float(wd[j] << 16);
          float c1 = __uint_as_float(wd[j] & 0xffff0000u);
          if (scale_rows) {
            c0 = bf16r(c0 * s_w[i0 + u]);
            c1 = bf16r(c1 * s_w[i0 + u]);
          }
          acc[2 * j] = bf16r(acc[2 * j] + c0);
          acc[2 * j + 1] = bf16r(acc[2 * j + 1] + c1);
        }
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out + t * ld_out)[v] = o;
  }
}

// Slot-sum combine (order SLOT_SUM): out[t] = bf16 of torch's CUDA sum over
// the slot dimension of the [T, K, H] contributions, the local combine of the
// W8A8 path (efficient_kernels.py:269-273). A thread keeps four fp32
// accumulators per column, slot k adding into a[k % 4] in ascending k, and
// folds them as ((a0 + a1) + a2) + a3: the order in which torch's reduction
// kernel sums a strided dimension within one thread (four accumulators in
// flight). A contribution is bf16(c * bf16(w)) with scaling; slots that are
// dropped or outside [lo, hi) add +0, which leaves an fp32 sum that started
// at +0 unchanged, so they are skipped.
__global__ void __launch_bounds__(128) combine_slot_sum_kernel(
    const __nv_bfloat16* __restrict__ rows, long long ld_rows, const int* __restrict__ inverse,
    const long long* __restrict__ indices, int T, int K, int H, int lo, int hi, int scale_rows,
    const void* __restrict__ weights, int weights_bf16, __nv_bfloat16* __restrict__ out,
    long long ld_out) {
  const int t = blockIdx.x;
  __shared__ int s_row[kMaxK];
  __shared__ float s_w[kMaxK];
  if (threadIdx.x < K) {
    const int k = threadIdx.x;
    const long long e = indices[(long long)t * K + k];
    const int r = inverse[(long long)t * K + k];
    const bool valid = !(r < 0 || e < lo || e >= hi);
    float wv = 1.f;
    if (valid && scale_rows)
      wv = weights_bf16
               ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(weights)[(long long)t * K + k])
               : bf16r(reinterpret_cast<const float*>(weights)[(long long)t * K + k]);
    s_row[k] = valid ? r : -1;
    s_w[k] = wv;
  }
  __syncthreads();
  const int nvec = H >> 3;
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    float acc[4][8];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[a][j] = 0.f;
    for (int k0 = 0; k0 < K; k0 += 4) {
      uint4 q[4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
        if (k0 + a < K && s_row[k0 + a] >= 0)
          q[a] = __ldg(reinterpret_cast<const uint4*>(rows + s_row[k0 + a] * ld_rows) + v);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        if (k0 + a >= K || s_row[k0 + a] < 0) continue;
        const float w = s_w[k0 + a];
        const uint32_t wd[4] = {q[a].x, q[a].y, q[a].z, q[a].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float c0 = __uint_as_float(wd[j] << 16);
          float c1 = __uint_as_float(wd[j] & 0xffff0000u);
          if (scale_rows) {
            c0 = bf16r(__fmul_rn(c0, w));
            c1 = bf16r(__fmul_rn(c1, w));
          }
          acc[a][2 * j] = __fadd_rn(acc[a][2 * j], c0);
          acc[a][2 * j + 1] = __fadd_rn(acc[a][2 * j + 1], c1);
        }
      }
    }
    float s[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      s[j] = __fadd_rn(__fadd_rn(__fadd_rn(acc[0][j], acc[1][j]), acc[2][j]), acc[3][j]);
    uint4 o;
    o.x = pack_bf16x2(s[0], s[1]);
    o.y = pack_bf16x2(s[2], s[3]);
    o.z = pack_bf16x2(s[4], s[5]);
    o.w = pack_bf16x2(s[6], s[7]);
    reinterpret_cast<uint4*>(out + t * ld_out)[v] = o;
  }
}

// out[t] = bf16( sum over the token's slots k in order of
// fp32(bf16(rows[inverse[t*K + k]] * fp32(w[t, k]))) ), in fp32 with one
// final rounding; only experts in [lo, hi). The scatter-reduce of the fused
// MXFP4 path (matmul_ogs with gammas, efficient_kernels.py:195-205): its
// epilogue scales each (token, slot) row of acc + bias by the gamma and
// stores it in the output dtype, then a grouped reduction sums each token's
// rows in fp32.
__global__ void __launch_bounds__(128) combine_f32_kernel(
    const float* __restrict__ rows, long long ld_rows, const int* __restrict__ inverse,
    const long long* __restrict__ indices, int T, int K, int H, int lo, int hi,
    const void* __restrict__ weights, int weights_bf16, __nv_bfloat16* __restrict__ out,
    long long ld_out) {
  const int t = blockIdx.x;
  const int nvec = H >> 2;
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < K; ++k) {
      const long long e = indices[(long long)t * K + k];
      const int r = inverse[(long long)t * K + k];
      if (r < 0 || e < lo || e >= hi) continue;
      const float w = weights_bf16
                          ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(weights)[(long long)t * K + k])
                          : reinterpret_cast<const float*>(weights)[(long long)t * K + k];
      const float4 y = __ldg(reinterpret_cast<const float4*>(rows + r * ld_rows) + v);
      acc.x += bf16r(__fmul_rn(y.x, w));
      acc.y += bf16r(__fmul_rn(y.y, w));
      acc.z += bf16r(__fmul_rn(y.z, w));
      acc.w += bf16r(__fmul_rn(y.w, w));
    }
    uint2 o;
    o.x = pack_bf16x2(acc.x, acc.y);
    o.y = pack_bf16x2(acc.z, acc.w);
    reinterpret_cast<uint2*>(out + t * ld_out)[v] = o;
  }
}

__global__ void __launch_bounds__(128) gather_rows_kernel(const __nv_bfloat16* __restrict__ src,
                                                           long long ld_src,
                                                           const int* __restrict__ map, int div,
                                                           int n, int H,
                                                           __nv_bfloat16* __restrict__ dst,
                                                           long long ld_dst) {
  const int i = blockIdx.x;
  if (i >= n) return;
  const int m = map[i];
  const int nvec = H >> 3;
  uint4* b = reinterpret_cast<uint4*>(dst + i * ld_dst);
  if (m < 0) {  // a dropped assignment (inverse entry -1): zero row
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) b[v] = make_uint4(0, 0, 0, 0);
    return;
  }
  const long long s = m / div;
  const uint4* a = reinterpret_cast<const uint4*>(src + s * ld_src);
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) b[v] = __ldg(a + v);
}

// Rows [offsets[lo], offsets[hi]) of the permuted order only (the local
// experts' rows under expert parallelism), grid-strided.
__global__ void __launch_bounds__(128) gather_rows_range_kernel(
    const __nv_bfloat16* __restrict__ src, long long ld_src, const int* __restrict__ map, int div,
    int n, int H, __nv_bfloat16* __restrict__ dst, long long ld_dst, const int* __restrict__ offsets,
    int lo, int hi) {
  const int r0 = max(0, min(n, offsets[lo])), r1 = max(r0, min(n, offsets[hi]));
  const int nvec = H >> 3;
  for (int i = r0 + blockIdx.x; i < r1; i += gridDim.x) {
    const int m = map[i];
    uint4* b = reinterpret_cast<uint4*>(dst + i * ld_dst);
    if (m < 0) {
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) b[v] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const uint4* a = reinterpret_cast<const uint4*>(src + (long long)(m / div) * ld_src);
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) b[v] = __ldg(a + v);
  }
}

// The shared expert as one more routed slot of every token: slot K of row t
// is expert `shared` with weight bf16(1 / (1 + exp(-f32(logit[t])))), the
// value torch.sigmoid gives for the bf16 score logit; slots 0..K-1 copy the
// routed expert ids and their weights rounded to bf16.
__global__ void __launch_bounds__(256) append_shared_slot_kernel(
    const long long* __restrict__ indices, const void* __restrict__ weights, int weights_bf16,
    const __nv_bfloat16* __restrict__ logit, long long ld_logit, int T, int K, long long shared,
    long long* __restrict__ out_idx, __nv_bfloat16* __restrict__ out_w) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int K1 = K + 1;
  if (i >= (long long)T * K1) return;
  const long long t = i / K1;
  const int k = static_cast<int>(i - t * K1);
  if (k < K) {
    const long long j = t * K + k;
    out_idx[i] = indices[j];
    out_w[i] = weights_bf16 ? reinterpret_cast<const __nv_bfloat16*>(weights)[j]
                            : __float2bfloat16_rn(reinterpret_cast<const float*>(weights)[j]);
  } else {
    const float x = __bfloat162float(logit[t * ld_logit]);
    out_idx[i] = shared;
    out_w[i] = __float2bfloat16_rn(1.f / (1.f + expf(-x)));
  }
}

}  // namespace

cudaError_t launch_gather_rows_range(cudaStream_t st, const void* src, long long ld_src,
                                     const int* map, int div, int n, int H, void* dst,
                                     long long ld_dst, const int* offsets, int expert_lo,
                                     int expert_hi, int max_blocks) {
  if (n == 0) return cudaSuccess;
  const int blocks = n < max_blocks ? n : max_blocks;
  gather_rows_range_kernel<<<blocks, 128, 0, st>>>(static_cast<const __nv_bfloat16*>(src), ld_src,
                                                   map, div, n, H, static_cast<__nv_bfloat16*>(dst),
                                                   ld_dst, offsets, expert_lo, expert_hi);
  return cudaGetLastError();
}

cudaError_t launch_combine_f32(cudaStream_t st, const float* rows, long long ld_rows,
                               const int* inverse, const long long* indices, int T, int K, int H,
                               int lo, int hi, const void* weights, int weights_bf16, void* out,
                               long long ld_out) {
  combine_f32_kernel<<<T, 128, 0, st>>>(rows, ld_rows, inverse, indices, T, K, H, lo, hi, weights,
                                        weights_bf16, static_cast<__nv_bfloat16*>(out), ld_out);
  return cudaGetLastError();
}

cudaError_t launch_combine(cudaStream_t st, const void* rows, long long ld_rows,
                           const int* inverse, const long long* indices, int T, int K, int H,
                           int order, int experts_per_rank, int expert_lo, int expert_hi,
                           int scale_rows, const void* weights, int weights_bf16, void* out,
                           long long ld_out) {
  if (T == 0) return cudaSuccess;
  if (order == 2) {
    combine_slot_sum_kernel<<<T, 128, 0, st>>>(static_cast<const __nv_bfloat16*>(rows), ld_rows, inverse,
                                               indices, T, K, H, expert_lo, expert_hi, scale_rows, weights,
                                               weights_bf16, static_cast<__nv_bfloat16*>(out), ld_out);
    return cudaGetLastError();
  }
  combine_kernel<<<T, 128, 0, st>>>(static_cast<const __nv_bfloat16*>(rows), ld_rows, inverse,
                                    indices, T, K, H, order, experts_per_rank, expert_lo,
                                    expert_hi, scale_rows, weights, weights_bf16,
                                    static_cast<__nv_bfloat16*>(out), ld_out);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(cudaStream_t st, const void* src, long long ld_src,
                               const int* map, int div, int n, int H, void* dst,
                               long long ld_dst) {
  if (n == 0) return cudaSuccess;
  gather_rows_kernel<<<n, 128, 0, st>>>(static_cast<const __nv_bfloat16*>(src), ld_src, map,
                                        div, n, H, static_cast<__nv_bfloat16*>(dst), ld_dst);
  return cudaGetLastError();
}

cudaError_t launch_append_shared_slot(cudaStream_t st, const long long* indices, const void* weights,
                                      int weights_bf16, const void* logit, long long ld_logit, int T, int K,
                                      long long shared, long long* out_idx, void* out_w) {
  const long long n = (long long)T * (K + 1);
  if (n == 0) return cudaSuccess;
  append_shared_slot_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(
      indices, weights, weights_bf16, static_cast<const __nv_bfloat16*>(logit), ld_logit, T, K, shared, out_idx,
      static_cast<__nv_bfloat16*>(out_w));
  return cudaGetLastError();
}


}  // namespace b200

