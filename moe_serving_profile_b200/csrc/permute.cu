// Expert-contiguous permutation of the T*K routing assignments.
//
// The assignments are visited in slot-major order j = k*T + t (the order of
// torch.where(indices.T == e)) and placed with a stable counting sort by
// expert, so rows of one expert come out ordered by (slot, token).
//
// Small problems (T*K <= kSmallMax) run in one CTA. Larger ones use chunks
// of 1024 assignments: a per-chunk histogram kernel, a single-CTA scan, and a
// placement kernel that ranks equal experts inside a chunk with
// __match_any_sync plus a per-warp prefix in shared memory.
#include "b200moe.h"
#include "block_scan.cuh"
#include "internal.h"
#include "ptx.cuh"

// Chunk-histogram scratch of b200moe_permute_noalloc: one fixed array per
// device, written by the histogram kernel before the scan and placement
// kernels read it, so it never needs clearing.
static __device__ __align__(256) int g_permute_scratch[B200MOE_PERMUTE_SCRATCH_BYTES / sizeof(int)];

namespace b200 {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kChunk = 1024;
constexpr int kSmallMax = 8192;

__device__ __forceinline__ int load_expert(const long long* __restrict__ idx, int T, int K, int E,
                                           int j, int* src_out, int* inverse, int* status) {
  const int k = j / T;
  const int t = j - k * T;
  const int src = t * K + k;
  *src_out = src;
  const long long v = idx[src];
  if (v < 0 || v >= E) {
    inverse[src] = -1;
    atomicOr(status, kStatusBadIndex);
    return -1;
  }
  return static_cast<int>(v);
}

// Place the assignments j in [c0, c0 + 1024) given base[e] = first position
// of expert e's rows in this chunk. wc is shared [32][E]; tot (shared [E])
// receives the per-expert count of this chunk.
__device__ void place_chunk(const long long* __restrict__ idx, int T, int K, int E, int R, int c0,
                            const int* base, int* wc, int* tot, int* __restrict__ perm_src,
                            int* __restrict__ inverse, int* status) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 32 * E; i += blockDim.x) wc[i] = 0;
  __syncthreads();
  const int j = c0 + tid;
  int e = -1, src = -1;
  if (j < R) e = load_expert(idx, T, K, E, j, &src, inverse, status);
  const unsigned m = __match_any_sync(kFull, e);
  const int rank = __popc(m & ((1u << lane) - 1u));
  if (e >= 0 && rank == 0) wc[warp * E + e] = __popc(m);
  __syncthreads();
  for (int ee = tid; ee < E; ee += blockDim.x) {
    int s = 0;
#pragma unroll 4
    for (int w = 0; w < 32; ++w) {
      const int c = wc[w * E + ee];
      wc[w * E + ee] = s;
      s += c;
    }
    tot[ee] = s;
  }
  __syncthreads();
  if (e >= 0) {
    const int pos = base[e] + wc[warp * E + e] + rank;
    perm_src[pos] = src;
    inverse[src] = pos;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(1024) permute_small_kernel(const long long* __restrict__ idx,
                                                              int T, int K, int E,
                                                              int* __restrict__ counts,
                                                              int* __restrict__ offsets,
                                                              int* __restrict__ perm_src,
                                                              int* __restrict__ inverse,
                                                              int* status) {
  extern __shared__ int sm[];
  int* hist = sm;              // [E]
  int* run = hist + E;         // [E]
  int* tot = run + E;          // [E]
  int* scratch = tot + E;      // [40]
  int* wc = scratch + 40;      // [32 * E]
  const int R = T * K;
  const int tid = threadIdx.x;
  for (int i = tid; i < E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int j = tid; j < R; j += blockDim.x) {
    int src;
    const int e = load_expert(idx, T, K, E, j, &src, inverse, status);
    if (e >= 0) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  int total;
  const int h = tid < E ? hist[tid] : 0;
  const int ex = block_exclusive_scan(h, E, scratch, &total);
  if (tid < E) {
    counts[tid] = h;
    offsets[tid] = ex;
    run[tid] = ex;
  }
  if (tid == 0) offsets[E] = total;
  __syncthreads();
  for (int c0 = 0; c0 < R; c0 += kChunk) {
    place_chunk(idx, T, K, E, R, c0, run, wc, tot, perm_src, inverse, status);
    for (int i = tid; i < E; i += blockDim.x) run[i] += tot[i];
    __syncthreads();
  }
}

__global__ void __launch_bounds__(1024) permute_hist_kernel(const long long* __restrict__ idx,
                                                             int T, int K, int E,
                                                             int* __restrict__ chist,
                                                             int* __restrict__ inverse,
                                                             int* status) {
  extern __shared__ int sm[];
  int* hist = sm;
  const int R = T * K;
  for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int j = blockIdx.x * kChunk + threadIdx.x;
  if (j < R) {
    int src;
    const int e = load_expert(idx, T, K, E, j, &src, inverse, status);
    if (e >= 0) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x)
    chist[(long long)blockIdx.x * E + i] = hist[i];
}

// chist[c][e] -> absolute first position of expert e's rows in chunk c.
// Warp w scans the chunks of experts w, w + 32, ..., its lanes taking 32
// chunks at a time with a carry (one thread per expert walking every chunk
// serially cost 11 us at 4096 tokens x 8 slots); then one block-wide scan
// over the experts' totals, and every entry gets its expert's offset.
__global__ void __launch_bounds__(1024) permute_scan_kernel(int E, int nchunks,
                                                             int* __restrict__ chist,
                                                             int* __restrict__ counts,
                                                             int* __restrict__ offsets) {
  __shared__ int scratch[40];
  __shared__ int s_tot[1024];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = warp; e < E; e += 32) {
    int carry = 0;
    for (int c0 = 0; c0 < nchunks; c0 += 32) {
      const int c = c0 + lane;
      const int v = c < nchunks ? chist[(long long)c * E + e] : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += u;
      }
      if (c < nchunks) chist[(long long)c * E + e] = carry + incl - v;
      carry += __shfl_sync(kFull, incl, 31);
    }
    if (lane == 0) s_tot[e] = carry;
  }
  __syncthreads();
  const int s = tid < E ? s_tot[tid] : 0;
  int total;
  const int ex = block_exclusive_scan(s, E, scratch, &total);
  if (tid < E) {
    counts[tid] = s;
    offsets[tid] = ex;
    s_tot[tid] = ex;   // every thread read its total before the scan's barriers
  }
  if (tid == 0) offsets[E] = total;
  __syncthreads();
  const long long n = (long long)nchunks * E;
  for (long long i = tid; i < n; i += blockDim.x) chist[i] += s_tot[static_cast<int>(i % E)];
}

__global__ void __launch_bounds__(1024) permute_place_kernel(const long long* __restrict__ idx,
                                                              int T, int K, int E,
                                                              const int* __restrict__ chist,
                                                              int* __restrict__ perm_src,
                                                              int* __restrict__ inverse,
                                                              int* status) {
  extern __shared__ int sm[];
  int* base = sm;          // [E]
  int* tot = base + E;     // [E]
  int* wc = tot + E;       // [32 * E]
  const int R = T * K;
  for (int i = threadIdx.x; i < E; i += blockDim.x)
    base[i] = chist[(long long)blockIdx.x * E + i];
  __syncthreads();
  place_chunk(idx, T, K, E, R, blockIdx.x * kChunk, base, wc, tot, perm_src, inverse, status);
}

}  // namespace

size_t permute_workspace_bytes(int T, int K, int E) {
  const long long R = (long long)T * K;
  if (R <= kSmallMax) return 0;
  const long long nchunks = (R + kChunk - 1) / kChunk;
  return static_cast<size_t>(nchunks * E * sizeof(int));
}

cudaError_t permute_static_scratch(void** ptr) {
  return cudaGetSymbolAddress(ptr, g_permute_scratch);
}

cudaError_t launch_permute(cudaStream_t st, const long long* indices, int T, int K, int E,
                           int* counts, int* offsets, int* perm_src, int* inverse,
                           void* workspace, int* status) {
  const int R = T * K;
  if (R <= kSmallMax) {
    const size_t smem = (size_t)(3 * E + 40 + 32 * E) * sizeof(int);
    cudaError_t err = cudaFuncSetAttribute(permute_small_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    permute_small_kernel<<<1, 1024, smem, st>>>(indices, T, K, E, counts, offsets, perm_src,
                                                inverse, status);
    return cudaGetLastError();
  }
  const int nchunks = (R + kChunk - 1) / kChunk;
  int* chist = static_cast<int*>(workspace);
  permute_hist_kernel<<<nchunks, 1024, E * sizeof(int), st>>>(indices, T, K, E, chist, inverse,
                                                              status);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  permute_scan_kernel<<<1, 1024, 0, st>>>(E, nchunks, chist, counts, offsets);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  const size_t smem = (size_t)(2 * E + 32 * E) * sizeof(int);
  err = cudaFuncSetAttribute(permute_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  permute_place_kernel<<<nchunks, 1024, smem, st>>>(indices, T, K, E, chist, perm_src, inverse,
                                                    status);
  return cudaGetLastError();
}

}  // namespace b200
