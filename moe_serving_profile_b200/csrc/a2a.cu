// Receive-side plan of the token all-to-all (moe_serving/moe.py:110-137).
//
// After the dispatch exchange a rank holds its rows grouped by source rank
// and, inside one source, by local expert (each sender's expert-major
// permutation is already destination-major because a rank's experts are a
// contiguous id range). The grouped GEMM wants each local expert's rows
// contiguous, so this kernel builds the transposition of the
// [source][expert] segments into [expert][source] order:
//   offsets[e]      first expert-major position of local expert e
//   map_in[p]       arrival row at expert-major position p
//   map_back[j]     expert-major position of arrival row j
// Inside one expert the sources stay ascending and each source's rows keep
// their arrival order.
//
// Every CTA rebuilds the segment bases (at most 1024 segments) in shared
// memory and then maps a grid-stride share of the rows; one launch, no
// workspace.
#include "block_scan.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace b200 {
namespace {

constexpr int kMaxSegments = 1024;

__global__ void __launch_bounds__(1024) a2a_recv_plan_kernel(const int* __restrict__ counts,
                                                              int ep, int el, int rows,
                                                              int* __restrict__ offsets,
                                                              int* __restrict__ map_in,
                                                              int* __restrict__ map_back,
                                                              int* status) {
  __shared__ int arr_base[kMaxSegments];  // [s * el + e]: first arrival row of segment
  __shared__ int em_base[kMaxSegments];   // [s * el + e]: first expert-major position
  __shared__ int scratch[40];
  const int n = ep * el;
  const int tid = threadIdx.x;
  // arrival order: segments in (source, expert) order
  const int c_arr = tid < n ? counts[tid] : 0;
  int total_arr;
  const int ex_arr = block_exclusive_scan(c_arr, n, scratch, &total_arr);
  if (tid < n) arr_base[tid] = ex_arr;
  // expert-major order: thread tid takes segment (e, s) with tid = e * ep + s
  int c_em = 0, seg = 0;
  if (tid < n) {
    const int e = tid / ep, s = tid - e * ep;
    seg = s * el + e;
    c_em = counts[seg];
  }
  int total_em;
  const int ex_em = block_exclusive_scan(c_em, n, scratch, &total_em);
  if (tid < n) {
    em_base[seg] = ex_em;
    if (blockIdx.x == 0 && tid % ep == 0) offsets[tid / ep] = ex_em;
  }
  if (blockIdx.x == 0 && tid == 0) {
    offsets[el] = total_em;
    if (total_em != rows) atomicOr(status, kStatusBadTile);
  }
  __syncthreads();
  for (int j = blockIdx.x * blockDim.x + tid; j < rows; j += gridDim.x * blockDim.x) {
    // largest segment g with arr_base[g] <= j (later empty segments share the
    // base of the next non-empty one, so the largest such g holds row j)
    int lo = 0, hi = n - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (arr_base[mid] <= j) lo = mid;
      else hi = mid - 1;
    }
    const int pos = em_base[lo] + (j - arr_base[lo]);
    if (j - arr_base[lo] >= counts[lo] || pos >= rows) {
      atomicOr(status, kStatusBadTile);
      continue;
    }
    map_in[pos] = j;
    map_back[j] = pos;
  }
}

}  // namespace

cudaError_t launch_a2a_recv_plan(cudaStream_t st, const int* counts, int ep, int el, int rows,
                                 int* offsets, int* map_in, int* map_back, int sm_count,
                                 int* status) {
  int blocks = (rows + 1023) / 1024;
  if (blocks < 1) blocks = 1;
  if (blocks > sm_count) blocks = sm_count;
  a2a_recv_plan_kernel<<<blocks, 1024, 0, st>>>(counts, ep, el, rows, offsets, map_in, map_back,
                                                 status);
  return cudaGetLastError();
}

}  // namespace b200
