// Block-wide exclusive scan shared by the permutation kernels.
#pragma once

namespace b200 {

// Exclusive scan of vals[0..n) (n <= 1024) held one per thread; returns the
// exclusive prefix for this thread, total in *total. Uses scratch[32].
__device__ __forceinline__ int block_exclusive_scan(int v, int n, int* scratch, int* total) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid >= n) v = 0;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    int s = lane < nw ? scratch[lane] : 0;
    int si = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, si, o);
      if (lane >= o) si += u;
    }
    scratch[lane] = si - s;  // exclusive warp offsets
    if (lane == 31) scratch[32] = si;
  }
  __syncthreads();
  const int res = scratch[warp] + incl - v;
  *total = scratch[32];
  __syncthreads();
  return res;
}

}  // namespace b200
