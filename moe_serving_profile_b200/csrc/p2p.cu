// Combine + cross-rank reduction in one kernel over NVLink peer memory: the
// replicated-token expert-parallel layer's "fast" exchange
// (moe_serving/qwen3_parallel.py:105-118 combines each rank's own experts and
// all-reduces the [T, H] partial sums) without a separate collective launch.
//
// Every rank owns one exchange buffer (cudaMalloc'd, mapped into the other
// ranks' address spaces with CUDA IPC; plain loads and stores, no multicast):
//   [2][kP2PBlocks][8] u32    flags: slot (phase, b, src) = the epoch of
//                             block b's last phase signal from rank src,
//                             written by rank src
//   [kP2PBlocks] u32          this rank's epoch per block (local)
//   [2][world][A][H] bf16     inbox: partial rows sent here, by source rank
//   [2][t_cap][H] bf16        finished rows (two-shot)
// (the leading [2] of the row areas is the epoch parity). Block b owns the
// rows t = b (mod kP2PBlocks) on every rank (the grid is min(T, kP2PBlocks)
// blocks), so a row's writer and readers are the same block everywhere and
// every block keeps its own epoch sequence. A block first combines its rows:
// partial[t] = bf16 running sum of the row's local-expert contributions in
// ascending expert order (the combine kernel's order). Then:
//   one-shot (T * H * 2 * (world - 1) <= kP2POneShotBytes):
//     push partial[t] into inbox [rank][t] of every rank (posted NVLink
//     stores); signal every peer, wait for every peer (bounded); out[t] =
//     bf16(fp32 sum of inbox [0 .. world)[t] in rank order), local reads.
//   two-shot (larger exchanges, world sizes dividing kP2PBlocks: 2, 4, 8):
//     the rows of block b belong to rank o = b % world (= t % world); push
//     partial[t] only to inbox [rank][t / world] of rank o and signal it;
//     rank o waits for every source, sums in rank order as above, pushes the
//     finished row into every rank's finished area [t] and signals them; every
//     rank copies its finished rows to out. Each rank sends about
//     2 T H 2 (world - 1) / world bytes instead of T H 2 (world - 1).
// Epoch parity selects the row areas, so a rank writes an area of a peer
// again only two calls later, after that peer has signalled the call in
// between, which it does only after it has read the area.
#include "internal.h"
#include "ptx.cuh"

namespace b200 {
namespace {

constexpr int kMaxK = 32;

struct P2PParams {
  const __nv_bfloat16* rows;
  long long ld_rows;
  const int* inverse;
  const long long* indices;
  int T, K, H, lo, hi, scale_rows, weights_bf16, world, rank, t_cap, a_rows, two_shot;
  const void* weights;
  uint8_t* peer[kP2PMaxRanks];   // every rank's exchange buffer (peer[rank] is local)
  __nv_bfloat16* out;
  long long ld_out;
  unsigned long long timeout_ns;
  int* status;
};

__device__ __forceinline__ uint32_t* flags_of(uint8_t* base, int phase) {
  return reinterpret_cast<uint32_t*>(base) + phase * kP2PBlocks * kP2PMaxRanks;
}
__device__ __forceinline__ uint32_t* seq_of(uint8_t* base) {
  return reinterpret_cast<uint32_t*>(base) + 2 * kP2PBlocks * kP2PMaxRanks;
}
// inbox row [parity][src][i]
__device__ __forceinline__ __nv_bfloat16* inbox_row(uint8_t* base, const P2PParams& p, int parity,
                                                    int src, int i) {
  return reinterpret_cast<__nv_bfloat16*>(base + kP2PHeaderBytes) +
         (((long long)parity * p.world + src) * p.a_rows + i) * p.H;
}
// finished row [parity][t]
__device__ __forceinline__ __nv_bfloat16* final_row(uint8_t* base, const P2PParams& p, int parity, int t) {
  return reinterpret_cast<__nv_bfloat16*>(base + kP2PHeaderBytes) +
         (2ll * p.world * p.a_rows + (long long)parity * p.t_cap + t) * p.H;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0: fence this block's stores, then store the epoch into slot
// (phase, b, rank) of every listed peer.
__device__ __forceinline__ void signal_peers(const P2PParams& p, int phase, int b, uint32_t epoch,
                                             int only) {
  __threadfence_system();
  for (int q = 0; q < p.world; ++q)
    if (q != p.rank && (only < 0 || q == only))
      st_release_sys(flags_of(p.peer[q], phase) + b * kP2PMaxRanks + p.rank, epoch);
}

// Thread 0: wait until slot (phase, b, q) here holds the epoch for every
// listed source q (bounded). Returns false after the timeout (status set).
__device__ __forceinline__ bool wait_peers(const P2PParams& p, int phase, int b, uint32_t epoch,
                                           int only) {
  const uint64_t t0 = globaltimer_ns();
  for (int q = 0; q < p.world; ++q) {
    if (q == p.rank || (only >= 0 && q != only)) continue;
    const uint32_t* f = flags_of(p.peer[p.rank], phase) + b * kP2PMaxRanks + q;
    while (static_cast<int>(ld_acquire_sys(f) - epoch) < 0) {
      if (globaltimer_ns() - t0 > p.timeout_ns) {
        atomicOr(p.status, kStatusPeerTimeout);
        return false;
      }
      __nanosleep(64);
    }
  }
  __threadfence();
  return true;
}

__device__ __forceinline__ void acc_row(float (&acc)[8], const uint4& u) {
  const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc[2 * j] += __uint_as_float(wd[j] << 16);
    acc[2 * j + 1] += __uint_as_float(wd[j] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint4 pack_row(const float (&acc)[8]) {
  uint4 o;
  o.x = pack_bf16x2(acc[0], acc[1]);
  o.y = pack_bf16x2(acc[2], acc[3]);
  o.z = pack_bf16x2(acc[4], acc[5]);
  o.w = pack_bf16x2(acc[6], acc[7]);
  return o;
}

__global__ void __launch_bounds__(128) combine_allreduce_kernel(const __grid_constant__ P2PParams p) {
  const int b = blockIdx.x;
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  uint8_t* mine = p.peer[p.rank];
  if (threadIdx.x == 0) s_epoch = seq_of(mine)[b] + 1;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int parity = static_cast<int>(epoch & 1u);
  const int nvec = p.H >> 3;
  const int owner = b % p.world;   // two-shot: the rank that finishes this block's rows

  // ---- 1. partial sums of this block's rows, pushed to the inbox(es)
  // The row's local contributions in (expert, slot) order: lane k of warp 0
  // reads slot k, its rank among the valid slots (keys are distinct) is its
  // position, and the sorted rows and slots go to shared memory for the block.
  __shared__ int s_row[kMaxK];
  __shared__ int s_slot[kMaxK];
  __shared__ int s_n;
  for (int t = b; t < p.T; t += kP2PBlocks) {   // gridDim.x == min(T, kP2PBlocks)
    __syncthreads();   // the previous row's list is no longer read
    if (threadIdx.x < 32) {
      const int k = threadIdx.x;
      bool valid = false;
      long long kk = 0;
      int r = -1;
      if (k < p.K) {
        const long long e = p.indices[(long long)t * p.K + k];
        r = p.inverse[(long long)t * p.K + k];
        valid = !(r < 0 || e < p.lo || e >= p.hi);
        kk = e * kMaxK + k;
      }
      const unsigned vmask = __ballot_sync(0xffffffffu, valid);
      int pos = 0;
      for (int j = 0; j < p.K; ++j) {
        const long long kj = __shfl_sync(0xffffffffu, kk, j);
        if (((vmask >> j) & 1u) && kj < kk) ++pos;
      }
      if (valid) {
        s_row[pos] = r;
        s_slot[pos] = k;
      }
      if (k == 0) s_n = __popc(vmask);
    }
    __syncthreads();
    const int n = s_n;
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      // up to 8 rows' vectors are loaded before any is added (same order)
      for (int i0 = 0; i0 < n; i0 += 8) {
        uint4 qv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (i0 + u < n) qv[u] = __ldg(reinterpret_cast<const uint4*>(p.rows + s_row[i0 + u] * p.ld_rows) + v);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (i0 + u >= n) break;
          float wv = 1.f;
          if (p.scale_rows) {
            const long long wi = (long long)t * p.K + s_slot[i0 + u];
            wv = p.weights_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.weights)[wi])
                                : reinterpret_cast<const float*>(p.weights)[wi];
          }
          const uint32_t wd[4] = {qv[u].x, qv[u].y, qv[u].z, qv[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float c0 = __uint_as_float(wd[j] << 16);
            float c1 = __uint_as_float(wd[j] & 0xffff0000u);
            if (p.scale_rows) {
              c0 = bf16r(c0 * wv);
              c1 = bf16r(c1 * wv);
            }
            acc[2 * j] = bf16r(acc[2 * j] + c0);
            acc[2 * j + 1] = bf16r(acc[2 * j + 1] + c1);
          }
        }
      }
      const uint4 o = pack_row(acc);
      if (p.two_shot) {
        reinterpret_cast<uint4*>(inbox_row(p.peer[owner], p, parity, p.rank, t / p.world))[v] = o;
      } else {
        for (int q = 0; q < p.world; ++q)
          reinterpret_cast<uint4*>(inbox_row(p.peer[q], p, parity, p.rank, t))[v] = o;
      }
    }
  }

  // ---- 2. exchange
  __syncthreads();
  if (threadIdx.x == 0) {
    seq_of(mine)[b] = epoch;
    if (!p.two_shot) {
      signal_peers(p, 0, b, epoch, -1);
      s_ok = wait_peers(p, 0, b, epoch, -1);
    } else if (owner != p.rank) {
      signal_peers(p, 0, b, epoch, owner);
      s_ok = 1;
    } else {
      s_ok = wait_peers(p, 0, b, epoch, -1);
    }
  }
  __syncthreads();
  if (!s_ok) return;   // the status word reports it; the output rows are not written

  if (!p.two_shot) {
    // ---- 3. sum the inbox rows in rank order (fp32), one bf16 rounding
    for (int t = b; t < p.T; t += kP2PBlocks) {
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int q = 0; q < p.world; ++q)   // L2 reads: peers rewrite the inbox
          acc_row(acc, __ldcg(reinterpret_cast<const uint4*>(inbox_row(mine, p, parity, q, t)) + v));
        reinterpret_cast<uint4*>(p.out + t * p.ld_out)[v] = pack_row(acc);
      }
    }
    return;
  }

  if (owner == p.rank) {
    // ---- 3a. the owner finishes the rows and pushes them to every rank
    for (int t = b; t < p.T; t += kP2PBlocks) {
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int q = 0; q < p.world; ++q)
          acc_row(acc, __ldcg(reinterpret_cast<const uint4*>(inbox_row(mine, p, parity, q, t / p.world)) + v));
        const uint4 o = pack_row(acc);
        for (int q = 0; q < p.world; ++q)
          if (q != p.rank) reinterpret_cast<uint4*>(final_row(p.peer[q], p, parity, t))[v] = o;
        reinterpret_cast<uint4*>(p.out + t * p.ld_out)[v] = o;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) signal_peers(p, 1, b, epoch, -1);
    return;
  }
  // ---- 3b. the other ranks wait for the owner's finished rows
  if (threadIdx.x == 0) s_ok = wait_peers(p, 1, b, epoch, owner);
  __syncthreads();
  if (!s_ok) return;
  for (int t = b; t < p.T; t += kP2PBlocks)
    for (int v = threadIdx.x; v < nvec; v += blockDim.x)
      reinterpret_cast<uint4*>(p.out + t * p.ld_out)[v] =
          __ldcg(reinterpret_cast<const uint4*>(final_row(mine, p, parity, t)) + v);
}

}  // namespace

cudaError_t launch_combine_allreduce(cudaStream_t st, const void* rows, long long ld_rows,
                                     const int* inverse, const long long* indices, int T, int K,
                                     int H, int expert_lo, int expert_hi, int scale_rows,
                                     const void* weights, int weights_bf16, int world, int rank,
                                     void* const* peers, int t_cap, void* out, long long ld_out,
                                     unsigned long long timeout_ns, int* status) {
  P2PParams p{};
  p.rows = static_cast<const __nv_bfloat16*>(rows);
  p.ld_rows = ld_rows;
  p.inverse = inverse;
  p.indices = indices;
  p.T = T;
  p.K = K;
  p.H = H;
  p.lo = expert_lo;
  p.hi = expert_hi;
  p.scale_rows = scale_rows;
  p.weights = weights;
  p.weights_bf16 = weights_bf16;
  p.world = world;
  p.rank = rank;
  p.t_cap = t_cap;
  p.a_rows = p2p_inbox_rows(t_cap, H, world);
  p.two_shot = p2p_two_shot(T, H, world) ? 1 : 0;
  for (int i = 0; i < world; ++i) p.peer[i] = static_cast<uint8_t*>(peers[i]);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.timeout_ns = timeout_ns;
  p.status = status;
  // every rank launches the same grid; at most kP2PBlocks blocks of 128
  // threads, which fit on the device at once, so no block waits on one that
  // cannot start. T = 0 launches nothing (no block's epoch advances anywhere).
  if (T == 0) return cudaSuccess;
  combine_allreduce_kernel<<<T < kP2PBlocks ? T : kP2PBlocks, 128, 0, st>>>(p);
  return cudaGetLastError();
}

}  // namespace b200
