// Expert-parallel row exchanges over NVLink peer memory (CUDA IPC mappings,
// plain 16-byte loads and stores, no multicast, no TMA):
//
//   token all-to-all (moe_serving/moe.py:110-137, distributed.py:33-46)
//     a2a_counts    every rank writes its per-expert row counts into every
//                   rank's count board, waits for the others' boards, and
//                   derives all placements on the device: where its rows go
//                   in each destination, its own experts' segments, and where
//                   each computed row goes back (no host read of any count)
//     a2a_dispatch  pushes each routed row straight into the destination's
//                   receive area, already in the destination's expert-major
//                   order (expert, then source rank, then the source's
//                   permuted order), so the grouped GEMMs read it in place
//     a2a_return    pushes each computed row back into its source's return
//                   area at the source's own permuted position; the source
//                   combines from there in (rank, slot) order
//   replicated-token exact gather (moe_serving/parallel_numerics.py:13-36)
//     ep_gather     (after a handshake saying every rank's previous combine
//                   from its area A is done) every rank pushes its experts'
//                   contribution rows (already
//                   at their global permuted positions) into every peer's
//                   area, so each rank holds all T*K rows and runs the ordered
//                   global-expert combine locally: the reference numerics at
//                   any EP size with (world - 1) / world of the rows moved
//                   instead of an all-reduce of all of them
//
// Buffer of one rank: PeerRowsHeader, area A [cap_a][H] bf16 (receive /
// gathered rows), area B [cap_b][H] bf16 (returned rows). A phase ends with
// the last block of the grid (a done counter) storing the call's epoch into
// its slot (phase, rank) of every peer's flag table and waiting, bounded, for
// every peer's slot (phase, peer) here. Epochs only grow, so nothing is
// reset between calls and the calls replay from CUDA graphs.
//
// Reuse of the single-buffered areas is ordered by the exchange itself: a
// rank writes a peer's board or receive area for call n + 1 only after it
// has every peer's returned rows of call n, which each peer sends after its
// reads of call n (its GEMMs and its board reads precede its return signal
// in stream order); a peer's return area is written for call n + 1 only
// after that peer's dispatch of call n + 1, which follows its combine of
// call n.
#include "internal.h"
#include "ptx.cuh"

namespace b200 {
namespace {

constexpr int kPhaseCounts = 0, kPhaseDispatch = 1, kPhaseReturn = 2, kPhaseGather = 3,
              kPhaseGatherReady = 4;

__device__ __forceinline__ PeerRowsHeader* hdr(void* base) {
  return reinterpret_cast<PeerRowsHeader*>(base);
}
__device__ __forceinline__ uint4* area_a(void* base, int H, long long row) {
  return reinterpret_cast<uint4*>(static_cast<uint8_t*>(base) + kPeerRowsHeaderBytes +
                                  row * static_cast<long long>(H) * 2);
}
__device__ __forceinline__ uint4* area_b(void* base, int H, long long cap_a, long long row) {
  return reinterpret_cast<uint4*>(static_cast<uint8_t*>(base) + kPeerRowsHeaderBytes +
                                  (cap_a + row) * static_cast<long long>(H) * 2);
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct PeerSet {
  void* p[kP2PMaxRanks];
};

// One thread: store `epoch` into slot (phase, rank) of every other rank,
// after fencing this grid's stores, then wait (bounded) until every other
// rank's slot (phase, q) here holds it. Returns false on timeout (status set).
__device__ bool signal_and_wait(const PeerSet& ps, int world, int rank, int phase, uint32_t epoch,
                                unsigned long long timeout_ns, int* status) {
  __threadfence_system();
  for (int q = 0; q < world; ++q)
    if (q != rank) st_release_sys(&hdr(ps.p[q])->flags[phase][rank], epoch);
  const uint64_t t0 = globaltimer_ns();
  for (int q = 0; q < world; ++q) {
    if (q == rank) continue;
    const uint32_t* f = &hdr(ps.p[rank])->flags[phase][q];
    while (static_cast<int>(ld_acquire_sys(f) - epoch) < 0) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        atomicOr(status, kStatusPeerTimeout);
        return false;
      }
      __nanosleep(64);
    }
  }
  __threadfence_system();
  return true;
}

// Block-wide exclusive scan of one int per thread (blockDim.x == 1024).
__device__ int block_scan_excl(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  __syncthreads();
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += u;
    }
    warp_sums[lane] = wi - w;
    if (lane == 31) warp_sums[32] = wi;
  }
  __syncthreads();
  const int r = incl - v + warp_sums[warp];
  if (total) *total = warp_sums[32];
  __syncthreads();
  return r;
}

// One block of 1024 threads. E <= 1024 experts, el = E / world.
__global__ void __launch_bounds__(1024) a2a_counts_kernel(PeerSet ps, int world, int rank, int E,
                                                          const int* __restrict__ counts,
                                                          int* __restrict__ recv_offsets_out,
                                                          long long cap_a, long long cap_b,
                                                          unsigned long long timeout_ns, int* status) {
  __shared__ int warp_sums[33];
  __shared__ int tot_s[1024];
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  const int tid = threadIdx.x;
  const int el = E / world;
  PeerRowsHeader* me = hdr(ps.p[rank]);
  if (tid == 0) {
    s_epoch = me->a2a_epoch + 1u;
    me->a2a_epoch = s_epoch;
    me->ctr_dispatch = 0u;
    me->ctr_return = 0u;
  }
  // my counts into row `rank` of every board (mine included)
  const int c = tid < E ? counts[tid] : 0;
  if (tid < E)
    for (int q = 0; q < world; ++q) hdr(ps.p[q])->board[rank][tid] = c;
  __threadfence_system();
  __syncthreads();
  if (tid == 0) s_ok = signal_and_wait(ps, world, rank, kPhaseCounts, s_epoch, timeout_ns, status) ? 1 : 0;
  __syncthreads();
  if (!s_ok) return;
  // per-expert totals over the sources, and the rows of sources below me
  int tot = 0, below = 0;
  if (tid < E) {
    for (int s = 0; s < world; ++s) {
      const int v = me->board[s][tid];
      tot += v;
      if (s < rank) below += v;
    }
  }
  tot_s[tid] = tot;
  int all_rows = 0;
  const int ex = block_scan_excl(tot, warp_sums, &all_rows);   // over all experts
  __syncthreads();
  // segment base inside the destination: subtract the scan at its first expert
  __shared__ int dest_first[kP2PMaxRanks];
  if (tid < E && tid % el == 0) dest_first[tid / el] = ex;
  __syncthreads();
  if (tid < E) me->dst_base[tid] = ex - dest_first[tid / el] + below;
  // my experts: receive segments in (expert, source) order and the sources'
  // own permuted offsets of those experts
  const int g0 = rank * el;
  const int mine_total = (rank + 1 < world ? dest_first[rank + 1] : all_rows) - dest_first[rank];
  // my receive offsets and (expert, source) segment starts, in order
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < el; ++e) {
      const int lim = acc < cap_a ? acc : static_cast<int>(cap_a);
      me->recv_offsets[e] = lim;
      if (recv_offsets_out) recv_offsets_out[e] = lim;
      int sacc = acc;
      for (int s = 0; s < world; ++s) {
        me->seg_start[e * world + s] = sacc;
        sacc += me->board[s][g0 + e];
      }
      acc += tot_s[g0 + e];
    }
    const int lim = acc < cap_a ? acc : static_cast<int>(cap_a);
    me->seg_start[el * world] = lim;
    me->recv_offsets[el] = lim;
    if (recv_offsets_out) recv_offsets_out[el] = lim;
    me->recv_total = lim;
    if (acc > cap_a || mine_total != acc) atomicOr(status, kStatusBadTile);
  }
  // ret_base[e * world + s] = source s's permuted offset of expert g0 + e:
  // the exclusive scan of board[s][0 .. E) at g0 + e
  for (int s = 0; s < world; ++s) {
    const int v = tid < E ? me->board[s][tid] : 0;
    int src_total = 0;
    const int exs = block_scan_excl(v, warp_sums, &src_total);
    if (tid >= g0 && tid < g0 + el) me->ret_base[(tid - g0) * world + s] = exs;
    if (s == rank && tid == 0 && src_total > cap_b) atomicOr(status, kStatusBadTile);
  }
}

// Copy one row of H bf16 (H % 8 == 0) with a warp, 16 bytes per lane per step.
__device__ __forceinline__ void copy_row(uint4* dst, const uint4* src, int n16, int lane) {
  for (int i = lane; i < n16; i += 32) dst[i] = src[i];
}

// Last block of the grid to finish: returns true in thread 0 of it.
__device__ bool last_block(uint32_t* ctr) {
  __shared__ int s_last;
  __threadfence_system();   // this thread's peer stores, before the block's arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t old = atomicAdd(ctr, 1u);
    s_last = old == gridDim.x - 1 ? 1 : 0;
  }
  __syncthreads();
  return s_last != 0 && threadIdx.x == 0;
}

__global__ void __launch_bounds__(256) a2a_dispatch_kernel(
    PeerSet ps, int world, int rank, int E, const __nv_bfloat16* __restrict__ hidden, long long ldh,
    int H, const long long* __restrict__ indices, const int* __restrict__ perm_src,
    const int* __restrict__ offsets, int K, long long cap_a, unsigned long long timeout_ns,
    int* status) {
  PeerRowsHeader* me = hdr(ps.p[rank]);
  const int el = E / world;
  const int n16 = H / 8;
  const int rows = offsets[E];
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int j = blockIdx.x * wpb + (threadIdx.x >> 5); j < rows; j += gridDim.x * wpb) {
    const int src = perm_src[j];
    const int e = static_cast<int>(indices[src]);
    if (e < 0 || e >= E) continue;
    const int d = e / el;
    const long long dst = static_cast<long long>(me->dst_base[e]) + (j - offsets[e]);
    if (dst < 0 || dst >= cap_a) {
      if (lane == 0) atomicOr(status, kStatusBadTile);
      continue;
    }
    copy_row(area_a(ps.p[d], H, dst),
             reinterpret_cast<const uint4*>(hidden + static_cast<long long>(src / K) * ldh), n16, lane);
  }
  if (last_block(&me->ctr_dispatch))
    signal_and_wait(ps, world, rank, kPhaseDispatch, me->a2a_epoch, timeout_ns, status);
}

__global__ void __launch_bounds__(256) a2a_return_kernel(PeerSet ps, int world, int rank, int E,
                                                         const __nv_bfloat16* __restrict__ y,
                                                         long long ldy, int H, long long cap_a,
                                                         long long cap_b,
                                                         unsigned long long timeout_ns, int* status) {
  PeerRowsHeader* me = hdr(ps.p[rank]);
  const int el = E / world;
  const int nseg = el * world;
  const int n16 = H / 8;
  const int rows = me->recv_total;
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int r = blockIdx.x * wpb + (threadIdx.x >> 5); r < rows; r += gridDim.x * wpb) {
    // segment (e, s): the last with seg_start <= r
    int lo = 0, hi = nseg;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (me->seg_start[mid] <= r) lo = mid; else hi = mid;
    }
    const int s = lo % world;
    const long long dst = static_cast<long long>(me->ret_base[lo]) + (r - me->seg_start[lo]);
    if (dst < 0 || dst >= cap_b) {
      if (lane == 0) atomicOr(status, kStatusBadTile);
      continue;
    }
    copy_row(area_b(ps.p[s], H, cap_a, dst),
             reinterpret_cast<const uint4*>(y + static_cast<long long>(r) * ldy), n16, lane);
  }
  if (last_block(&me->ctr_return))
    signal_and_wait(ps, world, rank, kPhaseReturn, me->a2a_epoch, timeout_ns, status);
}

// Before a gather writes any peer's area A, every rank says that its last
// combine from area A is done (this launch follows it in stream order) and
// waits for the others: one thread.
__global__ void ep_gather_ready_kernel(PeerSet ps, int world, int rank, unsigned long long timeout_ns,
                                       int* status) {
  if (threadIdx.x != 0) return;
  const uint32_t epoch = hdr(ps.p[rank])->gather_epoch + 1u;
  signal_and_wait(ps, world, rank, kPhaseGatherReady, epoch, timeout_ns, status);
}

// Rows [offsets[lo], offsets[hi]) of this rank's area A go to the same rows of
// every other rank's area A.
__global__ void __launch_bounds__(256) ep_gather_kernel(PeerSet ps, int world, int rank, int H,
                                                        const int* __restrict__ offsets, int lo,
                                                        int hi, long long cap_a,
                                                        unsigned long long timeout_ns, int* status) {
  PeerRowsHeader* me = hdr(ps.p[rank]);
  const uint32_t epoch = me->gather_epoch + 1u;   // every block reads it before the last one ends
  const int n16 = H / 8;
  const int r0 = offsets[lo];
  const int r1 = offsets[hi];
  if (r1 > cap_a && threadIdx.x == 0 && blockIdx.x == 0) atomicOr(status, kStatusBadTile);
  const int rend = r1 < cap_a ? r1 : static_cast<int>(cap_a);
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  // one (row, peer) pair per warp step, so every link carries traffic at once
  const long long n = static_cast<long long>(rend > r0 ? rend - r0 : 0) * (world - 1);
  for (long long w = blockIdx.x * wpb + (threadIdx.x >> 5); w < n; w += (long long)gridDim.x * wpb) {
    const int r = r0 + static_cast<int>(w / (world - 1));
    int q = static_cast<int>(w % (world - 1));
    q += q >= rank ? 1 : 0;
    copy_row(area_a(ps.p[q], H, r), area_a(ps.p[rank], H, r), n16, lane);
  }
  if (last_block(&me->ctr_gather)) {
    signal_and_wait(ps, world, rank, kPhaseGather, epoch, timeout_ns, status);
    me->ctr_gather = 0u;
    me->gather_epoch = epoch;
  }
}

PeerSet peer_set(void* const* peers, int world) {
  PeerSet ps{};
  for (int i = 0; i < world; ++i) ps.p[i] = peers[i];
  return ps;
}

int copy_grid(long long rows, int sm_count) {
  const long long want = (rows + 7) / 8;   // 8 warps per block, a row per warp
  const long long cap = 4ll * sm_count;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

}  // namespace

cudaError_t launch_a2a_counts(cudaStream_t st, void* const* peers, int world, int rank, int E,
                              const int* counts, int* recv_offsets, long long cap_a, long long cap_b,
                              unsigned long long timeout_ns, int* status) {
  a2a_counts_kernel<<<1, 1024, 0, st>>>(peer_set(peers, world), world, rank, E, counts, recv_offsets,
                                        cap_a, cap_b, timeout_ns, status);
  return cudaGetLastError();
}

cudaError_t launch_a2a_dispatch(cudaStream_t st, void* const* peers, int world, int rank, int E,
                                const void* hidden, long long ldh, int H, const long long* indices,
                                const int* perm_src, const int* offsets, int rows_cap, int K,
                                long long cap_a, int sm_count, unsigned long long timeout_ns,
                                int* status) {
  a2a_dispatch_kernel<<<copy_grid(rows_cap, sm_count), 256, 0, st>>>(
      peer_set(peers, world), world, rank, E, static_cast<const __nv_bfloat16*>(hidden), ldh, H,
      indices, perm_src, offsets, K, cap_a, timeout_ns, status);
  return cudaGetLastError();
}

cudaError_t launch_a2a_return(cudaStream_t st, void* const* peers, int world, int rank, int E,
                              const void* y, long long ldy, int H, long long cap_a, long long cap_b,
                              int sm_count, unsigned long long timeout_ns, int* status) {
  a2a_return_kernel<<<copy_grid(cap_a, sm_count), 256, 0, st>>>(
      peer_set(peers, world), world, rank, E, static_cast<const __nv_bfloat16*>(y), ldy, H, cap_a,
      cap_b, timeout_ns, status);
  return cudaGetLastError();
}

cudaError_t launch_ep_gather(cudaStream_t st, void* const* peers, int world, int rank, int H,
                             const int* offsets, int lo, int hi, long long rows_cap, long long cap_a,
                             int sm_count, unsigned long long timeout_ns, int* status) {
  ep_gather_ready_kernel<<<1, 32, 0, st>>>(peer_set(peers, world), world, rank, timeout_ns, status);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  ep_gather_kernel<<<copy_grid(rows_cap * (world > 1 ? world - 1 : 1), sm_count), 256, 0, st>>>(
      peer_set(peers, world), world, rank, H, offsets, lo, hi, cap_a, timeout_ns, status);
  return cudaGetLastError();
}

}  // namespace b200
