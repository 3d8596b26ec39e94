// Launchers shared between the kernel translation units and the C ABI layer.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace b200 {

// Returns a cudaError_t from the launch (cudaSuccess if enqueued).
cudaError_t launch_router_logits(cudaStream_t st, int mode, const void* hidden, long long ldx,
                                 const void* weight, const void* bias, int T, int H, int E,
                                 void* logits);
cudaError_t launch_router_select(cudaStream_t st, int mode, const void* logits, int T, int E,
                                 int K, int normalize, void* probs, void* scores,
                                 long long* indices, int* counts);

cudaError_t launch_route_record(cudaStream_t st, const long long* indices, const void* scores,
                                int scores_bf16, long long n, void* out_idx, void* out_scores);

// Per-(row, 128-column) FP8 activation quantisation (w8a8.cu).
cudaError_t launch_act_quant(cudaStream_t st, const void* x, long long ldx, const int* map, int div,
                             int rows, int k_valid, int k_pad, void* q, float* s, const int* range_offsets,
                             int expert_lo, int expert_hi);

// W8A8 grouped GEMM (w8a8.cu): kernel parameters, filled by the host.
struct W8A8Params {
  const int* offsets;          // permuted-row offsets of the global experts
  int expert_begin, n_experts;
  int gated, feat_tiles, n_feat, nkb, ngroups;
  const uint8_t* wblob;        // FP8 blobs (one fp32 scale per 64-row half)
  uint32_t blob_bytes;
  const float* qs;             // activation scales [rows][qs_groups]
  int qs_groups;
  const void* row_w;
  int row_w_bf16;
  const int* row_src;
  __nv_bfloat16* out;
  long long ldo;
  int* status;
  int ns;                      // pipeline stages
  uint32_t stage_bytes, x_off, bar_off, tmem_cols;
};
constexpr int kW8A8Threads = 320;   // copy warp, MMA warp, 8 promotion + epilogue warps
uint32_t w8a8_epilogue_bytes(int bn, int gated);
int w8a8_tmem_buffers(int bn);      // group accumulators in tensor memory (4: the MMAs run 3 groups ahead)
const void* w8a8_kernel_ptr(int bn);   // token tile 16, 32, 64 or 128; else NULL

size_t permute_workspace_bytes(int T, int K, int E);
cudaError_t launch_permute(cudaStream_t st, const long long* indices, int T, int K, int E,
                           int* counts, int* offsets, int* perm_src, int* inverse,
                           void* workspace, int* status);
// Address, on the current device, of the fixed permutation scratch array
// (B200MOE_PERMUTE_SCRATCH_BYTES).
cudaError_t permute_static_scratch(void** ptr);

// Receive-side plan of the token all-to-all (a2a.cu).
cudaError_t launch_a2a_recv_plan(cudaStream_t st, const int* counts, int ep, int el, int rows,
                                 int* offsets, int* map_in, int* map_back, int sm_count,
                                 int* status);

cudaError_t launch_append_shared_slot(cudaStream_t st, const long long* indices, const void* weights,
                                      int weights_bf16, const void* logit, long long ld_logit, int T, int K,
                                      long long shared, long long* out_idx, void* out_w);
cudaError_t launch_combine(cudaStream_t st, const void* rows, long long ld_rows,
                           const int* inverse, const long long* indices, int T, int K, int H,
                           int order, int experts_per_rank, int expert_lo, int expert_hi,
                           int scale_rows, const void* weights, int weights_bf16, void* out,
                           long long ld_out);

cudaError_t launch_combine_f32(cudaStream_t st, const float* rows, long long ld_rows,
                               const int* inverse, const long long* indices, int T, int K, int H,
                               int lo, int hi, const void* weights, int weights_bf16, void* out,
                               long long ld_out);

// Exchange-buffer layout of the fused combine + all-reduce (p2p.cu).
constexpr int kP2PBlocks = 1024;    // block b owns rows t = b (mod 1024)
constexpr int kP2PMaxRanks = 8;
constexpr size_t kP2PHeaderBytes = 69632;  // flags [2][1024][8] u32 + epochs [1024] u32
static_assert(2 * kP2PBlocks * kP2PMaxRanks * 4 + kP2PBlocks * 4 <= kP2PHeaderBytes, "p2p header");
constexpr long long kP2POneShotBytes = 16ll << 20;   // one-shot up to this many pushed bytes per rank

// The exchange of T rows pushes every partial row to every rank (one-shot)
// or to its row's owner only (two-shot; the owner of row t is t % world and
// its inbox slot t / world, which needs world to divide kP2PBlocks).
inline bool p2p_two_shot(int T, int H, int world) {
  return world > 1 && (long long)T * H * 2 * (world - 1) > kP2POneShotBytes;
}
inline bool p2p_supported(int T, int H, int world) {
  return !p2p_two_shot(T, H, world) || kP2PBlocks % world == 0;
}
// Inbox rows per (parity, source) of a buffer for up to t_cap rows.
inline int p2p_inbox_rows(int t_cap, int H, int world) {
  long long one = world > 1 ? kP2POneShotBytes / ((long long)H * 2 * (world - 1)) : t_cap;
  if (one > t_cap) one = t_cap;
  const int two = (t_cap + world - 1) / world;
  return static_cast<int>(one > two ? one : two);
}

cudaError_t launch_combine_allreduce(cudaStream_t st, const void* rows, long long ld_rows,
                                     const int* inverse, const long long* indices, int T, int K,
                                     int H, int expert_lo, int expert_hi, int scale_rows,
                                     const void* weights, int weights_bf16, int world, int rank,
                                     void* const* peers, int t_cap, void* out, long long ld_out,
                                     unsigned long long timeout_ns, int* status);

// Row-exchange buffer of the peer-memory all-to-all and gather (a2a_p2p.cu):
// this header, then area A [cap_a][H] bf16 and area B [cap_b][H] bf16.
struct PeerRowsHeader {
  uint32_t flags[5][kP2PMaxRanks];   // [phase][source]: epoch of the source's last signal
  uint32_t a2a_epoch, gather_epoch, ctr_dispatch, ctr_return, ctr_gather;
  int recv_total;                    // rows received by the last all-to-all
  uint32_t pad[18];
  int board[kP2PMaxRanks][1024];     // [source][expert]: row counts of the last all-to-all
  int dst_base[1024];                // [expert]: first row of my rows of it in its owner's area A
  int seg_start[1025];               // [my expert * world + source]: first receive row
  int ret_base[1024];                // [my expert * world + source]: source's permuted offset
  int recv_offsets[1025];            // [my expert]: first receive row (expert-major)
};
constexpr size_t kPeerRowsHeaderBytes = 65536;
static_assert(sizeof(PeerRowsHeader) <= kPeerRowsHeaderBytes, "peer rows header");

cudaError_t launch_a2a_counts(cudaStream_t st, void* const* peers, int world, int rank, int E,
                              const int* counts, int* recv_offsets, long long cap_a, long long cap_b,
                              unsigned long long timeout_ns, int* status);
cudaError_t launch_a2a_dispatch(cudaStream_t st, void* const* peers, int world, int rank, int E,
                                const void* hidden, long long ldh, int H, const long long* indices,
                                const int* perm_src, const int* offsets, int rows_cap, int K,
                                long long cap_a, int sm_count, unsigned long long timeout_ns,
                                int* status);
cudaError_t launch_a2a_return(cudaStream_t st, void* const* peers, int world, int rank, int E,
                              const void* y, long long ldy, int H, long long cap_a, long long cap_b,
                              int sm_count, unsigned long long timeout_ns, int* status);
cudaError_t launch_ep_gather(cudaStream_t st, void* const* peers, int world, int rank, int H,
                             const int* offsets, int lo, int hi, long long rows_cap, long long cap_a,
                             int sm_count, unsigned long long timeout_ns, int* status);

cudaError_t launch_gather_rows_range(cudaStream_t st, const void* src, long long ld_src,
                                     const int* map, int div, int n, int H, void* dst,
                                     long long ld_dst, const int* offsets, int expert_lo,
                                     int expert_hi, int max_blocks);

cudaError_t launch_gather_rows(cudaStream_t st, const void* src, long long ld_src,
                               const int* map, int div, int n, int H, void* dst,
                               long long ld_dst);

}  // namespace b200
