/*
 * b200moe — C ABI of the sm_100a MoE expert layer.
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t
 * (passed as void*), enqueues work on that stream without any host
 * synchronisation, and returns an int status (B200MOE_OK or an error code;
 * b200moe_last_error() gives the message for the calling thread). The
 * library never allocates or frees caller memory: all outputs and workspaces
 * are owned by the caller (torch's caching allocator on the Python side).
 *
 * The reference (moe_serving, pure Python) has no foreign-function boundary;
 * each function names the reference code path it replaces, by file:line in
 * the reference project. Router formulas live in Transformers; the cited
 * lines are those of the installed transformers 5.5.0 proxy of the pinned
 * 5.20.0 tree (models/qwen3_moe/modeling_qwen3_moe.py and
 * models/gpt_oss/modeling_gpt_oss.py).
 */
#ifndef B200MOE_H_
#define B200MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */
#define B200MOE_OK 0
#define B200MOE_ERR_INVALID 1     /* bad argument / shape */
#define B200MOE_ERR_UNSUPPORTED 2 /* valid but outside what the kernels implement */
#define B200MOE_ERR_CUDA 3        /* a CUDA runtime call failed */

/* Device status bits (b200moe_device_status): set by kernels, never fatal. */
#define B200MOE_STATUS_WAIT_TIMEOUT 1 /* a bounded device wait gave up */
#define B200MOE_STATUS_BAD_TILE 2     /* inconsistent tile bookkeeping */
#define B200MOE_STATUS_BAD_INDEX 4    /* an expert id outside [0, E) was dropped */
#define B200MOE_STATUS_PEER_TIMEOUT 8 /* a wait for another rank's signal gave up */

/* Message describing the last non-zero return on this host thread. */
const char* b200moe_last_error(void);

/* Library version string. */
const char* b200moe_version(void);

/* Read (and optionally clear) the per-device status word that kernels OR
 * B200MOE_STATUS_* bits into. Synchronises the device. */
int b200moe_device_status(int device, int clear, int* out_status);

/* ------------------------------------------------------------ router
 * Fused router: logits = hidden[T,H] . weight[E,H]^T (+ bias) accumulated in
 * fp32 in a fixed order (H split into 64-column segments, each one fmaf
 * chain in increasing h from 0, the segment sums then added in increasing
 * order; H % 8 == 0, H <= 8192), followed by softmax / top-k / per-expert
 * counts.
 * Top-k order: value descending, equal values by ascending expert id.
 *
 * mode B200MOE_ROUTER_QWEN3 replaces Qwen3MoeTopKRouter.forward
 *   (qwen3_moe/modeling_qwen3_moe.py:263-272), hooked at
 *   moe_serving/qwen3_parallel.py:42-44: bf16 logits, fp32 softmax over E,
 *   top-k, optional renormalisation; probs fp32 [T,E], scores fp32 [T,K].
 * mode B200MOE_ROUTER_GPT_OSS replaces GptOssTopKRouter.forward
 *   (gpt_oss/modeling_gpt_oss.py:126-131), hooked at
 *   moe_serving/gpt_oss_parallel.py:256-258: bf16 logits with bias, top-k on
 *   the logits, softmax over the k values in bf16; scores bf16 [T,K].
 * mode B200MOE_ROUTER_NATIVE replaces moe_serving/moe.py:97-107 (route):
 *   fp32 logits, fp32 softmax, top-k, renormalise with clamp 1e-20; scores
 *   are written as bf16 [T,K] (the hidden dtype).
 *
 * bias: bf16 [E], required for GPT_OSS; optional for QWEN3 (added to the
 *   fp32 sum before the bf16 rounding, as F.linear(h, W, b) does); ignored
 *   for NATIVE.
 * logits: workspace/output, bf16 [T,E] (QWEN3, GPT_OSS) or fp32 [T,E]
 *   (NATIVE). With logits_given != 0 the GEMV is skipped and the selection
 *   runs on the caller's logits (used to test selection on identical inputs).
 * counts: int32 [E] or NULL; zeroed and filled on the stream.
 */
#define B200MOE_ROUTER_QWEN3 0
#define B200MOE_ROUTER_GPT_OSS 1
#define B200MOE_ROUTER_NATIVE 2

int b200moe_router(int device, void* stream, int mode, const void* hidden,
                   long long ld_hidden, const void* weight, const void* bias, int T, int H,
                   int E, int K, int normalize, void* logits, void* probs, void* scores,
                   long long* indices, int* counts, int logits_given);

/* Compact routing record of one router call (the per-layer capture of
 * moe_serving/record_routing.py:71-77: expert ids as int16, routing weights
 * as fp16): out_indices[i] = (int16) indices[i], out_scores[i] =
 * fp16_rn(scores[i]) for i < n, scores fp32 (scores_bf16 = 0) or bf16 (1).
 * Written on the device so a recorder reads a whole step back with one
 * copy instead of converting and copying at every layer. Ids must fit int16. */
int b200moe_route_record(int device, void* stream, const long long* indices, const void* scores,
                         int scores_bf16, long long n, void* out_indices, void* out_scores);

/* Dynamic FP8 activation quantisation of the W8A8 ("efficient") FP8 path
 * (moe_serving/efficient_kernels.py:243-274, the activation side of the hub
 * finegrained-fp8 matmul_grouped): per row r and 128-column group g,
 * s[r,g] = amax / 448 over the group's bf16 values (1 for an all-zero
 * group) and q[r,c] = e4m3fn(x[src(r),c] / s[r,g]), round to nearest even,
 * saturating at +-448; q = 0 for k_valid <= c < k_pad.
 * x: bf16 rows of stride ldx elements; src(r) = map[r] / map_div when map is
 * given (the permuted-row gather perm_src / K), else r. q: e4m3 [rows, k_pad];
 * s: fp32 [rows, ceil(k_pad / 128)]. Needs k_valid % 4 == 0, ldx % 4 == 0,
 * k_pad % 16 == 0 and k_valid <= k_pad.
 * row_offsets (device int32 [E+1], b200moe_permute's offsets) or NULL: when
 * given, only rows r in [row_offsets[expert_lo], row_offsets[expert_hi]) are
 * quantised (the rows of one rank's experts; the others are left unwritten,
 * as the rank's GEMM never reads them). */
int b200moe_act_quant_fp8(int device, void* stream, const void* x, long long ldx, const int* map,
                          int map_div, int rows, int k_valid, int k_pad, void* q, float* s,
                          const int* row_offsets, int expert_lo, int expert_hi);

/* ------------------------------------------------------------ permutation
 * Expert-contiguous permutation of the T*K (token, slot) assignments.
 * Within an expert, rows are ordered slot-major then by token, the order of
 * torch.where(indices.T == e) in moe_serving/parallel_numerics.py:21-26 (and
 * the native Transformers expert loop). Replaces that host loop and the
 * sort/histc bookkeeping of moe_serving/efficient_kernels.py:244-253 and
 * :160-178.
 *
 * indices: int64 [T,K] global expert ids. Outputs (int32): counts [E],
 * offsets [E+1] (exclusive prefix of counts), perm_src [T*K] (permuted row
 * -> t*K + k), inverse [T*K] (t*K + k -> permuted row, -1 if dropped).
 * Ids outside [0,E) are dropped and flagged with B200MOE_STATUS_BAD_INDEX.
 */
int b200moe_permute_workspace(int T, int K, int E, size_t* bytes);
int b200moe_permute(int device, void* stream, const long long* indices, int T, int K, int E,
                    int* counts, int* offsets, int* perm_src, int* inverse, void* workspace,
                    size_t workspace_bytes);

/* Permutation without a caller workspace (no counterpart in the reference,
 * whose bookkeeping runs on the host). Same arguments, outputs, ordering and
 * errors as b200moe_permute; the per-chunk histograms live in one fixed
 * device array of B200MOE_PERMUTE_SCRATCH_BYTES per device instead of the
 * workspace, so the call makes no allocation (no cudaMalloc/cudaFree, no
 * allocating library call). It is for callers that cannot allocate: a host
 * binding that owns only buffers pre-sized by its engine's memory planner,
 * and a serving step that must not call cudaMalloc/cudaFree because those
 * can synchronise the whole device and stall its other streams.
 *
 * Limit: b200moe_permute_workspace(T, K, E) must be at most
 * B200MOE_PERMUTE_SCRATCH_BYTES (1 MiB: e.g. T*K up to 2,097,152 at E = 128);
 * larger problems return B200MOE_ERR_UNSUPPORTED.
 * Setup: the first call on a device looks up the array's address on that
 * device; make that first call before any stream capture.
 * Zeroing: none needed; every scratch word a call reads was written earlier
 * in the same call.
 * Races: calls on one device share the array, so calls that overlap in time
 * (different streams without an ordering between them, or different host
 * threads) race; order them on one stream or with events.
 */
#define B200MOE_PERMUTE_SCRATCH_BYTES (1u << 20)

int b200moe_permute_noalloc(int device, void* stream, const long long* indices, int T, int K,
                            int E, int* counts, int* offsets, int* perm_src, int* inverse);

/* ------------------------------------------------------------ grouped GEMM
 * One launch computes, for every expert in [expert_begin, expert_begin +
 * n_experts) and every permuted row of that expert, either
 *   gated (planes = 2): act[r, f] = epilogue(x_r . Wgate[e,f], x_r . Wup[e,f])
 *   down  (planes = 1): out[r, f] = epilogue(a_r . Wdown[e,f])
 * on tcgen05 tensor cores (BF16 x BF16 -> FP32 in TMEM) by a persistent
 * kernel (one CTA per SM looping over (expert, token tile, feature tile)
 * tiles; gated tiles cover 64 features, down tiles 128). Weights, logically
 * [n_experts][planes][feat_pad][k_pad], are passed as
 *   B200MOE_W_BF16     bf16 in that layout (K contiguous)
 *   B200MOE_W_FP8      e4m3 with fp32 block scales (block sc_br x sc_bc),
 *                      converted on chip to bf16(fp32(w) * scale), the
 *                      arithmetic of moe_serving/qwen3_parallel.py:48-53
 *   B200MOE_W_MXFP4    e2m1 pairs (low nibble first) with ue8m0 scales per
 *                      32 values, decoded exactly to bf16 as transformers'
 *                      _convert_moe_packed_tensors does (called at
 *                      moe_serving/gpt_oss_parallel.py:183-193)
 * Quantised weights are packed once at load time into blobs, one per
 * (expert, feature tile, 64-column k-block), stored
 * [n_experts][feat_pad / tile_rows_per_plane][k_pad / 64][blob_bytes]:
 *   rows: a feature tile is 64 features of both planes (rows 0-63 gate,
 *     64-127 up) when planes = 2, or 128 features when planes = 1;
 *   data: 128 rows of 64 bytes (FP8) or 32 bytes (MXFP4), the 16-byte chunk
 *     c of row r stored at chunk position c ^ ((r >> 1) & 3) (FP8) or
 *     c ^ ((r >> 2) & 1) (MXFP4);
 *   scales after the data: FP8 with sc_br and sc_bc multiples of 64, the
 *     fp32 scales of rows 0-63 and 64-127 then 8 zero bytes (blob 8208 B);
 *     other FP8 blocks, fp32 [128 rows][4 chunks of 16 columns] (blob
 *     10240 B); MXFP4, ue8m0 [128 rows][2 groups of 32 columns] (blob 4352 B).
 * Quantised weights are converted by the CTA into tensor memory: up to
 * 128-token tiles beside 8 A stages, 160-token tiles beside 6, both with two
 * accumulator slots; with a 256-token tile the accumulator has one slot (the
 * epilogue of a tile does not overlap the next tile's main loop).
 * Epilogues:
 *   B200MOE_EPI_SWIGLU     bf16(bf16(silu(bf16 g)) * bf16 u)
 *                          (moe_serving/qwen3_parallel.py:84-94)
 *   B200MOE_EPI_CLAMP_SWIGLU  +bias, clamp(g<=limit, |u|<=limit),
 *                          g*sigmoid(alpha g)*(u+1), bf16 after each op
 *                          (moe_serving/gpt_oss_parallel.py:195-202)
 *   B200MOE_EPI_DOWN       bf16(acc) (+bias, bf16), then optionally
 *                          * routing weight of the row, bf16
 *                          (gpt_oss_parallel.py:203-204,
 *                          parallel_numerics.py:27)
 * Replaces the per-expert loops of qwen3_parallel.py:84-118 and
 * gpt_oss_parallel.py:195-244 and the grouped kernels called at
 * efficient_kernels.py:255-269 and :188-205.
 */
#define B200MOE_W_BF16 0
#define B200MOE_W_FP8 1
#define B200MOE_W_MXFP4 2

#define B200MOE_EPI_SWIGLU 0
#define B200MOE_EPI_CLAMP_SWIGLU 1
#define B200MOE_EPI_DOWN 2
/* The fused MXFP4 path of the reference's efficient GPT-OSS numerics
 * (matmul_ogs with a fused SwiGLU and fp32 biases, efficient_kernels.py:157-206,
 * biases cast to fp32 at gpt_oss_parallel.py:438-446): fp32 throughout the
 * epilogue. CLAMP_SWIGLU_F32 (gated): g = acc_g + bias_g, u = acc_u + bias_u,
 * g = min(g, limit), u = clamp(u, -limit, limit), out = bf16(g / (1 +
 * exp(-alpha g)) * (u + 1)). DOWN_F32: out is fp32, out = acc + bias (no
 * rounding, no row weight; ldo in floats, a multiple of 4). */
#define B200MOE_EPI_CLAMP_SWIGLU_F32 3
#define B200MOE_EPI_DOWN_F32 4

typedef struct b200moe_gemm_args {
  /* rows */
  const int* offsets;   /* [E_global + 1] permuted-row offsets (device) */
  int expert_begin;     /* first global expert id handled by this launch */
  int n_experts;        /* local experts in the weight stack */
  int max_rows;         /* upper bound on rows of these experts (T*K) */
  int token_tile;       /* 0 = choose (a power of two covering 1.5x the mean rows per
                           expert; 160 instead of 256 for quantised weights);
                           else 16, 32, 64, 128, 160 or 256 */
  int split_k;          /* reserved: must be 0 or 1 */
  /* weights (A operand) */
  int wfmt;             /* B200MOE_W_* */
  int planes;           /* 2 = gated gate/up, 1 = single projection */
  int feat_pad;         /* padded features per plane, multiple of 128 */
  int n_feat;           /* valid features per plane */
  int k_pad;            /* padded reduction length, multiple of 64 */
  const void* weight;   /* device: bf16 tiles or packed blobs (above) */
  int sc_br, sc_bc;     /* FP8 scale block, selects the blob's scale form */
  /* activations (B operand): row r reads b_src[src(r) * ldb + k], k < k_valid,
     src(r) = b_map ? b_map[r] / b_div : r */
  const void* b_src;
  long long ldb;
  int b_rows;           /* rows of b_src (tokens T, or T*K permuted rows) */
  int k_valid;
  const int* b_map;
  int b_div;
  /* epilogue */
  int epilogue;         /* B200MOE_EPI_* */
  const void* bias;     /* bf16 [n_experts][planes][feat_pad] or NULL */
  float alpha, limit;
  const void* row_weight;   /* routing weights [T*K] (fp32 or bf16) or NULL */
  int row_weight_bf16;
  const int* row_src;       /* permuted row -> t*K + k (for row_weight) */
  void* out;                /* bf16, row r at out + r * ldo */
  long long ldo;
} b200moe_gemm_args;

int b200moe_expert_gemm(int device, void* stream, const b200moe_gemm_args* args);

/* sizeof(b200moe_gemm_args), so foreign bindings can check their mirror. */
size_t b200moe_gemm_args_size(void);

/* W8A8 grouped GEMM of the reference's efficient FP8 mode: replaces the
 * hub finegrained-fp8 matmul_grouped calls of grouped_fp8
 * (moe_serving/efficient_kernels.py:255-265). The B operand is e4m3 token
 * rows already quantised per (row, 128-column group) by
 * b200moe_act_quant_fp8, in permuted row order: q [b_rows, k_pad] and
 * q_scale fp32 [b_rows, ceil(k_pad / 128)]. Weights are the packed FP8
 * blobs of b200moe_expert_gemm (wfmt = B200MOE_W_FP8, scale blocks of a
 * multiple of 64 rows x 128 columns). For weight row f and permuted row n:
 *   D[n, f] = sum_g sw[f, g] * q_scale[n, g] * sum_{k in g} W[f, k] * q[n, k]
 * (tensor-core fp32 inner sums, fp32 promotion). Epilogues: planes = 2 with
 * B200MOE_EPI_SWIGLU writes bf16(bf16(silu(bf16 gate)) * bf16 up) (the
 * reference's act_fn(gate) * up on the bf16 GEMM output); planes = 1 with
 * B200MOE_EPI_DOWN writes bf16(D), times the row's routing weight when
 * row_weight is given (bf16(bf16(D) * w)). b_src, ldb, k_valid, b_map and
 * bias must be NULL / unused; token_tile is 0 (choose) or 16, 32, 64, 128. */
int b200moe_w8a8_gemm(int device, void* stream, const b200moe_gemm_args* args, const void* q,
                      const float* q_scale);

/* ------------------------------------------------------------ combine
 * out[t, :] = ordered bf16 sum over the slots k of token t of the
 * contribution rows c[inverse[t*K+k], :], starting from bf16 zero and
 * rounding to bf16 after every add (index_add_ on a bf16 tensor).
 *   order B200MOE_ORDER_EXPERT: ascending global expert id — the order of
 *     moe_serving/parallel_numerics.py:21-35 (ordered_expert_merge)
 *   order B200MOE_ORDER_RANK_SLOT: ascending (expert / experts_per_rank,
 *     slot) — the order of index_add_ over the dest-sorted rows at
 *     moe_serving/moe.py:123-136
 * Only experts in [expert_lo, expert_hi) are added (the rank-local partial
 * sum of the reference's fast mode, qwen3_parallel.py:105-118).
 * scale_rows != 0: the contribution is bf16(f32(c) * w[t*K+k]) (weights fp32
 * or bf16); otherwise rows are already scaled (EPI_DOWN with row_weight).
 *   order B200MOE_ORDER_SLOT_SUM: the local combine of the reference's W8A8
 *     path (grouped_fp8, moe_serving/efficient_kernels.py:269-273:
 *     values * weights.to(bf16), masked rows 0, then
 *     values[inverse].reshape(T, K, H).sum(1)). The contribution of slot k is
 *     bf16(f32(c) * f32(bf16(w[t*K+k]))) with scale_rows (c as is without);
 *     slots that are dropped or outside [expert_lo, expert_hi) are +0. The
 *     sum is torch's CUDA reduction over the slot dimension: fp32
 *     accumulators a[k % 4] += contribution in ascending k, then
 *     ((a0 + a1) + a2) + a3, rounded once to bf16. experts_per_rank unused.
 */
#define B200MOE_ORDER_EXPERT 0
#define B200MOE_ORDER_RANK_SLOT 1
#define B200MOE_ORDER_SLOT_SUM 2

int b200moe_combine(int device, void* stream, const void* rows, long long ld_rows,
                    const int* inverse, const long long* indices, int T, int K, int H,
                    int order, int experts_per_rank, int expert_lo, int expert_hi,
                    int scale_rows, const void* weights, int weights_bf16, void* out,
                    long long ld_out);

/* The shared expert as one more routed slot of every token (the shared
 * expert of moe_serving/moe.py:84-95, added to the routed output at
 * moe.py:161-162), so that one permutation, one pair of grouped GEMMs and
 * one combine cover both: for t < T,
 *   out_indices[t][k] = indices[t][k], out_weights[t][k] = bf16(weights[t][k])
 *     for k < K (weights fp32 or bf16 [T][K]);
 *   out_indices[t][K] = shared_expert,
 *   out_weights[t][K] = bf16(1 / (1 + exp(-f32(score_logit[t * ld_logit]))))
 *     (score_logit: the bf16 [T, 1] output of F.linear(hidden, score); the
 *     value torch.sigmoid gives for it).
 * out_indices int64 [T][K+1], out_weights bf16 [T][K+1]. K < 32. With the
 * shared expert packed as expert shared_expert of the launch and the combine
 * in RANK_SLOT order over K + 1 slots, the result is bitwise the routed sum
 * plus the shared expert's output (one more bf16 add). */
int b200moe_append_shared_slot(int device, void* stream, const long long* indices, const void* weights,
                               int weights_bf16, const void* score_logit, long long ld_logit, int T, int K,
                               long long shared_expert, long long* out_indices, void* out_weights);

/* The scatter-reduce of the reference's fused MXFP4 path (matmul_ogs with
 * gammas and a scatter index, efficient_kernels.py:195-205), replacing the
 * index_add_-order combine there: rows are the fp32 outputs of
 * B200MOE_EPI_DOWN_F32 (acc + bias), each (token, slot) row is scaled by
 * its routing weight and rounded to bf16 (matmul_ogs's epilogue stores the
 * gamma-scaled rows in the output dtype), and the token's rows are summed in
 * fp32 (its grouped reduction):
 *   out[t, :] = bf16( sum over k = 0 .. K-1 in order of
 *                     fp32(bf16(rows[inverse[t*K+k], :] * fp32(weights[t*K+k]))) )
 * over the slots whose expert is in [expert_lo, expert_hi). weights fp32 or
 * bf16 [T][K]. H % 4 == 0. */
int b200moe_combine_f32(int device, void* stream, const float* rows, long long ld_rows,
                        const int* inverse, const long long* indices, int T, int K, int H,
                        int expert_lo, int expert_hi, const void* weights, int weights_bf16, void* out,
                        long long ld_out);

/* ------------------------------------------------------------ row gather
 * dst[i, :H] = src[map[i] / div, :H] for i < n (bf16 rows; a negative
 * map[i], a dropped assignment, gives a zero row). The dispatch
 * packing of moe_serving/moe.py:127 (hidden[token_index[order]]) and the
 * un-permute of received rows.
 */
int b200moe_gather_rows(int device, void* stream, const void* src, long long ld_src,
                        const int* map, int div, int n, int H, void* dst, long long ld_dst);

/* ------------------------------------------------------------ NVLink exchange
 * Fused combine + all-reduce of the replicated-token expert-parallel layer
 * ("fast" numerics, moe_serving/qwen3_parallel.py:105-118: every rank
 * combines its own experts' rows, the [T, H] partial sums are all-reduced)
 * in one kernel over peer memory, replacing b200moe_combine (expert order,
 * [expert_lo, expert_hi)) followed by an NCCL all-reduce:
 *   out[t] = bf16( sum over ranks p = 0 .. world-1 in order of
 *                  fp32(partial_p[t]) ),
 *   partial_p[t] = rank p's ordered combine of its experts' rows (bf16
 *                  running sum, b200moe_combine's arithmetic).
 * Every rank owns one exchange buffer of b200moe_p2p_buffer_bytes(t_cap, H,
 * world) bytes from b200moe_p2p_alloc (zeroed): per-block flags, an inbox
 * that ranks push partial rows into and an area for finished rows. Up to
 * 16 MiB pushed per rank (T * H * 2 * (world - 1)) every rank pushes its
 * partial rows to every rank (one-shot); above, each row goes to one owner
 * rank, which sums it and pushes the finished row to every rank (two-shot).
 * The result is the same either way. Two-shot needs a world size of 2, 4 or
 * 8 (B200MOE_ERR_UNSUPPORTED otherwise). It is exported with b200moe_p2p_export
 * and mapped by the other ranks with b200moe_p2p_import (CUDA IPC; plain
 * peer loads and stores over NVLink, no multicast objects). peers[world] are
 * the buffers' addresses in this process, peers[rank] the local one. All
 * ranks must call with the same T (<= t_cap), K, H, world, in the same order;
 * calls are ordered by per-block epochs kept inside the buffers (block b
 * owns rows t = b mod 1024), so they can be captured in a CUDA graph and
 * replayed. A peer that does not arrive within
 * timeout_ns (0: 2 s) sets B200MOE_STATUS_PEER_TIMEOUT; those rows of out are
 * then not written. world <= 8, K <= 32, H % 8 == 0.
 */
size_t b200moe_p2p_buffer_bytes(int t_cap, int H, int world);
int b200moe_p2p_alloc(int device, size_t bytes, void** out_ptr);
int b200moe_p2p_free(int device, void* ptr);
/* handle: 64 bytes (cudaIpcMemHandle_t) */
int b200moe_p2p_export(int device, void* ptr, unsigned char* handle);
int b200moe_p2p_import(int device, const unsigned char* handle, void** out_ptr);
int b200moe_p2p_close(int device, void* ptr);
int b200moe_combine_allreduce(int device, void* stream, const void* rows, long long ld_rows,
                              const int* inverse, const long long* indices, int T, int K, int H,
                              int expert_lo, int expert_hi, int scale_rows, const void* weights,
                              int weights_bf16, int world, int rank, void* const* peers,
                              int t_cap, void* out, long long ld_out,
                              unsigned long long timeout_ns);

/* As b200moe_gather_rows, restricted to the rows [offsets[expert_lo],
 * offsets[expert_hi]) (device offsets of b200moe_permute, 0 <= expert_lo <=
 * expert_hi <= E): the rows of one rank's experts under expert parallelism.
 * Other rows of dst are left as they are. */
int b200moe_gather_rows_range(int device, void* stream, const void* src, long long ld_src,
                              const int* map, int div, int n, int H, void* dst, long long ld_dst,
                              const int* offsets, int expert_lo, int expert_hi);

/* ------------------------------------------------------------ token all-to-all
 * Receive-side plan of the dispatch exchange of moe_serving/moe.py:123-131
 * (collective.exchange of rows grouped by destination rank). After the
 * exchange a rank holds rows grouped by source rank and, inside a source, by
 * local expert. counts: int32 [ep * experts_per_rank], counts[s * el + e] =
 * rows source s sent for local expert e. Outputs (int32):
 *   offsets [el + 1]  expert-major segment starts (sources ascending inside
 *                     an expert, each source's rows in arrival order)
 *   map_in  [rows]    expert-major position -> arrival row
 *   map_back[rows]    arrival row -> expert-major position
 * rows must equal the sum of counts (else B200MOE_STATUS_BAD_TILE is raised
 * in the device status). ep * experts_per_rank <= 1024.
 */
int b200moe_a2a_recv_plan(int device, void* stream, const int* counts, int ep,
                          int experts_per_rank, int rows, int* offsets, int* map_in,
                          int* map_back);

/* ------------------------------------------------------------ one call per expert layer
 * The whole single-GPU expert layer of ParallelExperts.forward
 * (moe_serving/qwen3_parallel.py:96-118, gpt_oss_parallel.py:206-244 with
 * ParallelGroup(1); parallel_numerics.ordered_expert_merge, :13-36) in one
 * call: b200moe_permute of the routing, the row gather (token tiles of 64 or
 * more), the gate/up and down grouped GEMMs (b200moe_expert_gemm with the
 * automatic token tile of 1.5x the mean rows per expert, at most 160 for
 * quantised weights) and b200moe_combine in ascending global expert order.
 * Results are those of the separate calls, bit for bit. The weights are the
 * packed stacks b200moe_expert_gemm takes (w1 gate/up, planes 2, feat_pad =
 * ceil(I/128)*128, k_pad = ceil(H/64)*64; w2 down, feat_pad = ceil(H/128)*128,
 * k_pad = feat_pad of w1; optional bf16 biases b1 / b2). workspace:
 * b200moe_layer_workspace(args) bytes of device memory the call may
 * overwrite, 256-byte aligned; it must not be in use by another call that
 * may run at the same time. out: bf16 [T][ldo].
 */
typedef struct b200moe_layer_args {
  const long long* indices;   /* [T][K] global expert ids (device) */
  const void* weights;        /* [T][K] routing weights, fp32 or bf16 (device) */
  int weights_bf16;
  int T, K, E;                /* tokens, top-k, global experts */
  int expert_begin;           /* global id of the stack's first expert */
  const void* hidden;         /* bf16 [T][ldh] */
  long long ldh;
  int H, I;                   /* hidden and intermediate sizes */
  int wfmt, n_experts;        /* B200MOE_W_*, experts in the stacks */
  const void* w1;
  const void* w2;
  const void* b1;
  const void* b2;
  int sc_br, sc_bc;           /* FP8 scale block */
  int gated_epilogue;         /* B200MOE_EPI_SWIGLU or B200MOE_EPI_CLAMP_SWIGLU */
  float alpha, limit;
  void* out;
  long long ldo;
} b200moe_layer_args;

size_t b200moe_layer_workspace(const b200moe_layer_args* args);
int b200moe_expert_layer(int device, void* stream, const b200moe_layer_args* args, void* workspace,
                         size_t workspace_bytes);
/* sizeof(b200moe_layer_args), so foreign bindings can check their mirror. */
size_t b200moe_layer_args_size(void);

/* ------------------------------------------------------------ peer-memory row exchanges
 * The token all-to-all of moe_serving/moe.py:110-137 (replacing the three
 * ProcessGroupCollective.exchange calls of distributed.py:33-46, each an
 * NCCL count exchange, a host read of the split sizes and an
 * all_to_all_single) and the replicated-token exact gather of
 * moe_serving/parallel_numerics.py:13-36 (every expert's contribution rows on
 * every rank), over NVLink peer memory.
 *
 * Every rank of the group owns one buffer of b200moe_peer_rows_bytes(H,
 * cap_a, cap_b) bytes from b200moe_p2p_alloc (zeroed), exported and imported
 * with b200moe_p2p_export / b200moe_p2p_import like the combine buffers;
 * peers[world] are the buffers' addresses in this process, peers[rank] the
 * local one. A buffer is a 64 KB header (flags, the count board, placements),
 * area A [cap_a][H] bf16 at byte offset 65536 and area B [cap_b][H] bf16
 * after it. All ranks call the same sequence of functions with the same E,
 * H, world and caps; each waits (bounded, timeout_ns, 0: 2 s) for the other
 * ranks of its phase and sets B200MOE_STATUS_PEER_TIMEOUT when one does not
 * arrive. A row that would fall outside an area is skipped and sets
 * B200MOE_STATUS_BAD_TILE. world <= 8, E <= 1024, E % world == 0, H % 8 == 0.
 *
 * Token all-to-all, per layer call (rank r holds its own tokens):
 *   b200moe_a2a_counts    counts: int32 [E], this rank's rows per global
 *                         expert (b200moe_permute's counts). Exchanges them
 *                         with every rank and writes recv_offsets (int32
 *                         [E / world + 1], device): the receive-area segment
 *                         starts of this rank's experts. Area A of rank d will
 *                         hold d's experts' rows in (expert, source rank,
 *                         source's permuted order) order; cap_a bounds the
 *                         received rows (world * max tokens per rank * K),
 *                         cap_b this rank's own rows (tokens * K).
 *   b200moe_a2a_dispatch  pushes row j of this rank's permutation (hidden row
 *                         perm_src[j] / K, expert indices[perm_src[j]]) into
 *                         its owner's area A; returns once every rank's rows
 *                         for this rank have landed. The grouped GEMMs then
 *                         read area A in place with recv_offsets.
 *   b200moe_a2a_return    y: [cap_a][ldy] bf16, the expert outputs in receive
 *                         order; pushes every row back to its source's area B
 *                         at the source's own permuted position, and returns
 *                         once this rank's rows have all come back. Area B
 *                         rows [0, T * K) are then the returned rows in this
 *                         rank's permuted order (combine them with
 *                         b200moe_combine, order RANK_SLOT, as moe.py:134-136
 *                         adds them).
 * Replicated-token exact gather:
 *   b200moe_ep_gather     rows [offsets[expert_lo], offsets[expert_hi]) of
 *                         this rank's area A (its experts' contribution rows,
 *                         written there by the down GEMM) are copied to the
 *                         same rows of every other rank's area A; returns once
 *                         every rank's rows have landed here, so area A holds
 *                         all rows_total rows for the ordered combine.
 */
size_t b200moe_peer_rows_bytes(int H, long long cap_a, long long cap_b);
int b200moe_a2a_counts(int device, void* stream, void* const* peers, int world, int rank, int E,
                       const int* counts, int* recv_offsets, long long cap_a, long long cap_b,
                       unsigned long long timeout_ns);
int b200moe_a2a_dispatch(int device, void* stream, void* const* peers, int world, int rank, int E,
                         const void* hidden, long long ldh, int H, const long long* indices,
                         const int* perm_src, const int* offsets, int rows, int K,
                         long long cap_a, unsigned long long timeout_ns);
int b200moe_a2a_return(int device, void* stream, void* const* peers, int world, int rank, int E,
                       const void* y, long long ldy, int H, long long cap_a, long long cap_b,
                       unsigned long long timeout_ns);
int b200moe_ep_gather(int device, void* stream, void* const* peers, int world, int rank, int H,
                      const int* offsets, int expert_lo, int expert_hi, int rows_total,
                      long long cap_a, unsigned long long timeout_ns);

#ifdef __cplusplus
}
#endif

#endif /* B200MOE_H_ */
