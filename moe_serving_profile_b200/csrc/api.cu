// C ABI of the b200moe library: argument validation, launch shapes, TMA
// descriptors and the per-device status word. See include/b200moe.h.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <algorithm>

#include "b200moe.h"
#include "gemm_params.h"
#include "internal.h"
#include "ptx.cuh"

// One status word per device: kernels OR StatusBits into it.
__device__ int g_b200moe_status;

namespace {

thread_local std::string t_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_error = buf;
  return code;
}

#define B200_CUDA(expr)                                                                   \
  do {                                                                                    \
    cudaError_t e_ = (expr);                                                              \
    if (e_ != cudaSuccess)                                                                \
      return fail(B200MOE_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_));     \
  } while (0)

#define B200_CHECK(cond, ...)                                \
  do {                                                       \
    if (!(cond)) return fail(B200MOE_ERR_INVALID, __VA_ARGS__); \
  } while (0)

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int* g_status_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
bool g_gemm_attr[kMaxDevices] = {};
bool g_w8a8_attr[kMaxDevices][4] = {};
void* g_permute_scratch_ptr[kMaxDevices] = {};

int use_device(int device, int** status) {
  B200_CHECK(device >= 0 && device < kMaxDevices, "device %d out of range", device);
  B200_CUDA(cudaSetDevice(device));
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_status_ptr[device] == nullptr) {
    void* p = nullptr;
    B200_CUDA(cudaGetSymbolAddress(&p, g_b200moe_status));
    g_status_ptr[device] = static_cast<int*>(p);
    int sms = 0;
    B200_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    g_sm_count[device] = sms;
  }
  if (status) *status = g_status_ptr[device];
  return B200MOE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

int pow2_ceil(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

}  // namespace

extern "C" {

const char* b200moe_last_error(void) { return t_error.c_str(); }

const char* b200moe_version(void) { return "b200moe 0.1 (sm_100a)"; }

size_t b200moe_gemm_args_size(void) { return sizeof(b200moe_gemm_args); }

int b200moe_device_status(int device, int clear, int* out_status) {
  int* sp = nullptr;
  int rc = use_device(device, &sp);
  if (rc) return rc;
  B200_CHECK(out_status != nullptr, "out_status is NULL");
  B200_CUDA(cudaDeviceSynchronize());
  int v = 0;
  B200_CUDA(cudaMemcpy(&v, sp, sizeof(int), cudaMemcpyDeviceToHost));
  *out_status = v;
  if (clear) {
    const int zero = 0;
    B200_CUDA(cudaMemcpy(sp, &zero, sizeof(int), cudaMemcpyHostToDevice));
  }
  return B200MOE_OK;
}

int b200moe_router(int device, void* stream, int mode, const void* hidden, long long ld_hidden,
                   const void* weight, const void* bias, int T, int H, int E, int K,
                   int normalize, void* logits, void* probs, void* scores, long long* indices,
                   int* counts, int logits_given) {
  B200_CHECK(mode >= B200MOE_ROUTER_QWEN3 && mode <= B200MOE_ROUTER_NATIVE, "bad router mode %d", mode);
  B200_CHECK(T >= 0 && E >= 1 && K >= 1, "bad sizes T=%d E=%d K=%d", T, E, K);
  if (E > 512 || K > 32 || K > E)
    return fail(B200MOE_ERR_UNSUPPORTED, "router supports E <= 512 and K <= min(32, E) (E=%d K=%d)", E, K);
  B200_CHECK(T == 0 || (logits && scores && indices), "logits, scores and indices are required");
  if (mode == B200MOE_ROUTER_GPT_OSS) B200_CHECK(bias != nullptr, "GPT-OSS router needs a bias");
  if (!logits_given && T > 0) {
    B200_CHECK(hidden && weight, "hidden and weight are required");
    if (H % 8 != 0 || H > 8192)
      return fail(B200MOE_ERR_UNSUPPORTED, "router needs H %% 8 == 0 and H <= 8192 (H=%d)", H);
    B200_CHECK(aligned16(hidden) && aligned16(weight) && ld_hidden % 8 == 0 && ld_hidden >= H,
               "hidden/weight must be 16-byte aligned with ld %% 8 == 0");
  }
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (counts) B200_CUDA(cudaMemsetAsync(counts, 0, sizeof(int) * E, st));
  if (T == 0) return B200MOE_OK;
  if (!logits_given) {
    B200_CUDA(b200::launch_router_logits(st, mode, hidden, ld_hidden, weight,
                                         mode == B200MOE_ROUTER_NATIVE ? nullptr : bias, T, H, E,
                                         logits));
  }
  B200_CUDA(b200::launch_router_select(st, mode, logits, T, E, K, normalize,
                                       mode == B200MOE_ROUTER_QWEN3 ? probs : nullptr, scores,
                                       indices, counts));
  return B200MOE_OK;
}

int b200moe_route_record(int device, void* stream, const long long* indices, const void* scores,
                         int scores_bf16, long long n, void* out_indices, void* out_scores) {
  B200_CHECK(n >= 0 && (scores_bf16 == 0 || scores_bf16 == 1), "bad record arguments");
  if (n == 0) return B200MOE_OK;
  B200_CHECK(indices && scores && out_indices && out_scores, "indices, scores and outputs are required");
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  B200_CUDA(b200::launch_route_record(static_cast<cudaStream_t>(stream), indices, scores, scores_bf16, n,
                                      out_indices, out_scores));
  return B200MOE_OK;
}

int b200moe_act_quant_fp8(int device, void* stream, const void* x, long long ldx, const int* map,
                          int map_div, int rows, int k_valid, int k_pad, void* q, float* s,
                          const int* row_offsets, int expert_lo, int expert_hi) {
  B200_CHECK(rows >= 0 && k_valid >= 0 && k_pad >= k_valid, "bad sizes rows=%d k_valid=%d k_pad=%d", rows,
             k_valid, k_pad);
  B200_CHECK(k_valid % 4 == 0 && k_pad % 16 == 0 && ldx % 4 == 0 && ldx >= k_valid,
             "need k_valid %% 4 == 0, k_pad %% 16 == 0, ldx %% 4 == 0 and ldx >= k_valid");
  B200_CHECK(map == nullptr || map_div >= 1, "map_div must be >= 1");
  B200_CHECK((long long)rows * ((k_pad + 127) / 128) < (1ll << 40), "too many groups");
  B200_CHECK(row_offsets == nullptr || (expert_lo >= 0 && expert_hi >= expert_lo), "bad expert range");
  if (rows == 0 || k_pad == 0) return B200MOE_OK;
  B200_CHECK(x && q && s, "x, q and s are required");
  B200_CHECK(reinterpret_cast<uintptr_t>(x) % 8 == 0 && reinterpret_cast<uintptr_t>(q) % 4 == 0,
             "x must be 8-byte and q 4-byte aligned");
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  B200_CUDA(b200::launch_act_quant(static_cast<cudaStream_t>(stream), x, ldx, map, map_div, rows, k_valid,
                                   k_pad, q, s, row_offsets, expert_lo, expert_hi));
  return B200MOE_OK;
}

int b200moe_permute_workspace(int T, int K, int E, size_t* bytes) {
  B200_CHECK(bytes != nullptr, "bytes is NULL");
  B200_CHECK(T >= 0 && K >= 1 && E >= 1, "bad sizes");
  *bytes = b200::permute_workspace_bytes(T, K, E);
  return B200MOE_OK;
}

int b200moe_permute(int device, void* stream, const long long* indices, int T, int K, int E,
                    int* counts, int* offsets, int* perm_src, int* inverse, void* workspace,
                    size_t workspace_bytes) {
  B200_CHECK(T >= 0 && K >= 1 && E >= 1, "bad sizes T=%d K=%d E=%d", T, K, E);
  if (E > 1024) return fail(B200MOE_ERR_UNSUPPORTED, "permute supports E <= 1024 (E=%d)", E);
  B200_CHECK((long long)T * K < (1ll << 30), "T*K too large");
  B200_CHECK(counts && offsets, "counts and offsets are required");
  const bool empty = (long long)T * K == 0;
  const size_t need = b200::permute_workspace_bytes(T, K, E);
  if (!empty) {
    B200_CHECK(indices && perm_src && inverse, "indices, perm_src and inverse are required");
    B200_CHECK(workspace_bytes >= need && (need == 0 || workspace != nullptr),
               "permute workspace too small: %zu < %zu", workspace_bytes, need);
  }
  int* sp = nullptr;
  int rc = use_device(device, &sp);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (empty) {
    B200_CUDA(cudaMemsetAsync(counts, 0, sizeof(int) * E, st));
    B200_CUDA(cudaMemsetAsync(offsets, 0, sizeof(int) * (E + 1), st));
    return B200MOE_OK;
  }
  B200_CUDA(b200::launch_permute(st, indices, T, K, E, counts, offsets, perm_src, inverse,
                                 workspace, sp));
  return B200MOE_OK;
}

int b200moe_permute_noalloc(int device, void* stream, const long long* indices, int T, int K,
                            int E, int* counts, int* offsets, int* perm_src, int* inverse) {
  B200_CHECK(T >= 0 && K >= 1 && E >= 1, "bad sizes T=%d K=%d E=%d", T, K, E);
  if (E > 1024) return fail(B200MOE_ERR_UNSUPPORTED, "permute supports E <= 1024 (E=%d)", E);
  B200_CHECK((long long)T * K < (1ll << 30), "T*K too large");
  B200_CHECK(counts && offsets, "counts and offsets are required");
  const bool empty = (long long)T * K == 0;
  if (!empty) B200_CHECK(indices && perm_src && inverse, "indices, perm_src and inverse are required");
  const size_t need = b200::permute_workspace_bytes(T, K, E);
  if (need > B200MOE_PERMUTE_SCRATCH_BYTES)
    return fail(B200MOE_ERR_UNSUPPORTED,
                "permute_noalloc needs %zu scratch bytes, more than its fixed %u (T=%d K=%d E=%d)",
                need, B200MOE_PERMUTE_SCRATCH_BYTES, T, K, E);
  int* sp = nullptr;
  int rc = use_device(device, &sp);
  if (rc) return rc;
  void* scratch = nullptr;
  {
    // first call on this device: look up the array's address with the device current
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_permute_scratch_ptr[device] == nullptr) {
      void* p = nullptr;
      B200_CUDA(b200::permute_static_scratch(&p));
      g_permute_scratch_ptr[device] = p;
    }
    scratch = g_permute_scratch_ptr[device];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (empty) {
    B200_CUDA(cudaMemsetAsync(counts, 0, sizeof(int) * E, st));
    B200_CUDA(cudaMemsetAsync(offsets, 0, sizeof(int) * (E + 1), st));
    return B200MOE_OK;
  }
  B200_CUDA(b200::launch_permute(st, indices, T, K, E, counts, offsets, perm_src, inverse,
                                 scratch, sp));
  return B200MOE_OK;
}

int b200moe_expert_gemm(int device, void* stream, const b200moe_gemm_args* a) {
  B200_CHECK(a != nullptr, "args is NULL");
  if (a->max_rows <= 0) return B200MOE_OK;
  B200_CHECK(a->offsets && a->weight && a->b_src && a->out, "offsets, weight, b_src, out are required");
  B200_CHECK(a->wfmt >= B200MOE_W_BF16 && a->wfmt <= B200MOE_W_MXFP4, "bad weight format %d", a->wfmt);
  B200_CHECK(a->planes == 1 || a->planes == 2, "planes must be 1 or 2");
  B200_CHECK(a->epilogue >= B200MOE_EPI_SWIGLU && a->epilogue <= B200MOE_EPI_DOWN_F32, "bad epilogue");
  const bool down_epi = a->epilogue == B200MOE_EPI_DOWN || a->epilogue == B200MOE_EPI_DOWN_F32;
  B200_CHECK(down_epi == (a->planes == 1),
             "gated epilogues need planes == 2, the down epilogues planes == 1");
  B200_CHECK(a->epilogue != B200MOE_EPI_DOWN_F32 || (a->row_weight == nullptr && a->ldo % 4 == 0),
             "the fp32 down epilogue takes no row weights and needs ldo %% 4 == 0");
  B200_CHECK(a->n_experts >= 1 && a->expert_begin >= 0, "bad expert range");
  if (a->n_experts > 1024) return fail(B200MOE_ERR_UNSUPPORTED, "at most 1024 experts per launch");
  B200_CHECK(a->feat_pad >= 128 && a->feat_pad % 128 == 0, "feat_pad must be a positive multiple of 128");
  B200_CHECK(a->n_feat >= 1 && a->n_feat <= a->feat_pad, "n_feat out of range");
  B200_CHECK(a->k_pad >= 64 && a->k_pad % 64 == 0, "k_pad must be a positive multiple of 64");
  B200_CHECK(a->k_valid >= 1 && a->k_valid <= a->k_pad && a->k_valid % 8 == 0,
             "k_valid must be in [1, k_pad] and a multiple of 8");
  B200_CHECK(a->ldb >= a->k_valid && a->ldb % 8 == 0 && aligned16(a->b_src), "B rows must be 16-byte aligned");
  B200_CHECK(a->b_rows >= 1, "b_rows must be positive");
  B200_CHECK(aligned16(a->weight), "weight must be 16-byte aligned");
  B200_CHECK(a->ldo >= a->n_feat, "ldo too small");
  B200_CHECK(a->ldo % 8 == 0 && a->n_feat % 8 == 0 && aligned16(a->out),
             "output rows must be 16-byte aligned (ldo %% 8 == 0, n_feat %% 8 == 0)");
  B200_CHECK(a->b_map == nullptr || a->b_div >= 1, "b_div must be >= 1");
  if (a->wfmt == B200MOE_W_FP8)
    B200_CHECK(a->sc_br >= 1 && a->sc_bc >= 16 && a->sc_bc % 16 == 0,
               "fp8 weights need a scale block with columns a multiple of 16");
  if (a->row_weight) B200_CHECK(a->row_src != nullptr, "row_weight needs row_src");
  B200_CHECK(a->token_tile == 0 || a->token_tile == 16 || a->token_tile == 32 ||
                 a->token_tile == 64 || a->token_tile == 128 || a->token_tile == 160 ||
                 a->token_tile == 256,
             "token_tile must be 0, 16, 32, 64, 128, 160 or 256");
  if (a->split_k > 1) return fail(B200MOE_ERR_UNSUPPORTED, "split_k > 1 is not implemented");
  B200_CHECK(a->split_k >= 0, "split_k must be 0 or 1");
  int* sp = nullptr;
  int rc = use_device(device, &sp);
  if (rc) return rc;

  const bool gated = a->planes == 2;
  int bn = a->token_tile;
  if (bn == 0) {
    // quantised weights: at most 160 tokens, the largest tile with two
    // accumulator slots beside the tensor-memory A stages
    const int max_auto = a->wfmt == B200MOE_W_BF16 ? 256 : 160;
    // 1.5x the mean rows per expert, so that one tile usually holds an
    // expert's rows
    const long long avg = (3ll * a->max_rows + 2ll * a->n_experts - 1) / (2ll * a->n_experts);
    bn = std::min(max_auto, std::max(16, pow2_ceil(static_cast<int>(std::min(avg, 1ll << 20)))));
  }
  // quantised weights at 256-row tiles: converted weights in shared-memory A
  // stages (the tensor-memory A stages leave room for one 256-column slot)
  const bool a_smem = a->wfmt != B200MOE_W_BF16 && bn == 256 && a->b_map == nullptr;
  const int feat_tile = gated ? 64 : 128;
  const int feat_tiles = a->feat_pad / feat_tile;
  const long long tiles_ub =
      (long long)(std::min(a->n_experts, a->max_rows) + a->max_rows / bn) * feat_tiles;

  // shared memory plan: raw weight ring, bf16 A ring, token-row ring, epilogue
  // exchange buffer, barriers + tile prefix
  // quantised weights: one blob per (expert, feature tile, k-block), staged
  // on 1024-byte boundaries
  const bool fp8_half = a->sc_br % 64 == 0 && a->sc_bc % 64 == 0;
  const uint32_t blob_bytes = a->wfmt == B200MOE_W_FP8 ? 8192u + (fp8_half ? 16u : 2048u)
                              : (a->wfmt == B200MOE_W_MXFP4 ? 4096u + 256u : 0u);
  const uint32_t rpb = (blob_bytes + 1023u) & ~1023u;
  if (a->wfmt != B200MOE_W_BF16 && (bn == 16 || bn == 32) && a->b_map == nullptr) {
    // short token tiles over contiguous permuted rows: the register-operand
    // decode kernel (decode.cu). Shared memory: nr weight stages (blob on a
    // 128-byte boundary), nr token boxes of bn x 128 bytes from a 1024-byte
    // boundary, the warp pairs' double-buffered accumulator exchange (4
    // pairs x 2 x 32 lanes x bn / 2 floats), then full/empty barriers per stage,
    // the tile total and the tile prefix.
    b200::DecodeParams d{};
    d.offsets = a->offsets;
    d.expert_begin = a->expert_begin;
    d.n_experts = a->n_experts;
    d.bn = bn;
    d.wfmt = a->wfmt;
    d.gated = gated ? 1 : 0;
    d.feat_tiles = feat_tiles;
    d.feat_pad = a->feat_pad;
    d.n_feat = a->n_feat;
    d.nkb = a->k_pad / 64;
    d.wblob = static_cast<const uint8_t*>(a->weight);
    d.blob_bytes = blob_bytes;
    d.scale_form = a->wfmt == B200MOE_W_MXFP4 ? 2 : (fp8_half ? 0 : 1);
    d.epi = a->epilogue;
    d.bias = static_cast<const __nv_bfloat16*>(a->bias);
    d.alpha = a->alpha;
    d.limit = a->limit;
    d.row_w = a->row_weight;
    d.row_w_bf16 = a->row_weight_bf16;
    d.row_src = a->row_src;
    d.out = a->out;
    d.ldo = a->ldo;
    d.status = sp;
    d.stage_bytes = (blob_bytes + 127u) & ~127u;
    const uint32_t tok_stage = static_cast<uint32_t>(bn) * 128u;
    const uint32_t xb = 4u * 2u * 32u * static_cast<uint32_t>(bn) * 4u;
    const uint32_t tail = 8u + 4u * static_cast<uint32_t>(a->n_experts + 1);
    const uint32_t room = b200::kDecodeSmemMax - 1024u - 1024u - xb - tail;
    d.nr = std::min<int>(32, static_cast<int>(room / (d.stage_bytes + tok_stage + 16u))) & ~1;
    if (d.nr < 4) return fail(B200MOE_ERR_UNSUPPORTED, "decode shared memory plan does not fit");
    d.tok_off = (static_cast<uint32_t>(d.nr) * d.stage_bytes + 1023u) & ~1023u;
    d.x_off = d.tok_off + static_cast<uint32_t>(d.nr) * tok_stage;
    d.bar_off = d.x_off + xb;
    const uint32_t smem = d.bar_off + 16u * static_cast<uint32_t>(d.nr) + tail + 1024u;   // + alignment slack
    PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
    if (!enc) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    CUtensorMap tmap;
    std::memset(&tmap, 0, sizeof(tmap));
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a->k_valid), static_cast<cuuint64_t>(a->b_rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a->ldb) * 2};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(bn)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult cr = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a->b_src), dims, strides, box,
                      estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(B200MOE_ERR_CUDA, "activation tensor map failed (%d)", (int)cr);
    const int grid = static_cast<int>(std::min<long long>(g_sm_count[device], tiles_ub));
    const int e = b200::launch_decode_gemm(tmap, d, grid, smem, static_cast<cudaStream_t>(stream));
    if (e != 0) return fail(B200MOE_ERR_CUDA, "decode GEMM launch failed: %s",
                            cudaGetErrorString(static_cast<cudaError_t>(e)));
    return B200MOE_OK;
  }
  const uint32_t a_stage = 128u * 128u;
  const uint32_t b_stage = static_cast<uint32_t>(bn) * 128u;
  // epilogue: exchange buffer (8 KB), two bf16 staging chunks (8 KB), row weights (1 KB)
  const uint32_t xbytes = 8192u + 8192u + 1024u;
  const uint32_t barbytes = (((96u * 8u + 16u + 4u * (a->n_experts + 1)) + 1023u) / 1024u) * 1024u;
  const uint32_t budget = 232448u - 2048u;
  // BF16 weights: a ring of na shared-memory A stages filled by TMA and nb
  // token-row stages. Quantised weights: na = 8 tensor-memory A stages (TMEM
  // columns 256..511, beside the two accumulator slots of at most 128 columns
  // each), nb token-row stages and as many raw stages as fit (even, <= 24).
  int na = 0, nb = 0, nr = 0;
  if (a_smem) {
    // A and token-row stages in step (one commit releases both), then as
    // many raw stages as fit, at most 8
    na = nb = 3;
    const uint32_t fixed = na * a_stage + nb * b_stage + xbytes + barbytes;
    nr = fixed < budget ? static_cast<int>((budget - fixed) / rpb) : 0;
    nr = std::min(8, nr);
    if (nr < 3)
      return fail(B200MOE_ERR_UNSUPPORTED, "shared memory plan does not fit (token_tile=%d)", bn);
  } else if (rpb == 0) {
    na = 8;
    nb = 6;
    auto total = [&](int a_, int b_) { return a_ * a_stage + b_ * b_stage + xbytes + barbytes; };
    while (total(na, nb) > budget) {
      if (nb > 3) --nb;
      else if (na > 4) --na;
      else if (nb > 2) --nb;
      else if (na > 2) --na;
      else break;
    }
    if (total(na, nb) > budget)
      return fail(B200MOE_ERR_UNSUPPORTED, "shared memory plan does not fit (token_tile=%d)", bn);
  } else {
    // token-row stages: 8, matching the A stages (one commit releases both),
    // while at least 8 raw stages still fit; else 4. A 160-token tile keeps
    // two accumulator slots (columns 0..319) beside 6 A stages (320..511).
    na = bn == 160 ? 6 : 8;
    nb = na;
    if (nb * b_stage + xbytes + barbytes + 8 * rpb > budget) nb = 4;
    const uint32_t fixed = nb * b_stage + xbytes + barbytes;
    nr = fixed < budget ? static_cast<int>((budget - fixed) / rpb) : 0;
    nr = std::min(24, nr) & ~1;
    if (nr < 4)
      return fail(B200MOE_ERR_UNSUPPORTED, "shared memory plan does not fit (token_tile=%d)", bn);
  }

  b200::GemmParams p{};
  p.offsets = a->offsets;
  p.expert_begin = a->expert_begin;
  p.n_experts = a->n_experts;
  p.bn = bn;
  p.wfmt = a->wfmt;
  p.gated = gated ? 1 : 0;
  p.feat_tile = feat_tile;
  p.feat_tiles = feat_tiles;
  p.feat_pad = a->feat_pad;
  p.n_feat = a->n_feat;
  p.k_pad = a->k_pad;
  p.nkb = a->k_pad / 64;
  p.wblob = static_cast<const uint8_t*>(a->weight);
  p.blob_bytes = blob_bytes;
  p.stage_bytes = rpb;
  p.scale_form = a->wfmt == B200MOE_W_MXFP4 ? 2 : (fp8_half ? 0 : 1);
  p.b_gather = a->b_map != nullptr ? 1 : 0;
  p.b_map = a->b_map;
  p.b_div = a->b_map ? a->b_div : 1;
  p.epi = a->epilogue;
  p.bias = static_cast<const __nv_bfloat16*>(a->bias);
  p.alpha = a->alpha;
  p.limit = a->limit;
  p.row_w = a->row_weight;
  p.row_w_bf16 = a->row_weight_bf16;
  p.row_src = a->row_src;
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.ldo = a->ldo;
  p.status = sp;
  p.nr = nr;
  p.na = na;
  p.nb = nb;
  uint32_t off = 0;
  p.raw_off = off;
  off += nr * rpb;
  p.a_off = off;
  if (rpb == 0 || a_smem) off += na * a_stage;
  p.b_off = off;
  off += nb * b_stage;
  p.x_off = off;
  off += xbytes;
  p.bar_off = off;
  off += barbytes;
  const uint32_t smem = off + 1024u;  // + alignment slack
  // independent accumulator chains for short token tiles: 2 slots x nacc
  // banks x bn columns stay within the 256 columns below the A stages
  p.nacc = std::max(1, std::min(4, 128 / bn));
  p.nbanks = std::min(p.nacc, p.nkb);
  // quantised weights keep their A stages in TMEM columns 256..511, so a
  // 256-token tile gets a single accumulator slot
  p.acc_slots = (rpb && bn > 160 && !a_smem) ? 1 : 2;
  p.a_smem = a_smem ? 1 : 0;
  p.joint_ab = na == nb ? 1 : 0;
  // two MMA issuers when there are banks for both and the A / B rings split
  // evenly between them
  p.n_issuers = (p.nacc % 2 == 0 && na % 2 == 0 && nb % 2 == 0) ? 2 : 1;
  p.tmem_cols = (rpb && !a_smem) ? 512u
                                 : static_cast<uint32_t>(std::max(32, pow2_ceil(p.acc_slots * p.nacc * bn)));
  p.a_col0 = (rpb && bn == 160) ? 320u : 256u;

  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (!enc) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  // BF16 weights: [n_experts * planes * feat_pad rows] x [k_pad] tiles
  CUtensorMap wmap, bmap;
  std::memset(&wmap, 0, sizeof(wmap));
  if (a->wfmt == B200MOE_W_BF16) {
    const cuuint64_t rows = static_cast<cuuint64_t>(a->n_experts) * a->planes * a->feat_pad;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a->k_pad), rows};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a->k_pad) * 2};
    const cuuint32_t box[2] = {64, gated ? 64u : 128u};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
    CUresult cr = enc(&wmap, dt, 2, const_cast<void*>(a->weight), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(B200MOE_ERR_CUDA, "weight tensor map failed (%d)", (int)cr);
  }
  // token rows: [b_rows] x [k_valid] bf16 (columns past k_valid read as zero);
  // one-row boxes for tile::gather4, token_tile-row boxes for contiguous rows
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a->k_valid), static_cast<cuuint64_t>(a->b_rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a->ldb) * 2};
    const cuuint32_t box[2] = {64, a->b_map ? 1u : (a_smem ? 64u : static_cast<cuuint32_t>(bn))};
    const cuuint32_t estr[2] = {1, 1};
    CUresult cr = enc(&bmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a->b_src), dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(B200MOE_ERR_CUDA, "activation tensor map failed (%d)", (int)cr);
  }

  const void* kern = b200::gemm_kernel_ptr();
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_gemm_attr[device]) {
      B200_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448 - 1024));
      g_gemm_attr[device] = true;
    }
  }
  const int grid = static_cast<int>(std::min<long long>(g_sm_count[device], tiles_ub));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(512, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  void* args[] = {&wmap, &bmap, &p};
  B200_CUDA(cudaLaunchKernelExC(&cfg, kern, args));
  return B200MOE_OK;
}

int b200moe_w8a8_gemm(int device, void* stream, const b200moe_gemm_args* a, const void* q,
                      const float* q_scale) {
  B200_CHECK(a != nullptr, "args is NULL");
  if (a->max_rows <= 0) return B200MOE_OK;
  B200_CHECK(a->offsets && a->weight && q && q_scale && a->out, "offsets, weight, q, q_scale, out are required");
  B200_CHECK(a->wfmt == B200MOE_W_FP8, "W8A8 needs FP8 weights");
  B200_CHECK(a->sc_br >= 64 && a->sc_br % 64 == 0 && a->sc_bc == 128,
             "W8A8 needs FP8 scale blocks of 128 columns and a multiple of 64 rows");
  B200_CHECK(a->planes == 1 || a->planes == 2, "planes must be 1 or 2");
  B200_CHECK((a->planes == 2 && a->epilogue == B200MOE_EPI_SWIGLU) ||
                 (a->planes == 1 && a->epilogue == B200MOE_EPI_DOWN),
             "W8A8 supports the SwiGLU gate/up and the down epilogues");
  B200_CHECK(a->bias == nullptr, "W8A8 has no bias");
  B200_CHECK(a->b_map == nullptr, "W8A8 reads quantised permuted rows (b_map must be NULL)");
  B200_CHECK(a->n_experts >= 1 && a->expert_begin >= 0, "bad expert range");
  if (a->n_experts > 1024) return fail(B200MOE_ERR_UNSUPPORTED, "at most 1024 experts per launch");
  B200_CHECK(a->feat_pad >= 128 && a->feat_pad % 128 == 0, "feat_pad must be a positive multiple of 128");
  B200_CHECK(a->n_feat >= 1 && a->n_feat <= a->feat_pad, "n_feat out of range");
  B200_CHECK(a->k_pad >= 64 && a->k_pad % 64 == 0, "k_pad must be a positive multiple of 64");
  B200_CHECK(a->b_rows >= 1 && aligned16(q), "q must be 16-byte aligned with b_rows >= 1");
  B200_CHECK(aligned16(a->weight), "weight must be 16-byte aligned");
  B200_CHECK(a->ldo >= a->n_feat && a->ldo % 8 == 0 && a->n_feat % 8 == 0 && aligned16(a->out),
             "output rows must be 16-byte aligned (ldo %% 8 == 0, n_feat %% 8 == 0)");
  if (a->row_weight) B200_CHECK(a->row_src != nullptr, "row_weight needs row_src");
  B200_CHECK(a->token_tile == 0 || a->token_tile == 16 || a->token_tile == 32 || a->token_tile == 64 ||
                 a->token_tile == 128,
             "W8A8 token_tile must be 0, 16, 32, 64 or 128");
  int* sp = nullptr;
  int rc = use_device(device, &sp);
  if (rc) return rc;

  const bool gated = a->planes == 2;
  int bn = a->token_tile;
  if (bn == 0) {
    const long long avg = (3ll * a->max_rows + 2ll * a->n_experts - 1) / (2ll * a->n_experts);
    bn = std::min(128, std::max(16, pow2_ceil(static_cast<int>(std::min(avg, 1ll << 20)))));
  }
  const int feat_tiles = a->feat_pad / (gated ? 64 : 128);
  const long long tiles_ub = (long long)(std::min(a->n_experts, a->max_rows) + a->max_rows / bn) * feat_tiles;

  b200::W8A8Params p{};
  p.offsets = a->offsets;
  p.expert_begin = a->expert_begin;
  p.n_experts = a->n_experts;
  p.gated = gated ? 1 : 0;
  p.feat_tiles = feat_tiles;
  p.n_feat = a->n_feat;
  p.nkb = a->k_pad / 64;
  p.ngroups = (p.nkb + 1) / 2;
  p.wblob = static_cast<const uint8_t*>(a->weight);
  p.blob_bytes = 8192u + 16u;   // e4m3 rows + one fp32 scale per 64-row half
  p.qs = q_scale;
  p.qs_groups = (a->k_pad + 127) / 128;
  p.row_w = a->row_weight;
  p.row_w_bf16 = a->row_weight_bf16;
  p.row_src = a->row_src;
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.ldo = a->ldo;
  p.status = sp;
  // shared memory: stages of (two 8 KB weight blobs + bn x 128 B token rows) on
  // 1024-byte boundaries, the epilogue buffers, barriers + tile prefix
  const uint32_t budget = 232448u - 2048u;
  p.stage_bytes = (16384u + static_cast<uint32_t>(bn) * 128u + 1023u) & ~1023u;   // one 128-column group
  const uint32_t xbytes = (b200::w8a8_epilogue_bytes(bn, p.gated) + 1023u) & ~1023u;
  const uint32_t nbuf = static_cast<uint32_t>(b200::w8a8_tmem_buffers(bn));
  // full/empty per stage, acc_full/acc_empty per TMEM buffer, mma_done; tmem
  // address, tile total, tile prefix
  const uint32_t barbytes =
      ((8u * (2u * 16u + 2u * nbuf + 1u) + 8u + 4u * (a->n_experts + 1) + 1023u) / 1024u) * 1024u;
  p.ns = static_cast<int>(std::min<uint32_t>(16u, (budget - xbytes - barbytes) / p.stage_bytes));
  if (p.ns < 2) return fail(B200MOE_ERR_UNSUPPORTED, "shared memory plan does not fit (token_tile=%d)", bn);
  p.x_off = p.ns * p.stage_bytes;
  p.bar_off = p.x_off + xbytes;
  const uint32_t smem = p.bar_off + barbytes + 1024u;   // + alignment slack
  p.tmem_cols = static_cast<uint32_t>(std::max(32, pow2_ceil(static_cast<int>(nbuf) * bn)));

  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (!enc) return fail(B200MOE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  CUtensorMap qmap;
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a->k_pad), static_cast<cuuint64_t>(a->b_rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a->k_pad)};
    const cuuint32_t box[2] = {128, static_cast<cuuint32_t>(bn)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult cr = enc(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(q), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(B200MOE_ERR_CUDA, "activation tensor map failed (%d)", (int)cr);
  }
  const int ti = bn == 16 ? 0 : bn == 32 ? 1 : bn == 64 ? 2 : 3;
  const void* kern = b200::w8a8_kernel_ptr(bn);
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_w8a8_attr[device][ti]) {
      B200_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448 - 1024));
      g_w8a8_attr[device][ti] = true;
    }
  }
  const int grid = static_cast<int>(std::min<long long>(g_sm_count[device], tiles_ub));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(b200::kW8A8Threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  void* args[] = {&qmap, &p};
  B200_CUDA(cudaLaunchKernelExC(&cfg, kern, args));
  return B200MOE_OK;
}

int b200moe_combine(int device, void* stream, const void* rows, long long ld_rows,
                    const int* inverse, const long long* indices, int T, int K, int H, int order,
                    int experts_per_rank, int expert_lo, int expert_hi, int scale_rows,
                    const void* weights, int weights_bf16, void* out, long long ld_out) {
  B200_CHECK(T >= 0 && K >= 1 && H >= 8, "bad sizes");
  if (K > 32 || H % 8 != 0) return fail(B200MOE_ERR_UNSUPPORTED, "combine needs K <= 32 and H %% 8 == 0");
  B200_CHECK(order == B200MOE_ORDER_EXPERT || order == B200MOE_ORDER_RANK_SLOT ||
                 order == B200MOE_ORDER_SLOT_SUM,
             "bad order");
  B200_CHECK(order != B200MOE_ORDER_RANK_SLOT || experts_per_rank >= 1, "experts_per_rank must be >= 1");
  if (T == 0) return B200MOE_OK;
  B200_CHECK(out && inverse && indices && rows, "rows, out, inverse and indices are required");
  B200_CHECK(!scale_rows || weights, "scale_rows needs weights");
  B200_CHECK(aligned16(rows) && aligned16(out) && ld_rows % 8 == 0 && ld_out % 8 == 0,
             "rows/out must be 16-byte aligned with ld %% 8 == 0");
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  B200_CUDA(b200::launch_combine(static_cast<cudaStream_t>(stream), rows, ld_rows, inverse, indices,
                                 T, K, H, order, experts_per_rank, expert_lo, expert_hi, scale_rows,
                                 weights, weights_bf16, out, ld_out));
  return B200MOE_OK;
}

int b200moe_append_shared_slot(int device, void* stream, const long long* indices, const void* weights,
                               int weights_bf16, const void* score_logit, long long ld_logit, int T, int K,
                               long long shared_expert, long long* out_indices, void* out_weights) {
  B200_CHECK(T >= 0 && K >= 1 && K < 32, "bad sizes (1 <= K < 32)");
  B200_CHECK(shared_expert >= 0 && ld_logit >= 1, "bad shared expert id or logit stride");
  if (T == 0) return B200MOE_OK;
  B200_CHECK(indices && weights && score_logit && out_indices && out_weights, "all pointers are required");
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  B200_CUDA(b200::launch_append_shared_slot(static_cast<cudaStream_t>(stream), indices, weights, weights_bf16,
                                            score_logit, ld_logit, T, K, shared_expert, out_indices, out_weights));
  return B200MOE_OK;
}

int b200moe_combine_f32(int device, void* stream, const float* rows, long long ld_rows,
                        const int* inverse, const long long* indices, int T, int K, int H,
                        int expert_lo, int expert_hi, const void* weights, int weights_bf16, void* out,
                        long long ld_out) {
  B200_CHECK(T >= 0 && K >= 1 && H >= 4, "bad sizes");
  if (H % 4 != 0) return fail(B200MOE_ERR_UNSUPPORTED, "combine_f32 needs H %% 4 == 0");
  if (T == 0) return B200MOE_OK;
  B200_CHECK(rows && inverse && indices && weights && out, "rows, inverse, indices, weights and out are required");
  B200_CHECK(aligned16(rows) && ld_rows % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 7) == 0 && ld_out % 4 == 0,
             "rows must be 16-byte aligned (ld %% 4 == 0), out 8-byte aligned (ld %% 4 == 0)");
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  B200_CUDA(b200::launch_combine_f32(static_cast<cudaStream_t>(stream), rows, ld_rows, inverse, indices, T, K,
                                     H, expert_lo, expert_hi, weights, weights_bf16, out, ld_out));
  return B200MOE_OK;
}

size_t b200moe_p2p_buffer_bytes(int t_cap, int H, int world) {
  if (t_cap < 0 || H < 8 || world < 1 || world > b200::kP2PMaxRanks) return 0;
  const size_t rows = 2ull * world * static_cast<size_t>(b200::p2p_inbox_rows(t_cap, H, world)) +
                      2ull * static_cast<size_t>(t_cap);
  return b200::kP2PHeaderBytes + rows * static_cast<size_t>(H) * 2ull;
}

int b200moe_p2p_alloc(int device, size_t bytes, void** out_ptr) {
  B200_CHECK(out_ptr != nullptr && bytes >= b200::kP2PHeaderBytes, "bad exchange buffer request");
  *out_ptr = nullptr;
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  void* p = nullptr;
  B200_CUDA(cudaMalloc(&p, bytes));   // its own allocation: the IPC handle covers exactly it
  const cudaError_t err = cudaMemset(p, 0, bytes);
  if (err != cudaSuccess) {
    cudaFree(p);
    return fail(B200MOE_ERR_CUDA, "exchange buffer clear failed: %s", cudaGetErrorString(err));
  }
  B200_CUDA(cudaDeviceSynchronize());
  *out_ptr = p;
  return B200MOE_OK;
}

int b200moe_p2p_free(int device, void* ptr) {
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  if (ptr) B200_CUDA(cudaFree(ptr));
  return B200MOE_OK;
}

int b200moe_p2p_export(int device, void* ptr, unsigned char* handle) {
  B200_CHECK(ptr && handle, "ptr and handle are required");
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  B200_CUDA(cudaIpcGetMemHandle(&h, ptr));
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
  std::memcpy(handle, &h, sizeof(h));
  return B200MOE_OK;
}

int b200moe_p2p_import(int device, const unsigned char* handle, void** out_ptr) {
  B200_CHECK(handle && out_ptr, "handle and out_ptr are required");
  *out_ptr = nullptr;
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  B200_CUDA(cudaIpcOpenMemHandle(out_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return B200MOE_OK;
}

int b200moe_p2p_close(int device, void* ptr) {
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  if (ptr) B200_CUDA(cudaIpcCloseMemHandle(ptr));
  return B200MOE_OK;
}

int b200moe_combine_allreduce(int device, void* stream, const void* rows, long long ld_rows,
                              const int* inverse, const long long* indices, int T, int K, int H,
                              int expert_lo, int expert_hi, int scale_rows, const void* weights,
                              int weights_bf16, int world, int rank, void* const* peers,
                              int t_cap, void* out, long long ld_out,
                              unsigned long long timeout_ns) {
  B200_CHECK(T >= 0 && K >= 1 && H >= 8 && t_cap >= 0, "bad sizes");
  if (K > 32 || H % 8 != 0)
    return fail(B200MOE_ERR_UNSUPPORTED, "combine_allreduce needs K <= 32 and H %% 8 == 0");
  if (world < 1 || world > b200::kP2PMaxRanks)
    return fail(B200MOE_ERR_UNSUPPORTED, "combine_allreduce supports 1..%d ranks", b200::kP2PMaxRanks);
  B200_CHECK(rank >= 0 && rank < world, "rank %d outside [0, %d)", rank, world);
  B200_CHECK(T <= t_cap, "T=%d exceeds the exchange buffer's %d rows", T, t_cap);
  if (!b200::p2p_supported(T, H, world))
    return fail(B200MOE_ERR_UNSUPPORTED,
                "exchanges above 16 MiB per rank need a world size dividing 1024 (world=%d)", world);
  B200_CHECK(peers != nullptr, "peers are required");
  for (int i = 0; i < world; ++i)
    B200_CHECK(peers[i] != nullptr && aligned16(peers[i]), "peer buffer %d missing or unaligned", i);
  B200_CHECK(!scale_rows || weights, "scale_rows needs weights");
  if (T > 0) {
    B200_CHECK(out && inverse && indices && rows, "rows, out, inverse and indices are required");
    B200_CHECK(aligned16(rows) && aligned16(out) && ld_rows % 8 == 0 && ld_out % 8 == 0,
               "rows/out must be 16-byte aligned with ld %% 8 == 0");
  }
  int* sp = nullptr;
  int rc = use_device(device, &sp);
  if (rc) return rc;
  B200_CUDA(b200::launch_combine_allreduce(static_cast<cudaStream_t>(stream), rows, ld_rows, inverse,
                                           indices, T, K, H, expert_lo, expert_hi, scale_rows,
                                           weights, weights_bf16, world, rank, peers, t_cap, out,
                                           ld_out, timeout_ns ? timeout_ns : b200::kWaitLimitNs, sp));
  return B200MOE_OK;
}

int b200moe_gather_rows_range(int device, void* stream, const void* src, long long ld_src,
                              const int* map, int div, int n, int H, void* dst, long long ld_dst,
                              const int* offsets, int expert_lo, int expert_hi) {
  B200_CHECK(n >= 0 && H >= 8 && div >= 1, "bad sizes");
  B200_CHECK(expert_lo >= 0 && expert_hi >= expert_lo, "bad expert range");
  if (H % 8 != 0) return fail(B200MOE_ERR_UNSUPPORTED, "gather_rows needs H %% 8 == 0");
  if (n == 0 || expert_hi == expert_lo) return B200MOE_OK;
  B200_CHECK(src && map && dst && offsets, "src, map, dst and offsets are required");
  B200_CHECK(aligned16(src) && aligned16(dst) && ld_src % 8 == 0 && ld_dst % 8 == 0,
             "rows must be 16-byte aligned with ld %% 8 == 0");
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  B200_CUDA(b200::launch_gather_rows_range(static_cast<cudaStream_t>(stream), src, ld_src, map, div,
                                           n, H, dst, ld_dst, offsets, expert_lo, expert_hi,
                                           32 * g_sm_count[device]));
  return B200MOE_OK;
}

int b200moe_gather_rows(int device, void* stream, const void* src, long long ld_src,
                        const int* map, int div, int n, int H, void* dst, long long ld_dst) {
  B200_CHECK(n >= 0 && H >= 8 && div >= 1, "bad sizes");
  if (H % 8 != 0) return fail(B200MOE_ERR_UNSUPPORTED, "gather_rows needs H %% 8 == 0");
  if (n == 0) return B200MOE_OK;
  B200_CHECK(src && map && dst, "src, map and dst are required");
  B200_CHECK(aligned16(src) && aligned16(dst) && ld_src % 8 == 0 && ld_dst % 8 == 0,
             "rows must be 16-byte aligned with ld %% 8 == 0");
  int rc = use_device(device, nullptr);
  if (rc) return rc;
  B200_CUDA(b200::launch_gather_rows(static_cast<cudaStream_t>(stream), src, ld_src, map, div, n, H,
                                     dst, ld_dst));
  return B200MOE_OK;
}

// ---------------------------------------------------------------- one call per expert layer
namespace {

struct LayerPlan {
  int bn, R;
  size_t off_counts, off_offsets, off_perm, off_inv, off_scratch, off_rows, off_act, off_contrib, total;
  size_t scratch;
  bool gather;
};

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

// Token tile of the separate-call path (experts.tile_policy): the smallest
// power of two from 16 covering 1.5x the mean rows per expert, capped at
// 256 (BF16) or 160 (quantised weights).
int layer_tile(int T, int K, int E, int wfmt) {
  const int max_tile = wfmt == B200MOE_W_BF16 ? 256 : 160;
  const double rows = 1.5 * static_cast<double>(T) * K / E;
  int bn = 16;
  while (bn < max_tile && bn < rows) bn *= 2;
  return std::min(bn, max_tile);
}

LayerPlan layer_plan(const b200moe_layer_args* a) {
  LayerPlan p{};
  p.R = a->T * a->K;
  p.bn = layer_tile(a->T, a->K, a->E, a->wfmt);
  // permuted rows gathered once: for large tiles (plain 2D TMA tiles
  // instead of per-row gathers) and for the decode kernel of quantised
  // weights, which reads contiguous rows only
  p.gather = p.bn >= 64 || a->wfmt != B200MOE_W_BF16;
  const size_t R = static_cast<size_t>(p.R);
  const size_t i_pad = static_cast<size_t>((a->I + 127) / 128 * 128);
  const size_t h_k = static_cast<size_t>((a->H + 63) / 64 * 64);
  p.scratch = b200::permute_workspace_bytes(a->T, a->K, a->E);
  size_t off = 0;
  p.off_counts = off;  off = align256(off + 4ull * a->E);
  p.off_offsets = off; off = align256(off + 4ull * (a->E + 1));
  p.off_perm = off;    off = align256(off + 4ull * R);
  p.off_inv = off;     off = align256(off + 4ull * R);
  p.off_scratch = off; off = align256(off + p.scratch);
  p.off_rows = off;    off = align256(off + (p.gather ? 2ull * R * h_k : 0));
  p.off_act = off;     off = align256(off + 2ull * R * i_pad);
  p.off_contrib = off; off = align256(off + 2ull * R * static_cast<size_t>(a->H));
  p.total = off;
  return p;
}

}  // namespace

size_t b200moe_layer_args_size(void) { return sizeof(b200moe_layer_args); }

size_t b200moe_layer_workspace(const b200moe_layer_args* a) {
  if (!a || a->T < 0 || a->K < 1 || a->E < 1 || a->H < 8 || a->I < 8) return 0;
  return layer_plan(a).total;
}

int b200moe_expert_layer(int device, void* stream, const b200moe_layer_args* a, void* workspace,
                         size_t workspace_bytes) {
  B200_CHECK(a != nullptr, "args is NULL");
  B200_CHECK(a->T >= 0 && a->K >= 1 && a->E >= 1 && a->H >= 8 && a->I >= 8, "bad sizes");
  B200_CHECK(a->n_experts >= 1 && a->expert_begin >= 0 && a->expert_begin + a->n_experts <= a->E,
             "bad expert range");
  B200_CHECK(a->gated_epilogue == B200MOE_EPI_SWIGLU || a->gated_epilogue == B200MOE_EPI_CLAMP_SWIGLU,
             "bad gated epilogue");
  if (a->T == 0) return B200MOE_OK;
  B200_CHECK((long long)a->T * a->K < (1ll << 30), "T*K too large");
  B200_CHECK(a->indices && a->weights && a->hidden && a->out && a->w1 && a->w2,
             "indices, weights, hidden, out, w1 and w2 are required");
  const LayerPlan p = layer_plan(a);
  B200_CHECK(workspace != nullptr && workspace_bytes >= p.total && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
             "workspace must be 256-byte aligned and hold %zu bytes (got %zu)", p.total, workspace_bytes);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* counts = reinterpret_cast<int*>(ws + p.off_counts);
  int* offsets = reinterpret_cast<int*>(ws + p.off_offsets);
  int* perm = reinterpret_cast<int*>(ws + p.off_perm);
  int* inv = reinterpret_cast<int*>(ws + p.off_inv);
  __nv_bfloat16* rows = reinterpret_cast<__nv_bfloat16*>(ws + p.off_rows);
  __nv_bfloat16* act = reinterpret_cast<__nv_bfloat16*>(ws + p.off_act);
  __nv_bfloat16* contrib = reinterpret_cast<__nv_bfloat16*>(ws + p.off_contrib);
  const int i_pad = (a->I + 127) / 128 * 128;
  const int h_k = (a->H + 63) / 64 * 64;
  const int h_f = (a->H + 127) / 128 * 128;
  int rc = b200moe_permute(device, stream, a->indices, a->T, a->K, a->E, counts, offsets, perm, inv,
                           ws + p.off_scratch, p.scratch);
  if (rc) return rc;
  const int lo = a->expert_begin, hi = a->expert_begin + a->n_experts;
  if (p.gather) {
    rc = b200moe_gather_rows_range(device, stream, a->hidden, a->ldh, perm, a->K, p.R, a->H, rows, h_k,
                                   offsets, lo, hi);
    if (rc) return rc;
  }
  b200moe_gemm_args g{};
  g.offsets = offsets;
  g.expert_begin = lo;
  g.n_experts = a->n_experts;
  g.max_rows = p.R;
  g.token_tile = p.bn;
  g.wfmt = a->wfmt;
  g.sc_br = a->sc_br;
  g.sc_bc = a->sc_bc;
  g.alpha = a->alpha;
  g.limit = a->limit;
  // gate / up
  g.planes = 2;
  g.feat_pad = i_pad;
  g.n_feat = a->I;
  g.k_pad = h_k;
  g.weight = a->w1;
  g.b_src = p.gather ? static_cast<const void*>(rows) : a->hidden;
  g.ldb = p.gather ? h_k : a->ldh;
  g.b_rows = p.gather ? p.R : a->T;
  g.k_valid = a->H;
  g.b_map = p.gather ? nullptr : perm;
  g.b_div = p.gather ? 1 : a->K;
  g.epilogue = a->gated_epilogue;
  g.bias = a->b1;
  g.out = act;
  g.ldo = i_pad;
  rc = b200moe_expert_gemm(device, stream, &g);
  if (rc) return rc;
  // down, scaled by the routing weights
  g.planes = 1;
  g.feat_pad = h_f;
  g.n_feat = a->H;
  g.k_pad = i_pad;
  g.weight = a->w2;
  g.b_src = act;
  g.ldb = i_pad;
  g.b_rows = p.R;
  g.k_valid = a->I;
  g.b_map = nullptr;
  g.b_div = 1;
  g.epilogue = B200MOE_EPI_DOWN;
  g.bias = a->b2;
  g.row_weight = a->weights;
  g.row_weight_bf16 = a->weights_bf16;
  g.row_src = perm;
  g.out = contrib;
  g.ldo = a->H;
  rc = b200moe_expert_gemm(device, stream, &g);
  if (rc) return rc;
  // a stack holding every expert combines every assignment, as the separate
  // combine call does (expert range [0, 2^30))
  const bool all = lo == 0 && hi == a->E;
  return b200moe_combine(device, stream, contrib, a->H, inv, a->indices, a->T, a->K, a->H,
                         B200MOE_ORDER_EXPERT, 1, all ? 0 : lo, all ? (1 << 30) : hi, 0, nullptr, 0,
                         a->out, a->ldo);
}

// ---------------------------------------------------------------- peer-memory row exchanges
size_t b200moe_peer_rows_bytes(int H, long long cap_a, long long cap_b) {
  if (H < 8 || cap_a < 0 || cap_b < 0) return 0;
  return b200::kPeerRowsHeaderBytes + static_cast<size_t>(cap_a + cap_b) * static_cast<size_t>(H) * 2ull;
}

static int check_peers(void* const* peers, int world, int rank) {
  if (world < 1 || world > b200::kP2PMaxRanks)
    return fail(B200MOE_ERR_UNSUPPORTED, "peer exchanges support 1..%d ranks", b200::kP2PMaxRanks);
  B200_CHECK(rank >= 0 && rank < world, "rank %d outside [0, %d)", rank, world);
  B200_CHECK(peers != nullptr, "peers are required");
  for (int i = 0; i < world; ++i)
    B200_CHECK(peers[i] != nullptr && aligned16(peers[i]), "peer buffer %d missing or unaligned", i);
  return B200MOE_OK;
}

int b200moe_a2a_counts(int device, void* stream, void* const* peers, int world, int rank, int E,
                       const int* counts, int* recv_offsets, long long cap_a, long long cap_b,
                       unsigned long long timeout_ns) {
  int rc = check_peers(peers, world, rank);
  if (rc) return rc;
  B200_CHECK(E >= 1 && cap_a >= 0 && cap_b >= 0, "bad sizes");
  if (E > 1024 || E % world != 0)
    return fail(B200MOE_ERR_UNSUPPORTED, "the all-to-all needs E <= 1024 and E %% world == 0");
  B200_CHECK(counts != nullptr, "counts are required");
  int* sp = nullptr;
  rc = use_device(device, &sp);
  if (rc) return rc;
  B200_CUDA(b200::launch_a2a_counts(static_cast<cudaStream_t>(stream), peers, world, rank, E, counts,
                                    recv_offsets, cap_a, cap_b,
                                    timeout_ns ? timeout_ns : b200::kWaitLimitNs, sp));
  return B200MOE_OK;
}

int b200moe_a2a_dispatch(int device, void* stream, void* const* peers, int world, int rank, int E,
                         const void* hidden, long long ldh, int H, const long long* indices,
                         const int* perm_src, const int* offsets, int rows, int K,
                         long long cap_a, unsigned long long timeout_ns) {
  int rc = check_peers(peers, world, rank);
  if (rc) return rc;
  B200_CHECK(E >= 1 && rows >= 0 && K >= 1 && cap_a >= 0, "bad sizes");
  if (E > 1024 || E % world != 0 || H % 8 != 0 || H < 8)
    return fail(B200MOE_ERR_UNSUPPORTED, "the all-to-all needs E <= 1024, E %% world == 0, H %% 8 == 0");
  B200_CHECK(offsets != nullptr, "offsets are required");
  if (rows > 0) {
    B200_CHECK(hidden && indices && perm_src, "hidden, indices and perm_src are required");
    B200_CHECK(aligned16(hidden) && ldh % 8 == 0 && ldh >= H, "hidden rows must be 16-byte aligned");
  }
  int* sp = nullptr;
  rc = use_device(device, &sp);
  if (rc) return rc;
  B200_CUDA(b200::launch_a2a_dispatch(static_cast<cudaStream_t>(stream), peers, world, rank, E, hidden,
                                      ldh, H, indices, perm_src, offsets, rows, K, cap_a,
                                      g_sm_count[device], timeout_ns ? timeout_ns : b200::kWaitLimitNs,
                                      sp));
  return B200MOE_OK;
}

int b200moe_a2a_return(int device, void* stream, void* const* peers, int world, int rank, int E,
                       const void* y, long long ldy, int H, long long cap_a, long long cap_b,
                       unsigned long long timeout_ns) {
  int rc = check_peers(peers, world, rank);
  if (rc) return rc;
  B200_CHECK(E >= 1 && cap_a >= 0 && cap_b >= 0, "bad sizes");
  if (E > 1024 || E % world != 0 || H % 8 != 0 || H < 8)
    return fail(B200MOE_ERR_UNSUPPORTED, "the all-to-all needs E <= 1024, E %% world == 0, H %% 8 == 0");
  if (cap_a > 0) B200_CHECK(y && aligned16(y) && ldy % 8 == 0 && ldy >= H, "y rows must be 16-byte aligned");
  int* sp = nullptr;
  rc = use_device(device, &sp);
  if (rc) return rc;
  B200_CUDA(b200::launch_a2a_return(static_cast<cudaStream_t>(stream), peers, world, rank, E, y, ldy, H,
                                    cap_a, cap_b, g_sm_count[device],
                                    timeout_ns ? timeout_ns : b200::kWaitLimitNs, sp));
  return B200MOE_OK;
}

int b200moe_ep_gather(int device, void* stream, void* const* peers, int world, int rank, int H,
                      const int* offsets, int expert_lo, int expert_hi, int rows_total,
                      long long cap_a, unsigned long long timeout_ns) {
  int rc = check_peers(peers, world, rank);
  if (rc) return rc;
  B200_CHECK(expert_lo >= 0 && expert_hi >= expert_lo && rows_total >= 0 && cap_a >= 0, "bad sizes");
  if (H % 8 != 0 || H < 8) return fail(B200MOE_ERR_UNSUPPORTED, "the gather needs H %% 8 == 0");
  B200_CHECK(offsets != nullptr, "offsets are required");
  B200_CHECK(rows_total <= cap_a, "rows_total %d exceeds area A's %lld rows", rows_total, cap_a);
  int* sp = nullptr;
  rc = use_device(device, &sp);
  if (rc) return rc;
  B200_CUDA(b200::launch_ep_gather(static_cast<cudaStream_t>(stream), peers, world, rank, H, offsets,
                                   expert_lo, expert_hi, rows_total, cap_a, g_sm_count[device],
                                   timeout_ns ? timeout_ns : b200::kWaitLimitNs, sp));
  return B200MOE_OK;
}

int b200moe_a2a_recv_plan(int device, void* stream, const int* counts, int ep,
                          int experts_per_rank, int rows, int* offsets, int* map_in,
                          int* map_back) {
  B200_CHECK(ep >= 1 && experts_per_rank >= 1 && rows >= 0, "bad sizes ep=%d el=%d rows=%d", ep,
             experts_per_rank, rows);
  if ((long long)ep * experts_per_rank > 1024)
    return fail(B200MOE_ERR_UNSUPPORTED, "a2a_recv_plan supports ep * experts_per_rank <= 1024");
  B200_CHECK(counts && offsets, "counts and offsets are required");
  B200_CHECK(rows == 0 || (map_in && map_back), "map_in and map_back are required");
  int* sp = nullptr;
  int rc = use_device(device, &sp);
  if (rc) return rc;
  B200_CUDA(b200::launch_a2a_recv_plan(static_cast<cudaStream_t>(stream), counts, ep,
                                       experts_per_rank, rows, offsets, map_in, map_back,
                                       g_sm_count[device], sp));
  return B200MOE_OK;
}

}  // extern "C"
