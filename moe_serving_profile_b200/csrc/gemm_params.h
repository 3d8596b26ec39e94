// Kernel parameters of the grouped expert GEMM (host-filled, passed by value).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

struct GemmParams {
  // rows: permuted-row offsets of the global experts, this launch's slice
  const int* offsets;
  int expert_begin, n_experts;
  int bn;            // token tile (MMA N): 16..256
  // weights (MMA A): 128 rows per tile. Gated: 64 gate + 64 up rows of the
  // same 64 features; down: 128 features.
  int wfmt, gated, feat_tile, feat_tiles, feat_pad, n_feat, k_pad, nkb;
  // quantised weights: one blob per (expert, feature tile, k-block) of
  // blob_bytes (128 rows of e4m3 / e2m1 bytes, then the k-block's scales in
  // form scale_form: 0 FP8 one fp32 per 64-row half, 1 FP8 fp32 per (row,
  // 16-column chunk), 2 MXFP4 two ue8m0 bytes per row), staged in shared
  // memory every stage_bytes
  const uint8_t* wblob;
  uint32_t blob_bytes, stage_bytes;
  int scale_form;
  // activations (MMA B): rows gathered by token (b_map / b_div) or contiguous
  int b_gather;
  const int* b_map;
  int b_div;
  // epilogue
  int epi;
  const __nv_bfloat16* bias;
  float alpha, limit;
  const void* row_w;
  int row_w_bf16;
  const int* row_src;
  __nv_bfloat16* out;
  long long ldo;
  int* status;
  // pipeline plan: nr raw weight stages in shared memory (quantised
  // weights), na A stages (BF16 weights: shared memory; quantised weights:
  // tensor memory at column a_col0, 32 columns each), nb token-row stages
  int nr, na, nb;
  // accumulator banks per tile: CTA-wide k-block i accumulates into bank
  // i % nacc (independent MMA chains; the epilogue adds the banks in order);
  // banks used per tile = min(nacc, nkb)
  int nacc, nbanks;
  // MMA issuer threads (2 when nacc is even: k-block i goes to issuer i % 2)
  int n_issuers;
  // accumulator slots (2: tile t + 1 accumulates while tile t's epilogue
  // drains; 1: 256-token tiles of quantised weights, whose A stages take the
  // other half of tensor memory)
  int acc_slots;
  // joint_ab: A and B rings have the same number of stages and k-block i
  // uses stage i % na of both, so one commit to a_empty releases both (the
  // token-row producer waits on a_empty; b_empty is unused)
  int joint_ab;
  // a_smem (quantised weights, token tiles up to 256): the converters write
  // the bf16 weight tile into shared-memory A stages (128-byte-swizzled
  // K-major, the layout a TMA SWIZZLE_128B load produces), all eight
  // converter warps share every k-block, and tensor memory holds two
  // accumulator slots of bn columns. An expert's rows are cut into
  // ceil(rows / bn) chunks of equal size (rounded up to 16, the MMA's N
  // granule), each chunk one tile whose MMA N is its row count rounded up
  // to 16; token rows arrive as 64-row TMA boxes.
  int a_smem;
  uint32_t raw_off, a_off, b_off, x_off, bar_off, tmem_cols, a_col0;
};

// Address of the grouped GEMM kernel (for cudaLaunchKernelExC).
const void* gemm_kernel_ptr();

// Kernel parameters of the register-operand decode GEMM (quantised weights,
// token tiles of 16 or 32 rows). Weights, epilogue and tile order as
// GemmParams; token rows are contiguous permuted rows, read through a 2D
// tensor map (64-column boxes of bn rows, 128-byte swizzle).
struct DecodeParams {
  const int* offsets;
  int expert_begin, n_experts;
  int bn;            // 16 or 32 token rows per tile
  int wfmt, gated, feat_tiles, feat_pad, n_feat, nkb;
  const uint8_t* wblob;
  uint32_t blob_bytes;
  int scale_form;
  int epi;
  const __nv_bfloat16* bias;
  float alpha, limit;
  const void* row_w;
  int row_w_bf16;
  const int* row_src;
  void* out;
  long long ldo;
  int* status;
  // ring of nr stages (nr even): weight blobs every stage_bytes from 0, the
  // token boxes (bn x 128 bytes each) from tok_off (1024-byte aligned); the
  // warp pairs' accumulator exchange at x_off; barriers and the tile prefix
  // at bar_off
  int nr;
  uint32_t stage_bytes, tok_off, x_off, bar_off;
};

// Largest dynamic shared memory of a decode GEMM launch, and the device
// ordinals the launcher tracks.
constexpr uint32_t kDecodeSmemMax = 232448u - 1024u;
constexpr int kDecodeMaxDevices = 64;

// Launch the decode GEMM: one CTA of 576 threads per SM, smem bytes of
// dynamic shared memory (at most kDecodeSmemMax), tmap the token rows'
// tensor map. Returns a cudaError_t.
int launch_decode_gemm(const CUtensorMap& tmap, const DecodeParams& p, int grid, uint32_t smem,
                       cudaStream_t stream);

}  // namespace b200
