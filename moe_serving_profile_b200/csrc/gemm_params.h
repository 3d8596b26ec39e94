// Kernel parameters of the grouped expert GEMM (host-filled, passed by value).
#pragma once

#include <cuda_bf16.h>
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
  const float* fp8_scale;
  int sc_br, sc_bc, sc_nbr, sc_nbc;
  const uint8_t* mx_scale;
  int mx_groups;
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
  // shared-memory plan
  int nr, na, nb;
  uint32_t raw_off, a_off, b_off, x_off, bar_off, tmem_cols;
};

// Address of the grouped GEMM kernel (for cudaLaunchKernelExC).
const void* gemm_kernel_ptr();

}  // namespace b200
