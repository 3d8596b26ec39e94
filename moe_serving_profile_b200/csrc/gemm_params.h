// Kernel parameters of the grouped expert GEMM (host-filled, passed by value).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace b200 {

struct GemmParams {
  const int* offsets;
  int expert_begin, n_experts, bn, ks, feat_tiles;
  int wfmt, planes, feat_pad, n_feat, k_pad, nkb;
  const float* fp8_scale;
  int sc_br, sc_bc, sc_nbr, sc_nbc;
  const uint8_t* mx_scale;
  int mx_groups;
  const __nv_bfloat16* b_src;
  long long ldb;
  int k_valid;
  const int* b_map;
  int b_div;
  int epi;
  const __nv_bfloat16* bias;
  float alpha, limit;
  const void* row_w;
  int row_w_bf16;
  const int* row_src;
  __nv_bfloat16* out;
  long long ldo;
  int* status;
  int nr, na, nb;
  uint32_t raw_off, a_off, b_off, red_off, bar_off, tmem_cols;
};

// Address of the grouped GEMM kernel (for cudaLaunchKernelExC).
const void* gemm_kernel_ptr();

}  // namespace b200
