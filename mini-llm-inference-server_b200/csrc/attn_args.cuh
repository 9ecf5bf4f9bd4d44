// Kernel parameters of the paged-attention launch, shared by the kernels and the C-ABI layer.
#pragma once

#include "common.cuh"

namespace mlb {

struct AttnArgs {
  const char* q;
  int64_t q_st, q_sh;  // q strides (tokens, heads) in elements
  const char* k_cache;
  const char* v_cache;
  int64_t num_blocks;
  int h, hkv, group, tile_tokens;
  float sl2;  // softmax scale * log2(e)
  const int32_t* bt;
  int64_t bt_stride;
  const int32_t* seq_lens;
  const int32_t* qo;
  const mlb_work_unit* units;
  const mlb_shared_unit* shared_units;
  const mlb_share_member* members;
  float* part_o;
  float* part_lse;
  char* out;
  int64_t o_st, o_sh;  // out strides (tokens, heads) in elements
  int32_t* err;
};

}  // namespace mlb
