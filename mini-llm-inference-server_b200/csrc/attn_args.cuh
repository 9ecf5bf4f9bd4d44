// Kernel parameters of the paged-attention launch, shared by the kernels and the C-ABI layer.
#pragma once

#include <type_traits>

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
  int64_t part_rows;  // rows of part_o / part_lse (writes beyond are skipped and flagged)
  mlb_out_targets out;  // final rows: one or more destinations (the call's `out`, or every rank's buffer)
  int out_vec;          // out_vec_ok(out): rows may be stored with packed 16-byte-aligned stores
  int32_t* err;
  // fused append (mlb_paged_attention_append), app_k == nullptr otherwise: the step's new rows, taken from
  // here for every page that holds them and stored into the pools at app_slots by the row's last query tile
  const char* app_k;
  const char* app_v;
  int64_t app_k_st, app_k_sh, app_v_st, app_v_sh;  // strides in elements
  const int64_t* app_slots;
};

// Query tokens per 8-column tile of the per-sequence kernel (columns = tokens x query heads of one KV head).
// The planner numbers partial rows with it and the split-K reduction reads them with it: every entry point
// takes it from here.
inline int tokens_per_tile(int num_heads, int num_kv_heads) {
  const int group = num_heads / num_kv_heads;
  return group >= 8 ? 1 : 8 / group;
}

// True when every destination row start is 16-byte aligned (bases and both strides), so a run of
// consecutive elements of one row can go out as one packed store.
inline bool out_vec_ok(const mlb_out_targets& t, int elt_bytes) {
  if ((t.stride_tok * elt_bytes) % 16 || (t.stride_head * elt_bytes) % 16) return false;
  for (int i = 0; i < t.num_dests; ++i)
    if (reinterpret_cast<uintptr_t>(t.dests[i]) % 16) return false;
  return true;
}

template <int B>
__device__ __forceinline__ void store_bytes(char* p, const uint32_t* w) {
  if constexpr (B == 4) {
    *reinterpret_cast<uint32_t*>(p) = w[0];
  } else if constexpr (B == 8) {
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  } else {
#pragma unroll
    for (int k = 0; k < B / 16; ++k)
      reinterpret_cast<uint4*>(p)[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
  }
}

// Store N consecutive output elements (dims d .. d + N - 1, d a multiple of N) into every destination.
// With `vec` they leave as packed stores of N x element bytes (one NVLink / L2 transaction per lane
// instead of N), otherwise one element at a time.  The casts are store_f32's.
template <int DT, int N>
__device__ __forceinline__ void store_out_n(const mlb_out_targets& t, bool vec, int64_t tok, int head, int d,
                                            const float (&v)[N]) {
  constexpr int EB = Elt<DT>::bytes;
  const int64_t off = (tok * t.stride_tok + static_cast<int64_t>(t.head_offset + head) * t.stride_head + d) * EB;
  if (vec) {
    uint32_t w[N * EB / 4];
    if constexpr (DT == MLB_F32) {
#pragma unroll
      for (int k = 0; k < N; ++k) w[k] = __float_as_uint(v[k]);
    } else {
#pragma unroll
      for (int k = 0; k < N / 2; ++k) {
        const uint32_t lo = DT == MLB_BF16 ? f32_to_bf16_bits(v[2 * k]) : f32_to_f16_bits(v[2 * k]);
        const uint32_t hi = DT == MLB_BF16 ? f32_to_bf16_bits(v[2 * k + 1]) : f32_to_f16_bits(v[2 * k + 1]);
        w[k] = lo | (hi << 16);
      }
    }
#pragma unroll
    for (int i = 0; i < MLB_MAX_OUT_DESTS; ++i)
      if (i < t.num_dests) store_bytes<N * EB>(static_cast<char*>(t.dests[i]) + off, w);
  } else {
#pragma unroll
    for (int i = 0; i < MLB_MAX_OUT_DESTS; ++i)
      if (i < t.num_dests)
#pragma unroll
        for (int k = 0; k < N; ++k) store_f32<DT>(static_cast<char*>(t.dests[i]) + off + k * EB, v[k]);
  }
}


// Store one output element (token tok, head of this call, dim d) into every destination.
template <int DT>
__device__ __forceinline__ void store_out1(const mlb_out_targets& t, int64_t tok, int head, int d, float v) {
  const int64_t off = (tok * t.stride_tok + static_cast<int64_t>(t.head_offset + head) * t.stride_head + d) *
                      Elt<DT>::bytes;
#pragma unroll
  for (int i = 0; i < MLB_MAX_OUT_DESTS; ++i)
    if (i < t.num_dests) store_f32<DT>(static_cast<char*>(t.dests[i]) + off, v);
}

template <int B>
__device__ __forceinline__ void load_bytes(const char* p, uint32_t* w) {
  if constexpr (B == 4) {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  } else if constexpr (B == 8) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x;
    w[1] = v.y;
  } else {
#pragma unroll
    for (int k = 0; k < B / 16; ++k) {
      const uint4 v = reinterpret_cast<const uint4*>(p)[k];
      w[4 * k] = v.x;
      w[4 * k + 1] = v.y;
      w[4 * k + 2] = v.z;
      w[4 * k + 3] = v.w;
    }
  }
}

// Copy N consecutive output elements of one row from destination `self` to every other destination.
template <int DT, int N>
__device__ __forceinline__ void copy_out_n(const mlb_out_targets& t, bool vec, int self, int64_t tok, int head,
                                           int d) {
  constexpr int EB = Elt<DT>::bytes;
  const int64_t off = (tok * t.stride_tok + static_cast<int64_t>(t.head_offset + head) * t.stride_head + d) * EB;
  const char* src = nullptr;
#pragma unroll
  for (int i = 0; i < MLB_MAX_OUT_DESTS; ++i)
    if (i == self) src = static_cast<const char*>(t.dests[i]) + off;
  if (vec) {
    uint32_t w[N * EB / 4];
    load_bytes<N * EB>(src, w);
#pragma unroll
    for (int i = 0; i < MLB_MAX_OUT_DESTS; ++i)
      if (i < t.num_dests && i != self) store_bytes<N * EB>(static_cast<char*>(t.dests[i]) + off, w);
  } else {
    using U = typename std::conditional<EB == 4, uint32_t, uint16_t>::type;
    U x[N];
#pragma unroll
    for (int k = 0; k < N; ++k) x[k] = reinterpret_cast<const U*>(src)[k];
#pragma unroll
    for (int i = 0; i < MLB_MAX_OUT_DESTS; ++i)
      if (i < t.num_dests && i != self)
#pragma unroll
        for (int k = 0; k < N; ++k) reinterpret_cast<U*>(static_cast<char*>(t.dests[i]) + off)[k] = x[k];
  }
}

}  // namespace mlb
