// K1 — KV append: scatter this step's k/v rows into the paged pools through slot_mapping.
//
// Replaces write_kv (src/minillm/attention/paged_torch_ref.py:23-28): two torch index_copy_ launches
// per layer become one launch that writes K and V.  One thread moves one 16-byte vector of one
// (token, head) row; consecutive threads take consecutive vectors of the same row, so both the read
// of the (possibly strided) input row and the write of the pool row are coalesced 16-byte accesses.
// Casting (e.g. fp32 rows into a bf16 pool) rounds to nearest even, bit-identical to Tensor.to.
#include "common.cuh"

namespace mlb {
namespace {

struct AppendArgs {
  char* k_cache;
  char* v_cache;
  const int64_t* slots;
  const char* k;
  const char* v;
  int64_t k_st, k_sh, v_st, v_sh;  // input strides in elements
  int64_t num_slots;
  int64_t num_tokens;
  int hkv, dh;
  int vecs_per_row;  // 16-byte output vectors per (token, head) row
  int32_t* err;
};

template <int IN, int OUT>
__device__ __forceinline__ void convert_vec(const char* src, char* dst, int n_out) {
  // n_out = elements in one 16-byte output vector
  using Ti = typename Elt<IN>::T;
  const Ti* s = reinterpret_cast<const Ti*>(src);
  alignas(16) uint8_t buf[16];
  if constexpr (OUT == MLB_F32) {
    float* o = reinterpret_cast<float*>(buf);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = to_f32(s[i]);
  } else {
    uint16_t* o = reinterpret_cast<uint16_t*>(buf);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float x = to_f32(s[i]);
      o[i] = OUT == MLB_BF16 ? f32_to_bf16_bits(x) : f32_to_f16_bits(x);
    }
  }
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(buf);
}

// VEC: input rows start 16-byte aligned and the whole vector can be read with wide loads.
template <int IN, int OUT, bool VEC>
__global__ void __launch_bounds__(256) kv_append_kernel(AppendArgs a) {
  constexpr int in_b = Elt<IN>::bytes, out_b = Elt<OUT>::bytes;
  constexpr int per_vec = 16 / out_b;  // elements per output vector
  griddep_begin();
  const int64_t rows = a.num_tokens * a.hkv;
  const int64_t total = 2 * rows * a.vecs_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int which = i >= rows * a.vecs_per_row;  // 0: K, 1: V
    const int64_t j = i - which * rows * a.vecs_per_row;
    const int c = static_cast<int>(j % a.vecs_per_row);
    const int64_t row = j / a.vecs_per_row;
    const int h = static_cast<int>(row % a.hkv);
    const int64_t tok = row / a.hkv;
    const int64_t slot = __ldg(a.slots + tok);
    if (slot < 0 || slot >= a.num_slots) {
      if (c == 0 && h == 0 && which == 0) flag_error(a.err, MLB_DEV_SLOT_RANGE);
      continue;
    }
    const char* src = which ? a.v : a.k;
    const int64_t st = which ? a.v_st : a.k_st, sh = which ? a.v_sh : a.k_sh;
    src += ((tok * st + h * sh) + static_cast<int64_t>(c) * per_vec) * in_b;
    char* dst = (which ? a.v_cache : a.k_cache) + ((slot * a.hkv + h) * a.dh + static_cast<int64_t>(c) * per_vec) * out_b;
    if constexpr (IN == OUT) {
      if constexpr (VEC) {
        *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
      } else {
        using T = typename Elt<IN>::T;
        alignas(16) T buf[per_vec];
#pragma unroll
        for (int e = 0; e < per_vec; ++e) buf[e] = reinterpret_cast<const T*>(src)[e];
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(buf);
      }
    } else {
      constexpr int src_bytes = per_vec * in_b;  // 8 (16-bit -> f32) or 32 (f32 -> 16-bit) or 16
      alignas(16) uint8_t sb[src_bytes < 16 ? 16 : src_bytes];
      if constexpr (VEC) {
#pragma unroll
        for (int e = 0; e < src_bytes / 8; ++e)
          reinterpret_cast<uint2*>(sb)[e] = __ldg(reinterpret_cast<const uint2*>(src) + e);
      } else {
        using Ti = typename Elt<IN>::T;
#pragma unroll
        for (int e = 0; e < per_vec; ++e) reinterpret_cast<Ti*>(sb)[e] = reinterpret_cast<const Ti*>(src)[e];
      }
      convert_vec<IN, OUT>(reinterpret_cast<const char*>(sb), dst, per_vec);
    }
  }
}

template <int IN, int OUT>
cudaError_t launch_typed(const AppendArgs& a, bool vec, cudaStream_t s) {
  const int64_t total = 2 * a.num_tokens * a.hkv * a.vecs_per_row;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 64) blocks = 148 * 64;  // grid-stride beyond 64 CTAs per SM
  if (blocks < 1) blocks = 1;
  if (vec)
    return launch_k(kv_append_kernel<IN, OUT, true>, dim3(static_cast<unsigned>(blocks)), dim3(threads), 0, s, a);
  return launch_k(kv_append_kernel<IN, OUT, false>, dim3(static_cast<unsigned>(blocks)), dim3(threads), 0, s, a);
}

}  // namespace

cudaError_t launch_kv_append(void* k_cache, void* v_cache, int cache_dtype, int64_t num_slots,
                             const int64_t* slots, const void* k, int64_t k_st, int64_t k_sh, const void* v,
                             int64_t v_st, int64_t v_sh, int in_dtype, int64_t num_tokens, int hkv, int dh,
                             bool vec, int32_t* err, cudaStream_t s) {
  const int out_b = cache_dtype == MLB_F32 ? 4 : 2;
  AppendArgs a{static_cast<char*>(k_cache), static_cast<char*>(v_cache), slots,
               static_cast<const char*>(k), static_cast<const char*>(v), k_st, k_sh, v_st, v_sh, num_slots,
               num_tokens, hkv, dh, dh * out_b / 16, err};
#define MLB_APPEND_CASE(I, O) \
  if (in_dtype == I && cache_dtype == O) return launch_typed<I, O>(a, vec, s);
  MLB_APPEND_CASE(MLB_F32, MLB_F32)
  MLB_APPEND_CASE(MLB_F32, MLB_BF16)
  MLB_APPEND_CASE(MLB_F32, MLB_F16)
  MLB_APPEND_CASE(MLB_BF16, MLB_BF16)
  MLB_APPEND_CASE(MLB_BF16, MLB_F32)
  MLB_APPEND_CASE(MLB_BF16, MLB_F16)
  MLB_APPEND_CASE(MLB_F16, MLB_F16)
  MLB_APPEND_CASE(MLB_F16, MLB_F32)
  MLB_APPEND_CASE(MLB_F16, MLB_BF16)
#undef MLB_APPEND_CASE
  return cudaErrorInvalidValue;
}

}  // namespace mlb
