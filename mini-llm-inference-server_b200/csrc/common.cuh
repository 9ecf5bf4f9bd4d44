// Shared device helpers for the sm_100a paged-KV kernels: dtype traits, RNE casts, and thin inline-PTX
// wrappers for 16-byte cp.async, ldmatrix / movmatrix and the m16n8k16 tensor-core MMA.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "mlb_paged_kv.h"

namespace mlb {

constexpr int kBlockSize = 16;  // tokens per page: the reference's BLOCK_SIZE (cache/paged.py:21)
constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------- dtype traits

template <int DT> struct Elt;
template <> struct Elt<MLB_F32> { using T = float; static constexpr int bytes = 4; };
template <> struct Elt<MLB_F16> { using T = __half; static constexpr int bytes = 2; };
template <> struct Elt<MLB_BF16> { using T = __nv_bfloat16; static constexpr int bytes = 2; };

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

// float -> bf16 bits, round to nearest even.  NaN becomes 0xFFFF, the pattern the reference's CPU cast
// (torch's vectorised float->bfloat16 conversion) stores.  Overflow rounds to +-inf as IEEE requires.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0xffffu;
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

// float -> fp16 bits, round to nearest even (cvt.rn.f16.f32); NaN keeps its sign with payload 0x7E00,
// the pattern the reference's CPU cast stores.
__device__ __forceinline__ uint16_t f32_to_f16_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>(((u >> 16) & 0x8000u) | 0x7e00u);
  return __half_as_ushort(__float2half_rn(x));
}

template <int DT> __device__ __forceinline__ void store_f32(void* p, float x);
template <> __device__ __forceinline__ void store_f32<MLB_F32>(void* p, float x) { *static_cast<float*>(p) = x; }
template <> __device__ __forceinline__ void store_f32<MLB_F16>(void* p, float x) {
  *static_cast<uint16_t*>(p) = f32_to_f16_bits(x);
}
template <> __device__ __forceinline__ void store_f32<MLB_BF16>(void* p, float x) {
  *static_cast<uint16_t*>(p) = f32_to_bf16_bits(x);
}

// ---------------------------------------------------------------- misc

__device__ __forceinline__ void flag_error(int32_t* err, int bit) {
  if (err) atomicOr(err, bit);
}

__device__ __forceinline__ float fast_exp2(float x) {  // ex2.approx: 2^x, -inf -> +0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- programmatic dependent launch

// Every kernel of this library begins with griddep_begin().  Launched with programmatic stream
// serialisation (launch_k), a kernel's CTAs may become resident while its predecessor on the stream is
// still finishing; griddepcontrol.wait holds them until that grid has completed and its memory is
// visible, so no input is read early (the split-K reductions' plan arrays, uploaded before the attention
// launch they follow, are the one exception).  Then launch_dependents lets the next kernel's CTAs do the
// same, so each launch's latency hides behind the tail of the one before.  Launched normally, both are
// no-ops.  Every kernel triggers only after its own wait, so when a kernel's CTAs run, every grid two or
// more launches before it on the stream has completed.
__device__ __forceinline__ void griddep_begin() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

bool programmatic_launch();  // host: the library-wide setting (mlb_set_programmatic_launch)

// kernel<<<grid, block, smem, s>>>(args...), with programmatic stream serialisation when enabled
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = programmatic_launch() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- 16-byte asynchronous copies (LDGSTS)

// global -> shared, 16 bytes, cached in L2 only (.cg): each thread's copies form commit groups
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {  // at most N of this thread's groups still pending
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarriers (shared memory)

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n.reg .b64 st;\nmbarrier.arrive.shared::cta.b64 st, [%0];\n}\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// ---------------------------------------------------------------- warp-level tensor-core fragments

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// pack (lo, hi) into a 16-bit pair; lo lands in the low half
template <int DT> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<MLB_BF16>(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
template <> __device__ __forceinline__ uint32_t pack2<MLB_F16>(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// D = A(16x16, row) * B(16x8, col) + D, fp32 accumulate
template <int DT> __device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                                           uint32_t a3, uint32_t b0, uint32_t b1);
template <> __device__ __forceinline__ void mma16816<MLB_BF16>(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <> __device__ __forceinline__ void mma16816<MLB_F16>(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

}  // namespace mlb
