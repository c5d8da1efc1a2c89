// Shared helpers for the kadllm_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/kadllm_b200.h"

namespace kb {

// ---------------------------------------------------------------------------
// Status reporting: every entry point returns a kadllm_status and leaves a
// message retrievable with kadllm_last_error() on the calling thread.
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);

#define KB_REQUIRE(cond, code, ...)         \
  do {                                      \
    if (!(cond)) {                          \
      ::kb::set_error(__VA_ARGS__);         \
      return (code);                        \
    }                                       \
  } while (0)

#define KB_CHECK_LAUNCH(what)                                                       \
  do {                                                                              \
    cudaError_t _e = cudaGetLastError();                                            \
    if (_e != cudaSuccess) {                                                        \
      ::kb::set_error("%s: %s", what, cudaGetErrorString(_e));                      \
      return KADLLM_ECUDA;                                                          \
    }                                                                               \
  } while (0)

inline bool valid_dtype(int d) { return d == KADLLM_F32 || d == KADLLM_F16 || d == KADLLM_BF16; }
inline int dtype_size(int d) { return d == KADLLM_F32 ? 4 : 2; }

// ---------------------------------------------------------------------------
// Scalar conversions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_as_float(const void* p, int64_t i, int dtype) {
  if (dtype == KADLLM_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == KADLLM_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// Elements i, i + 1 (i even, the row 4- / 8-byte aligned) as a float pair, in one load.
__device__ __forceinline__ float2 load2_as_float(const void* p, int64_t i, int dtype) {
  if (dtype == KADLLM_BF16) return __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(p)[i >> 1]);
  if (dtype == KADLLM_F16) return __half22float2(reinterpret_cast<const __half2*>(p)[i >> 1]);
  return reinterpret_cast<const float2*>(p)[i >> 1];
}

__device__ __forceinline__ void store_from_float(void* p, int64_t i, int dtype, float v) {
  if (dtype == KADLLM_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dtype == KADLLM_F16)
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}

// Round a float to the nearest value representable in `dtype` (identity for fp32).
__device__ __forceinline__ float round_to(float v, int dtype) {
  if (dtype == KADLLM_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == KADLLM_F16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Load 4 consecutive elements as floats (pointer + element offset, offset % 4 == 0).
__device__ __forceinline__ void load4(const void* p, int64_t i, int dtype, float out[4]) {
  if (dtype == KADLLM_BF16) {
    const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(p) + i);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
    out[0] = __low2float(a); out[1] = __high2float(a);
    out[2] = __low2float(b); out[3] = __high2float(b);
  } else if (dtype == KADLLM_F16) {
    const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(p) + i);
    const __half2 a = *reinterpret_cast<const __half2*>(&u.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&u.y);
    out[0] = __low2float(a); out[1] = __high2float(a);
    out[2] = __low2float(b); out[3] = __high2float(b);
  } else {
    const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    out[0] = f.x; out[1] = f.y; out[2] = f.z; out[3] = f.w;
  }
}

__device__ __forceinline__ void store4(void* p, int64_t i, int dtype, const float v[4]) {
  if (dtype == KADLLM_BF16) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p) + i) = u;
  } else if (dtype == KADLLM_F16) {
    __half2 a = __floats2half2_rn(v[0], v[1]);
    __half2 b = __floats2half2_rn(v[2], v[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(p) + i) = u;
  } else {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }
// SiLU with the fast approximate divide; for values rounded to bf16 right after
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + __expf(-x)); }
// torch.nn.functional.softplus with beta=1, threshold=20
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(__expf(x)); }

// ---------------------------------------------------------------------------
// Tensor-core fragments (mma.sync m16n8k16, bf16 in, fp32 accumulate)
// ---------------------------------------------------------------------------
// Packed fp32 pairs (sm_100 f32x2 arithmetic: each lane an independent fp32 op, round to nearest).
__device__ __forceinline__ uint64_t pk2(float2 v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};\n" : "=l"(r) : "f"(v.x), "f"(v.y));
  return r;
}
__device__ __forceinline__ float2 upk2(uint64_t r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;\n" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)), "l"(pk2(c)));
  return upk2(d);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)));
  return upk2(d);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)));
  return upk2(d);
}
__device__ __forceinline__ float fast_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fast_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
// SiLU of a pair: v / (1 + 2^(-v log2 e)) with the approximate exp2 / reciprocal units.
__device__ __forceinline__ float2 silu2(float2 v) {
  const float2 t = mul2(v, make_float2(-1.4426950408889634f, -1.4426950408889634f));
  const float2 d = add2(make_float2(fast_ex2(t.x), fast_ex2(t.y)), make_float2(1.f, 1.f));
  return mul2(v, make_float2(fast_rcp(d.x), fast_rcp(d.y)));
}
// (low, high) fp32 -> bf16x2 word, round to nearest even
__device__ __forceinline__ uint32_t bf2_pack(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t bf2_pack_f2(float2 v) { return bf2_pack(v.x, v.y); }
// bf16x2 word -> (low, high) fp32 pair
__device__ __forceinline__ float2 bf2f(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t r[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldmatrix_x2(uint32_t r[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(p)));
}

// D = A(16x16 row) * B(16x8 col) + D
__device__ __forceinline__ void mma_bf16_16816(float d[4], const uint32_t a[4], const uint32_t b[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

}  // namespace kb
