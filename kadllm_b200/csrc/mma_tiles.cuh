// Warp-level bf16 tensor-core tile products on shared-memory operands.
#pragma once
#include "common.cuh"

namespace kb {

// acc[NT][4] += A(16 x K) * B(K x 8*NT) for one warp.
//   A_T = false: A stored row-major [m][k] (lda elements per row), tile rows m0..m0+15
//   A_T = true : A stored as [k][m] (the transpose), tile columns m0..m0+15
//   B_T = false: B stored as [n][k] (each output column's k values contiguous)
//   B_T = true : B stored row-major [k][n]
// k0 / n0 select the sub-block; K and NT (even) are compile-time.
template <int K, int NT, bool A_T, bool B_T>
__device__ __forceinline__ void warp_mma(float (&acc)[NT][4], const __nv_bfloat16* A, int lda, int m0, int ka0,
                                         const __nv_bfloat16* B, int ldb, int kb0, int n0) {
  static_assert(NT % 2 == 0, "NT must be even");
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int kk = 0; kk < K; kk += 16) {
    uint32_t a[4];
    if constexpr (A_T) {
      ldmatrix_x4_trans(a, A + (ka0 + kk + (lane & 7) + ((lane >> 4) << 3)) * lda + m0 + ((lane >> 3) & 1) * 8);
    } else {
      ldmatrix_x4(a, A + (m0 + (lane & 15)) * lda + ka0 + kk + (lane >> 4) * 8);
    }
#pragma unroll
    for (int np = 0; np < NT / 2; ++np) {
      uint32_t b[4];
      const int n = n0 + np * 16;
      if constexpr (B_T) {
        ldmatrix_x4_trans(b, B + (kb0 + kk + (lane & 15)) * ldb + n + (lane >> 4) * 8);
      } else {
        ldmatrix_x4(b, B + (n + (lane & 7) + ((lane >> 4) << 3)) * ldb + kb0 + kk + ((lane >> 3) & 1) * 8);
      }
      const uint32_t b0[2] = {b[0], b[1]}, b1[2] = {b[2], b[3]};
      mma_bf16_16816(acc[2 * np], a, b0);
      mma_bf16_16816(acc[2 * np + 1], a, b1);
    }
  }
}

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return r;
}

// D = A(16x8 row, tf32) * B(8x8 col, tf32) + D
__device__ __forceinline__ void mma_tf32_1688(float d[4], const uint32_t a[4], const uint32_t b[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// acc[NT][4] += A(16 x K) * B(K x 8*NT) from row-major fp32 shared-memory blocks, TF32 tensor cores.
template <int K, int NT>
__device__ __forceinline__ void warp_mma_tf32(float (&acc)[NT][4], const float* A, int lda, const float* B, int ldb) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int k0 = 0; k0 < K; k0 += 8) {
    uint32_t a[4];
    a[0] = to_tf32(A[g * lda + k0 + tq]);
    a[1] = to_tf32(A[(g + 8) * lda + k0 + tq]);
    a[2] = to_tf32(A[g * lda + k0 + tq + 4]);
    a[3] = to_tf32(A[(g + 8) * lda + k0 + tq + 4]);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      uint32_t b[2];
      b[0] = to_tf32(B[(k0 + tq) * ldb + j * 8 + g]);
      b[1] = to_tf32(B[(k0 + tq + 4) * ldb + j * 8 + g]);
      mma_tf32_1688(acc[j], a, b);
    }
  }
}

// Store a 16 x 8*NT fp32 accumulator tile (scaled by `mul`) to row-major shared memory.
template <int NT>
__device__ __forceinline__ void store_acc(float* C, int ldc, const float (&acc)[NT][4], float mul) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    C[g * ldc + j * 8 + 2 * tq] = mul * acc[j][0];
    C[g * ldc + j * 8 + 2 * tq + 1] = mul * acc[j][1];
    C[(g + 8) * ldc + j * 8 + 2 * tq] = mul * acc[j][2];
    C[(g + 8) * ldc + j * 8 + 2 * tq + 1] = mul * acc[j][3];
  }
}

template <int NT>
__device__ __forceinline__ void zero_acc(float (&acc)[NT][4]) {
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
}

}  // namespace kb
