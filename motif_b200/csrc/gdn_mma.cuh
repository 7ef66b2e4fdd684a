// Shared pieces of the 16-bit chunked delta-rule kernels: chunk size, warp count, stride
// struct and the ldmatrix / mma operand helpers (row-major shared-memory tiles with padded
// row strides).
#pragma once

#include "common.cuh"

namespace mb {
namespace gdnk {

constexpr int C = 64;
constexpr int NW = 8;
constexpr int NT = NW * 32;

struct Strides18 {
  int64_t s[18];
};

// ldmatrix address helpers -------------------------------------------------------------
// A operand (16x16, row-major [m][k] in smem): x4 non-trans.
template <typename T>
__device__ __forceinline__ void lda(uint32_t* a, const T* base, int stride, int m0, int k0) {
  const int lane = threadIdx.x & 31;
  ldmatrix_x4(a, base + (m0 + (lane & 15)) * stride + k0 + (lane >> 4) * 8);
}
// A operand from a matrix stored transposed ([k][m] in smem): x4 trans.
template <typename T>
__device__ __forceinline__ void lda_t(uint32_t* a, const T* base, int stride, int m0, int k0) {
  const int lane = threadIdx.x & 31;
  const int mi = lane >> 3;
  ldmatrix_x4_trans(a, base + (k0 + (lane & 7) + (mi >> 1) * 8) * stride + m0 + (mi & 1) * 8);
}
// B operands for two n8 tiles (n0, n0+8) from a matrix stored [k][n] (row-major): x4 trans.
template <typename T>
__device__ __forceinline__ void ldb_t(uint32_t* b, const T* base, int stride, int k0, int n0) {
  const int lane = threadIdx.x & 31;
  ldmatrix_x4_trans(b, base + (k0 + (lane & 15)) * stride + n0 + (lane >> 4) * 8);
}
// B operands for one n8 tile from [k][n] storage: x2 trans.
__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t* r, const void* smem) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(smem)));
}
template <typename T>
__device__ __forceinline__ void ldb_t1(uint32_t* b, const T* base, int stride, int k0, int n0) {
  const int lane = threadIdx.x & 31;
  ldmatrix_x2_trans(b, base + (k0 + (lane & 15)) * stride + n0);
}
// B operands for two n8 tiles from a matrix stored [n][k] (B = M^T): x4 non-trans.
template <typename T>
__device__ __forceinline__ void ldb_n(uint32_t* b, const T* base, int stride, int k0, int n0) {
  const int lane = threadIdx.x & 31;
  ldmatrix_x4(b, base + (n0 + (lane & 7) + (lane >> 4) * 8) * stride + k0 + ((lane >> 3) & 1) * 8);
}

template <typename T>
__device__ __forceinline__ void st2(T* p, float a, float b) {
  *reinterpret_cast<uint32_t*>(p) = pack2<T>(a, b);
}
template <typename T>
__device__ __forceinline__ float2 ld2(const T* p) {
  const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
  const T* e = reinterpret_cast<const T*>(&u);
  return make_float2(to_f(e[0]), to_f(e[1]));
}

}  // namespace gdnk
}  // namespace mb
