// Shared device helpers for the DF-SSM B200 decode kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define DFSSM_HEADDIM 64
#define DFSSM_DSTATE 128
#define DFSSM_RANK 16
#define DFSSM_DCONV 4

namespace dfssm {

// fp16(1e-4): the clamp floor of the reference's activation scale
// (inference/gpu/df_ssm_inference.py:150, clamp(min=1e-4) on an fp16 tensor).
__device__ __forceinline__ float qscale_floor() { return __half2float(__ushort_as_half((unsigned short)0x068Eu)); }

__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }
__device__ __forceinline__ __half f2h(float f) { return __float2half_rn(f); }
__device__ __forceinline__ float round_h(float f) { return __half2float(__float2half_rn(f)); }

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide reductions with a fixed combination order (deterministic across CTAs).
template <int NW>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NW; ++i) s += red[i];
  return s;
}
template <int NW>
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = red[0];
#pragma unroll
  for (int i = 1; i < NW; ++i) s = fmaxf(s, red[i]);
  return s;
}
template <int NW>
__device__ __forceinline__ int block_isum(int v, int* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  int s = 0;
#pragma unroll
  for (int i = 0; i < NW; ++i) s += red[i];
  return s;
}

// Streaming (read-once) 128-bit load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// dp4a with unsigned a (0/1 bytes of the sign mask) and signed b (int8 activations).
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Byte position of column `col` inside the permuted activation layout used by the
// 1-bit GEMV: within each 32-column word block, byte 4*i + m holds column 8*m + i,
// so that ((bits >> i) & 0x01010101) lines up with one 32-bit activation word.
__host__ __device__ __forceinline__ int qperm_index(int col) {
  return (col & ~31) + ((col & 7) << 2) + ((col >> 3) & 3);
}

// Orderable 16-bit key of an fp16 value (monotone in the value for non-NaN inputs).
__device__ __forceinline__ uint32_t f16_order_key(__half h) {
  uint32_t u = __half_as_ushort(h);
  return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
}
// 64-bit argmax key: larger fp16 value wins, ties go to the smaller index (torch.argmax).
__device__ __forceinline__ unsigned long long argmax_key(__half v, uint32_t idx) {
  return ((unsigned long long)f16_order_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t argmax_key_index(unsigned long long k) {
  return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
}

}  // namespace dfssm
