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
// Round an fp32 value to the nearest fp16 value (ties to even), returned as fp32, using two
// exact-rounding fp32 additions instead of the F2H/H2F conversion pair (which issue on the
// low-throughput conversion pipe): adding M = 1.5 * 2^(E+13), E the value's binary exponent
// clamped to fp16's subnormal floor 2^-14, leaves the sum with fp16's spacing 2^(E-10) as its
// last fp32 bit, so fp32's own round-to-nearest-even performs the fp16 rounding.  Results with
// magnitude above 65504 are fp16 overflow and become +-inf, as __float2half_rn does.
__device__ __forceinline__ float round_h(float v) {
  unsigned e = (__float_as_uint(v) >> 23) & 0xffu;
  e = e < 113u ? 113u : (e > 160u ? 160u : e);
  const float M = __uint_as_float(((e + 13u) << 23) | 0x400000u);
  const float r = copysignf(__fsub_rn(__fadd_rn(v, M), M), v);  // keeps -0 for tiny negatives
  return fabsf(r) > 65504.f ? copysignf(__int_as_float(0x7f800000), v) : r;
}
// The same fp16 rounding with the hardware conversions (cvt.rn.f16.f32, then widening):
// 2 instructions instead of 8-13, for per-element prologue code that is issue-bound.
__device__ __forceinline__ float round_hc(float v) { return __half2float(__float2half_rn(v)); }
// Correctly rounded a / b from rb = RN(1/b) with two FMAs (Markstein's theorem: with rb within
// half an ulp of 1/b and q0 = RN(a*rb) within an ulp of a/b, the remainder r = a - b*q0 is exact
// and RN(q0 + r*rb) = RN(a/b)), valid while a/b, a and b stay normal fp32 -- true for fp16
// operands.  One exception: a = -0 gives +0 (the quantiser maps both zeros to q = 0).  dfssm_selftest_division checks it against IEEE division over every fp16 pair the
// quantiser can meet.
__device__ __forceinline__ float div_rn_rcp(float a, float b, float rb) {
  const float q0 = __fmul_rn(a, rb);
  const float r = __fmaf_rn(-q0, b, a);
  return __fmaf_rn(r, rb, q0);
}
// Round to the nearest integer, ties to even (|v| < 2^22): same trick with M = 1.5 * 2^23.
__device__ __forceinline__ float rint_alu(float v) { return __fsub_rn(__fadd_rn(v, 12582912.0f), 12582912.0f); }
// Signed byte j of w as fp32 without I2F: w ^ 0x80808080 biases the bytes to 0..255, a byte
// permute places byte j in the mantissa of 2^23, and one exact subtraction removes 2^23 + 128.
__device__ __forceinline__ float i8_to_f(unsigned w_biased, int j) {
  return __fsub_rn(__uint_as_float(__byte_perm(w_biased, 0x4B000000u, 0x7540u | (unsigned)j)), 8388736.0f);
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// Warp-wide max of non-negative floats in one instruction: their bit patterns order as unsigned
// integers, so redux.sync's integer max gives the float max exactly.
__device__ __forceinline__ float warp_max_nonneg(float v) {
  return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
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

// ---- TMA bulk copies, mbarriers and release/acquire counters
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until the mbarrier phase with `parity` completes; bounded (a copy from valid memory always
// completes, the bound only keeps a fault elsewhere from turning into an endless spin).  Returns
// false if the wait ran out; the caller records that in an error word the host checks.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity) {
  for (unsigned it = 0; it < (1u << 24); ++it)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// fp16 tensor-core MMA m16n8k16 with fp32 accumulation (the LM head kernels)
__device__ __forceinline__ void mma_f16(float (&d)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3,
                                        unsigned b0, unsigned b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// two int8 of a biased word (w ^ 0x80808080) as an exact half2: bytes (lo, lo+1) or (lo+2, lo+3)
__device__ __forceinline__ unsigned i8x2_to_h2(unsigned wb, unsigned sel) {
  const unsigned h = __byte_perm(wb, 0x64646464u, sel);
  const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h), __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
  return *reinterpret_cast<const unsigned*>(&r);
}

}  // namespace dfssm
