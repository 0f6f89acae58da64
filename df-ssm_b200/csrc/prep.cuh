// Shared prologue of the projections: RMSNorm -> per-row int8 quantisation -> LoRA
// down-projection for 512-thread CTAs where each thread owns KPT consecutive columns in
// registers (used by the persistent step kernel and by act_prep_fast_kernel).
#pragma once
#include "types.cuh"

namespace dfssm {

constexpr int kPrepFastThreads = 512;
constexpr int kPrepFastWarps = kPrepFastThreads / 32;

// Barrier of the 512 compute threads (named barrier 1).  Blocks of exactly 512 threads use it
// like __syncthreads; the persistent kernel adds a copy-issuing warp that never joins it.
__device__ __forceinline__ void cta_sync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

// ---- block reductions over kPrepFastThreads (512) threads
// Block-wide sum / max of N values per thread with a fixed combination order.  Warp partials
// go to red[w*N + i]; thread i < N combines column i into red[kPrepFastWarps*N + i]; every thread then
// reads the N totals.  `red` holds (kPrepFastWarps + 1) * N floats.
template <int N>
__device__ __forceinline__ void block_sum_n(float (&v)[N], float* red) {
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = warp_sum(v[i]);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  cta_sync();
  if (l == 0)
#pragma unroll
    for (int i = 0; i < N; ++i) red[w * N + i] = v[i];
  cta_sync();
  if (threadIdx.x < N) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kPrepFastWarps; ++j) s += red[j * N + threadIdx.x];
    red[kPrepFastWarps * N + threadIdx.x] = s;
  }
  cta_sync();
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = red[kPrepFastWarps * N + i];
}
template <int N>
__device__ __forceinline__ void block_max_n(float (&v)[N], float* red) {  // v >= 0 (absolute values)
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = warp_max_nonneg(v[i]);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  cta_sync();
  if (l == 0)
#pragma unroll
    for (int i = 0; i < N; ++i) red[w * N + i] = v[i];
  cta_sync();
  if (threadIdx.x < N) {
    float s = red[threadIdx.x];
#pragma unroll
    for (int j = 1; j < kPrepFastWarps; ++j) s = fmaxf(s, red[j * N + threadIdx.x]);
    red[kPrepFastWarps * N + threadIdx.x] = s;
  }
  cta_sync();
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = red[kPrepFastWarps * N + i];
}

// Single-barrier block sum / max: warp partials go to red[w*N + i], one cta_sync, then every
// thread combines the 16 partials of each value itself, in the same fixed order, so all
// threads hold identical totals.  `red` must not still be read by the previous reduction that
// used it: callers rotate buffers so that a barrier separates the two uses.
// The 16 x N warp partials at red (16-byte aligned), read with vector loads for N <= 2.
template <int N>
__device__ __forceinline__ void load_partials(const float* red, float (&p)[kPrepFastWarps * N]) {
  if constexpr (N <= 2) {
#pragma unroll
    for (int j = 0; j < kPrepFastWarps * N / 4; ++j) {
      const float4 t = reinterpret_cast<const float4*>(red)[j];
      p[4 * j] = t.x, p[4 * j + 1] = t.y, p[4 * j + 2] = t.z, p[4 * j + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < kPrepFastWarps * N; ++j) p[j] = red[j];
  }
}
template <int N>
__device__ __forceinline__ void block_sum1(float (&v)[N], float* red) {
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = warp_sum(v[i]);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0)
#pragma unroll
    for (int i = 0; i < N; ++i) red[w * N + i] = v[i];
  cta_sync();
  float p[kPrepFastWarps * N];
  load_partials<N>(red, p);
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kPrepFastWarps; ++j) s += p[j * N + i];
    v[i] = s;
  }
}
template <int N>
__device__ __forceinline__ void block_max1(float (&v)[N], float* red) {  // v >= 0 (absolute values)
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = warp_max_nonneg(v[i]);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0)
#pragma unroll
    for (int i = 0; i < N; ++i) red[w * N + i] = v[i];
  cta_sync();
  float p[kPrepFastWarps * N];
  load_partials<N>(red, p);
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float s = p[i];
#pragma unroll
    for (int j = 1; j < kPrepFastWarps; ++j) s = fmaxf(s, p[j * N + i]);
    v[i] = s;
  }
}

// Like block_sum_n but only threads i < N receive total i (returned), for the LoRA partials.
template <int N>
__device__ __forceinline__ float block_sum_scatter(float (&v)[N], float* red) {
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = warp_sum(v[i]);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  cta_sync();
  if (l == 0)
#pragma unroll
    for (int i = 0; i < N; ++i) red[w * N + i] = v[i];
  cta_sync();
  float s = 0.f;
  if (threadIdx.x < N)
#pragma unroll
    for (int j = 0; j < kPrepFastWarps; ++j) s += red[j * N + threadIdx.x];
  return s;
}

template <int KPT>
struct RankHalves;  // KPT fp16 LoRA-B values of one rank for this thread's columns
template <> struct RankHalves<1> { using T = unsigned short; };
template <> struct RankHalves<2> { using T = unsigned; };
template <> struct RankHalves<4> { using T = uint2; };
template <> struct RankHalves<8> { using T = uint4; };
// widths that are not a power of two (the 2.7B shape: d_model 2560 = 512 x 5, d_inner 5120 = 512 x 10):
// the halves packed in pairs into 32-bit words, half j in the low (j even) or high half of word j / 2
template <int N>
struct HalfPack {
  unsigned w[(N + 1) / 2];
};
template <> struct RankHalves<5> { using T = HalfPack<5>; };
template <> struct RankHalves<10> { using T = HalfPack<10>; };

// KPT consecutive fp16 values at p (read-only data), in this thread's RankHalves form
template <int KPT>
__device__ __forceinline__ typename RankHalves<KPT>::T ld_halves(const __half* p) {
  using T = typename RankHalves<KPT>::T;
  if constexpr (KPT == 5 || KPT == 10) {
    T v;
    const unsigned short* h = reinterpret_cast<const unsigned short*>(p);
    if constexpr (KPT % 2 == 0) {  // 4-byte aligned: one word per pair
#pragma unroll
      for (int i = 0; i < KPT / 2; ++i) v.w[i] = __ldg(reinterpret_cast<const unsigned*>(p) + i);
    } else {
#pragma unroll
      for (int i = 0; i < (KPT + 1) / 2; ++i) {
        const unsigned lo = __ldg(h + 2 * i), hi = 2 * i + 1 < KPT ? __ldg(h + 2 * i + 1) : 0u;
        v.w[i] = lo | (hi << 16);
      }
    }
    return v;
  } else {
    return __ldg(reinterpret_cast<const T*>(p));
  }
}

template <int KPT>
__device__ __forceinline__ void load_lora_b(const __half* B16, int K, typename RankHalves<KPT>::T (&out)[DFSSM_RANK]) {
  const int k0 = threadIdx.x * KPT;
#pragma unroll
  for (int r = 0; r < DFSSM_RANK; ++r) out[r] = ld_halves<KPT>(B16 + (size_t)r * K + k0);
}
// NR rank rows starting at r0.
template <int KPT, int NR>
__device__ __forceinline__ void load_lora_b_ranks(const __half* B16, int K, int r0,
                                                  typename RankHalves<KPT>::T (&out)[NR]) {
  const int k0 = threadIdx.x * KPT;
#pragma unroll
  for (int r = 0; r < NR; ++r) out[r] = ld_halves<KPT>(B16 + (size_t)(r0 + r) * K + k0);
}

template <int KPT>
__device__ __forceinline__ float half_of(const typename RankHalves<KPT>::T& v, int j) {
  const unsigned short* h = reinterpret_cast<const unsigned short*>(&v);
  return __half2float(__ushort_as_half(h[j]));
}

// Shared-memory position of permuted activation byte p: 16-byte unit u of 128-byte chunk c is
// stored at unit u ^ (c & 7), so the 8 lanes of a quarter-warp that read unit u of chunks
// c..c+7 hit 8 different bank groups.
__device__ __forceinline__ int qswz(int p) {
  const int c = p >> 7;
  return (p & ~127) | ((((p >> 4) & 7) ^ (c & 7)) << 4) | (p & 15);
}

// RMSNorm + per-row int8 quantisation + LoRA down-projection of this thread's KPT columns of
// B activation rows.  vals[b][j]: fp16-exact inputs of columns k0 + j.  Writes q (permuted) to
// sq[b][*] and xs/qsum/t to smem; returns after a cta_sync.
// SWZ: store q in the swizzled shared-memory order of the persistent kernel (qswz) instead of
// the plain permuted order read by the per-op GEMV kernels.  NR: LoRA ranks computed here (lb
// holds NR consecutive rank rows; s_t receives [B][NR]).
template <int B, int KPT, bool SWZ = true, int NR = DFSSM_RANK>
__device__ void prep_rows(float (&vals)[B][KPT], const float (&w)[KPT], int K,
                          const typename RankHalves<KPT>::T (&lb)[NR], int8_t* sq, int Kq,
                          float* s_xs, int* s_qsum, float* s_t, float* red) {
  const int k0 = threadIdx.x * KPT;
  float ss[B];
#pragma unroll
  for (int b = 0; b < B; ++b) {
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < KPT; ++j) a = __fadd_rn(a, __fmul_rn(vals[b][j], vals[b][j]));
    ss[b] = a;
  }
  block_sum_n<B>(ss, red);
  float am[B];
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const float r = rsqrtf(__fadd_rn(__fmul_rn(ss[b], 1.0f / (float)K), 1e-5f));
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < KPT; ++j) {
      const float xn = round_hc(__fmul_rn(__fmul_rn(vals[b][j], r), w[j]));
      vals[b][j] = xn;
      a = fmaxf(a, fabsf(xn));
    }
    am[b] = a;
  }
  block_max_n<B>(am, red);
  float all[B * NR + B];  // LoRA partials t[b][r] = sum_j xn_j * q_rj, then the q sums
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const float s = round_h(__fmul_rn(fmaxf(am[b], qscale_floor()), 1.0f / 127.0f));
    const float rs = __frcp_rn(s);
    int qsum = 0;
#pragma unroll
    for (int j = 0; j < KPT; ++j) {
      int q = __float2int_rn(round_hc(div_rn_rcp(vals[b][j], s, rs)));
      q = max(-128, min(127, q));
      sq[b * Kq + (SWZ ? qswz(qperm_index(k0 + j)) : qperm_index(k0 + j))] = (int8_t)q;
      qsum += q;
    }
    all[B * NR + b] = (float)qsum;
    if (threadIdx.x == 0) s_xs[b] = s;
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      float a = 0.f;
#pragma unroll
      for (int j = 0; j < KPT; ++j) a = fmaf(vals[b][j], half_of<KPT>(lb[r], j), a);
      all[b * NR + r] = a;
    }
  }
  const float tot = block_sum_scatter<B * NR + B>(all, red);
  if (threadIdx.x < B * NR) s_t[threadIdx.x] = round_h(tot);
  else if (threadIdx.x < B * NR + B) s_qsum[threadIdx.x - B * NR] = (int)tot;
  cta_sync();
}


// RMSNorm (first half of the quantising prologue): on return vals[b][j] holds the fp16-exact
// normalised values.
template <int B, int KPT>
__device__ __forceinline__ void prep_norm(float (&vals)[B][KPT], const float (&w)[KPT], int K, float* red) {
  float ss[B];
#pragma unroll
  for (int b = 0; b < B; ++b) {
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < KPT; ++j) a = __fadd_rn(a, __fmul_rn(vals[b][j], vals[b][j]));
    ss[b] = a;
  }
  block_sum1<B>(ss, red);
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const float r = rsqrtf(__fadd_rn(__fmul_rn(ss[b], 1.0f / (float)K), 1e-5f));
#pragma unroll
    for (int j = 0; j < KPT; ++j) vals[b][j] = round_hc(__fmul_rn(__fmul_rn(vals[b][j], r), w[j]));
  }
}

// Per-row int8 quantisation of normalised values (second half): q in sq (swizzled if SWZ),
// the scale in s_xs, and per-warp partial q sums in s_qpart[b][warp] (see qsum_of); returns
// after a cta_sync.  One barrier for the amax, one for the stores.
template <int B, int KPT, bool SWZ = true>
__device__ void prep_quantize(const float (&vals)[B][KPT], int8_t* sq, int Kq, float* s_xs, int* s_qpart, float* red) {
  const int k0 = threadIdx.x * KPT;
  float am[B];
#pragma unroll
  for (int b = 0; b < B; ++b) {
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < KPT; ++j) a = fmaxf(a, fabsf(vals[b][j]));
    am[b] = a;
  }
  block_max1<B>(am, red);
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const float s = round_h(__fmul_rn(fmaxf(am[b], qscale_floor()), 1.0f / 127.0f));
    const float rs = __frcp_rn(s);
    int qsum = 0;
#pragma unroll
    for (int j = 0; j < KPT; ++j) {
      // q = rne(fp16(x / s)); |x / s| <= 127 * (1 + 2^-11) since s is amax/127 rounded to fp16,
      // so the clamp only guards the int8 store
      int q = __float2int_rn(round_hc(div_rn_rcp(vals[b][j], s, rs)));
      q = max(-128, min(127, q));
      sq[b * Kq + (SWZ ? qswz(qperm_index(k0 + j)) : qperm_index(k0 + j))] = (int8_t)q;
      qsum += q;
    }
    qsum = __reduce_add_sync(0xffffffffu, qsum);
    if ((threadIdx.x & 31) == 0) s_qpart[b * kPrepFastWarps + (threadIdx.x >> 5)] = qsum;
    if (threadIdx.x == 0) s_xs[b] = s;
  }
  cta_sync();
}

// Total q sum of activation row b from the per-warp partials of prep_quantize.
__device__ __forceinline__ int qsum_of(const int* s_qpart, int b) {
  int s = 0;
#pragma unroll
  for (int j = 0; j < kPrepFastWarps; ++j) s += s_qpart[b * kPrepFastWarps + j];
  return s;
}

// One rank r of the LoRA down-projection, t[b] = fp16(sum_k xn[b][k] * B16[r][k]), from the
// thread-resident normalised values of prep_quant.  Every thread returns the B totals.
// This thread's KPT fp16 values of LoRA-B row r (B16 is [16][K]).
template <int KPT>
__device__ __forceinline__ typename RankHalves<KPT>::T load_rank_b(const __half* B16, int K, int r) {
  return ld_halves<KPT>(B16 + (size_t)r * K + threadIdx.x * KPT);
}

// t[b] = fp16(sum_k vals[b][k] * B16[r][k]) for one rank r whose values bv are already in registers.
template <int B, int KPT>
__device__ __forceinline__ void lora_t_rank_v(const float (&vals)[B][KPT], typename RankHalves<KPT>::T bv,
                                              float (&t)[B], float* red) {
#pragma unroll
  for (int b = 0; b < B; ++b) {
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < KPT; ++j) a = fmaf(vals[b][j], half_of<KPT>(bv, j), a);
    t[b] = a;
  }
  block_sum1<B>(t, red);
#pragma unroll
  for (int b = 0; b < B; ++b) t[b] = round_h(t[b]);
}

template <int B, int KPT>
__device__ __forceinline__ void lora_t_rank(const float (&vals)[B][KPT], const __half* B16, int K, int r,
                                            float (&t)[B], float* red) {
  lora_t_rank_v<B, KPT>(vals, load_rank_b<KPT>(B16, K, r), t, red);
}

}  // namespace dfssm
