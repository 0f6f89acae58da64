// Sampling epilogue: the token selection of the reference's qualitative generation loop
// (eval/gen_test.py:54-95, generate) on the device, one CTA per sequence row:
//   l = logits / T;  l[seen] /= rep_penalty  (every token already in the sequence; the reference
//   divides whatever the sign);  p = softmax(l);  keep the nucleus: in descending p order, a token
//   is kept while the probability mass ranked before it is <= top_p;  draw one kept token with
//   probability p / (kept mass).
// The nucleus is found without sorting: with A(k) = sum of p_i over tokens whose fp32 bit
// pattern exceeds k (positive floats order like their bit patterns), the kept set is
// {i : bits(p_i) >= k*}, k* = min{k : A(k) <= top_p * sum(p)}, found by bisection over k.  For
// distinct probabilities this is exactly the reference's sorted-cumsum rule; tokens tied at the
// boundary are all kept (the reference's unstable sort keeps an arbitrary subset of them).
// The draw scans the kept tokens in vocabulary order (any fixed order gives the same
// distribution) against u * kept mass, u from splitmix64(seed, row, per-row counter).
#pragma once
#include "common.cuh"

namespace dfssm {

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;

__device__ __forceinline__ unsigned long long splitmix64(unsigned long long x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Sum / max over the CTA with a fixed order; every thread gets the total.
__device__ __forceinline__ float sample_block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll 8
  for (int j = 0; j < kSampleWarps; ++j) s += red[j];
  return s;
}
__device__ __forceinline__ float sample_block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = red[0];
#pragma unroll 8
  for (int j = 1; j < kSampleWarps; ++j) s = fmaxf(s, red[j]);
  return s;
}

// logits fp32 [B][V] (divided by temp, then seen ones by rep); seen bitmap uint32 [B][W] (W = ceil(V / 32)); counters uint64 [B] (one
// draw each, incremented); next int32 [B].  Optional: kept_mass [B] (kept mass / total mass) and
// kept_count [B].  Dynamic shared memory: V floats.
__global__ void __launch_bounds__(kSampleThreads)
sample_kernel(const float* __restrict__ logits, int V, const uint32_t* __restrict__ seen, int W, float temp,
              float top_p, float rep, unsigned long long seed, unsigned long long* __restrict__ counters,
              int* __restrict__ next, float* __restrict__ kept_mass, int* __restrict__ kept_count) {
  extern __shared__ float sp[];  // [V]: penalised scaled logits, then unnormalised probabilities
  __shared__ float red[kSampleWarps];
  __shared__ float s_scan[kSampleWarps];
  __shared__ int s_pick;
  const int row = blockIdx.x, tid = threadIdx.x;
  const float* lg = logits + (size_t)row * V;
  const uint32_t* sb = seen + (size_t)row * W;
  float m = -INFINITY;
  for (int i = tid; i < V; i += kSampleThreads) {
    float l = __fdiv_rn(lg[i], temp);  // divisions as in the reference, not reciprocal products
    if ((sb[i >> 5] >> (i & 31)) & 1u) l = __fdiv_rn(l, rep);
    sp[i] = l;
    m = fmaxf(m, l);
  }
  m = sample_block_max(m, red);
  float z = 0.f;
  for (int i = tid; i < V; i += kSampleThreads) {
    const float p = expf(sp[i] - m);
    sp[i] = p;
    z += p;
  }
  z = sample_block_sum(z, red);
  // bisection for k* over bit patterns [0, bits(1.0f)]: p <= 1 after subtracting the max
  const float lim = top_p * z;
  unsigned lo = 0u, hi = __float_as_uint(1.0f);  // A(hi) = 0 <= lim always
  while (lo < hi) {
    const unsigned mid = lo + ((hi - lo) >> 1);
    float a = 0.f;
    for (int i = tid; i < V; i += kSampleThreads) a += __float_as_uint(sp[i]) > mid ? sp[i] : 0.f;
    a = sample_block_sum(a, red);
    if (a <= lim) hi = mid;
    else lo = mid + 1;
  }
  const unsigned kstar = lo;
  // kept mass per thread over a contiguous chunk, then an exclusive scan over threads
  const int chunk = (V + kSampleThreads - 1) / kSampleThreads, c0 = tid * chunk, c1 = min(V, c0 + chunk);
  float mine = 0.f;
  int cnt = 0;
  for (int i = c0; i < c1; ++i)
    if (__float_as_uint(sp[i]) >= kstar) {
      mine += sp[i];
      ++cnt;
    }
  // inclusive warp scan, then warp totals
  const int lane = tid & 31, wid = tid >> 5;
  float inc = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) s_scan[wid] = inc;
  __syncthreads();
  float wbase = 0.f, total = 0.f;
  for (int j = 0; j < kSampleWarps; ++j) {
    const float v = s_scan[j];
    if (j < wid) wbase += v;
    total += v;
  }
  const float excl = wbase + inc - mine;
  const int kept = (int)sample_block_sum((float)cnt, red);
  if (tid == 0) s_pick = -1;
  __syncthreads();
  const unsigned long long ctr = counters[row];
  const unsigned long long r = splitmix64(seed ^ splitmix64(((unsigned long long)row << 40) ^ ctr));
  const float target = (float)(r >> 40) * (1.0f / 16777216.0f) * total;  // u in [0, 1) with 24 bits
  if (mine > 0.f && target >= excl && target < excl + mine) {
    float acc = excl;
    int pick = -1;
    for (int i = c0; i < c1; ++i)
      if (__float_as_uint(sp[i]) >= kstar) {
        acc += sp[i];
        pick = i;
        if (target < acc) break;
      }
    atomicMax(&s_pick, pick);  // one thread normally; rounding at a chunk edge may give two
  }
  __syncthreads();
  if (tid == 0) {
    int pick = s_pick;
    if (pick < 0) {  // target rounded past the last kept token: take the last kept token
      for (int i = V - 1; i >= 0; --i)
        if (__float_as_uint(sp[i]) >= kstar && sp[i] > 0.f) {
          pick = i;
          break;
        }
    }
    next[row] = pick;
    counters[row] = ctr + 1;
    if (kept_mass) kept_mass[row] = total / z;
    if (kept_count) kept_count[row] = kept;
  }
}

// Marks tokens[b] in row b of the seen bitmap.
__global__ void mark_seen_kernel(const int* __restrict__ tokens, int B, int V, uint32_t* __restrict__ seen, int W) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) {
    const int t = tokens[b];
    if (t >= 0 && t < V) atomicOr(seen + (size_t)b * W + (t >> 5), 1u << (t & 31));
  }
}

}  // namespace dfssm
