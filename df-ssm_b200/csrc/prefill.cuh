// Prompt prefill: T prompt tokens of every sequence in one pass per layer.  The projections run
// as one batched GEMM over all B*T token rows (proj_mma MODE 3, then MODE 1 for out_proj with the
// residual), and one CTA per (head, sequence) runs the recurrence over time for its head: the
// conv1d shift register over the T raw xBC values, then the state update, C.h + D.x and the gate
// token by token with the 64x128 fp32 state held in registers, so the state is read and written
// once per layer instead of once per token.  The arithmetic per token is that of the decode
// kernels (the in_proj conv epilogue and ssm_gate_kernel), in the same order.
#pragma once
#include <algorithm>

#include "common.cuh"

namespace dfssm {

constexpr int kScanThreads = 512;
constexpr int kScanMaxT = 64;  // tokens per scan launch (longer prompts run in chunks)

// proj fp16 [B*T rows][n_in]: z [d_inner] | x [d_inner] | B [d_state] | C [d_state] | dt [nheads]
// (row b*T + t).  Writes gated fp16 [B*T][d_inner]; updates this layer's conv state
// [B][3][d_xbc] (tap-major) and SSM state [B][nheads][64][128].
// Grid (nheads * SPLIT, B): CTA (h * SPLIT + part, b) owns channels p in [part * kScanRows,
// +kScanRows) of head h, kScanRows = 64 / SPLIT; SPLIT = 2 when one CTA per (head, sequence) leaves
// SMs idle and runs the conv of its x channels and of all B/C
// channels (the B/C conv is repeated by every CTA of the sequence; head 0 part 0 stores its state).
// Everything the token loop reads is staged in shared memory first, by coalesced row reads, so the
// loop itself touches no global memory: raw conv inputs (channel-major, 3 taps + T), conv + SiLU
// outputs (time-major, so a lane's 4 B/C values of one token are one conflict-free float4), the
// SiLU(z) gate factors, softplus(dt) and exp(A dt) per token, and the gated outputs (written to HBM
// as whole rows at the end).
// ---- SSD (chunked matrix) form of the chunk's recurrence, on the tensor cores
// With s_t = sum_{u <= t} dt_u A (A = -exp(A_log)), the state after token t is
//   h_t = e^{s_t} h_0 + sum_{u <= t} e^{s_t - s_u} dt_u x_u B_u^T
// so the chunk's outputs and final state are four small GEMMs per (head, sequence):
//   G = C B^T (T x T),  M = G o [u <= t] e^{s_t - s_u} dt_u,  Y = M X + diag(e^s) C h_0^T + D X,
//   h_T = e^{s_T} h_0 + (X^T diag(e^{s_T - s_u} dt_u)) B.
// They run as mma.sync m16n8k8 TF32 with fp32 accumulation.  x, B and C are fp16 values (the conv
// outputs), exact in TF32; the fp32 operands (M, h_0, the weighted X^T) are split into a TF32 high
// part and a TF32 remainder, two MMAs, so every product keeps ~22 significant bits.  The sums run
// in another order than the token loop's, within fp32 rounding of it.
__device__ __forceinline__ unsigned tf32_hi(float v) {
  unsigned r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ void tf32_split(float v, unsigned& hi, unsigned& lo) {
  hi = tf32_hi(v);
  lo = tf32_hi(v - __uint_as_float(hi));
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3, unsigned b0,
                                         unsigned b1) {
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared-memory floats of the SSD step for T tokens and R state rows: M [Tp][Tp+4], h_0 [R][N+4]
// (Tp = T rounded up to 16), then the gated outputs (fp16 [T][R]).
__host__ __device__ inline size_t ssd_smem_floats(int T, int rows, int d_state) {
  const size_t Tp = (size_t)(T + 15) / 16 * 16;
  return Tp * (Tp + 4) + (size_t)rows * (d_state + 4) + ((size_t)T * rows + 1) / 2;
}

// The SSD step of one CTA: its R state rows of one head over a chunk of T <= 64 tokens.  cvo holds
// the conv outputs time-major ([T][NCP]: x of the R rows, then B, then C), zg the SiLU(z) gate
// factors ([T][R + 1]), dts softplus(dt + bias); hv is this thread's part of h_0 (rows
// wid * R / 16 + r, columns 4 lane ..), hs the rows' fp32 state in HBM (written with h_T).  Writes
// the gated outputs to gs ([T][R] fp16).  Uses cum and wv ([T] each), M ([Tp][Tp + 4]) and h0s
// ([R][d_state + 4]).
template <int R>
__device__ void ssd_chunk(int T, int Tp, int N, int NCP, const float* cvo, const float* zg, const float* dts,
                          float Ah, float Dh, float* cum, float* wv, float* M, float* h0s, __half* gs,
                          const float4 (&hv)[R / 16], float* hs) {
  constexpr int RPW = R / 16;
  const int tid = threadIdx.x, wid = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const int MS = Tp + 4, HS = N + 4, ZS = R + 1;
  const float* xb = cvo;          // x[t][p] = xb[t * NCP + p]
  const float* Bm = cvo + R;      // B[t][n]
  const float* Cm = cvo + R + N;  // C[t][n]
#pragma unroll
  for (int r = 0; r < RPW; ++r)
    *reinterpret_cast<float4*>(h0s + (wid * RPW + r) * HS + 4 * lane) = hv[r];
  if (tid == 0) {  // s_t = sum_{u <= t} dt_u A, in token order
    float a = 0.f;
    for (int t = 0; t < T; ++t) {
      a += dts[t] * Ah;
      cum[t] = a;
    }
  }
  __syncthreads();
  const float sT = cum[T - 1];
  for (int t = tid; t < Tp; t += kScanThreads) wv[t] = t < T ? expf(sT - cum[t]) * dts[t] : 0.f;
  auto fp = [](float v) { return __float_as_uint(v); };  // fp16-exact values are exact TF32 operands
  // G = C B^T, masked and decayed into M
  const int nmt = Tp / 16, nnt = Tp / 8;
  for (int tile = wid; tile < nmt * nnt; tile += kScanThreads / 32) {
    const int mt = tile / nnt, nt = tile - mt * nnt;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const int ta = 16 * mt + g, tb = ta + 8, u = 8 * nt + g;
    if (8 * nt <= 16 * mt + 15) {  // tiles wholly above the diagonal stay zero
      const bool va = ta < T, vb = tb < T, vu = u < T;
      for (int k0 = 0; k0 < N; k0 += 8) {
        const unsigned a0 = va ? fp(Cm[ta * NCP + k0 + c]) : 0u, a2 = va ? fp(Cm[ta * NCP + k0 + c + 4]) : 0u;
        const unsigned a1 = vb ? fp(Cm[tb * NCP + k0 + c]) : 0u, a3 = vb ? fp(Cm[tb * NCP + k0 + c + 4]) : 0u;
        const unsigned b0 = vu ? fp(Bm[u * NCP + k0 + c]) : 0u, b1 = vu ? fp(Bm[u * NCP + k0 + c + 4]) : 0u;
        mma_tf32(acc, a0, a1, a2, a3, b0, b1);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = i < 2 ? ta : tb, v = 8 * nt + 2 * c + (i & 1);
      M[t * MS + v] = (v <= t && t < T) ? acc[i] * expf(cum[t] - cum[v]) * dts[v] : 0.f;
    }
  }
  __syncthreads();
  // outputs: Y = M X + diag(e^s) C h_0^T + D X, gated
  const int nyt = nmt * (R / 8);
  for (int tile = wid; tile < nyt; tile += kScanThreads / 32) {
    const int mt = tile / (R / 8), nt = tile - mt * (R / 8);
    const int ta = 16 * mt + g, tb = ta + 8, p = 8 * nt + g;
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc3[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < Tp; k0 += 8) {
      unsigned ah[4], al[4];
      tf32_split(M[ta * MS + k0 + c], ah[0], al[0]);
      tf32_split(M[tb * MS + k0 + c], ah[1], al[1]);
      tf32_split(M[ta * MS + k0 + c + 4], ah[2], al[2]);
      tf32_split(M[tb * MS + k0 + c + 4], ah[3], al[3]);
      const int u0 = k0 + c, u1 = u0 + 4;
      const unsigned b0 = u0 < T ? fp(xb[u0 * NCP + p]) : 0u, b1 = u1 < T ? fp(xb[u1 * NCP + p]) : 0u;
      mma_tf32(acc, ah[0], ah[1], ah[2], ah[3], b0, b1);
      mma_tf32(acc, al[0], al[1], al[2], al[3], b0, b1);
    }
    const bool va = ta < T, vb = tb < T;
    for (int k0 = 0; k0 < N; k0 += 8) {
      const unsigned a0 = va ? fp(Cm[ta * NCP + k0 + c]) : 0u, a2 = va ? fp(Cm[ta * NCP + k0 + c + 4]) : 0u;
      const unsigned a1 = vb ? fp(Cm[tb * NCP + k0 + c]) : 0u, a3 = vb ? fp(Cm[tb * NCP + k0 + c + 4]) : 0u;
      unsigned bh0, bl0, bh1, bl1;
      tf32_split(h0s[p * HS + k0 + c], bh0, bl0);
      tf32_split(h0s[p * HS + k0 + c + 4], bh1, bl1);
      mma_tf32(acc3, a0, a1, a2, a3, bh0, bh1);
      mma_tf32(acc3, a0, a1, a2, a3, bl0, bl1);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = i < 2 ? ta : tb, q = 8 * nt + 2 * c + (i & 1);
      if (t < T) {
        const float xv = xb[t * NCP + q];
        const float y = acc[i] + expf(cum[t]) * acc3[i] + xv * Dh;
        gs[t * R + q] = f2h(h2f(f2h(y)) * zg[t * ZS + q]);
      }
    }
  }
  // h_T = e^{s_T} h_0 + (X^T diag(wv)) B
  const float esT = expf(sT);
  const int nht = (R / 16) * (N / 8);
  for (int tile = wid; tile < nht; tile += kScanThreads / 32) {
    const int mt = tile / (N / 8), nt = tile - mt * (N / 8);
    const int pa = 16 * mt + g, pb = pa + 8, n = 8 * nt + g;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < Tp; k0 += 8) {
      const int u0 = k0 + c, u1 = u0 + 4;
      const float w0 = wv[u0], w1 = wv[u1];
      unsigned ah[4], al[4];
      tf32_split(u0 < T ? xb[u0 * NCP + pa] * w0 : 0.f, ah[0], al[0]);
      tf32_split(u0 < T ? xb[u0 * NCP + pb] * w0 : 0.f, ah[1], al[1]);
      tf32_split(u1 < T ? xb[u1 * NCP + pa] * w1 : 0.f, ah[2], al[2]);
      tf32_split(u1 < T ? xb[u1 * NCP + pb] * w1 : 0.f, ah[3], al[3]);
      const unsigned b0 = u0 < T ? fp(Bm[u0 * NCP + n]) : 0u, b1 = u1 < T ? fp(Bm[u1 * NCP + n]) : 0u;
      mma_tf32(acc, ah[0], ah[1], ah[2], ah[3], b0, b1);
      mma_tf32(acc, al[0], al[1], al[2], al[3], b0, b1);
    }
    const int nc = 8 * nt + 2 * c;
    const float2 ra = *reinterpret_cast<const float2*>(h0s + pa * HS + nc);
    const float2 rb = *reinterpret_cast<const float2*>(h0s + pb * HS + nc);
    __stcs(reinterpret_cast<float2*>(hs + (size_t)pa * N + nc), make_float2(acc[0] + esT * ra.x, acc[1] + esT * ra.y));
    __stcs(reinterpret_cast<float2*>(hs + (size_t)pb * N + nc), make_float2(acc[2] + esT * rb.x, acc[3] + esT * rb.y));
  }
}

template <int SPLIT, bool SSD>
__global__ void __launch_bounds__(kScanThreads)
prefill_scan_kernel(const __half* __restrict__ proj, int n_in, int T, int d_inner, int d_state, int nheads,
                    const __half* __restrict__ conv_w, const __half* __restrict__ conv_b,
                    const float* __restrict__ dt_bias, const float* __restrict__ A_log, const float* __restrict__ Dp,
                    float* __restrict__ conv_state, float* __restrict__ hstate, __half* __restrict__ gated) {
  constexpr int kScanRows = DFSSM_HEADDIM / SPLIT;           // state rows (head channels) per CTA
  constexpr int kScanRPW = kScanRows / (kScanThreads / 32);  // state rows per warp
  extern __shared__ float sm[];
  const int h = blockIdx.x / SPLIT, part = blockIdx.x - h * SPLIT, b = blockIdx.y, tid = threadIdx.x;
  const int c0 = h * DFSSM_HEADDIM + part * kScanRows;  // first head channel of this CTA
  const int d_xbc = d_inner + 2 * d_state;
  const int NC = kScanRows + 2 * d_state;  // this CTA's x channels, then all B and C channels
  const int NCP = NC + 4;                   // cvo row stride (padded against bank conflicts)
  const int TS = T + 3;
  const int Tp = (T + 15) & ~15;
  // raw is dead once the conv has run: the gated outputs (and the SSD step's M and h_0) reuse it
  const size_t raw_floats =
      ((SSD ? max((size_t)NC * TS, ssd_smem_floats(T, kScanRows, d_state)) : (size_t)NC * TS) + 3) & ~(size_t)3;
  float* raw = sm;                          // [NC][T + 3]: 3 taps of conv state, then the T raw inputs
  float* cvo = raw + raw_floats;            // [T][NCP]: fp16-exact conv + SiLU outputs
  constexpr int ZS = kScanRows + 1;         // padded: the staging stores run along t
  float* zg = cvo + NCP * T;                // [T][ZS]: fp16-exact SiLU(z)
  float* dts = zg + T * ZS;                 // [Tp]: softplus(dt + bias)
  float* abar = dts + Tp;                   // [Tp]: exp(A dt) (SSD: the state-update weights)
  float* cum = abar + Tp;                   // [Tp]: s_t (SSD)
  float* Msm = raw;                         // SSD: [Tp][Tp + 4]
  float* h0s = Msm + (size_t)Tp * (Tp + 4);  // SSD: [kScanRows][d_state + 4]
  __half* gs = reinterpret_cast<__half*>(SSD ? h0s + (size_t)kScanRows * (d_state + 4) : raw);  // [T][kScanRows]
  auto chan = [&](int c) { return c < kScanRows ? c0 + c : d_inner + (c - kScanRows); };
  // state tile: first, so the HBM stream starts before anything else
  const int wid = tid >> 5, lane = tid & 31, n0 = lane * 4;
  float* hs = hstate + ((size_t)b * nheads + h) * (DFSSM_HEADDIM * DFSSM_DSTATE) +
              (size_t)part * kScanRows * DFSSM_DSTATE;
  float4 hv[kScanRPW];
#pragma unroll
  for (int r = 0; r < kScanRPW; ++r)
    hv[r] = __ldcs(reinterpret_cast<const float4*>(hs + (wid * kScanRPW + r) * DFSSM_DSTATE + n0));
  const float Ah = -expf(A_log[h]), Dh = Dp[h], dtb = dt_bias[h];
  const __half* pb = proj + (size_t)b * T * n_in;
  const float* cs = conv_state + (size_t)b * 3 * d_xbc;
  for (int i = tid; i < NC * 3; i += kScanThreads) {
    const int k = i / NC, c = i - k * NC;
    raw[c * TS + k] = cs[(size_t)k * d_xbc + chan(c)];
  }
  // raw inputs and z by 16-byte loads, kU of them in flight per thread: a row t holds ux units of
  // this CTA's x channels, d_state/4 units of B and C, and ux units of z.  Unit u is (unit k = u / T,
  // token t = u % T), so a warp's shared-memory stores of one channel hit consecutive words.
  {
    constexpr int kU = 4;
    constexpr int ux = kScanRows / 8;
    const int ubc = 2 * d_state / 8, upr = ux + ubc + ux;  // units per row
    const int nu = T * upr;
    for (int u0 = tid; u0 < nu; u0 += kScanThreads * kU) {
      uint4 v[kU];
#pragma unroll
      for (int j = 0; j < kU; ++j) {
        const int u = u0 + j * kScanThreads;
        if (u < nu) {
          const int k = u / T, t = u - k * T;  // consecutive threads: consecutive tokens of one unit
          const size_t col = k < ux ? (size_t)d_inner + c0 + 8 * k
                                    : (k < ux + ubc ? (size_t)2 * d_inner + 8 * (k - ux)
                                                    : (size_t)c0 + 8 * (k - ux - ubc));
          v[j] = __ldcs(reinterpret_cast<const uint4*>(pb + (size_t)t * n_in + col));
        }
      }
#pragma unroll
      for (int j = 0; j < kU; ++j) {
        const int u = u0 + j * kScanThreads;
        if (u < nu) {
          const int k = u / T, t = u - k * T;
          const __half* hv8 = reinterpret_cast<const __half*>(&v[j]);
          if (k < ux + ubc) {
#pragma unroll
            for (int e = 0; e < 8; ++e) raw[(8 * k + e) * TS + 3 + t] = h2f(hv8[e]);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float z = h2f(hv8[e]);
              const float sig = round_h(1.0f / (1.0f + expf(-z)));
              zg[t * ZS + 8 * (k - ux - ubc) + e] = round_h(z * sig);
            }
          }
        }
      }
    }
  }
  for (int t = tid; t < T; t += kScanThreads) {
    const float dtv = log1pf(expf(h2f(pb[(size_t)t * n_in + d_inner + d_xbc + h]) + dtb));
    dts[t] = dtv;
    abar[t] = expf(dtv * Ah);
  }
  __syncthreads();
  // conv + SiLU: a thread owns a channel over a run of TL tokens and slides the 4-tap window
  const int nseg = T >= 32 ? 4 : 1, TL = (T + nseg - 1) / nseg;
  for (int item = tid; item < NC * nseg; item += kScanThreads) {
    const int seg = item / NC, c = item - seg * NC, ch = chan(c);
    const uint2 wv = *reinterpret_cast<const uint2*>(conv_w + ch * DFSSM_DCONV);
    const __half* w4 = reinterpret_cast<const __half*>(&wv);
    const float w0 = h2f(w4[0]), w1 = h2f(w4[1]), w2 = h2f(w4[2]), w3 = h2f(w4[3]), cb = h2f(conv_b[ch]);
    const int t0 = seg * TL, t1 = min(T, t0 + TL);
    const float* rr = raw + c * TS;
    float s0 = rr[t0], s1 = rr[t0 + 1], s2 = rr[t0 + 2];
    for (int t = t0; t < t1; ++t) {
      const float v = rr[3 + t];
      const float o2 = s0 * w0 + s1 * w1 + s2 * w2 + v * w3 + cb;
      const float sig = 1.0f / (1.0f + expf(-o2));
      cvo[t * NCP + c] = h2f(f2h(o2 * sig));
      s0 = s1;
      s1 = s2;
      s2 = v;
    }
  }
  // conv state after the prompt: the last three raw inputs (B/C channels written by one CTA)
  float* csw = conv_state + (size_t)b * 3 * d_xbc;
  for (int i = tid; i < NC * 3; i += kScanThreads) {
    const int k = i / NC, c = i - k * NC;
    if (c >= kScanRows && blockIdx.x != 0) continue;
    csw[(size_t)k * d_xbc + chan(c)] = raw[c * TS + T + k];
  }
  __syncthreads();
  if constexpr (SSD) {
    ssd_chunk<kScanRows>(T, Tp, d_state, NCP, cvo, zg, dts, Ah, Dh, cum, abar, Msm, h0s, gs, hv, hs);
  } else {
  for (int t = 0; t < T; ++t) {
    const float* ct = cvo + t * NCP;
    const float dtv = dts[t], Abar = abar[t];
    const float4 Bn = *reinterpret_cast<const float4*>(ct + kScanRows + n0);
    const float4 Cn = *reinterpret_cast<const float4*>(ct + kScanRows + d_state + n0);
    float part_[kScanRPW];
#pragma unroll
    for (int r = 0; r < kScanRPW; ++r) {
      const float X = ct[wid * kScanRPW + r] * dtv;
      float4 o;
      o.x = Abar * hv[r].x + X * Bn.x;
      o.y = Abar * hv[r].y + X * Bn.y;
      o.z = Abar * hv[r].z + X * Bn.z;
      o.w = Abar * hv[r].w + X * Bn.w;
      hv[r] = o;
      part_[r] = Cn.x * o.x + Cn.y * o.y + Cn.z * o.z + Cn.w * o.w;
    }
    // C.h of the warp's rows summed over the 32 lanes as a transposing butterfly: each exchange
    // halves the values a lane holds, so kScanRPW rows cost kScanRPW - 1 + 5 - log2(kScanRPW)
    // shuffles instead of 5 kScanRPW; the lane ends with the sum of row `rw`
    int rw = 0, off = 16;
#pragma unroll
    for (int n = kScanRPW; n > 1; n >>= 1, off >>= 1) {
      const bool hi = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < n / 2; ++i) {
        const float send = hi ? part_[i] : part_[i + n / 2];
        const float keep = hi ? part_[i + n / 2] : part_[i];
        part_[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
      rw += hi ? n / 2 : 0;
    }
#pragma unroll
    for (int o = off; o > 0; o >>= 1) part_[0] += __shfl_xor_sync(0xffffffffu, part_[0], o);
    if ((lane & (2 * off - 1)) == 0) {  // one lane per row
      const int pp = wid * kScanRPW + rw;
      const float y = part_[0] + ct[pp] * Dh;
      gs[t * kScanRows + pp] = f2h(h2f(f2h(y)) * zg[t * ZS + pp]);
    }
  }
#pragma unroll
  for (int r = 0; r < kScanRPW; ++r)
    __stcs(reinterpret_cast<float4*>(hs + (wid * kScanRPW + r) * DFSSM_DSTATE + n0), hv[r]);
  }
  __syncthreads();
  for (int i = tid; i < T * kScanRows / 2; i += kScanThreads) {
    const int t = i / (kScanRows / 2), p2 = i - t * (kScanRows / 2);
    reinterpret_cast<__half2*>(gated + ((size_t)b * T + t) * d_inner + c0)[p2] = reinterpret_cast<const __half2*>(gs)[i];
  }
}

inline size_t prefill_scan_smem(int T, int d_state, int split, bool ssd) {
  const size_t rows = DFSSM_HEADDIM / split, nc = rows + 2 * d_state;
  size_t raw = nc * (T + 3);
  if (ssd) raw = std::max(raw, ssd_smem_floats(T, (int)rows, d_state));
  raw = (raw + 3) & ~(size_t)3;
  const size_t Tp = (size_t)(T + 15) / 16 * 16;
  return (raw + (nc + 4) * T + (size_t)T * (rows + 1) + 3 * Tp) * sizeof(float);
}

// x rows b*T + t = the embedding of tokens[b][t] (fp16, as embed_kernel).
__global__ void embed_rows_kernel(const int* __restrict__ tokens, const int8_t* __restrict__ Eq,
                                  const float* __restrict__ Es, int d_model, int vocab, __half* __restrict__ x) {
  const int r = blockIdx.x;
  int tok = tokens[r];
  tok = min(max(tok, 0), vocab - 1);
  const float s = Es[tok];
  const int8_t* er = Eq + (size_t)tok * d_model;
  for (int k = threadIdx.x; k < d_model; k += blockDim.x) x[(size_t)r * d_model + k] = f2h((float)er[k] * s);
}

// Row b*T + T - 1 of src -> row b of dst (the last prompt token of every sequence).
__global__ void last_rows_kernel(const __half* __restrict__ src, int T, int width, __half* __restrict__ dst) {
  const int b = blockIdx.x;
  const __half* s = src + ((size_t)b * T + T - 1) * width;
  for (int k = threadIdx.x; k < width; k += blockDim.x) dst[(size_t)b * width + k] = s[k];
}

// Marks tokens[b][t] in row b of the seen bitmap.
__global__ void mark_seen_rows_kernel(const int* __restrict__ tokens, int B, int T, int V, uint32_t* __restrict__ seen,
                                      int W) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < B * T) {
    const int b = i / T, tok = tokens[i];
    if (tok >= 0 && tok < V) atomicOr(seen + (size_t)b * W + (tok >> 5), 1u << (tok & 31));
  }
}

}  // namespace dfssm
