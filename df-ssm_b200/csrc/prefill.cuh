// Prompt prefill: T prompt tokens of every sequence in one pass per layer.  The projections run
// as one batched GEMM over all B*T token rows (proj_mma MODE 3, then MODE 1 for out_proj with the
// residual), and one CTA per (head, sequence) runs the recurrence over time for its head: the
// conv1d shift register over the T raw xBC values, then the state update, C.h + D.x and the gate
// token by token with the 64x128 fp32 state held in registers, so the state is read and written
// once per layer instead of once per token.  The arithmetic per token is that of the decode
// kernels (the in_proj conv epilogue and ssm_gate_kernel), in the same order.
#pragma once
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
template <int SPLIT>
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
  const int TS = T + 3;
  float* raw = sm;                          // [NC][T + 3]: 3 taps of conv state, then the T raw inputs
  float* cvo = raw + NC * TS;               // [T][NC]: fp16-exact conv + SiLU outputs
  constexpr int ZS = kScanRows + 1;         // padded: the staging stores run along t
  float* zg = cvo + NC * T;                 // [T][ZS]: fp16-exact SiLU(z)
  float* dts = zg + T * ZS;                 // [T]: softplus(dt + bias)
  float* abar = dts + T;                    // [T]: exp(A dt)
  __half* gs = reinterpret_cast<__half*>(raw);  // [T][kScanRows] gated outputs (raw is dead by then)
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
      cvo[t * NC + c] = h2f(f2h(o2 * sig));
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
  for (int t = 0; t < T; ++t) {
    const float* ct = cvo + t * NC;
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
  __syncthreads();
  for (int i = tid; i < T * kScanRows / 2; i += kScanThreads) {
    const int t = i / (kScanRows / 2), p2 = i - t * (kScanRows / 2);
    reinterpret_cast<__half2*>(gated + ((size_t)b * T + t) * d_inner + c0)[p2] = reinterpret_cast<const __half2*>(gs)[i];
  }
}

inline size_t prefill_scan_smem(int T, int d_state, int split) {
  const size_t rows = DFSSM_HEADDIM / split, nc = rows + 2 * d_state;
  return (nc * (2 * T + 3) + (size_t)T * (rows + 1) + 2 * T) * sizeof(float);
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
