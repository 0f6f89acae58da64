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

constexpr int kScanThreads = 256;
constexpr int kScanMaxT = 64;  // tokens per scan launch (longer prompts run in chunks)

// proj fp16 [B*T rows][n_in]: z [d_inner] | x [d_inner] | B [d_state] | C [d_state] | dt [nheads]
// (row b*T + t).  Writes gated fp16 [B*T][d_inner]; updates this layer's conv state
// [B][3][d_xbc] (tap-major) and SSM state [B][nheads][64][128].
// Dynamic shared memory: (64 + 2*d_state) channels x (T + 3) fp32 raw inputs, then the same
// channels x T conv outputs.
__global__ void __launch_bounds__(kScanThreads)
prefill_scan_kernel(const __half* __restrict__ proj, int n_in, int T, int d_inner, int d_state, int nheads,
                    const __half* __restrict__ conv_w, const __half* __restrict__ conv_b,
                    const float* __restrict__ dt_bias, const float* __restrict__ A_log, const float* __restrict__ Dp,
                    float* __restrict__ conv_state, float* __restrict__ hstate, __half* __restrict__ gated) {
  extern __shared__ float sm[];
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int d_xbc = d_inner + 2 * d_state;
  const int NC = DFSSM_HEADDIM + 2 * d_state;  // this head's x channels, then all B and C channels
  const int TS = T + 3;
  float* raw = sm;                  // [NC][T + 3]: 3 taps of conv state, then the T raw inputs
  float* cvo = sm + NC * TS;        // [NC][T]: fp16-exact conv + SiLU outputs
  auto chan = [&](int c) { return c < DFSSM_HEADDIM ? h * DFSSM_HEADDIM + c : d_inner + (c - DFSSM_HEADDIM); };
  // state tile: first, so the HBM stream starts before anything else
  const int wid = tid >> 5, lane = tid & 31, n0 = lane * 4;
  float* hs = hstate + ((size_t)b * nheads + h) * (DFSSM_HEADDIM * DFSSM_DSTATE);
  float4 hv[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) hv[r] = __ldcs(reinterpret_cast<const float4*>(hs + (wid * 8 + r) * DFSSM_DSTATE + n0));
  const float* cs = conv_state + (size_t)b * 3 * d_xbc;
  for (int i = tid; i < NC * TS; i += kScanThreads) {
    const int c = i / TS, k = i - c * TS, ch = chan(c);
    raw[i] = k < 3 ? cs[(size_t)k * d_xbc + ch] : h2f(proj[((size_t)b * T + (k - 3)) * n_in + d_inner + ch]);
  }
  __syncthreads();
  for (int i = tid; i < NC * T; i += kScanThreads) {
    const int c = i / T, t = i - c * T, ch = chan(c);
    const float* rr = raw + c * TS + t;
    const __half* cw = conv_w + ch * DFSSM_DCONV;
    const float s0 = rr[0], s1 = rr[1], s2 = rr[2], v = rr[3];
    const float o2 = s0 * h2f(cw[0]) + s1 * h2f(cw[1]) + s2 * h2f(cw[2]) + v * h2f(cw[3]) + h2f(conv_b[ch]);
    const float sig = 1.0f / (1.0f + expf(-o2));
    cvo[i] = h2f(f2h(o2 * sig));
  }
  __syncthreads();
  // conv state after the prompt: the last three raw inputs (B/C channels written by head 0)
  float* csw = conv_state + (size_t)b * 3 * d_xbc;
  for (int i = tid; i < NC * 3; i += kScanThreads) {
    const int c = i / 3, k = i - c * 3;
    if (c >= DFSSM_HEADDIM && h != 0) continue;
    csw[(size_t)k * d_xbc + chan(c)] = raw[c * TS + T + k];
  }
  const float Ah = -expf(A_log[h]), Dh = Dp[h], dtb = dt_bias[h];
  const float* Bs = cvo + DFSSM_HEADDIM * T;  // channel-major: B channel n at Bs[n * T + t]
  const float* Cs = Bs + d_state * T;
  for (int t = 0; t < T; ++t) {
    const size_t row = (size_t)b * T + t;
    const __half* pr = proj + row * n_in;
    float dtv = h2f(pr[d_inner + d_xbc + h]) + dtb;
    dtv = log1pf(expf(dtv));
    const float Abar = expf(dtv * Ah);
    float Bn[4], Cn[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      Bn[i] = Bs[(n0 + i) * T + t];
      Cn[i] = Cs[(n0 + i) * T + t];
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int pp = wid * 8 + r;
      const float xv = cvo[pp * T + t];
      const float X = xv * dtv;
      float4 o;
      o.x = Abar * hv[r].x + X * Bn[0];
      o.y = Abar * hv[r].y + X * Bn[1];
      o.z = Abar * hv[r].z + X * Bn[2];
      o.w = Abar * hv[r].w + X * Bn[3];
      hv[r] = o;
      float part = Cn[0] * o.x + Cn[1] * o.y + Cn[2] * o.z + Cn[3] * o.w;
      part = warp_sum(part);
      if (lane == r) {
        const float y = part + xv * Dh;
        __half o16 = f2h(y);
        const float z = h2f(pr[h * DFSSM_HEADDIM + pp]);
        const float sig = round_h(1.0f / (1.0f + expf(-z)));
        const float silu = round_h(z * sig);
        o16 = f2h(h2f(o16) * silu);
        gated[row * d_inner + h * DFSSM_HEADDIM + pp] = o16;
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) __stcs(reinterpret_cast<float4*>(hs + (wid * 8 + r) * DFSSM_DSTATE + n0), hv[r]);
}

inline size_t prefill_scan_smem(int T, int d_state) {
  return (size_t)(DFSSM_HEADDIM + 2 * d_state) * (2 * T + 3) * sizeof(float);
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
