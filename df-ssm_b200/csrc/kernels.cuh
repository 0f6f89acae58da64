// Per-op decode kernels for sm_100a (any batch size).
//
// One decode step of one layer is, in launch order:
//   act_prep   (in)  RMSNorm(x)·ln_w -> fp16, per-row int8 quantisation, LoRA t = x·B^T
//   proj_gemv  (in)  packed 1-bit scaffold GEMV + dequant + LoRA + conv1d/SiLU epilogue
//   ssm_gate         dt softplus, exp(A·dt), state update, C·h + D·x, y·silu(z)
//   act_prep   (out) RMSNorm(gated)·norm_w, quantisation, LoRA t
//   proj_gemv  (out) scaffold GEMV + dequant + LoRA + residual add into x
// and once per step: embed (token -> x), act_prep (final norm), lm_head (int8 GEMV with
// a fused fp16-rounded argmax), finalize (winning token id).
//
// Every rounding point follows the reference GPU path
// (inference/gpu/df_ssm_inference.py:141-210, inference/gpu/df_ssm_kernels.cu:27-103).
#pragma once
#include "prep.cuh"

namespace dfssm {

// Error word of the per-op kernels' bounded waits (1: tcgen05 projection, 2: mma.sync projection
// activations, 4: tensor-core LM head activations); read and reported by dfssm_check_finite.
__device__ unsigned g_umma_err;

constexpr int kPrepThreads = 256;
constexpr int kGemvThreads = 256;
constexpr int kGemvBT = 16;      // batch rows per GEMV pass (one per lane of a half-warp)
constexpr int kSsmThreads = 256;
constexpr int kHeadThreads = 256;
constexpr int kHeadBT = 8;

// ---------------------------------------------------------------------------------------
// act_prep: one CTA per batch row.
//   xn = fp16((x * rsqrt(mean(x^2) + 1e-5)) * w)          df_ssm_inference.py:141-145
//   s  = fp16(max(amax|xn|, fp16(1e-4)) * (1/127))          df_ssm_inference.py:150
//   q  = clamp(rne(fp16(xn / s)), -128, 127)                df_ssm_inference.py:151
//   t_r = fp16(sum_k xn_k * B16[r][k])                      df_ssm_inference.py:92-97,173
// q is written in the permuted layout of qperm_index(); qsum = sum_k q_k.
// With quant == 0 only xn is produced (final norm before the LM head).
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kPrepThreads)
act_prep_kernel(const __half* __restrict__ in, int K, const float* __restrict__ w, int quant,
                __half* __restrict__ xn_out, int8_t* __restrict__ q_out, __half* __restrict__ xs_out,
                int* __restrict__ qsum_out, const __half* __restrict__ B16,
                __half* __restrict__ t_out) {
  extern __shared__ __align__(16) unsigned char smem[];
  __half* sxn = reinterpret_cast<__half*>(smem);
  __shared__ float red[kPrepThreads / 32];
  __shared__ int ired[kPrepThreads / 32];
  const int b = blockIdx.x;
  const __half* xr = in + (size_t)b * K;

  float ss = 0.f;
  for (int k = threadIdx.x; k < K; k += kPrepThreads) {
    float v = h2f(xr[k]);
    ss = __fadd_rn(ss, __fmul_rn(v, v));
  }
  ss = block_sum<kPrepThreads / 32>(ss, red);
  const float var = __fmul_rn(ss, 1.0f / (float)K);
  const float r = rsqrtf(__fadd_rn(var, 1e-5f));

  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += kPrepThreads) {
    __half xn = f2h(__fmul_rn(__fmul_rn(h2f(xr[k]), r), w[k]));
    sxn[k] = xn;
    amax = fmaxf(amax, fabsf(h2f(xn)));
    if (!quant) xn_out[(size_t)b * K + k] = xn;
  }
  if (!quant) return;
  amax = block_max<kPrepThreads / 32>(amax, red);
  const __half s16 = f2h(__fmul_rn(fmaxf(amax, qscale_floor()), 1.0f / 127.0f));
  const float s = h2f(s16);

  int qs = 0;
  int8_t* qrow = q_out + (size_t)b * K;
  for (int k = threadIdx.x; k < K; k += kPrepThreads) {
    float t = round_h(h2f(sxn[k]) / s);
    int q = (int)rint_alu(t);
    q = max(-128, min(127, q));
    qrow[qperm_index(k)] = (int8_t)q;
    qs += q;
  }
  qs = block_isum<kPrepThreads / 32>(qs, ired);
  if (threadIdx.x == 0) {
    xs_out[b] = s16;
    qsum_out[b] = qs;
  }
  // LoRA down-projection: warp w handles ranks 2w and 2w+1.
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int rk = wid * 2 + rr;
    const __half* brow = B16 + (size_t)rk * K;
    float acc = 0.f;
    if ((K & 255) == 0) {
      // 8 contiguous columns per lane per step: one 16-byte load of B and of x_norm
#pragma unroll 4
      for (int k = lane * 8; k < K; k += 256) {
        const uint4 bv = __ldg(reinterpret_cast<const uint4*>(brow + k));
        const uint4 xv = *reinterpret_cast<const uint4*>(sxn + k);
        const __half* bh = reinterpret_cast<const __half*>(&bv);
        const __half* xh = reinterpret_cast<const __half*>(&xv);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(h2f(xh[j]), h2f(bh[j]), acc);
      }
    } else {
      for (int k = lane; k < K; k += 32) acc = fmaf(h2f(sxn[k]), h2f(brow[k]), acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) t_out[b * DFSSM_RANK + rk] = f2h(acc);
  }
}

// act_prep_fast: the same prologue as act_prep_kernel (quantising variant) for K = 512 * KPT,
// with 512 threads that each keep KPT columns and their LoRA-B slices in registers and one
// combined block reduction for the LoRA partials and the q sum.  Grid (rows, PARTS): CTA (b, p)
// computes ranks p * 16 / PARTS.. of row b's LoRA down-projection (dividing each CTA's LoRA-B
// stream); all compute the identical q, xs and qsum, which CTA p = 0 stores.  More parts put more
// SMs on few rows.
template <int KPT, int PARTS = 2>
__global__ void __launch_bounds__(kPrepFastThreads)
act_prep_fast_kernel(const __half* __restrict__ in, int K, const float* __restrict__ w, int8_t* __restrict__ q_out,
                     __half* __restrict__ xs_out, int* __restrict__ qsum_out, const __half* __restrict__ B16,
                     __half* __restrict__ t_out) {
  constexpr int NR = DFSSM_RANK / PARTS;
  __shared__ float red[(kPrepFastWarps + 1) * (NR + 1)];
  __shared__ float s_t[NR];
  __shared__ float s_xs[1];
  __shared__ int s_qsum[1];
  __shared__ __align__(16) int8_t s_q[KPT * kPrepFastThreads];
  const int b = blockIdx.x, part = blockIdx.y, k0 = threadIdx.x * KPT;
  float wv[KPT];
  float vals[1][KPT];
  typename RankHalves<KPT>::T lb[NR];
  load_lora_b_ranks<KPT, NR>(B16, K, part * NR, lb);
  const __half* xr = in + (size_t)b * K + k0;
#pragma unroll
  for (int j = 0; j < KPT; ++j) {
    wv[j] = __ldg(w + k0 + j);
    vals[0][j] = h2f(xr[j]);
  }
  prep_rows<1, KPT, false, NR>(vals, wv, K, lb, s_q, K, s_xs, s_qsum, s_t, red);
  if (threadIdx.x < NR) t_out[b * DFSSM_RANK + part * NR + threadIdx.x] = f2h(s_t[threadIdx.x]);
  if (part == 0) {
    int4* dst = reinterpret_cast<int4*>(q_out + (size_t)b * K);
    const int4* src = reinterpret_cast<const int4*>(s_q);
    for (int i = threadIdx.x; i < K / 16; i += kPrepFastThreads) dst[i] = src[i];
    if (threadIdx.x == 0) {
      xs_out[b] = f2h(s_xs[0]);
      qsum_out[b] = s_qsum[0];
    }
  }
}

// Stand-alone RMSNorm + int8 quantisation of fp16 rows with the prologue functions of the
// persistent step kernel (prep_norm, prep_quantize): one 512-thread CTA per row, K = 512 KPT.
// Writes the normalised fp16 row, its fp16 scale and q in natural column order.
template <int KPT>
__global__ void __launch_bounds__(kPrepFastThreads)
rmsnorm_quant_kernel(const __half* __restrict__ in, int K, const float* __restrict__ w, __half* __restrict__ xn_out,
                     __half* __restrict__ xs_out, int8_t* __restrict__ q_out) {
  __shared__ __align__(16) float red[256];  // prep_norm uses red[0, 16), prep_quantize red[128, 144)
  __shared__ float s_xs[1];
  __shared__ int s_qpart[kPrepFastWarps];
  __shared__ __align__(16) int8_t s_q[KPT * kPrepFastThreads];
  const int b = blockIdx.x, k0 = threadIdx.x * KPT;
  float wv[KPT];
  float vals[1][KPT];
#pragma unroll
  for (int j = 0; j < KPT; ++j) {
    wv[j] = __ldg(w + k0 + j);
    vals[0][j] = h2f(in[(size_t)b * K + k0 + j]);
  }
  prep_norm<1, KPT>(vals, wv, K, red);
#pragma unroll
  for (int j = 0; j < KPT; ++j) xn_out[(size_t)b * K + k0 + j] = f2h(vals[0][j]);
  prep_quantize<1, KPT, false>(vals, s_q, K, s_xs, s_qpart, red + 128);
  for (int k = threadIdx.x; k < K; k += kPrepFastThreads) q_out[(size_t)b * K + k] = s_q[qperm_index(k)];
  if (threadIdx.x == 0) xs_out[b] = f2h(s_xs[0]);
}

// ---------------------------------------------------------------------------------------
// proj_gemv: packed 1-bit scaffold projection.
// Each half-warp owns one output row at a time; lane l16 streams 128-bit chunks
// c = l16, l16+16, ... of the row, expands the 128 sign bits into 32 0/1-byte masks
// ((word >> i) & 0x01010101) and dot-products them with the permuted int8 activations
// (dp4a).  sum_k s_k q_k = 2 * sum_{bit=1} q_k - sum_k q_k with s = +-1, so the int32
// result equals torch._int_mm on the unpacked +-1 weights bit for bit
// (df_ssm_inference.py:157).  The 16 per-batch partial sums of a half-warp are combined
// by a reduce-scatter so that lane l16 ends up with batch row l16 and runs its epilogue:
//   base = fp16(fp16(fp16(acc) * xs) * w_scale)                df_ssm_inference.py:158
//   v    = fp16(base + sum_r t_r * A16[n][r])                  df_ssm_inference.py:173,204
// MODE 0 (in_proj): rows in [d_inner, d_inner + d_xbc) also run the conv1d shift
// register + SiLU (df_ssm_kernels.cu:27-47) with fp32 state [B][3][d_xbc].
// MODE 1 (out_proj): x = fp16(x + v)                           df_ssm_inference.py:207
// MODE 2: raw int32 accumulators (stand-alone scaffold GEMM), `out` is int32 [B][ld_out].
// MODE 4: as MODE 2 from int8 activations in natural column order (q [B][K] row-major, qsum
// unused): each CTA permutes them into shared memory and sums the rows itself, so the stand-alone
// GEMM needs no separate permute launch.
// ---------------------------------------------------------------------------------------
template <int MODE>
__global__ void __launch_bounds__(kGemvThreads)
proj_gemv_kernel(ProjW p, const int8_t* __restrict__ q, const int* __restrict__ qsum,
                 const __half* __restrict__ xs, const __half* __restrict__ t, int B,
                 __half* __restrict__ out, int ld_out,
                 float* __restrict__ conv_state, const __half* __restrict__ conv_w,
                 const __half* __restrict__ conv_b, int d_inner, int d_xbc) {
  extern __shared__ __align__(16) unsigned char smem[];
  int8_t* sq = reinterpret_cast<int8_t*>(smem);  // [kGemvBT][K]
  __shared__ int s_qs[kGemvBT];                  // MODE 4: row sums of the staged activations
  const int K = p.K, N = p.N;
  const int C = K >> 7;  // 128-bit chunks per row
  const int lane = threadIdx.x & 31, l16 = lane & 15, half = lane >> 4;
  const int warp_g = blockIdx.x * (kGemvThreads / 32) + (threadIdx.x >> 5);
  const int warp_stride = gridDim.x * (kGemvThreads / 32);

  for (int bt0 = 0; bt0 < B; bt0 += kGemvBT) {
    const int nb = min(kGemvBT, B - bt0);
    __syncthreads();
    if (MODE == 4) {  // natural-order rows: permute into shared memory and sum them here
      if (threadIdx.x < kGemvBT) s_qs[threadIdx.x] = 0;
      __syncthreads();
      const int n16 = nb * K / 16;
      for (int i = threadIdx.x; i < n16; i += kGemvThreads) {
        const int r = (i * 16) / K, k0 = i * 16 - r * K;
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(q + (size_t)(bt0 + r) * K + k0));
        const int8_t* vb = reinterpret_cast<const int8_t*>(&v);
        int rs = 0;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          sq[r * K + qperm_index(k0 + e)] = vb[e];
          rs += vb[e];
        }
        atomicAdd(s_qs + r, rs);
      }
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(q + (size_t)bt0 * K);
      uint4* dst = reinterpret_cast<uint4*>(sq);
      const int n16 = nb * K / 16;
      for (int i = threadIdx.x; i < n16; i += kGemvThreads) dst[i] = src[i];
    }
    __syncthreads();
    for (int rp = warp_g; rp * 2 < N; rp += warp_stride) {
      const int row = rp * 2 + half;
      const bool valid = row < N;
      int acc[kGemvBT];
#pragma unroll
      for (int b = 0; b < kGemvBT; ++b) acc[b] = 0;
      if (valid) {
        const uint4* wrow = reinterpret_cast<const uint4*>(p.bits + (size_t)row * (K >> 5));
        for (int c = l16; c < C; c += 16) {
          const uint4 wv = ldg_stream(wrow + c);
          unsigned m[32];
          const unsigned ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int i = 0; i < 8; ++i) m[j * 8 + i] = (ws[j] >> i) & 0x01010101u;
#pragma unroll
          for (int b = 0; b < kGemvBT; ++b) {
            if (b < nb) {
              const int4* qv = reinterpret_cast<const int4*>(sq + b * K + c * 128);
              int a = acc[b];
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const int4 qq = qv[u];
                a = dp4a_us(m[4 * u + 0], qq.x, a);
                a = dp4a_us(m[4 * u + 1], qq.y, a);
                a = dp4a_us(m[4 * u + 2], qq.z, a);
                a = dp4a_us(m[4 * u + 3], qq.w, a);
              }
              acc[b] = a;
            }
          }
        }
      }
      // reduce-scatter across the 16 lanes of each half-warp: lane l16 <- batch row l16
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const bool up = l16 & 8;
        const int send = up ? acc[j] : acc[j + 8];
        const int keep = up ? acc[j + 8] : acc[j];
        acc[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const bool up = l16 & 4;
        const int send = up ? acc[j] : acc[j + 4];
        const int keep = up ? acc[j + 4] : acc[j];
        acc[j] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const bool up = l16 & 2;
        const int send = up ? acc[j] : acc[j + 2];
        const int keep = up ? acc[j + 2] : acc[j];
        acc[j] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
      }
      {
        const bool up = l16 & 1;
        const int send = up ? acc[0] : acc[1];
        const int keep = up ? acc[1] : acc[0];
        acc[0] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
      }
      const int b = bt0 + l16;
      if (!valid || l16 >= nb) continue;
      const int dot = 2 * acc[0] - (MODE == 4 ? s_qs[l16] : qsum[b]);
      if (MODE == 2 || MODE == 4) {
        reinterpret_cast<int*>(out)[(size_t)b * ld_out + row] = dot;
        continue;
      }
      const float base = round_h(round_h(round_h((float)dot) * h2f(xs[b])) * h2f(p.scale[row]));
      // LoRA up-projection
      const __half* arow = p.A16 + (size_t)row * DFSSM_RANK;
      const __half* tb = t + b * DFSSM_RANK;
      float la = 0.f;
#pragma unroll
      for (int r = 0; r < DFSSM_RANK; ++r) la = fmaf(h2f(tb[r]), h2f(arow[r]), la);
      const float v = round_h(base + round_h(la));
      if (MODE == 0) {
        float res = v;
        const int ch = row - d_inner;
        if (ch >= 0 && ch < d_xbc) {
          float* cs = conv_state + (size_t)b * 3 * d_xbc;
          const float s0 = cs[ch], s1 = cs[d_xbc + ch], s2 = cs[2 * d_xbc + ch];
          cs[ch] = s1;
          cs[d_xbc + ch] = s2;
          cs[2 * d_xbc + ch] = v;
          const __half* cw = conv_w + ch * DFSSM_DCONV;
          const float o = s0 * h2f(cw[0]) + s1 * h2f(cw[1]) + s2 * h2f(cw[2]) + v * h2f(cw[3]) + h2f(conv_b[ch]);
          const float sig = 1.0f / (1.0f + expf(-o));
          res = o * sig;
        }
        out[(size_t)b * ld_out + row] = f2h(res);
      } else {
        __half* xo = out + (size_t)b * ld_out + row;
        *xo = f2h(h2f(*xo) + v);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// proj_mma: the same projection as proj_gemv on int8 tensor cores, for batches of 8 or more.
// mma.sync m16n8k32 (s8 x s8 -> s32) with the weights on the M side: a warp owns 16 output rows
// and a slice of K, and the batch rows are the N side (NT tiles of 8).  The A fragment of row r
// for 32 columns is built straight from the packed word w of those columns: register
// (w >> j) & 0x01010101 holds the 0/1 signs of columns {j, 8+j, 16+j, 24+j}, which is exactly
// the permuted activation int j of that word (qperm_index), so lane (g, c) uses j = c and c + 4.
// sum_k s_k q_k = 2 * sum_{bit=1} q_k - sum_k q_k as in proj_gemv; the K slices of a CTA's warps
// are added exactly in int32 through shared memory before the shared epilogue.
// Activation rows sit in shared memory with a stride of K + 16 bytes (bank-conflict-free B loads).
// MODE 0: in_proj epilogue with the conv1d step; 1: out_proj with the residual add; 2: raw int32
// accumulators; 3: dequantised projection only (prompt rows, whose conv runs in the prefill scan).
// ---------------------------------------------------------------------------------------
constexpr int kMmaThreads = 256;
constexpr int kMmaNT = 4;  // most batch tiles of 8 per pass (32 rows)
constexpr int kMmaMaxBlk = 8;  // 16-byte weight blocks per warp slice (<= 32 words)

__device__ __forceinline__ void mma_s8(int (&d)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3, unsigned b0,
                                       unsigned b1) {
  asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two CTAs per SM (caps registers at 128): the in_proj grid has 266 CTAs, which one CTA per SM
// would run as two waves.
// NT batch tiles of 8 per pass (NB = 8 NT rows): the launcher picks the smallest NT that holds the
// batch (1, 2 or 4), so a batch of 8 does not run the MMAs, fragment loads and epilogue slots of 32.
template <int MODE, int RG, int NT = kMmaNT>
__global__ void __launch_bounds__(kMmaThreads, 2)
proj_mma_kernel(ProjW p, const int8_t* __restrict__ q, const int* __restrict__ qsum,
                const __half* __restrict__ xs, const __half* __restrict__ t, int B,
                __half* __restrict__ out, int ld_out,
                float* __restrict__ conv_state, const __half* __restrict__ conv_w,
                const __half* __restrict__ conv_b, int d_inner, int d_xbc) {
  constexpr int KS = (kMmaThreads / 32) / RG;  // K slices per CTA
  constexpr int NB = 8 * NT;                   // batch rows per pass
  constexpr int R = 16 * RG;                   // output rows per CTA
  extern __shared__ __align__(16) unsigned char smem[];
  const int K = p.K, N = p.N, W = K >> 5;
  const int SQ = K + 16;                                         // padded activation row stride
  int8_t* sq = reinterpret_cast<int8_t*>(smem);                  // [NB][SQ]
  int* red = reinterpret_cast<int*>(smem + NB * SQ);             // [KS][NB][R] (batch-major)
  // epilogue operands, loaded with independent loads before the MMA loop
  float* e_cs = reinterpret_cast<float*>(red + KS * R * NB);     // [NB][3][R] conv state (MODE 0)
  float* e_t = e_cs + NB * 3 * R;                                // [NB][16]
  float* e_a = e_t + NB * DFSSM_RANK;                            // [R][17] LoRA A (padded row)
  float* e_cw = e_a + R * (DFSSM_RANK + 1);                      // [R][4] conv weights
  float* e_misc = e_cw + R * 4;                                  // scale[R], conv_b[R], xs[NB], qsum[NB]
  float* e_scale = e_misc;
  float* e_cb = e_scale + R;
  float* e_xs = e_cb + R;
  int* e_qsum = reinterpret_cast<int*>(e_xs + NB);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const int rg = wid % RG, ks = wid / RG;
  const int row0 = blockIdx.x * R;
  const int wr = row0 + rg * 16;                                 // this warp's first row
  const int wpw = W / KS, kw0 = ks * wpw;                        // words per warp slice
  const int ra = min(wr + g, N - 1), rb = min(wr + g + 8, N - 1);
  const uint4* pa = reinterpret_cast<const uint4*>(p.bits + (size_t)ra * W);
  const uint4* pb = reinterpret_cast<const uint4*>(p.bits + (size_t)rb * W);
  __shared__ uint64_t qbar;
  // The first pass's activation copies and weight words go out before anything else, so their
  // round trips overlap the staging of the epilogue operands.
  auto issue_q = [&](int bt0, int nb) {
    if (wid == 0) {
      if (lane == 0) mbar_expect_tx(&qbar, (unsigned)(nb * K));
      __syncwarp();
      for (int b = lane; b < nb; b += 32) bulk_g2s(sq + b * SQ, q + (size_t)(bt0 + b) * K, (unsigned)K, &qbar);
    }
  };
  // this warp's weight words for the whole K slice (wpw <= 4 * kMmaMaxBlk words)
  uint4 wva[kMmaMaxBlk], wvb[kMmaMaxBlk];
  auto load_w = [&]() {
#pragma unroll
    for (int u = 0; u < kMmaMaxBlk; ++u) {
      if (4 * u < wpw) {
        wva[u] = ldg_stream(pa + (kw0 >> 2) + u);
        wvb[u] = ldg_stream(pb + (kw0 >> 2) + u);
      }
    }
  };
  if (threadIdx.x == 0) {
    mbar_init(&qbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  issue_q(0, min(NB, B));
  load_w();
  if (MODE != 2) {  // per-row epilogue operands (independent of the batch pass)
    constexpr int NF = DFSSM_RANK + 6, U = (R * NF + kMmaThreads - 1) / kMmaThreads;
    float v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = threadIdx.x + u * kMmaThreads, lr = i / NF, f = i - lr * NF;
      const int row = min(row0 + lr, N - 1), ch = min(max(row - d_inner, 0), d_xbc - 1);
      float x = 0.f;
      if (i < R * NF) {
        if (f < DFSSM_RANK) x = h2f(p.A16[(size_t)row * DFSSM_RANK + f]);
        else if (f == DFSSM_RANK) x = h2f(p.scale[row]);
        else if (MODE == 0 && f == DFSSM_RANK + 5) x = h2f(conv_b[ch]);
        else if (MODE == 0) x = h2f(conv_w[ch * DFSSM_DCONV + (f - DFSSM_RANK - 1)]);
      }
      v[u] = x;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = threadIdx.x + u * kMmaThreads, lr = i / NF, f = i - lr * NF;
      if (i >= R * NF) continue;
      if (f < DFSSM_RANK) e_a[lr * (DFSSM_RANK + 1) + f] = v[u];
      else if (f == DFSSM_RANK) e_scale[lr] = v[u];
      else if (f == DFSSM_RANK + 5) e_cb[lr] = v[u];
      else e_cw[lr * 4 + (f - DFSSM_RANK - 1)] = v[u];
    }
  }
  __syncthreads();
  unsigned phase = 0;
  for (int bt0 = 0; bt0 < B; bt0 += NB, phase ^= 1u) {
    const int nb = min(NB, B - bt0);
    __syncthreads();  // previous pass done with sq and the epilogue operands
    // activation rows -> shared memory by TMA bulk copies (rows >= nb keep stale bytes; their
    // output columns are never stored); the first pass's went out at kernel entry
    if (bt0 > 0) issue_q(bt0, nb);
    // per-batch epilogue operands
    {
      constexpr int NF = DFSSM_RANK + 2, U = (NB * NF + kMmaThreads - 1) / kMmaThreads;
      float v[U];
      int vq[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = threadIdx.x + u * kMmaThreads, b = i / NF, f = i - b * NF;
        v[u] = 0.f;
        vq[u] = 0;
        if (b < nb) {
          if (f < DFSSM_RANK) {
            if (MODE != 2) v[u] = h2f(t[(bt0 + b) * DFSSM_RANK + f]);
          } else if (f == DFSSM_RANK) {
            if (MODE != 2) v[u] = h2f(xs[bt0 + b]);
          } else {
            vq[u] = qsum[bt0 + b];
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = threadIdx.x + u * kMmaThreads, b = i / NF, f = i - b * NF;
        if (b >= NB) continue;
        if (f < DFSSM_RANK) e_t[b * DFSSM_RANK + f] = v[u];
        else if (f == DFSSM_RANK) e_xs[b] = v[u];
        else e_qsum[b] = vq[u];
      }
    }
    // staging loops issue all their global loads before the shared-memory stores (a load->store
    // loop with a runtime trip count would otherwise pay one memory round trip per iteration)
    if (MODE == 1) {  // residual values (the conv-state region is free in this mode)
      constexpr int U = (NB * R + kMmaThreads - 1) / kMmaThreads;
      float v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = threadIdx.x + u * kMmaThreads, b = i / R, lr = i - b * R;
        v[u] = (b < nb && row0 + lr < N) ? h2f(out[(size_t)(bt0 + b) * ld_out + row0 + lr]) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (threadIdx.x + u * kMmaThreads < NB * R) e_cs[threadIdx.x + u * kMmaThreads] = v[u];
    }
    if (MODE == 0) {
      constexpr int U = (NB * 3 * R + kMmaThreads - 1) / kMmaThreads;
      float v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = threadIdx.x + u * kMmaThreads;
        const int b = i / (3 * R), rem = i - b * 3 * R, tap = rem / R, lr = rem - tap * R;
        const int ch = row0 + lr - d_inner;
        v[u] = (b < nb && ch >= 0 && ch < d_xbc && row0 + lr < N)
                   ? conv_state[(size_t)(bt0 + b) * 3 * d_xbc + (size_t)tap * d_xbc + ch]
                   : 0.f;
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (threadIdx.x + u * kMmaThreads < NB * 3 * R) e_cs[threadIdx.x + u * kMmaThreads] = v[u];
    }
    if (bt0 > 0) load_w();
    if (!mbar_wait_bounded(&qbar, phase)) atomicOr(&g_umma_err, 2u);
    int acc[NT][4];
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[tt][i] = 0;
#pragma unroll
    for (int u = 0; u < kMmaMaxBlk; ++u) {
      if (4 * u >= wpw) break;
      const int kw = kw0 + 4 * u;
      const uint4 va = wva[u], vb = wvb[u];
      const unsigned wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const unsigned a0 = (wa[j] >> c) & 0x01010101u, a2 = (wa[j] >> (c + 4)) & 0x01010101u;
        const unsigned a1 = (wb[j] >> c) & 0x01010101u, a3 = (wb[j] >> (c + 4)) & 0x01010101u;
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
          const int8_t* qb = sq + (tt * 8 + g) * SQ + (kw + j) * 32;
          const unsigned b0 = *reinterpret_cast<const unsigned*>(qb + c * 4);
          const unsigned b1 = *reinterpret_cast<const unsigned*>(qb + (c + 4) * 4);
          mma_s8(acc[tt], a0, a1, a2, a3, b0, b1);
        }
      }
    }
    // D fragment: acc[tt][0..1] -> row g, batch cols 2c, 2c+1 of tile tt; [2..3] -> row g+8
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) {
      int* r = red + (ks * NB + tt * 8 + 2 * c) * R + rg * 16 + g;
      r[0] = acc[tt][0];
      r[R] = acc[tt][1];
      r[8] = acc[tt][2];
      r[R + 8] = acc[tt][3];
    }
    __syncthreads();
    // consecutive threads take consecutive rows of one batch row: coalesced stores of out and of
    // the conv state, conflict-free reads of the split-K partials
    for (int o = threadIdx.x; o < R * NB; o += kMmaThreads) {
      const int bb = o / R, lr = o - bb * R;
      const int row = row0 + lr, b = bt0 + bb;
      if (row >= N || bb >= nb) continue;
      int sacc = 0;
#pragma unroll
      for (int k2 = 0; k2 < KS; ++k2) sacc += red[(k2 * NB + bb) * R + lr];
      const int dot = 2 * sacc - e_qsum[bb];
      if (MODE == 2) {
        reinterpret_cast<int*>(out)[(size_t)b * ld_out + row] = dot;
        continue;
      }
      const float base = round_h(round_h(round_h((float)dot) * e_xs[bb]) * e_scale[lr]);
      float la = 0.f;
#pragma unroll
      for (int r = 0; r < DFSSM_RANK; ++r) la = fmaf(e_t[bb * DFSSM_RANK + r], e_a[lr * (DFSSM_RANK + 1) + r], la);
      const float v = round_h(base + round_h(la));
      if (MODE == 0) {
        float res = v;
        const int ch = row - d_inner;
        if (ch >= 0 && ch < d_xbc) {
          const float* es = e_cs + bb * 3 * R + lr;
          const float s0 = es[0], s1 = es[R], s2 = es[2 * R];
          float* cs = conv_state + (size_t)b * 3 * d_xbc;
          cs[ch] = s1;
          cs[d_xbc + ch] = s2;
          cs[2 * d_xbc + ch] = v;
          const float* cw = e_cw + lr * 4;
          const float o2 = s0 * cw[0] + s1 * cw[1] + s2 * cw[2] + v * cw[3] + e_cb[lr];
          const float sig = 1.0f / (1.0f + expf(-o2));
          res = o2 * sig;
        }
        out[(size_t)b * ld_out + row] = f2h(res);
      } else if (MODE == 3) {  // plain projection (the prefill scan applies the conv over time)
        out[(size_t)b * ld_out + row] = f2h(v);
      } else {
        out[(size_t)b * ld_out + row] = f2h(e_cs[bb * R + lr] + v);
      }
    }
  }
}

inline size_t proj_mma_smem(int K, int RG, int NT = kMmaNT) {
  const int NB = 8 * NT, KS = (kMmaThreads / 32) / RG, R = 16 * RG;
  return (size_t)NB * (K + 16) + (size_t)KS * R * NB * 4 +
         4 * ((size_t)NB * 3 * R + NB * DFSSM_RANK + R * (DFSSM_RANK + 1) + R * 4 + 2 * R + 2 * NB);
}

// ---------------------------------------------------------------------------------------
// ssm_gate: one CTA per (head, batch row); 64 x 128 fp32 state updated in place.
//   dt = softplus(dt_raw + dt_bias); Abar = exp(dt * -exp(A_log))   df_ssm_kernels.cu:77-79
//   h  = Abar * h + (x * dt) * B_n;  y = sum_n C_n h + D x           df_ssm_kernels.cu:80-101
//   gated = fp16(fp16(y) * fp16(z * fp16(sigmoid(z))))               df_ssm_inference.py:194-195
// Warp w owns rows p = 8w..8w+7, lane owns n = 4*lane..4*lane+3 (512 B coalesced per row).
// With zin == nullptr the ungated y is written instead (the reference ssm_step output).
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kSsmThreads)
ssm_gate_kernel(const __half* __restrict__ xbc, int ld_xbc, const __half* __restrict__ dtr, int ld_dt,
                const __half* __restrict__ zin, int ld_z, int d_inner, int d_state, int nheads,
                const float* __restrict__ dt_bias, const float* __restrict__ A_log,
                const float* __restrict__ Dp, float* __restrict__ hstate, __half* __restrict__ out, int ld_out) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = lane * 4;
  // the 32 KB state tile is requested first: its addresses depend on nothing else, so the HBM
  // stream starts before the small per-head inputs and the dt / exp arithmetic
  float* hs = hstate + ((size_t)b * nheads + h) * (DFSSM_HEADDIM * DFSSM_DSTATE);
  float4 hv[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) hv[r] = __ldcs(reinterpret_cast<const float4*>(hs + (wid * 8 + r) * DFSSM_DSTATE + n0));
  const __half* xc = xbc + (size_t)b * ld_xbc;     // conv'd x   [d_inner]
  const __half* Bc = xc + d_inner;                 // conv'd B   [d_state]
  const __half* Cc = xc + d_inner + d_state;       // conv'd C   [d_state]
  const uint2 bq = *reinterpret_cast<const uint2*>(Bc + n0);
  const uint2 cq = *reinterpret_cast<const uint2*>(Cc + n0);
  float dtv = h2f(dtr[(size_t)b * ld_dt + h]) + dt_bias[h];
  dtv = log1pf(expf(dtv));
  const float Abar = expf(dtv * (-expf(A_log[h])));
  const float Dh = Dp[h];
  float Bn[4], Cn[4];
  {
    const __half* bh = reinterpret_cast<const __half*>(&bq);
    const __half* ch = reinterpret_cast<const __half*>(&cq);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      Bn[i] = h2f(bh[i]);
      Cn[i] = h2f(ch[i]);
    }
  }
  float part[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int pp = wid * 8 + r;
    const float X = h2f(xc[h * DFSSM_HEADDIM + pp]) * dtv;
    float4 o;
    o.x = Abar * hv[r].x + X * Bn[0];
    o.y = Abar * hv[r].y + X * Bn[1];
    o.z = Abar * hv[r].z + X * Bn[2];
    o.w = Abar * hv[r].w + X * Bn[3];
    __stcs(reinterpret_cast<float4*>(hs + pp * DFSSM_DSTATE + n0), o);
    part[r] = Cn[0] * o.x + Cn[1] * o.y + Cn[2] * o.z + Cn[3] * o.w;
  }
  // C.h of the warp's 8 rows summed over the 32 lanes as a transposing butterfly: each exchange halves
  // the values a lane holds (7 shuffles), two more finish the sums, and lane 4k + 0 ends with the sum
  // of row rw (9 shuffles for 8 rows instead of 40); the 8 rows' epilogues then run in parallel
  int rw = 0;
#pragma unroll
  for (int n = 8, off = 16; n > 1; n >>= 1, off >>= 1) {
    const bool hi = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = hi ? part[i] : part[i + n / 2];
      const float keep = hi ? part[i + n / 2] : part[i];
      part[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
    rw += hi ? n / 2 : 0;
  }
  part[0] += __shfl_xor_sync(0xffffffffu, part[0], 2);
  part[0] += __shfl_xor_sync(0xffffffffu, part[0], 1);
  if ((lane & 3) == 0) {
    const int pp = wid * 8 + rw;
    const float y = part[0] + h2f(xc[h * DFSSM_HEADDIM + pp]) * Dh;
    __half o16 = f2h(y);
    if (zin != nullptr) {
      const float z = h2f(zin[(size_t)b * ld_z + h * DFSSM_HEADDIM + pp]);
      const float sig = round_h(1.0f / (1.0f + expf(-z)));
      const float silu = round_h(z * sig);
      o16 = f2h(h2f(o16) * silu);
    }
    out[(size_t)b * ld_out + h * DFSSM_HEADDIM + pp] = o16;
  }
}

// ---------------------------------------------------------------------------------------
// embed: x[b] = fp16(E_q[tok] * E_s[tok])  (the fp16 row the reference gathers,
// df_ssm_inference.py:220, for an int8 embedding with per-row scale).
// ---------------------------------------------------------------------------------------
__global__ void embed_kernel(const int* __restrict__ tokens, const int8_t* __restrict__ Eq,
                             const float* __restrict__ Es, int d_model, int vocab, __half* __restrict__ x) {
  const int b = blockIdx.x;
  int tok = tokens[b];
  tok = min(max(tok, 0), vocab - 1);
  const float s = Es[tok];
  const int8_t* er = Eq + (size_t)tok * d_model;
  for (int k = threadIdx.x; k < d_model; k += blockDim.x) x[(size_t)b * d_model + k] = f2h((float)er[k] * s);
}

// ---------------------------------------------------------------------------------------
// lm_head: logits[b][v] = E_s[v] * sum_k E_q[v][k] * xn[b][k] (fp32), plus an argmax over
// the fp16-rounded logits with first-index tie-breaking, as the reference's fp16 GEMM +
// argmax (df_ssm_inference.py:224,236).  One warp per vocabulary row; per-CTA best keys are
// merged with atomicMax into best[b] (reset by finalize_kernel).
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kHeadThreads)
lm_head_kernel(const int8_t* __restrict__ Eq, const float* __restrict__ Es, int vocab, int d,
               const __half* __restrict__ xn, int B, float* __restrict__ logits,
               unsigned long long* __restrict__ best) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* sx = reinterpret_cast<float*>(smem);  // [kHeadBT][d]
  __shared__ unsigned long long sbest[kHeadThreads / 32][kHeadBT];
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = d >> 4;  // 16-byte chunks per row
  for (int bt0 = 0; bt0 < B; bt0 += kHeadBT) {
    const int nb = min(kHeadBT, B - bt0);
    __syncthreads();
    for (int i = threadIdx.x; i < nb * d; i += kHeadThreads) sx[i] = h2f(xn[(size_t)bt0 * d + i]);
    __syncthreads();
    unsigned long long mybest[kHeadBT];
#pragma unroll
    for (int b = 0; b < kHeadBT; ++b) mybest[b] = 0ull;
    for (int v = blockIdx.x * (kHeadThreads / 32) + wid; v < vocab; v += gridDim.x * (kHeadThreads / 32)) {
      float acc[kHeadBT];
#pragma unroll
      for (int b = 0; b < kHeadBT; ++b) acc[b] = 0.f;
      const uint4* er = reinterpret_cast<const uint4*>(Eq + (size_t)v * d);
      // four 16-byte units per lane in flight (d = 2048 is one group); the sum runs over the
      // units in the same order as one at a time
      for (int cg = 0; cg < C; cg += 32 * 4) {
        uint4 evs[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int c = cg + lane + 32 * g;
          if (c < C) evs[g] = ldg_stream(er + c);
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int c = cg + lane + 32 * g;
          if (c >= C) break;
          const uint4 ev = evs[g];
          float e[16];
          const unsigned w4[4] = {ev.x ^ 0x80808080u, ev.y ^ 0x80808080u, ev.z ^ 0x80808080u, ev.w ^ 0x80808080u};
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) e[j * 4 + i] = i8_to_f(w4[j], i);
#pragma unroll
          for (int b = 0; b < kHeadBT; ++b) {
            if (b < nb) {
              const float4* xv = reinterpret_cast<const float4*>(sx + b * d + c * 16);
              float a = acc[b];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const float4 xx = xv[u];
                a = fmaf(e[4 * u + 0], xx.x, a);
                a = fmaf(e[4 * u + 1], xx.y, a);
                a = fmaf(e[4 * u + 2], xx.z, a);
                a = fmaf(e[4 * u + 3], xx.w, a);
              }
              acc[b] = a;
            }
          }
        }
      }
      const float sv = Es[v];
#pragma unroll
      for (int b = 0; b < kHeadBT; ++b) {
        if (b < nb) {
          const float s = warp_sum(acc[b]);
          const float lg = s * sv;
          if (lane == 0) {
            logits[(size_t)(bt0 + b) * vocab + v] = lg;
            const unsigned long long key = argmax_key(f2h(lg), (uint32_t)v);
            mybest[b] = key > mybest[b] ? key : mybest[b];
          }
        }
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int b = 0; b < kHeadBT; ++b) sbest[wid][b] = mybest[b];
    }
    __syncthreads();
    if (threadIdx.x < nb) {
      unsigned long long k = 0ull;
      for (int w = 0; w < kHeadThreads / 32; ++w) k = sbest[w][threadIdx.x] > k ? sbest[w][threadIdx.x] : k;
      atomicMax(best + bt0 + threadIdx.x, k);
    }
  }
}

// ---------------------------------------------------------------------------------------
// lm_head_mma: the LM head on fp16 tensor cores for batches of 8 or more (mma.sync m16n8k16,
// fp16 x fp16 -> fp32).  int8 embedding bytes become exact fp16 values with a byte permute that
// places them in the mantissa of 1024 (0x64xx) and one half2 subtraction of 1152; the fp16
// normalised activations are exact too, so every product is exact and only the fp32 summation
// order differs from the per-row kernel.  A warp owns 16 vocabulary rows at a time; per 64-column
// block lane (g, c) loads 16 bytes at 16c of rows g and g+8, which fixes the (consistent) k order
// of the A and B fragments.  logits = acc * E_s[v]; the argmax keys are merged per CTA and then
// with atomicMax into best[b].
// ---------------------------------------------------------------------------------------
constexpr int kHeadMmaWarps = 16;  // one CTA per SM (the activation tile fills shared memory)
constexpr int kHeadMmaThreads = 32 * kHeadMmaWarps;
constexpr int kHeadMmaU = 4;       // 64-column blocks whose embedding loads are issued together
constexpr int kHeadMmaNT = 4;  // most batch tiles of 8 per pass (32 rows)

// NT batch tiles of 8 per pass: the launcher takes the fewest that hold the batch (1, 2 or 4).
template <int NT = kHeadMmaNT>
__global__ void __launch_bounds__(kHeadMmaThreads, 1)
lm_head_mma_kernel(const int8_t* __restrict__ Eq, const float* __restrict__ Es, int vocab, int d,
                   const __half* __restrict__ xn, int B, float* __restrict__ logits,
                   unsigned long long* __restrict__ best) {
  constexpr int NB = 8 * NT;
  extern __shared__ __align__(16) unsigned char smem[];
  const int SX = d + 8;  // padded fp16 row stride
  __half* sx = reinterpret_cast<__half*>(smem);                                        // [NB][SX]
  unsigned long long* sbest = reinterpret_cast<unsigned long long*>(smem + (size_t)NB * SX * 2);  // [warps][NB]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const int ntiles = (vocab + 15) / 16;
  __shared__ uint64_t xbar;
  if (threadIdx.x == 0) {
    mbar_init(&xbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  unsigned phase = 0;
  for (int bt0 = 0; bt0 < B; bt0 += NB, phase ^= 1u) {
    const int nb = min(NB, B - bt0);
    __syncthreads();
    if (wid == 0) {
      if (lane == 0) mbar_expect_tx(&xbar, (unsigned)(nb * d * 2));
      __syncwarp();
      for (int b = lane; b < nb; b += 32)
        bulk_g2s(sx + b * SX, xn + (size_t)(bt0 + b) * d, (unsigned)(d * 2), &xbar);
    }
    if (!mbar_wait_bounded(&xbar, phase)) atomicOr(&g_umma_err, 4u);
    unsigned long long wbest[NT][2];
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) wbest[tt][0] = wbest[tt][1] = 0ull;
    for (int tile = blockIdx.x * kHeadMmaWarps + wid; tile < ntiles; tile += gridDim.x * kHeadMmaWarps) {
      const int v0 = tile * 16;
      const int va = min(v0 + g, vocab - 1), vb = min(v0 + g + 8, vocab - 1);
      const uint4* ra = reinterpret_cast<const uint4*>(Eq + (size_t)va * d);
      const uint4* rb = reinterpret_cast<const uint4*>(Eq + (size_t)vb * d);
      float acc[NT][4];
#pragma unroll
      for (int tt = 0; tt < NT; ++tt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[tt][i] = 0.f;
      // kHeadMmaU blocks' embedding loads go out together before their MMAs, so each lane keeps
      // 2 x kHeadMmaU 16-byte loads in flight (d / 64 is a multiple of kHeadMmaU: d % 256 == 0)
      for (int blk0 = 0; blk0 < d / 64; blk0 += kHeadMmaU) {
        uint4 ea[kHeadMmaU], eb[kHeadMmaU];
#pragma unroll
        for (int u = 0; u < kHeadMmaU; ++u) {
          ea[u] = ldg_stream(ra + (blk0 + u) * 4 + c);
          eb[u] = ldg_stream(rb + (blk0 + u) * 4 + c);
        }
#pragma unroll
        for (int u = 0; u < kHeadMmaU; ++u) {
          const unsigned wa[4] = {ea[u].x ^ 0x80808080u, ea[u].y ^ 0x80808080u, ea[u].z ^ 0x80808080u,
                                  ea[u].w ^ 0x80808080u};
          const unsigned wb[4] = {eb[u].x ^ 0x80808080u, eb[u].y ^ 0x80808080u, eb[u].z ^ 0x80808080u,
                                  eb[u].w ^ 0x80808080u};
#pragma unroll
          for (int s2 = 0; s2 < 4; ++s2) {
            const unsigned a0 = i8x2_to_h2(wa[s2], 0x4140u), a2 = i8x2_to_h2(wa[s2], 0x4342u);
            const unsigned a1 = i8x2_to_h2(wb[s2], 0x4140u), a3 = i8x2_to_h2(wb[s2], 0x4342u);
            const int col = (blk0 + u) * 64 + 16 * c + 4 * s2;
#pragma unroll
            for (int tt = 0; tt < NT; ++tt) {
              const uint2 bv = *reinterpret_cast<const uint2*>(sx + (tt * 8 + g) * SX + col);
              mma_f16(acc[tt], a0, a1, a2, a3, bv.x, bv.y);
            }
          }
        }
      }
      // D fragment: acc[tt][0..1] -> row v0+g, batch 2c, 2c+1 of tile tt; [2..3] -> row v0+g+8
#pragma unroll
      for (int tt = 0; tt < NT; ++tt) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int v = v0 + g + (i >= 2 ? 8 : 0);
          const int bb = tt * 8 + 2 * c + (i & 1);
          if (v < vocab && bb < nb) {
            const float lg = acc[tt][i] * Es[v];
            logits[(size_t)(bt0 + bb) * vocab + v] = lg;
            const unsigned long long key = argmax_key(f2h(lg), (uint32_t)v);
            wbest[tt][i & 1] = key > wbest[tt][i & 1] ? key : wbest[tt][i & 1];
          }
        }
      }
    }
    // reduce the per-lane bests over the 8 lanes that share c (same batch columns)
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        unsigned long long k = wbest[tt][j];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, k, o);
          k = k2 > k ? k2 : k;
        }
        if (g == 0) sbest[wid * NB + tt * 8 + 2 * c + j] = k;
      }
    __syncthreads();
    if (threadIdx.x < nb) {
      unsigned long long k = 0ull;
      for (int w = 0; w < kHeadMmaWarps; ++w) k = sbest[w * NB + threadIdx.x] > k ? sbest[w * NB + threadIdx.x] : k;
      atomicMax(best + bt0 + threadIdx.x, k);
    }
  }
}

inline size_t lm_head_mma_smem(int d, int NT = kHeadMmaNT) {
  return (size_t)8 * NT * (d + 8) * 2 + (size_t)kHeadMmaWarps * 8 * NT * 8;
}

__global__ void finalize_kernel(unsigned long long* __restrict__ best, int B, int* __restrict__ tokens) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) {
    tokens[b] = (int)argmax_key_index(best[b]);
    best[b] = 0ull;
  }
}

// ---------------------------------------------------------------------------------------
// permute_q: row-major int8 activations -> permuted layout + row sums (stand-alone GEMM).
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kPrepThreads)
permute_q_kernel(const int8_t* __restrict__ q, int K, int8_t* __restrict__ qp, int* __restrict__ qsum) {
  __shared__ int ired[kPrepThreads / 32];
  const int b = blockIdx.x;
  int s = 0;
  for (int k = threadIdx.x; k < K; k += kPrepThreads) {
    const int8_t v = q[(size_t)b * K + k];
    qp[(size_t)b * K + qperm_index(k)] = v;
    s += v;
  }
  s = block_isum<kPrepThreads / 32>(s, ired);
  if (threadIdx.x == 0) qsum[b] = s;
}

// ---------------------------------------------------------------------------------------
// conv_step: stand-alone conv1d shift register + SiLU (df_ssm_kernels.cu:27-47), fp32
// tap-major state [B][3][d_xbc], xbc fp16 in place.
// ---------------------------------------------------------------------------------------
__global__ void conv_step_kernel(float* __restrict__ conv_state, __half* __restrict__ xbc, int ld_xbc,
                                 const __half* __restrict__ conv_w, const __half* __restrict__ conv_b, int d_xbc) {
  const int b = blockIdx.y;
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= d_xbc) return;
  float* cs = conv_state + (size_t)b * 3 * d_xbc;
  __half* xr = xbc + (size_t)b * ld_xbc;
  const float s0 = cs[ch], s1 = cs[d_xbc + ch], s2 = cs[2 * d_xbc + ch];
  const float v = h2f(xr[ch]);
  cs[ch] = s1;
  cs[d_xbc + ch] = s2;
  cs[2 * d_xbc + ch] = v;
  const __half* cw = conv_w + ch * DFSSM_DCONV;
  const float o = s0 * h2f(cw[0]) + s1 * h2f(cw[1]) + s2 * h2f(cw[2]) + v * h2f(cw[3]) + h2f(conv_b[ch]);
  const float sig = 1.0f / (1.0f + expf(-o));
  xr[ch] = f2h(o * sig);
}

}  // namespace dfssm
