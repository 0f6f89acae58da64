// Persistent whole-step decode kernel for small batches (instances for 1 to 4 sequences per launch;
// larger batches in persistent mode run one launch per group of up to four): one cooperative launch
// per greedy decode step runs the embedding gather, every layer, the final norm, the LM head and
// the argmax.  One CTA per SM: 16 compute warps (512 threads, named barrier 1) and one warp
// that only issues the bulk copies of the weight/state ring.
//
// Per layer:
//   alpha: every CTA rebuilds RMSNorm(x) -> int8 q; 16 "producer" CTAs compute the in_proj
//          LoRA down-projection t (one rank each) and publish it.
//          "head" CTAs own half a head (32 channels p of head h): their z/x in_proj rows,
//          conv1d of their x channels, and their 32x128 slice of the fp32 SSM state.
//          "BC" CTAs own 8-row groups of the B, C and dt in_proj rows (and the conv1d channels
//          of B/C) and publish conv'd B/C and raw dt; head CTAs then run the state update,
//          C.h + D.x and the SiLU(z) gate and publish the gated vector.
//   beta:  every non-producer CTA owns 8-row groups of out_proj: gate-RMSNorm of the full
//          gated vector, quantisation, LoRA, the 1-bit GEMV and the residual add into x.
// There is no grid barrier.  Every exchanged value (x, LoRA t, conv'd B/C, gated) travels in
// a 64-bit word {32 data bits, 32-bit tag} written with one relaxed store; a consumer polls
// its words until every tag equals the tag of the expected (step, layer, kind), so the value
// and its readiness arrive in a single L2 round trip with no fence.  Tags come from an epoch
// base in device memory that the last CTA of each launch advances, so words left from
// earlier steps never match.  Exchange buffers alternate by layer parity; a writer of layer
// l+2 depends (through the exchange chain) on every reader of layer l having finished it.
// Weights and state of upcoming layers stream into a shared-memory ring with cp.async.bulk
// (TMA bulk copies completing on "full" mbarriers) while earlier layers compute, so the HBM
// stream is off the critical path.  The copy warp refills a slot once the compute threads
// release it on its "empty" mbarrier; issuing some 20 copies per stage takes the TMA unit about
// a microsecond, which no compute warp waits for.  Every wait is bounded: a timeout sets an error
// word (reported by dfssm_check_finite) and makes every later wait return at once, so a
// failed step ends quickly instead of hanging.
//
// Arithmetic follows the per-op kernels (kernels.cuh) and the reference rounding points;
// only fp32 summation orders differ.
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>
#include <vector>

#include "engine.h"
#include "prep.cuh"



using namespace dfssm;

namespace {

constexpr int kThreads = 512;              // compute threads (named barrier 1)
constexpr int kWarps = kThreads / 32;
constexpr int kBlockThreads = kThreads + 32;  // + one warp that issues the weight/state copies
constexpr unsigned kSpinLimit = 1u << 22;
// Polls after which a bounded wait gives up (kSpinLimit unless dfssm_debug_set_wait_limit lowered
// it for a test of the timeout path); read only every 256 polls.
__constant__ unsigned c_spin_limit = kSpinLimit;
__device__ __forceinline__ unsigned spin_limit() { return c_spin_limit; }
#ifndef DFSSM_GFIRST
#define DFSSM_GFIRST 2  // gated vector: take_words FIRST mode (a warp leader polls first: batch 1 1897 -> 1970 tok/s against 1)
#endif
#ifndef DFSSM_XFIRST
#define DFSSM_XFIRST 0  // x: take_words FIRST mode
#endif
constexpr int kMaxRPW = 2;  // SSM rows per warp (np = 32 channels over 16 warps)
constexpr int kDotRows = 64;  // in_proj / out_proj rows a CTA may own (GEMV results in shared memory)
// Reduction scratch: three rotating single-barrier buffers of 16 x B floats at red, red + 64 and
// red + 128 (B <= 4), the (16 + 1) x B floats of the final norm's reduction and the 16 x B argmax
// keys of the LM head.
constexpr int kRedFloats = 192;

struct CtaPlan {
  int role;       // 0 = head item, 1 = B/C rows, 2 = no in_proj rows
  int h, p0, np;  // head item
  int bc0, nbc;   // B/C rows [bc0, bc0 + nbc) within [0, 2*d_state)
  int o0, no;     // out_proj rows
  int v0, nv;     // LM head rows
  int tj;         // index among the B/C CTAs (LoRA-t producers are those with tj < n_t), else -1
  int tx;         // bytes of one ring stage (sum of this CTA's copies)
};

struct Layout {  // byte offsets inside one ring stage (identical for every CTA)
  int in_bits, in_scale, in_lA, in_lAs, conv_w, conv_b, out_bits, out_scale, out_lA, out_lAs, state, cstate;
  int stage_bytes;
};

struct PParams {
  LayerW lw0;          // layer 0's weights; layer l's arrays lie lstride bytes further per layer
  long long lstride;
  const CtaPlan* plans;
  Layout lay;
  int n_layer, d_model, d_inner, d_state, d_xbc, n_in, nheads, vocab;
  const int8_t* Eq;
  const float* Es;
  const float* norm_f;
  float* ssm;
  float* conv;
  long long ssm_layer, conv_layer;  // elements per layer
  __half* x_g;      // [B][d_model]
  __half* bc_g;     // [B][2*d_state]
  __half* gated_g;  // [B][d_inner]
  float* logits;    // [B][vocab]
  unsigned long long* best;
  int* tokens;
  unsigned* sync;  // [1] exit count, [3] error, [16] tag epoch base (never cleared by resets)
  // tagged exchange words {data, tag}, each [2 parities][B][...]:
  unsigned long long* xw;   // x as fp16 pairs        [d_model / 2]
  unsigned long long* bcw;  // conv'd B/C then raw dt, fp16 pairs [bcw_per_seq = d_state + nheads / 2]
  int bcw_per_seq;
  unsigned long long* gw;   // gated fp16 pairs       [d_inner / 2]
  unsigned long long* tw;   // LoRA t fp32, [2 parities][2: in, out][B][16]
  size_t rs;                // words between the replicas of the exchange region
  int l0, l1;      // layers run by this launch
  int from_x;      // 1: layer l0 starts from x_g instead of the token embedding
  int do_head;     // 1: final norm + LM head + argmax after layer l1-1
  int skew;        // test of the timeout path: CTA 0 runs with the next step's tags (never match)
  int n_bc;        // number of B/C CTAs
  int n_t;         // number of LoRA-t producer CTAs (the first n_t B/C CTAs; rank r -> producer r % n_t)
  int ns;          // ring stages
  int ring_off;    // byte offset of the ring in dynamic smem
  int tab_off;     // byte offset of the per-layer tables in dynamic smem
  unsigned long long* trace;  // optional: per-CTA globaltimer stamps (kTraceStride entries per CTA)
};

constexpr int kTracePerLayer = 16;
__device__ __forceinline__ void stamp(const PParams& P, int idx) {
  if (P.trace && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    P.trace[(size_t)blockIdx.x * (4 + kTracePerLayer * P.n_layer) + idx] = t;
  }
}

// Weight pointers of layer l: every layer's arrays sit at the same offsets within equal-sized
// slices of the weight arena (checked on the host when the plan is built).
__device__ __forceinline__ LayerW layer_w(const PParams& P, int l) {
  const long long o = (long long)l * P.lstride;
  LayerW L = P.lw0;
  auto mv = [o](auto*& p) { p = reinterpret_cast<std::remove_reference_t<decltype(p)>>(reinterpret_cast<const char*>(p) + o); };
  mv(L.in.bits), mv(L.in.scale), mv(L.in.A16), mv(L.in.B16);
  mv(L.out.bits), mv(L.out.scale), mv(L.out.A16), mv(L.out.B16);
  mv(L.conv_w), mv(L.conv_b), mv(L.A_log), mv(L.Dp), mv(L.dt_bias), mv(L.norm_w), mv(L.ln_w);
  return L;
}

// N consecutive fp32 values at p (16-byte aligned when N % 4 == 0) with the fewest load
// instructions: 512 threads issuing scalar loads at once queue them for ~0.5 us in the LSU.
template <int N>
__device__ __forceinline__ void ld_f32s(const float* p, float (&v)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int j = 0; j < N / 4; ++j) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(p) + j);
      v[4 * j] = t.x, v[4 * j + 1] = t.y, v[4 * j + 2] = t.z, v[4 * j + 3] = t.w;
    }
  } else if constexpr (N % 2 == 0) {
#pragma unroll
    for (int j = 0; j < N / 2; ++j) {
      const float2 t = __ldg(reinterpret_cast<const float2*>(p) + j);
      v[2 * j] = t.x, v[2 * j + 1] = t.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = __ldg(p + j);
  }
}

// ---- tagged exchange words
enum : unsigned { kTagX = 1, kTagTin = 2, kTagBC = 3, kTagGated = 4, kTagTout = 5, kTagsPerLayer = 8 };
__device__ __forceinline__ unsigned tag_of(unsigned base, int layer, unsigned kind) {
  return base + (unsigned)layer * kTagsPerLayer + kind;
}
__device__ __forceinline__ unsigned pack_h2(float a, float b) {
  return (unsigned)__half_as_ushort(f2h(a)) | ((unsigned)__half_as_ushort(f2h(b)) << 16);
}
__device__ __forceinline__ float lo_h(unsigned v) { return h2f(__ushort_as_half((unsigned short)(v & 0xffffu))); }
__device__ __forceinline__ float hi_h(unsigned v) { return h2f(__ushort_as_half((unsigned short)(v >> 16))); }
// Every exchange word is written to kReplicas copies kRepStride words apart and CTA c reads
// copy c % kReplicas: all CTAs polling one copy would concentrate their L2 requests on the
// few slices that hold it.
#ifndef DFSSM_XREPL
#define DFSSM_XREPL 8
#endif
constexpr int kReplicas = DFSSM_XREPL;
__device__ __forceinline__ void put_word(unsigned long long* p, size_t rstride, unsigned data, unsigned tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | data;
#pragma unroll
  for (int r = 0; r < kReplicas; ++r)
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p + r * rstride), "l"(w) : "memory");
}
// Poll G groups of N consecutive words (FIRST: first wait for word 0 of group 0 alone) (group g at p + g * gstride; N = 1, 2 or 4, each group
// 8*N-byte aligned for N > 1) until every tag equals `tag`; the data go to out[][].  All loads
// of one poll are issued together.  Bounded: after kSpinLimit polls the error word gets
// `code`, and once the error word is set every poll gives up at its next check.
// FIRST = 1: every thread first waits on its first word alone, then takes all; FIRST = 2: lane 0 of
// each warp waits on its first word while the other lanes wait at the warp's barrier (the whole warp
// must call), then the warp takes all (1/32 of the poll traffic while the words are not ready).
template <int G, int N, int FIRST = 0>
__device__ __forceinline__ void take_words(const unsigned long long* p, size_t gstride, unsigned tag,
                                           unsigned (&out)[G][N], unsigned* err, unsigned code) {
  unsigned long long w[G][N];
  if (FIRST == 1 || (FIRST == 2 && (threadIdx.x & 31) == 0)) {
    for (unsigned it = 0;; ++it) {
      unsigned long long w0;
      asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w0) : "l"(p) : "memory");
      if ((unsigned)(w0 >> 32) == tag) break;
      if ((it & 255u) == 255u && (ld_acquire(err) != 0 || it > spin_limit())) break;
    }
  }
  if (FIRST == 2) __syncwarp();
  for (unsigned it = 0;; ++it) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const unsigned long long* q = p + g * gstride;
      if (N == 1) {
        asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w[g][0]) : "l"(q) : "memory");
      } else {
#pragma unroll
        for (int k = 0; k < N; k += 2)
          asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];"
                       : "=l"(w[g][k]), "=l"(w[g][k + 1])
                       : "l"(q + k)
                       : "memory");
      }
    }
    bool ok = true;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int k = 0; k < N; ++k) ok &= (unsigned)(w[g][k] >> 32) == tag;
    if (ok) break;
    if ((it & 255u) == 255u) {
      if (ld_acquire(err) != 0) break;
      if (it > spin_limit()) {
        atomicOr(err, code);
        break;
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int k = 0; k < N; ++k) out[g][k] = (unsigned)w[g][k];
}

// Collect B x d_model/2 x words (KI = d_model / 512) into s_x.
template <int B, int KI>
__device__ __forceinline__ void take_x(const unsigned long long* xw, int n_words, unsigned tag, __half* s_x,
                                       unsigned* err) {
  constexpr int XPT = (B * KI) / 2 >= 4 ? 4 : ((B * KI) / 2 >= 2 ? 2 : 1);  // words per thread
  for (int i = threadIdx.x * XPT; i < n_words; i += kThreads * XPT) {
    unsigned v[1][XPT];
    take_words<1, XPT, DFSSM_XFIRST>(xw + i, 0, tag, v, err, 1u);
#pragma unroll
    for (int k = 0; k < XPT; ++k) reinterpret_cast<unsigned*>(s_x)[i + k] = v[0][k];
  }
  cta_sync();
}

// Wait for the ring slot of `layer` to hold its data (bounded).
__device__ __forceinline__ void wait_stage(const PParams& P, uint64_t* bars, int layer) {
  const int slot = (layer - P.l0) % P.ns;
  const unsigned parity = (unsigned)(((layer - P.l0) / P.ns) & 1);
  if (threadIdx.x == 0) {
    unsigned it = 0;
    while (!mbar_try_wait(bars + slot, parity)) {
      if ((++it & 1023u) == 0 && ld_acquire(P.sync + 3) != 0) break;
      if (it > spin_limit()) {
        atomicOr(P.sync + 3, 2u);
        break;
      }
    }
  }
  cta_sync();
}

// Issue the bulk copies that fill the ring slot of `layer` with this CTA's slice of it.
// Copy i (0..31) of this CTA's share of layer `layer`: source, byte offset in the ring stage and
// size (0 = none); all 16-byte aligned, sizes multiples of 16.  The byte total of a stage is
// precomputed on the host (CtaPlan::tx).
template <int B>
__device__ __forceinline__ void copy_desc(const PParams& P, const CtaPlan& pl, int layer, int i,
                                          const void*& src, int& dst, unsigned& bytes) {
  const LayerW L = layer_w(P, layer);
  const Layout& Y = P.lay;
  const int RB = P.d_model / 8, RBO = P.d_inner / 8;
  const void* s_ = nullptr;
  int d_ = 0;
  unsigned n_ = 0;
  const char* inb = reinterpret_cast<const char*>(L.in.bits);
  if (pl.role == 0) {
    const int c0 = pl.h * DFSSM_HEADDIM + pl.p0, np = pl.np;
    switch (i) {
      case 0: s_ = inb + (size_t)c0 * RB; d_ = Y.in_bits; n_ = np * RB; break;
      case 1: s_ = inb + (size_t)(P.d_inner + c0) * RB; d_ = Y.in_bits + np * RB; n_ = np * RB; break;
      case 3: s_ = L.in.scale + c0; d_ = Y.in_scale; n_ = np * 2; break;
      case 4: s_ = L.in.scale + P.d_inner + c0; d_ = Y.in_scale + np * 2; n_ = np * 2; break;
      case 5: s_ = L.in.A16 + (size_t)c0 * 16; d_ = Y.in_lA; n_ = np * 32; break;
      case 6: s_ = L.in.A16 + (size_t)(P.d_inner + c0) * 16; d_ = Y.in_lA + np * 32; n_ = np * 32; break;
      case 9: s_ = L.conv_w + (size_t)c0 * 4; d_ = Y.conv_w; n_ = np * 8; break;
      case 10: s_ = L.conv_b + c0; d_ = Y.conv_b; n_ = np * 2; break;
      default: break;
    }
    const int j = i - 15;
    if (j >= 0 && j < B) {
      s_ = P.ssm + (long long)layer * P.ssm_layer +
           ((long long)(j * P.nheads + pl.h) * DFSSM_HEADDIM + pl.p0) * DFSSM_DSTATE;
      d_ = Y.state + j * np * DFSSM_DSTATE * 4;
      n_ = np * DFSSM_DSTATE * 4;
    }
    const int k = i - 15 - B;
    if (k >= 0 && k < 3 * B) {
      s_ = P.conv + (long long)layer * P.conv_layer + (long long)k * P.d_xbc + c0;
      d_ = Y.cstate + k * np * 4;
      n_ = np * 4;
    }
  } else if (pl.role == 1) {
    // rows [bc0, bc0 + nbc) of the B/C/dt block; only the B/C channels have conv1d operands
    const int r0 = 2 * P.d_inner + pl.bc0, c0 = P.d_inner + pl.bc0, nb = pl.nbc;
    const int nconv = max(0, min(nb, 2 * DFSSM_DSTATE - pl.bc0));
    switch (i) {
      case 0: s_ = inb + (size_t)r0 * RB; d_ = Y.in_bits; n_ = nb * RB; break;
      case 3: s_ = L.in.scale + r0; d_ = Y.in_scale; n_ = nb * 2; break;
      case 5: s_ = L.in.A16 + (size_t)r0 * 16; d_ = Y.in_lA; n_ = nb * 32; break;
      case 9: s_ = L.conv_w + (size_t)c0 * 4; d_ = Y.conv_w; n_ = nconv * 8; break;
      case 10: s_ = L.conv_b + c0; d_ = Y.conv_b; n_ = nconv * 2; break;
      default: break;
    }
    const int k = i - 15 - B;
    if (k >= 0 && k < 3 * B) {
      s_ = P.conv + (long long)layer * P.conv_layer + (long long)k * P.d_xbc + c0;
      d_ = Y.cstate + k * nb * 4;
      n_ = nconv * 4;
    }
  }
  if (pl.no > 0) {
    const char* ob = reinterpret_cast<const char*>(L.out.bits);
    switch (i) {
      case 11: s_ = ob + (size_t)pl.o0 * RBO; d_ = Y.out_bits; n_ = pl.no * RBO; break;
      case 12: s_ = L.out.scale + pl.o0; d_ = Y.out_scale; n_ = pl.no * 2; break;
      case 13: s_ = L.out.A16 + (size_t)pl.o0 * 16; d_ = Y.out_lA; n_ = pl.no * 32; break;
      default: break;
    }
  }
  src = s_;
  dst = d_;
  bytes = n_;
}

// The ring stage of a layer is cut into pieces of at most kCopyPiece bytes, and piece p belongs
// to part floor(kParts * (its first byte) / (stage bytes)).  The compute threads release a
// slot in kParts steps spread over the following layer, so the ring's HBM traffic arrives as
// kParts small bursts instead of one large burst that would delay every CTA's exchange words.
constexpr unsigned kCopyPiece = 4096;
constexpr int kParts = 4;

// 1-bit GEMV of one row held in shared memory for B activation rows: returns the int32
// sum_k s_k q_k for every b in all 16 lanes of the half-warp.
template <int B>
struct Dots {
  int v[B];
};

template <int B>
__device__ __forceinline__ Dots<B> row_dot(const unsigned char* bits, int K, const int8_t* sq, int Kq, int l16,
                                        const int (&qs)[B]) {
  Dots<B> dot;
  int acc[B];
#pragma unroll
  for (int b = 0; b < B; ++b) acc[b] = 0;
  const int C = K >> 7;
  for (int c = l16; c < C; c += 16) {
    const uint4 wv = *reinterpret_cast<const uint4*>(bits + c * 16);
    const unsigned ws[4] = {wv.x, wv.y, wv.z, wv.w};
    unsigned m[32];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) m[j * 8 + i] = (ws[j] >> i) & 0x01010101u;
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const int4* qv = reinterpret_cast<const int4*>(sq + b * Kq + c * 128);
      int a = acc[b];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int4 qq = qv[u ^ (c & 7)];  // swizzled: see qswz()
        a = dp4a_us(m[4 * u + 0], qq.x, a);
        a = dp4a_us(m[4 * u + 1], qq.y, a);
        a = dp4a_us(m[4 * u + 2], qq.z, a);
        a = dp4a_us(m[4 * u + 3], qq.w, a);
      }
      acc[b] = a;
    }
  }
#pragma unroll
  for (int b = 0; b < B; ++b) {
    int a = acc[b];
    a += __shfl_xor_sync(0xffffffffu, a, 8);
    a += __shfl_xor_sync(0xffffffffu, a, 4);
    a += __shfl_xor_sync(0xffffffffu, a, 2);
    a += __shfl_xor_sync(0xffffffffu, a, 1);
    dot.v[b] = 2 * a - qs[b];
  }
  return dot;
}

// dequant + LoRA up-projection of one output row (reference rounding points).  A16 (16 fp16,
// 16-byte aligned) and t live in shared memory; the rank sum runs as 4 independent chains,
// since few threads run this epilogue and its latency is on the critical path.
__device__ __forceinline__ float proj_out(int dot, float xs, float wscale, const __half* A16, const float* t) {
  const float base = round_hc(round_hc(round_hc((float)dot) * xs) * wscale);
  const uint4 a0 = reinterpret_cast<const uint4*>(A16)[0], a1 = reinterpret_cast<const uint4*>(A16)[1];
  const unsigned aw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  float p[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&aw[i]));
    p[i & 3] = fmaf(t[2 * i], f.x, p[i & 3]);
    p[i & 3] = fmaf(t[2 * i + 1], f.y, p[i & 3]);
  }
  return round_hc(base + round_hc((p[0] + p[1]) + (p[2] + p[3])));
}

__device__ __forceinline__ float conv_silu(float s0, float s1, float s2, float v, const __half* cw, float cb) {
  const float o = s0 * h2f(cw[0]) + s1 * h2f(cw[1]) + s2 * h2f(cw[2]) + v * h2f(cw[3]) + cb;
  const float sig = 1.0f / (1.0f + expf(-o));
  return o * sig;
}

// LoRA-t producer: compute this CTA's ranks (r = tj, tj + n_t, ...) of t = fp16(xn . B16^T) and
// publish each as a tagged word.  The values of the first rank (r = tj) were loaded into b0
// before the wait for the activations, so the producer's path holds no HBM round trip for them.
template <int B, int KPT>
__device__ void publish_t(const PParams& P, int tj, const float (&vals)[B][KPT], typename RankHalves<KPT>::T b0,
                          const __half* B16, int K, unsigned long long* tw, unsigned tag, float* red) {
  // rank reductions alternate between red + 64 and red, the buffers the preceding norm did not
  // use last
  for (int r = tj, j = 0; r < DFSSM_RANK; r += P.n_t, ++j) {
    float t[B];
    lora_t_rank_v<B, KPT>(vals, r == tj ? b0 : load_rank_b<KPT>(B16, K, r), t, (j & 1) ? red : red + 64);
    if (threadIdx.x == 0)
#pragma unroll
      for (int b = 0; b < B; ++b) put_word(tw + b * DFSSM_RANK + r, P.rs, __float_as_uint(t[b]), tag);
  }
}

// One relaxed read of an exchange word, issued ahead of independent work so that its L2 round
// trip overlaps that work; take_word() then polls again only if the tag did not match yet.
__device__ __forceinline__ unsigned long long peek_word(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ unsigned take_word(const unsigned long long* p, unsigned long long early, unsigned tag,
                                              unsigned* err, unsigned code) {
  if ((unsigned)(early >> 32) == tag) return (unsigned)early;
  unsigned v[1][1];
  take_words<1, 1>(p, 0, tag, v, err, code);
  return v[0][0];
}

// This thread's LoRA-t word (threads < B x 16) of this CTA's replica.
template <int B>
__device__ __forceinline__ const unsigned long long* t_word(const PParams& P, const unsigned long long* tw) {
  return tw + (blockIdx.x % kReplicas) * P.rs + (threadIdx.x < B * DFSSM_RANK ? threadIdx.x : 0);
}

// Collect the B x 16 published LoRA t values into s_t; `early` is peek_word(t_word(...)) issued
// before the dot products.
template <int B>
__device__ __forceinline__ void fetch_t(const PParams& P, const unsigned long long* tw, unsigned tag, float* s_t,
                                        unsigned long long early) {
  if (threadIdx.x < B * DFSSM_RANK) s_t[threadIdx.x] = __uint_as_float(take_word(t_word<B>(P, tw), early, tag, P.sync + 3, 8u));
  cta_sync();
}

// The LoRA t words can be taken by the last warps of the CTA while the others run the dot products
// of `rows` rows (one per half-warp) when those warps have no row: kTWarps warps from thread kT0.
template <int B>
struct IdleT {
  static constexpr int kTWarps = (B * DFSSM_RANK + 31) / 32;
  static constexpr int kT0 = (kWarps - kTWarps) * 32;
  // (batches 3 and 4 measured 1-2% slower with it: their words are better read ahead of the dots)
  static __device__ __forceinline__ bool fits(int rows) { return B <= 2 && ((rows + 1) & ~1) <= kT0 / 16; }
  // the calling thread's t word, taken into s_t (threads outside [kT0, kT0 + B * 16) do nothing)
  static __device__ __forceinline__ void take(const PParams& P, const unsigned long long* tw, unsigned tag,
                                              float* s_t) {
    const int i = (int)threadIdx.x - kT0;
    if (i >= 0 && i < B * DFSSM_RANK)
      s_t[i] = __uint_as_float(
          take_word(tw + (blockIdx.x % kReplicas) * P.rs + i, 0ull, tag, P.sync + 3, 8u));
  }
};

// The copy-issuing warp: fills ring slot (k % ns) with layer l0 + k.  The first ns layers go
// out at once; later ones part by part, each as soon as the compute threads have released that
// part of the slot (empty barrier slot * kParts + part) while running the layer after the one
// that used it.  Lane i owns copy i of copy_desc, so a layer costs the warp one pass over the
// table; the warp shares its SM with 16 busy compute warps and must stay cheap.  The slot's
// previous contents were read by the compute threads before they released the part (an
// mbarrier arrive after their barrier), which lane 0 observed before the copies are issued.
// Bounded: gives up when a wait times out or the error word is set.
template <int B>
__device__ void copy_issuer(const PParams& P, const CtaPlan& pl, unsigned char* ring, uint64_t* full,
                            uint64_t* empty) {
  const int lane = threadIdx.x & 31;
  const int nl = P.l1 - P.l0;
  const unsigned tx = (unsigned)pl.tx;
  const unsigned b1 = tx / kParts, b2 = 2 * tx / kParts, b3 = 3 * tx / kParts;  // first bytes of parts 1..3
  const int RC = P.lay.stage_bytes / P.d_model;                 // embedding rows per head chunk
  const int nch = P.do_head ? (pl.nv + RC - 1) / RC : 0;
  for (int k = 0; k < nl + nch; ++k) {
    const int layer = P.l0 + k, slot = k % P.ns;
    unsigned char* st = ring + (size_t)slot * P.lay.stage_bytes;
    if (k >= nl) {  // LM head chunk: rows [r0, r0 + nr) of this CTA's vocabulary slice
      if (k >= P.ns) {
        int ok = 1;
        if (lane == 0) {
          const unsigned parity = (unsigned)((k / P.ns - 1) & 1);
          for (int part = 0; part < kParts && ok; ++part) {
            unsigned it = 0;
            while (!mbar_try_wait(empty + slot * kParts + part, parity)) {
              if ((++it & 1023u) == 0 && ld_acquire(P.sync + 3) != 0) {
                ok = 0;
                break;
              }
              if (it > spin_limit()) {
                atomicOr(P.sync + 3, 32u);
                ok = 0;
                break;
              }
            }
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) return;
      }
      const int r0 = pl.v0 + (k - nl) * RC, nr = min(RC, pl.v0 + pl.nv - r0);
      const unsigned bytes = (unsigned)nr * (unsigned)P.d_model;
      if (lane == 0) mbar_expect_tx(full + slot, bytes);
      __syncwarp();
      const char* src = reinterpret_cast<const char*>(P.Eq) + (size_t)r0 * P.d_model;
      for (unsigned off = lane * kCopyPiece; off < bytes; off += 32 * kCopyPiece)
        bulk_g2s(st + off, src + off, min(kCopyPiece, bytes - off), full + slot);
      __syncwarp();
      continue;
    }
    const void* src;
    int dst;
    unsigned n;
    copy_desc<B>(P, pl, layer, lane, src, dst, n);
    unsigned pre = n;  // inclusive prefix sum of the copy sizes over lanes -> first byte of mine
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned v = __shfl_up_sync(0xffffffffu, pre, o);
      if (lane >= o) pre += v;
    }
    pre -= n;
    for (int part = 0; part < kParts; ++part) {
      if (k >= P.ns) {
        int ok = 1;
        if (lane == 0) {
          const unsigned parity = (unsigned)((k / P.ns - 1) & 1);
          unsigned it = 0;
          while (!mbar_try_wait(empty + slot * kParts + part, parity)) {
            if ((++it & 1023u) == 0 && ld_acquire(P.sync + 3) != 0) {
              ok = 0;
              break;
            }
            if (it > spin_limit()) {
              atomicOr(P.sync + 3, 32u);
              ok = 0;
              break;
            }
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) return;
      }
      if (part == 0) {
        if (lane == 0) mbar_expect_tx(full + slot, tx);
        __syncwarp();
      }
      for (unsigned off = 0; off < n; off += kCopyPiece) {
        const unsigned at = pre + off;
        const int pp = (at >= b1) + (at >= b2) + (at >= b3);
        if (pp == part || k < P.ns)
          bulk_g2s(st + dst + off, reinterpret_cast<const char*>(src) + off, min(kCopyPiece, n - off), full + slot);
      }
      if (P.trace && lane == 0 && (part == 0 || part == kParts - 1)) {  // points 14 / 15 of the issued layer
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        P.trace[(size_t)blockIdx.x * (4 + kTracePerLayer * P.n_layer) + 2 + kTracePerLayer * layer + 14 +
                (part != 0)] = t;
      }
      __syncwarp();
      if (k < P.ns) break;  // the first ns layers: every piece went out with part 0
    }
  }
}

// Compute side: release part `part` of the ring slot used by the previous layer.
__device__ __forceinline__ void release_part(const PParams& P, uint64_t* empties, int layer, int part) {
  if (threadIdx.x == 0 && layer > P.l0) mbar_arrive(empties + ((layer - 1 - P.l0) % P.ns) * kParts + part);
}

template <int B, int KI, int KO>
__global__ void __launch_bounds__(kBlockThreads, 1) persistent_step_kernel(PParams P) {
  static_assert(B >= 1 && B <= 4, "the reduction scratch and the copy table hold up to four sequences");
  constexpr int kEpiLanes = (32 / (2 * B)) * (2 * B);  // epilogue entries per warp: whole row pairs
  extern __shared__ __align__(128) unsigned char smem[];
  const int d_model = P.d_model, d_inner = P.d_inner;
  // working smem (carve-up mirrored by build_plan)
  __half* s_x = reinterpret_cast<__half*>(smem);                   // [B][d_model]
  int8_t* s_q = reinterpret_cast<int8_t*>(smem + B * d_model * 2);  // [B][d_inner]
  float* s_misc = reinterpret_cast<float*>(smem + B * d_model * 2 + B * d_inner);
  // reduction buffers: red (norm, odd LoRA ranks), red + 64 (even LoRA ranks), red + 128
  // (quantisation amax) -- consecutive single-barrier reductions never share one
  float* red = s_misc;                              // [kRedFloats]
  float* s_t = red + kRedFloats;                    // [B*16]
  float* s_xs = s_t + B * 16;                       // [B]
  int* s_qpart = reinterpret_cast<int*>(s_xs + B);  // [B][kWarps] per-warp q sums
  float* s_abar = reinterpret_cast<float*>(s_qpart + B * kWarps);  // [16]: exp(A dt) per sequence
  float* s_z = s_abar + 16;                         // [B][64]: the SiLU(z) gate factors
  float* s_xc = s_z + B * 64;                       // [B][64]
  float* s_dt = s_xc + B * 64;                      // [B]
  float* s_bc = s_dt + B;                           // [B][2*d_state] (fp32)
  int* s_dot = reinterpret_cast<int*>(s_bc + B * 2 * DFSSM_DSTATE);  // [kDotRows][B] GEMV results
  // per-layer table copied once at kernel start (no dependent global loads inside the loop):
  // the layer pointer table, and this CTA's head scalars (dt_bias, A_log, D) for every layer
  float* s_hptab = reinterpret_cast<float*>(smem + P.tab_off);  // [n_layer][4], 16-byte aligned
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.ring_off - 8 * 8);      // ring slot full
  uint64_t* empties = reinterpret_cast<uint64_t*>(smem + P.ring_off - 8 * 8 - 8 * 4 * 8);  // [slot][part] released
  unsigned char* ring = smem + P.ring_off;

  const CtaPlan pl = P.plans[blockIdx.x];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, l16 = lane & 15, hw = tid >> 4;
  const unsigned ebase0 = __ldcg(P.sync + 16);  // tag epoch of this launch
  const unsigned step_tags = (unsigned)(P.n_layer + 1) * kTagsPerLayer;
  const unsigned ebase = ebase0 + (P.skew && blockIdx.x == 0 ? step_tags : 0u);
  const int XW = d_model / 2, GW = d_inner / 2;
  const size_t rep_off = (size_t)(blockIdx.x % kReplicas) * P.rs;  // this CTA's copy of the exchange words

  if (tid == 0) {
    for (int i = 0; i < P.ns; ++i) {
      mbar_init(bars + i, 1);
      for (int j = 0; j < kParts; ++j) mbar_init(empties + i * kParts + j, 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  stamp(P, 0);
  {
    if (pl.role == 0) {
      for (int l = tid; l < P.n_layer; l += kBlockThreads) {
        const LayerW G = layer_w(P, l);
        float* e = s_hptab + l * 4;
        e[0] = G.dt_bias[pl.h];
        e[1] = G.A_log[pl.h];
        e[2] = G.Dp[pl.h];
      }
    }
  }
  __syncthreads();
  if (wid == kWarps) {
    copy_issuer<B>(P, pl, ring, bars, empties);
    return;
  }

  // embedding gather (every CTA needs the full x of the first layer)
  for (int i = tid; i < B * d_model && !P.from_x; i += kThreads) {
    const int b = i / d_model, k = i - b * d_model;
    int tok = P.tokens[b];
    tok = min(max(tok, 0), P.vocab - 1);
    s_x[i] = f2h((float)P.Eq[(size_t)tok * d_model + k] * P.Es[tok]);
  }
  cta_sync();

  for (int layer = P.l0; layer < P.l1; ++layer) {
    const LayerW L = layer_w(P, layer);
    unsigned char* st = ring + (size_t)((layer - P.l0) % P.ns) * P.lay.stage_bytes;
    // ---------------- alpha: per-thread weights are loaded before waiting for x
    float w_in[KI];
    {
      ld_f32s<KI>(L.ln_w + tid * KI, w_in);
    }
    const bool t_producer = pl.role == 1 && pl.tj < P.n_t;
    typename RankHalves<KI>::T tb_in{};
    if (t_producer) tb_in = load_rank_b<KI>(L.in.B16, d_model, pl.tj);
    const int tb = 2 + kTracePerLayer * layer;
    stamp(P, tb + 0);
    const int par = layer & 1;
    if (layer > P.l0) {  // x of this layer, published word by word by the previous layer's out_proj
      take_x<B, KI>(P.xw + rep_off + (size_t)par * B * XW, B * XW, tag_of(ebase, layer, kTagX), s_x, P.sync + 3);
    } else if (P.from_x) {
      for (int i = tid; i < B * d_model / 8; i += kThreads)
        reinterpret_cast<uint4*>(s_x)[i] = __ldcg(reinterpret_cast<const uint4*>(P.x_g) + i);
      cta_sync();
    }
    stamp(P, tb + 1);
    release_part(P, empties, layer, 0);
    {
      float vals[B][KI];
#pragma unroll
      for (int b = 0; b < B; ++b)
#pragma unroll
        for (int j = 0; j < KI; ++j) vals[b][j] = h2f(s_x[b * d_model + tid * KI + j]);
      prep_norm<B, KI>(vals, w_in, d_model, red);
      if (t_producer) publish_t<B, KI>(P, pl.tj, vals, tb_in, L.in.B16, d_model, P.tw + (size_t)(par * 2 + 0) * B * DFSSM_RANK,
                                         tag_of(ebase, layer, kTagTin), red);  // publish before quantising
      prep_quantize<B, KI>(vals, s_q, d_inner, s_xs, s_qpart, red + 128);
    }
    int qs[B];
#pragma unroll
    for (int b = 0; b < B; ++b) qs[b] = qsum_of(s_qpart, b);
    stamp(P, tb + 3);
    wait_stage(P, bars, layer);
    stamp(P, tb + 4);
    const int RB = d_model / 8;
    // updated SSM state of a head CTA, written back after it arrives at the gated barrier so that
    // the barrier's release does not wait for these 16 KB of stores
    float4 hnew[B][kMaxRPW];
    if (pl.role == 0) {
      const int np = pl.np, nrows = 2 * np;  // z and x rows (the dt rows belong to the B/C CTAs)
      const __half* sc = reinterpret_cast<const __half*>(st + P.lay.in_scale);
      const __half* la = reinterpret_cast<const __half*>(st + P.lay.in_lA);
      const __half* cw = reinterpret_cast<const __half*>(st + P.lay.conv_w);
      const __half* cb = reinterpret_cast<const __half*>(st + P.lay.conv_b);
      const float* cst = reinterpret_cast<const float*>(st + P.lay.cstate);
      const unsigned long long t_early = peek_word(t_word<B>(P, P.tw + (size_t)(par * 2 + 0) * B * DFSSM_RANK));
      for (int i = hw; i < ((nrows + 1) & ~1); i += 2 * kWarps) {
        const int row = i < nrows ? i : nrows - 1;
        const Dots<B> dd = row_dot<B>(st + P.lay.in_bits + (size_t)row * RB, d_model, s_q, d_inner, l16, qs);
        if (i < nrows && l16 < B) s_dot[row * B + l16] = dd.v[l16];
      }
      cta_sync();
      stamp(P, tb + 12);
      release_part(P, empties, layer, 1);
      fetch_t<B>(P, P.tw + (size_t)(par * 2 + 0) * B * DFSSM_RANK, tag_of(ebase, layer, kTagTin), s_t, t_early);
      stamp(P, tb + 2);
      // word i < B * d_state is B/C word i % d_state of sequence i / d_state, word B * d_state + b
      // the one holding dt of head h for sequence b; thread tid takes word tid (read ahead once
      // here) and, where B * (d_state + 1) > kThreads, word tid + kThreads as well
      constexpr int kBcWords = B * (DFSSM_DSTATE + 1);
      auto bc_word = [&](int i) {
        const int b = i < B * DFSSM_DSTATE ? i / DFSSM_DSTATE : i - B * DFSSM_DSTATE;
        const int j = i < B * DFSSM_DSTATE ? i - b * DFSSM_DSTATE : DFSSM_DSTATE + pl.h / 2;
        return P.bcw + ((size_t)par * B + b) * P.bcw_per_seq + rep_off + j;
      };
      // The B/C and dt words: where there are enough threads without an epilogue entry (tid >= E) for
      // one word each, they wait for and take them while the others run the epilogue, so the wait
      // overlaps the epilogue instead of following it; else every thread takes them after the epilogue,
      // each thread's first word read once ahead of it (measured: batch 1 +2.6%; two words per idle
      // thread made batches 3 and 4 slower).
      const int E = nrows * B;  // epilogue entries, one per thread
      const bool bc_idle = E + kBcWords <= kThreads;
      auto take_bc = [&](int i, unsigned long long early) {
        const unsigned v = take_word(bc_word(i), early, tag_of(ebase, layer, kTagBC), P.sync + 3, 4u);
        if (i < B * DFSSM_DSTATE) {
          s_bc[2 * i] = lo_h(v);
          s_bc[2 * i + 1] = hi_h(v);
        } else {  // dt = softplus(raw + dt_bias) and exp(A dt), once per sequence
          const float* hp = s_hptab + layer * 4;
          const float dtv = log1pf(expf(((pl.h & 1) ? hi_h(v) : lo_h(v)) + hp[0]));
          s_dt[i - B * DFSSM_DSTATE] = dtv;
          s_abar[i - B * DFSSM_DSTATE] = expf(dtv * (-expf(hp[1])));
        }
      };
      if (bc_idle && tid >= E && tid - E < kBcWords) take_bc(tid - E, 0ull);
      const unsigned long long bc_early = !bc_idle && tid < kBcWords ? peek_word(bc_word(tid)) : 0ull;
      for (int e2 = tid; e2 < E; e2 += kThreads) {
        const int row = e2 / B, b = e2 - row * B;
        const int dot = s_dot[e2];
        const float v = proj_out(dot, s_xs[b], h2f(sc[row]), la + row * 16, s_t + b * 16);
        if (row < np) {  // the gate factor fp16(z fp16(sigmoid(z))) of this channel
          const float sig = round_h(1.0f / (1.0f + expf(-v)));
          s_z[b * 64 + row] = round_h(v * sig);
        } else {
          const int j = row - np, ch = pl.h * DFSSM_HEADDIM + pl.p0 + j;
          const float s0 = cst[(b * 3 + 0) * np + j], s1 = cst[(b * 3 + 1) * np + j], s2 = cst[(b * 3 + 2) * np + j];
          float* gcs = P.conv + (long long)layer * P.conv_layer + (long long)b * 3 * P.d_xbc + ch;
          gcs[0] = s1;
          gcs[P.d_xbc] = s2;
          gcs[2 * P.d_xbc] = v;
          s_xc[b * 64 + j] = round_hc(conv_silu(s0, s1, s2, v, cw + j * 4, h2f(cb[j])));
        }
      }
      if (!bc_idle)
        for (int i = tid; i < kBcWords; i += kThreads) take_bc(i, i == tid ? bc_early : 0ull);
      cta_sync();
      stamp(P, tb + 5);
      stamp(P, tb + 6);
      // SSM state update + gate; warp w owns rows p = 2w, 2w+1 (np = 2 * kWarps), lane owns
      // n = 4*lane..; lane 0 publishes the gated pair as one word
      unsigned long long* gw = P.gw + (size_t)par * B * GW;
      const unsigned tg_g = tag_of(ebase, layer, kTagGated);
      const float* sst = reinterpret_cast<const float*>(st + P.lay.state);
      const float* hp = s_hptab + layer * 4;
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const float dtv = s_dt[b], Abar = s_abar[b];
        const float Dh = hp[2];
        const float* bb = s_bc + b * 256 + lane * 4;
        const float4 Bn = make_float4(bb[0], bb[1], bb[2], bb[3]);
        const float4 Cn = make_float4(bb[128], bb[129], bb[130], bb[131]);
        float part[kMaxRPW];
#pragma unroll
        for (int rr = 0; rr < kMaxRPW; ++rr) {
          const int p = wid * kMaxRPW + rr;
          const float4 hv = *reinterpret_cast<const float4*>(sst + ((size_t)b * np + p) * DFSSM_DSTATE + lane * 4);
          const float X = s_xc[b * 64 + p] * dtv;
          float4 o;
          o.x = Abar * hv.x + X * Bn.x;
          o.y = Abar * hv.y + X * Bn.y;
          o.z = Abar * hv.z + X * Bn.z;
          o.w = Abar * hv.w + X * Bn.w;
          hnew[b][rr] = o;
          part[rr] = Cn.x * o.x + Cn.y * o.y + Cn.z * o.z + Cn.w * o.w;
        }
        // C.h of the two rows over the 32 lanes as a transposing butterfly (5 shuffles instead of 10):
        // lanes 0-15 end with row 0, lanes 16-31 with row 1; lanes 0 and 16 finish their row and lane 0
        // publishes the pair
        static_assert(kMaxRPW == 2, "the butterfly below pairs two rows per warp");
        const bool hi = (lane & 16) != 0;
        float sum = (hi ? part[1] : part[0]) + __shfl_xor_sync(0xffffffffu, hi ? part[0] : part[1], 16);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const int pr = wid * kMaxRPW + (hi ? 1 : 0);
        const float gmine = round_h(sum + s_xc[b * 64 + pr] * Dh) * s_z[b * 64 + pr];
        const float gnext = __shfl_sync(0xffffffffu, gmine, 16);
        if (lane == 0) {
          const int c = pl.h * DFSSM_HEADDIM + pl.p0 + wid * kMaxRPW;
          const unsigned w = pack_h2(gmine, gnext);
          put_word(gw + (size_t)b * GW + c / 2, P.rs, w, tg_g);
          *reinterpret_cast<unsigned*>(P.gated_g + (size_t)b * d_inner + c) = w;  // plain copy for the host API
        }
      }
    } else if (pl.role == 1) {
      const int nb = pl.nbc;
      const __half* sc = reinterpret_cast<const __half*>(st + P.lay.in_scale);
      const __half* la = reinterpret_cast<const __half*>(st + P.lay.in_lA);
      const __half* cw = reinterpret_cast<const __half*>(st + P.lay.conv_w);
      const __half* cb = reinterpret_cast<const __half*>(st + P.lay.conv_b);
      const float* cst = reinterpret_cast<const float*>(st + P.lay.cstate);
      const unsigned long long* tw_in = P.tw + (size_t)(par * 2 + 0) * B * DFSSM_RANK;
      const bool t_idle = IdleT<B>::fits(nb);  // warps without B/C rows take t during the dot products
      const unsigned long long t_early = t_idle ? 0ull : peek_word(t_word<B>(P, tw_in));
      for (int i = hw; i < ((nb + 1) & ~1); i += 2 * kWarps) {
        const int row = i < nb ? i : nb - 1;
        const Dots<B> dd = row_dot<B>(st + P.lay.in_bits + (size_t)row * RB, d_model, s_q, d_inner, l16, qs);
        if (i < nb && l16 < B) s_dot[row * B + l16] = dd.v[l16];
      }
      if (t_idle) IdleT<B>::take(P, tw_in, tag_of(ebase, layer, kTagTin), s_t);
      cta_sync();
      stamp(P, tb + 12);
      release_part(P, empties, layer, 1);
      if (!t_idle) fetch_t<B>(P, tw_in, tag_of(ebase, layer, kTagTin), s_t, t_early);
      stamp(P, tb + 2);
      unsigned long long* bcw = P.bcw + (size_t)par * B * P.bcw_per_seq;
      const unsigned tg_bc = tag_of(ebase, layer, kTagBC);
      // one thread per (row, b), e = row * B + b; a warp takes kEpiLanes consecutive entries (whole
      // row pairs), so the partner row of a pair sits B lanes up in the same warp, and the even
      // row's lane publishes the pair
      for (int e0 = wid * kEpiLanes; e0 < nb * B; e0 += kWarps * kEpiLanes) {
        const int e2 = e0 + lane, row = e2 / B, b = e2 - row * B;
        const bool mine = lane < kEpiLanes && e2 < nb * B;
        float o = 0.f;
        if (mine) {
          const float v = proj_out(s_dot[e2], s_xs[b], h2f(sc[row]), la + row * 16, s_t + b * 16);
          if (pl.bc0 + row < 2 * DFSSM_DSTATE) {  // B/C channel: conv1d + SiLU
            const int ch = d_inner + pl.bc0 + row;
            const float s0 = cst[(b * 3 + 0) * nb + row], s1 = cst[(b * 3 + 1) * nb + row], s2 = cst[(b * 3 + 2) * nb + row];
            float* gcs = P.conv + (long long)layer * P.conv_layer + (long long)b * 3 * P.d_xbc + ch;
            gcs[0] = s1;
            gcs[P.d_xbc] = s2;
            gcs[2 * P.d_xbc] = v;
            o = conv_silu(s0, s1, s2, v, cw + row * 4, h2f(cb[row]));
          } else {  // dt row of head bc0 + row - 2 d_state: raw projection (fp16-exact)
            o = v;
          }
        }
        const float o_next = __shfl_down_sync(0xffffffffu, o, B);
        if (mine && (row & 1) == 0)
          put_word(bcw + (size_t)b * P.bcw_per_seq + (pl.bc0 + row) / 2, P.rs, pack_h2(o, o_next), tg_bc);
      }
      cta_sync();
    } else {
      release_part(P, empties, layer, 1);  // no in_proj rows
    }
    stamp(P, tb + 7);
    // ---------------- beta: out_proj rows
    float w_out[KO];
    {
      ld_f32s<KO>(L.norm_w + tid * KO, w_out);
    }
    typename RankHalves<KO>::T tb_out{};
    if (t_producer) tb_out = load_rank_b<KO>(L.out.B16, d_inner, pl.tj);
    stamp(P, tb + 8);
    // head CTAs write their state back, then every CTA collects the gated vector
    cta_sync();
    release_part(P, empties, layer, 2);
    if (pl.role == 0) {
#pragma unroll
      for (int b = 0; b < B; ++b)
#pragma unroll
        for (int rr = 0; rr < kMaxRPW; ++rr) {
          const int p = wid * kMaxRPW + rr;
          float* gh = P.ssm + (long long)layer * P.ssm_layer +
                      ((long long)(b * P.nheads + pl.h) * DFSSM_HEADDIM + pl.p0 + p) * DFSSM_DSTATE + lane * 4;
          __stcs(reinterpret_cast<float4*>(gh), hnew[b][rr]);
        }
    }
    {
      float vals[B][KO];
      const unsigned long long* gw = P.gw + (size_t)par * B * GW;
      const unsigned tg_g = tag_of(ebase, layer, kTagGated);
      unsigned v[B][KO / 2];
      // the gated vector is the largest exchange (every CTA takes all of it while most wait for
      // the slowest head): poll one word per thread, then load the rest
      take_words<B, KO / 2, DFSSM_GFIRST>(gw + rep_off + tid * (KO / 2), GW, tg_g, v, P.sync + 3, 16u);
#pragma unroll
      for (int b = 0; b < B; ++b)
#pragma unroll
        for (int j = 0; j < KO / 2; ++j) {
          vals[b][2 * j] = lo_h(v[b][j]);
          vals[b][2 * j + 1] = hi_h(v[b][j]);
        }
      if (P.trace) cta_sync();  // point 9 marks the whole CTA holding the gated vector
      stamp(P, tb + 9);
      prep_norm<B, KO>(vals, w_out, d_inner, red);
      if (t_producer) publish_t<B, KO>(P, pl.tj, vals, tb_out, L.out.B16, d_inner, P.tw + (size_t)(par * 2 + 1) * B * DFSSM_RANK,
                                         tag_of(ebase, layer, kTagTout), red);  // publish before quantising
      prep_quantize<B, KO>(vals, s_q, d_inner, s_xs, s_qpart, red + 128);
    }
#pragma unroll
    for (int b = 0; b < B; ++b) qs[b] = qsum_of(s_qpart, b);
    stamp(P, tb + 10);
    release_part(P, empties, layer, 3);
    const unsigned long long* tw_out = P.tw + (size_t)(par * 2 + 1) * B * DFSSM_RANK;
    const bool to_idle = IdleT<B>::fits(pl.no);  // warps without out_proj rows take t meanwhile
    const unsigned long long to_early = pl.no > 0 && !to_idle ? peek_word(t_word<B>(P, tw_out)) : 0ull;
    if (pl.no > 0) {
      const int RBO = d_inner / 8;
      for (int i = hw; i < ((pl.no + 1) & ~1); i += 2 * kWarps) {
        const int row = i < pl.no ? i : pl.no - 1;
        const Dots<B> dd = row_dot<B>(st + P.lay.out_bits + (size_t)row * RBO, d_inner, s_q, d_inner, l16, qs);
        if (i < pl.no && l16 < B) s_dot[row * B + l16] = dd.v[l16];
      }
      if (to_idle) IdleT<B>::take(P, tw_out, tag_of(ebase, layer, kTagTout), s_t);
    }
    cta_sync();
    stamp(P, tb + 13);
    if (pl.no > 0) {
      if (!to_idle) fetch_t<B>(P, tw_out, tag_of(ebase, layer, kTagTout), s_t, to_early);
      const __half* sc = reinterpret_cast<const __half*>(st + P.lay.out_scale);
      const __half* la = reinterpret_cast<const __half*>(st + P.lay.out_lA);
      unsigned long long* xw = P.xw + (size_t)(par ^ 1) * B * XW;
      const unsigned tg_x = tag_of(ebase, layer + 1, kTagX);
      // one thread per (row, b) as in the B/C epilogue; the even row's lane publishes the pair
      for (int e0 = wid * kEpiLanes; e0 < pl.no * B; e0 += kWarps * kEpiLanes) {
        const int e2 = e0 + lane, row = e2 / B, b = e2 - row * B;
        const int o = pl.o0 + row;
        const bool mine = lane < kEpiLanes && e2 < pl.no * B;
        float xo = 0.f;
        if (mine) {
          const float v = proj_out(s_dot[e2], s_xs[b], h2f(sc[row]), la + row * 16, s_t + b * 16);
          xo = h2f(s_x[b * d_model + o]) + v;
        }
        const float xo_next = __shfl_down_sync(0xffffffffu, xo, B);
        if (mine && (row & 1) == 0) {
          const unsigned w = pack_h2(xo, xo_next);
          put_word(xw + (size_t)b * XW + o / 2, P.rs, w, tg_x);
          *reinterpret_cast<unsigned*>(P.x_g + (size_t)b * d_model + o) = w;  // plain copy for the host API
        }
      }
    }
    cta_sync();
    stamp(P, tb + 11);
  }

  // ---------------- final norm + LM head + argmax
  // The copy warp streams this CTA's embedding rows through the ring as items nl, nl + 1, ...
  // (RC rows each) once the compute threads release the slots, as it does for layers.
  stamp(P, 2 + kTracePerLayer * P.n_layer);
  const int nl = P.l1 - P.l0;
  if (tid == 0)  // the last layer's slot is free now
    for (int j = 0; j < kParts; ++j) mbar_arrive(empties + ((nl - 1) % P.ns) * kParts + j);
  if (P.do_head) {
    take_x<B, KI>(P.xw + rep_off + (size_t)(P.l1 & 1) * B * XW, B * XW, tag_of(ebase, P.l1, kTagX), s_x, P.sync + 3);
    stamp(P, 3 + kTracePerLayer * P.n_layer);
    {
      // normalised x, fp16-exact, written back over x in s_x (each thread rewrites its own columns)
      float vals[B][KI];
      float ss[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        float a = 0.f;
#pragma unroll
        for (int j = 0; j < KI; ++j) {
          vals[b][j] = h2f(s_x[b * d_model + tid * KI + j]);
          a = __fadd_rn(a, __fmul_rn(vals[b][j], vals[b][j]));
        }
        ss[b] = a;
      }
      block_sum_n<B>(ss, red);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const float r = rsqrtf(__fadd_rn(__fmul_rn(ss[b], 1.0f / (float)d_model), 1e-5f));
#pragma unroll
        for (int j = 0; j < KI; ++j) {
          const int k = tid * KI + j;
          s_x[b * d_model + k] = f2h(__fmul_rn(__fmul_rn(vals[b][j], r), P.norm_f[k]));
        }
      }
    }
    cta_sync();
    unsigned long long mybest[B];
#pragma unroll
    for (int b = 0; b < B; ++b) mybest[b] = 0ull;
    // Logits on the fp16 tensor cores (mma.sync m16n8k16, fp32 accumulation; the int8 rows become
    // exact fp16 by a byte permute, the normalised x is fp16, so every product is exact).  The rows
    // of a chunk go in 16-row tiles, two tiles per pass: warp w takes tile w / 8 of the pass and the
    // K slice w % 8 (d_model / 512 blocks of 64 columns), lane (g, c) loads 16 bytes at 16c of a
    // block's rows g and g + 8 (the k order of A and B agrees), batch column n = g of B (zero for
    // g >= B).  Partial sums [2][8 slices][16 rows][B] meet in s_q (free in the head phase) and are
    // added over the slices in a fixed order by one thread per (tile, row, sequence).
    const int RC = P.lay.stage_bytes / d_model, nch = (pl.nv + RC - 1) / RC;
    const int g = lane >> 2, c = lane & 3;
    const int nblk = d_model / 64, bps = nblk / 8;  // 64-column blocks, blocks per K slice
    const int wtile = wid >> 3, slice = wid & 7;
    float* part = reinterpret_cast<float*>(s_q);  // [2][8][16][B]
    for (int ch = 0; ch < nch; ++ch) {
      const int item = nl + ch;
      wait_stage(P, bars, P.l0 + item);
      const unsigned char* st = ring + (size_t)(item % P.ns) * P.lay.stage_bytes;
      const int r0 = pl.v0 + ch * RC, nr = min(RC, pl.v0 + pl.nv - r0);
      for (int t0 = 0; t0 < nr; t0 += 32) {  // a pass: tiles t0 / 16 and t0 / 16 + 1
        // the row scale of the thread that finishes (tile, row, sequence) below, requested before the
        // MMAs so that its memory round trip overlaps them
        float es_pre = 0.f;
        if (tid < 32 * B) {
          const int tile = tid / (16 * B), row = (tid - tile * 16 * B) / B, r = t0 + 16 * tile + row;
          if (r < nr) es_pre = __ldg(P.Es + r0 + r);
        }
        const int tr0 = t0 + 16 * wtile;      // this warp's tile's first row
        if (tr0 < nr) {
          const uint4* ra = reinterpret_cast<const uint4*>(st + (size_t)min(tr0 + g, nr - 1) * d_model);
          const uint4* rb = reinterpret_cast<const uint4*>(st + (size_t)min(tr0 + g + 8, nr - 1) * d_model);
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          for (int blk = slice * bps; blk < (slice + 1) * bps; ++blk) {
            const uint4 ea = ra[blk * 4 + c], eb = rb[blk * 4 + c];
            const unsigned wa[4] = {ea.x ^ 0x80808080u, ea.y ^ 0x80808080u, ea.z ^ 0x80808080u, ea.w ^ 0x80808080u};
            const unsigned wb[4] = {eb.x ^ 0x80808080u, eb.y ^ 0x80808080u, eb.z ^ 0x80808080u, eb.w ^ 0x80808080u};
#pragma unroll
            for (int s2 = 0; s2 < 4; ++s2) {
              const unsigned a0 = i8x2_to_h2(wa[s2], 0x4140u), a2 = i8x2_to_h2(wa[s2], 0x4342u);
              const unsigned a1 = i8x2_to_h2(wb[s2], 0x4140u), a3 = i8x2_to_h2(wb[s2], 0x4342u);
              uint2 bv = make_uint2(0u, 0u);
              if (g < B) bv = *reinterpret_cast<const uint2*>(s_x + g * d_model + blk * 64 + 16 * c + 4 * s2);
              mma_f16(acc, a0, a1, a2, a3, bv.x, bv.y);
            }
          }
          // D: acc[0..1] -> row g, columns 2c, 2c + 1; acc[2..3] -> row g + 8
          if (2 * c < B) {  // lane (g, c) holds batch columns 2c and 2c + 1
            float* pp = part + ((size_t)(wtile * 8 + slice) * 16) * B;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const int b = 2 * c + k;
              if (b < B) {
                pp[g * B + b] = acc[k];
                pp[(g + 8) * B + b] = acc[2 + k];
              }
            }
          }
        }
        cta_sync();
        if (tid < 32 * B) {  // (tile, row, sequence)
          const int tile = tid / (16 * B), rem = tid - tile * 16 * B, row = rem / B, b = rem - row * B;
          const int r = t0 + 16 * tile + row;
          if (r < nr) {
            const float* pp = part + ((size_t)(tile * 8) * 16 + row) * B + b;
            float sum = 0.f;
#pragma unroll
            for (int sl = 0; sl < 8; ++sl) sum += pp[(size_t)sl * 16 * B];
            const int vr = r0 + r;
            const float lg = sum * es_pre;
            P.logits[(size_t)b * P.vocab + vr] = lg;
            const unsigned long long key = argmax_key(f2h(lg), (uint32_t)vr);
#pragma unroll
            for (int bb = 0; bb < B; ++bb)  // static indices keep mybest in registers
              if (bb == b) mybest[bb] = key > mybest[bb] ? key : mybest[bb];
          }
        }
        cta_sync();  // the partials are read before the next pass (or chunk) writes them
      }
      if (tid == 0)  // every warp is done with the chunk: release its slot
        for (int j = 0; j < kParts; ++j) mbar_arrive(empties + (item % P.ns) * kParts + j);
    }
    // each thread's best keys -> the warp's best per sequence (lane 0)
#pragma unroll
    for (int b = 0; b < B; ++b)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, mybest[b], o);
        mybest[b] = k2 > mybest[b] ? k2 : mybest[b];
      }
    unsigned long long* sb = reinterpret_cast<unsigned long long*>(red);
    cta_sync();
    if (lane == 0)
#pragma unroll
      for (int b = 0; b < B; ++b) sb[wid * B + b] = mybest[b];
    cta_sync();
    if (tid < B) {
      unsigned long long k = 0ull;
      for (int w = 0; w < kWarps; ++w) k = sb[w * B + tid] > k ? sb[w * B + tid] : k;
      atomicMax(P.best + tid, k);
    }
  }  // do_head
  stamp(P, 1);
  cta_sync();
  // drain: no bulk copy into this CTA's ring may still be in flight when it exits (only
  // possible after a timed-out wait); bounded, ignores the error word
  if (tid == 0) {
    const int RC = P.lay.stage_bytes / d_model;
    const int ni = nl + (P.do_head ? (pl.nv + RC - 1) / RC : 0);  // ring items: layers, then head chunks
    for (int s = 0; s < P.ns && s < ni; ++s) {
      const int last = s + ((ni - 1 - s) / P.ns) * P.ns;
      unsigned it = 0;
      // a lowered test limit still leaves copies from valid memory ample time to land
      const unsigned lim = spin_limit() > (1u << 16) ? spin_limit() : (1u << 16);
      while (!mbar_try_wait(bars + s, (unsigned)((last / P.ns) & 1)) && ++it < lim) {
      }
    }
  }
  // exit protocol: the last CTA out publishes the tokens and resets the sync words
  if (tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(P.sync + 1, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence();
      for (int b = 0; b < B && P.do_head; ++b) {
        const unsigned long long k = atomicExch(P.best + b, 0ull);
        P.tokens[b] = (int)argmax_key_index(k);
      }
      // next launch's tags (past a skewed CTA's, so none of its words can match them)
      P.sync[16] = ebase0 + (P.skew ? 2u : 1u) * step_tags;
      __threadfence();
      P.sync[1] = 0;
    }
  }
}

// ------------------------------------------------------------------ host side

// Tagged exchange words of one replica for launch groups of up to G sequences.
size_t xch_words(const dfssm_dims& d, size_t G) {
  return 2 * G * (d.d_model / 2) + 2 * G * (d.d_state + d.nheads / 2) + 2 * G * (d.d_inner / 2) +
         2 * 2 * G * DFSSM_RANK;
}
constexpr size_t kXchSlack = 4096;  // spare words per replica (room for a layout pad)

struct PersistentState {
  int ready = 0;
  void* fn = nullptr;
  PParams params{};
  CtaPlan* d_plans = nullptr;
  int smem = 0;
  int grid = 0;
};

constexpr int kPersistGroupMax = 4;  // largest batch one launch of the kernel takes (instances 1 to 4)

struct PersistentSet {
  PersistentState st[kPersistGroupMax + 1];  // indexed by the group size: 1 to 4
  int skew_next = 0;      // dfssm_debug_skew_next_step: the next launch runs skewed
};

template <int B, int KI, int KO>
void* kernel_ptr() {
  return reinterpret_cast<void*>(persistent_step_kernel<B, KI, KO>);
}

void* pick_kernel(int B, int KI, int KO) {
#define DFSSM_PK(b, ki, ko) \
  if (B == b && KI == ki && KO == ko) return kernel_ptr<b, ki, ko>();
  DFSSM_PK(1, 4, 8)
  DFSSM_PK(2, 4, 8)
  DFSSM_PK(3, 4, 8)
  DFSSM_PK(4, 4, 8)
  DFSSM_PK(1, 1, 2)
  DFSSM_PK(2, 1, 2)
#undef DFSSM_PK
  return nullptr;
}

PersistentSet* set_of(const dfssm_engine* e) { return static_cast<PersistentSet*>(e->persist); }

// Per-CTA work plans and the ring-stage layout for batch B.  Returns 0 if the dims or the
// batch are not supported by the persistent kernel.
int build_plan(const dfssm_engine* e, int B, int grid, std::vector<CtaPlan>& plans, Layout& lay, int& ns,
               int& smem_total, int& n_bc, int& tab_off) {
  const dfssm_dims& d = e->d;
  if (d.d_model % 512 || d.d_inner % 512) return 0;
  const int KI = d.d_model / 512, KO = d.d_inner / 512;
  if (!pick_kernel(B, KI, KO)) return 0;
  const int S = 2, np = DFSSM_HEADDIM / S;
  const int n_items = d.nheads * S;
  n_bc = grid - n_items;
  if (d.d_state != DFSSM_DSTATE || d.nheads % 8) return 0;
  const int bc_groups = (2 * d.d_state + d.nheads) / 8;  // 8-row groups of the B, C and dt rows
  if (n_bc < 1) return 0;
  if (n_bc > bc_groups) n_bc = bc_groups;
  plans.assign(grid, CtaPlan{});
  const int og = d.d_model / 8;  // out rows in 8-row groups
  int max_no = 0, max_nbc = 0;
  // LoRA-t producers (the first min(16, n_bc) B/C CTAs) get no out_proj rows: they publish the
  // out_proj t while the others run their GEMV, and would otherwise arrive last at the x barrier
  const int n_t = n_bc < DFSSM_RANK ? n_bc : DFSSM_RANK;
  const int n_out = grid - n_t;
  int oc = 0;
  for (int c = 0; c < grid; ++c) {
    CtaPlan& p = plans[c];
    const bool producer = c >= n_items && c < n_items + n_t;
    if (producer) {
      p.o0 = 0;
      p.no = 0;
    } else {
      const int g0 = (int)((long long)og * oc / n_out), g1 = (int)((long long)og * (oc + 1) / n_out);
      p.o0 = g0 * 8;
      p.no = (g1 - g0) * 8;
      ++oc;
    }
    max_no = p.no > max_no ? p.no : max_no;
    const long long v0 = (long long)d.vocab * c / grid, v1 = (long long)d.vocab * (c + 1) / grid;
    p.v0 = (int)v0;
    p.nv = (int)(v1 - v0);
    if (c < n_items) {
      p.role = 0;
      p.h = c / S;
      p.p0 = (c % S) * np;
      p.np = np;
    } else if (c < n_items + n_bc) {
      const int j = c - n_items;
      const int b0 = bc_groups * j / n_bc, b1 = bc_groups * (j + 1) / n_bc;
      p.role = 1;
      p.tj = j;
      p.bc0 = b0 * 8;
      p.nbc = (b1 - b0) * 8;
      max_nbc = p.nbc > max_nbc ? p.nbc : max_nbc;
    } else {
      p.role = 2;
    }
  }
  const int RB = d.d_model / 8, RBO = d.d_inner / 8;
  for (CtaPlan& p : plans) {
    long long tx = 0;
    if (p.role == 0)
      tx += (long long)(2 * p.np) * RB + 2 * p.np * (2 + 32) + p.np * 8 + p.np * 2 +
            (long long)B * p.np * DFSSM_DSTATE * 4 + 3LL * B * p.np * 4;
    else if (p.role == 1) {
      const int nconv = std::max(0, std::min(p.nbc, 2 * d.d_state - p.bc0));
      tx += (long long)p.nbc * RB + p.nbc * (2 + 32) + nconv * 8 + nconv * 2 + 3LL * B * nconv * 4;
    }
    if (p.no > 0) tx += (long long)p.no * RBO + p.no * (2 + 32);
    p.tx = (int)tx;
  }
  const int rows_in = 2 * np > max_nbc ? 2 * np : max_nbc;
  const int ch = np > max_nbc ? np : max_nbc;
  auto a16 = [](int x) { return (x + 15) & ~15; };
  int off = 0;
  lay.in_bits = off; off += a16(rows_in * RB);
  lay.in_scale = off; off += a16(2 * ch * 2);
  lay.in_lA = off; off += a16(2 * ch * 32);  // fp16 LoRA A rows
  lay.in_lAs = off;
  lay.conv_w = off; off += a16(ch * 8);
  lay.conv_b = off; off += a16(ch * 2);
  lay.out_bits = off; off += a16(max_no * RBO);
  lay.out_scale = off; off += a16(max_no * 2);
  lay.out_lA = off; off += a16(max_no * 32);
  lay.out_lAs = off;
  lay.state = off; off += a16(B * np * DFSSM_DSTATE * 4);
  lay.cstate = off; off += a16(B * 3 * ch * 4);
  lay.stage_bytes = (off + 127) & ~127;
  if (2 * np > kDotRows || max_nbc > kDotRows || max_no > kDotRows) return 0;
  const int misc_floats = kRedFloats + B * 16 + B + B * kWarps + 16 + B * 64 * 2 + B + B * 256 + kDotRows * B + 8;
  int work = B * d.d_model * 2 + B * d.d_inner + misc_floats * 4;
  work = (work + 127) & ~127;
  tab_off = work;
  work += d.n_layer * 4 * 4;  // head scalars (dt_bias, A_log, D) of every layer
  work = (work + 127) & ~127;
  const int ring_off = work + 384;  // 8 full + 8 x 4 released mbarriers live just below the ring
  int max_smem = 0;
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, e->device);
  ns = (max_smem - ring_off) / lay.stage_bytes;
  if (ns > 6) ns = 6;
  if (ns < 2) return 0;
  if (ns * lay.stage_bytes < B * d.d_model * 4) return 0;  // the head phase reuses the ring
  smem_total = ring_off + ns * lay.stage_bytes;
  return 1;
}

}  // namespace

void persistent_destroy(dfssm_engine* e) {
  PersistentSet* ps = set_of(e);
  if (!ps) return;
  for (auto& s : ps->st)
    if (s.d_plans) cudaFree(s.d_plans);
  delete ps;
  e->persist = nullptr;
}

// Byte stride between consecutive layers' weights if every array of every layer sits at the
// same offset from its layer's first array (the arena's plan), else 0.
long long uniform_layer_stride(const dfssm_engine* e) {
  const auto& Ls = e->layers;
  if (Ls.size() < 2) return 0;
  auto fields = [](const LayerW& L) {
    return std::vector<const char*>{
        (const char*)L.in.bits, (const char*)L.in.scale, (const char*)L.in.A16, (const char*)L.in.B16,
        (const char*)L.out.bits, (const char*)L.out.scale, (const char*)L.out.A16, (const char*)L.out.B16,
        (const char*)L.conv_w, (const char*)L.conv_b, (const char*)L.A_log, (const char*)L.Dp,
        (const char*)L.dt_bias, (const char*)L.norm_w, (const char*)L.ln_w};
  };
  const auto f0 = fields(Ls[0]);
  const long long st = (long long)(fields(Ls[1])[0] - f0[0]);
  for (size_t l = 0; l < Ls.size(); ++l) {
    const auto fl = fields(Ls[l]);
    for (size_t i = 0; i < f0.size(); ++i)
      if ((long long)(fl[i] - f0[i]) != (long long)l * st) return 0;
  }
  return st;
}

int persistent_init(dfssm_engine* e) {
  if (!e->persist) e->persist = new PersistentSet();
  const long long lstride = e->d.n_layer > 1 ? uniform_layer_stride(e) : 0;
  if (e->d.n_layer > 1 && lstride == 0) return DFSSM_OK;  // no persistent kernel: it derives layer pointers
  for (int B = 1; B <= kPersistGroupMax; ++B) {
    PersistentState& ps = set_of(e)->st[B];
    ps.ready = 0;
    if (B > e->max_batch) continue;
    std::vector<CtaPlan> plans;
    Layout lay;
    int ns = 0, smem = 0, n_bc = 0, tab_off = 0;
    const int grid = e->sm_count;
    if (!build_plan(e, B, grid, plans, lay, ns, smem, n_bc, tab_off)) continue;
    const dfssm_dims& d = e->d;
    void* fn = pick_kernel(B, d.d_model / 512, d.d_inner / 512);
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    int nblk = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nblk, fn, kBlockThreads, smem) != cudaSuccess || nblk < 1) {
      cudaGetLastError();
      continue;
    }
    if (cudaMalloc(&ps.d_plans, sizeof(CtaPlan) * grid) != cudaSuccess) return dfssm_fail(DFSSM_ERR_OOM, "plan alloc");
    if (cudaMemcpy(ps.d_plans, plans.data(), sizeof(CtaPlan) * grid, cudaMemcpyHostToDevice) != cudaSuccess)
      return dfssm_fail(DFSSM_ERR_CUDA, "plan upload");
    PParams& P = ps.params;
    P.lw0 = e->layers[0];
    P.lstride = lstride;
    P.plans = ps.d_plans;
    P.lay = lay;
    P.n_layer = d.n_layer;
    P.d_model = d.d_model;
    P.d_inner = d.d_inner;
    P.d_state = d.d_state;
    P.d_xbc = d.d_xbc;
    P.n_in = d.n_in;
    P.nheads = d.nheads;
    P.vocab = d.vocab;
    P.Eq = e->Eq;
    P.Es = e->Es;
    P.norm_f = e->norm_f;
    P.ssm = e->ssm;
    P.conv = e->conv;
    P.ssm_layer = (long long)e->ssm_layer;
    P.conv_layer = (long long)e->conv_layer;
    P.x_g = e->x;
    P.xw = e->xch;
    // Every exchange region holds [2 parities][G sequences][...] with G = 2 for launches of one or
    // two sequences and 4 for four, then the next replica follows after `pad` more words
    // (DFSSM_XPAD; default 0).  Where the words fall among the L2 slices moves the batch-1 step by
    // up to +-3% (pads of 0..384 words on one box: 1768..1870 tok/s), but which pad is best changed
    // from box to box, so no pad is tuned in.
    const int G = B <= 2 ? 2 : kPersistGroupMax;  // (B = 3 and 4 share the four-sequence layout)
    static const size_t pad = [] {
      const char* v = getenv("DFSSM_XPAD");
      const long long p = v ? atoll(v) : 0;
      // whole 64-byte lines: the exchange words are also read as 16-byte pairs
      return (size_t)(p < 0 ? 0 : (p > (long long)kXchSlack ? (long long)kXchSlack : p)) & ~(size_t)7;
    }();
    P.rs = xch_words(d, G) + pad;
    P.bcw = P.xw + 2 * G * d.d_model / 2;
    P.bcw_per_seq = d.d_state + d.nheads / 2;
    P.gw = P.bcw + 2 * G * P.bcw_per_seq;
    P.tw = P.gw + 2 * G * d.d_inner / 2;
    P.gated_g = e->gated;
    P.logits = e->logits;
    P.best = e->best;
    P.tokens = e->tokens;
    P.sync = e->sync;
    P.l0 = 0;
    P.l1 = d.n_layer;
    P.from_x = 0;
    P.do_head = 1;
    P.n_bc = n_bc;
    P.n_t = n_bc < DFSSM_RANK ? n_bc : DFSSM_RANK;
    P.ns = ns;
    P.ring_off = smem - ns * lay.stage_bytes;
    P.trace = nullptr;
    P.tab_off = tab_off;
    ps.fn = fn;
    ps.smem = smem;
    ps.grid = grid;
    ps.ready = 1;
  }
  return DFSSM_OK;
}

size_t persistent_xch_words(const dfssm_dims& d) { return xch_words(d, kPersistGroupMax) + kXchSlack; }
size_t persistent_xch_bytes(const dfssm_dims& d) { return 8 * persistent_xch_words(d) * kReplicas; }

// Batches of up to kPersistMaxBatch sequences run as consecutive launches over groups of the
// largest sizes the kernel has (4, then the remaining 1 to 4), each group on its rows of the state and activation
// buffers.
constexpr int kPersistMaxBatch = 8;

// Size of the group that starts a batch of n remaining sequences (0 if no instance fits).
int group_size(const PersistentSet* ps, int n) {
  for (int g = n < kPersistGroupMax ? n : kPersistGroupMax; g >= 1; --g)
    if (ps->st[g].ready) return g;
  return 0;
}

bool persistent_supported(const dfssm_engine* e) {
  if (!e->persist || e->batch < 1 || e->batch > kPersistMaxBatch) return false;
  const PersistentSet* ps = set_of(e);
  for (int n = e->batch; n > 0;) {
    const int g = group_size(ps, n);
    if (!g) return false;
    n -= g;
  }
  return true;
}

int launch_persistent_layers(dfssm_engine* e, int l0, int l1, int from_x, int do_head, cudaStream_t s) {
  if (!persistent_supported(e)) return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "persistent kernel unavailable");
  if (l0 < 0 || l1 > e->d.n_layer || l0 >= l1) return dfssm_fail(DFSSM_ERR_ARG, "bad layer range [%d, %d)", l0, l1);
  const dfssm_dims& d = e->d;
  for (int b0 = 0, nb = 0; b0 < e->batch; b0 += nb) {
    nb = group_size(set_of(e), e->batch - b0);
    PersistentState& ps = set_of(e)->st[nb];
    PParams P = ps.params;
    // this group's rows of every per-sequence buffer (the layer strides stay those of max_batch)
    P.ssm += (size_t)b0 * d.nheads * DFSSM_HEADDIM * DFSSM_DSTATE;
    P.conv += (size_t)b0 * 3 * d.d_xbc;
    P.x_g += (size_t)b0 * d.d_model;
    P.gated_g += (size_t)b0 * d.d_inner;
    P.logits += (size_t)b0 * d.vocab;
    P.best += b0;
    P.tokens += b0;
    P.l0 = l0;
    P.l1 = l1;
    P.from_x = from_x;
    P.do_head = do_head;
    P.skew = set_of(e)->skew_next;
    void* args[] = {&P};
    cudaError_t ce = cudaLaunchCooperativeKernel(ps.fn, dim3(ps.grid), dim3(kBlockThreads), args, (size_t)ps.smem, s);
    if (ce != cudaSuccess) return dfssm_fail(DFSSM_ERR_CUDA, "cooperative launch failed: %s", cudaGetErrorString(ce));
  }
  set_of(e)->skew_next = 0;
  return DFSSM_OK;
}

int persistent_debug_skew(dfssm_engine* e) {
  if (!e->persist) return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "persistent kernel unavailable");
  set_of(e)->skew_next = 1;
  return DFSSM_OK;
}

int persistent_debug_wait_limit(dfssm_engine* e, unsigned polls) {
  const unsigned v = polls ? polls : kSpinLimit;
  if (cudaSetDevice(e->device) != cudaSuccess || cudaMemcpyToSymbol(c_spin_limit, &v, sizeof(v)) != cudaSuccess)
    return dfssm_fail(DFSSM_ERR_CUDA, "setting the wait limit failed");
  return DFSSM_OK;
}

int launch_persistent_step(dfssm_engine* e, cudaStream_t s) {
  return launch_persistent_layers(e, 0, e->d.n_layer, 0, 1, s);
}

size_t persistent_trace_entries(const dfssm_engine* e) {
  return (size_t)e->sm_count * (4 + kTracePerLayer * e->d.n_layer);
}

int launch_persistent_traced(dfssm_engine* e, unsigned long long* trace_dev, cudaStream_t s) {
  if (!persistent_supported(e) || group_size(set_of(e), e->batch) != e->batch)
    return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "the phase trace runs one persistent launch: batch 1 to 4");
  PersistentState& ps = set_of(e)->st[e->batch];
  PParams P = ps.params;
  P.trace = trace_dev;
  void* args[] = {&P};
  cudaError_t ce = cudaLaunchCooperativeKernel(ps.fn, dim3(ps.grid), dim3(kBlockThreads), args, (size_t)ps.smem, s);
  if (ce != cudaSuccess) return dfssm_fail(DFSSM_ERR_CUDA, "cooperative launch failed: %s", cudaGetErrorString(ce));
  return DFSSM_OK;
}
