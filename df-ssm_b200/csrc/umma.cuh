// Batched scaffold projection on the 5th-generation tensor cores (tcgen05, kind::i8), for batches
// of 64 and more (decode at large batch, prompt prefill rows, the stand-alone scaffold GEMM).
//
// One CTA computes a 128-row x NT-column tile of D = mask . q^T with the accumulator in tensor
// memory (TMEM): MMA M = 128 weight rows, N = NT batch rows, K in 256-byte chunks.
//   A (weights): the 0/1 sign masks as u8, built in shared memory from the packed bits: word w of
//     a row gives the 32 bytes (w >> j) & 0x01010101, j = 0..7 -- the permuted column order that
//     the quantised activations are stored in (qperm_index), so A and B columns line up.
//   B (activations): the permuted int8 q rows, as s8.
//   D (s32): sum over k of mask * q; the signed product is 2 D - sum_k q, as in the GEMV paths,
//     so the int32 result equals torch._int_mm on the +-1 weights bit for bit.
// Both operands use the K-major, no-swizzle canonical layout of 8-row x 16-byte core matrices:
// a row group's 16 core matrices along the chunk are contiguous (leading-byte offset 128 B) and
// row groups follow at 2 KB (stride-byte offset).  Two chunk buffers: threads fill one while the
// tensor core reads the other; an MMA batch signals its buffer free through tcgen05.commit on an
// mbarrier.  The epilogue reads D with tcgen05.ld (warp w and w + 4 own TMEM lanes 32(w % 4)..,
// i.e. output rows; each thread holds its row's dequant/LoRA/conv operands in registers) and
// runs the same per-element arithmetic as proj_mma_kernel.
#pragma once
#include <cuda.h>  // CUtensorMap (the map is encoded on the host through the driver entry point)

#include "common.cuh"

namespace dfssm {

constexpr int kUmmaThreads = 256;
#ifndef DFSSM_UMMA_KC
#define DFSSM_UMMA_KC 128
#endif
constexpr int kUmmaKC = DFSSM_UMMA_KC;  // K bytes per chunk (KC / 32 MMAs of K = 32)
constexpr int kUmmaMinBatch = 64;   // batches below this use proj_mma_kernel (mma.sync)
constexpr int kUmmaSpin = 1 << 22;  // bound of every mbarrier wait

__device__ __forceinline__ uint64_t umma_sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout = 0) {
  // start address, leading / stride byte offsets (16-byte units), descriptor version 1
  // (tcgen05), base offset 0, layout type (0 = no swizzle, 2 = 128-byte swizzle)
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

__device__ __forceinline__ bool umma_wait(uint64_t* bar, unsigned parity) {
  for (int it = 0; it < kUmmaSpin; ++it)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

inline size_t proj_umma_smem(int NT) {
  return 1024 + (size_t)2 * (128 + NT) * kUmmaKC + 2 * NT * 4 + NT * DFSSM_RANK * 4;  // + base alignment
}

// MODE as proj_mma_kernel: 0 in_proj + conv1d, 1 out_proj + residual, 2 raw int32, 3 plain.
// Grid (ceil(N / 128), ceil(B / NT), ksplit); (K / ksplit) % 256 == 0.  With ksplit > 1 the CTAs
// of a tile each take a K range (narrow projections would otherwise leave most SMs idle): the
// integer partials meet exactly, in any order, through atomicAdd -- into `out` for MODE 2 (zeroed
// by the caller), else into ws [B][N] int32 with a per-tile counter cnt, and the last CTA of the
// tile runs the epilogue and clears its part of ws and its counter.  err: set to 1 if a wait ran
// out.
// TMAB: the activation tiles arrive by TMA (tensor map tmq over q [B][K] int8, box 128 bytes x NT
// rows, 128-byte swizzle; rows past B read as zeros) and both operands use the 128-byte-swizzled
// K-major layout (8-row atoms of 1 KB, 16-byte unit u of row r at unit u ^ (r % 8)); otherwise the
// threads stage them in the no-swizzle core-matrix layout.
template <int MODE, int NT, bool TMAB>
__global__ void __launch_bounds__(kUmmaThreads, 1)
proj_umma_kernel(const __grid_constant__ CUtensorMap tmq, ProjW p, const int8_t* __restrict__ q,
                 const int* __restrict__ qsum, const __half* __restrict__ xs,
                 const __half* __restrict__ t, int B, __half* __restrict__ out, int ld_out,
                 float* __restrict__ conv_state, const __half* __restrict__ conv_w, const __half* __restrict__ conv_b,
                 int d_inner, int d_xbc, int ksplit, int* __restrict__ ws, unsigned* __restrict__ cnt,
                 unsigned* __restrict__ err) {
  constexpr int ABYTES = 128 * kUmmaKC, BBYTES = NT * kUmmaKC, SBO = kUmmaKC / 16 * 128;
  constexpr int WPR = kUmmaKC / 32, CPR = kUmmaKC / 16;  // words / 16-byte units per row and chunk
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // 1 KB-aligned base (the 128-byte swizzle atoms and TMA destinations need it)
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  static_assert(!TMAB || kUmmaKC == 128, "the swizzled layout holds one 128-byte row per chunk");
  // buffer k: A at smem + k (ABYTES + BBYTES), B right after it
  auto sA = [&](int k) { return smem + k * (ABYTES + BBYTES); };
  auto sB = [&](int k) { return smem + k * (ABYTES + BBYTES) + ABYTES; };
  float* e_xs = reinterpret_cast<float*>(smem + 2 * (ABYTES + BBYTES));  // [NT]
  int* e_qsum = reinterpret_cast<int*>(e_xs + NT);                         // [NT]
  float* e_t = reinterpret_cast<float*>(e_qsum + NT);                      // [NT][16]
  __shared__ uint64_t bars[2];
  __shared__ uint64_t fulls[2];  // TMAB: the B tile of a buffer has landed
  __shared__ uint32_t s_tmem;
  __shared__ int s_last;
  const int tid = threadIdx.x, wid = tid >> 5, lane = tid & 31;
  const int N = p.N, K = p.K, W = K >> 5;
  const int row0 = blockIdx.x * 128, b0 = blockIdx.y * NT, nb = min(NT, B - b0);
  if (wid == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)), "r"(NT));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init(&fulls[0], 1);
    mbar_init(&fulls[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // per-column operands of this batch tile
  for (int j = tid; j < NT; j += kUmmaThreads) {
    const int b = b0 + min(j, nb - 1);
    e_qsum[j] = qsum[b];
    e_xs[j] = MODE != 2 ? h2f(xs[b]) : 0.f;
  }
  if (MODE != 2)
    for (int i = tid; i < NT * DFSSM_RANK; i += kUmmaThreads) e_t[i] = h2f(t[(size_t)(b0 + min(i / DFSSM_RANK, nb - 1)) * DFSSM_RANK + i % DFSSM_RANK]);
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = s_tmem;
  const uint32_t idesc = (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(NT >> 3) << 17) | ((128u >> 4) << 24);

  // A chunk: 128 rows x WPR words; B chunk: NT rows x CPR 16-byte units.  A chunk's global loads
  // go to registers one chunk ahead of its shared-memory stores, so their latency overlaps the
  // tensor core working on the previous chunk.
  constexpr int AW = 128 * WPR / kUmmaThreads;  // words per thread
  constexpr int BU = NT * CPR / kUmmaThreads;   // 16-byte units per thread
  uint32_t rw[AW];
  uint4 rv[BU];
  auto load = [&](int kc) {
#pragma unroll
    for (int u = 0; u < AW; ++u) {
      const int i = tid + u * kUmmaThreads, r = i / WPR, j = i - r * WPR;
      rw[u] = __ldg(p.bits + (size_t)min(row0 + r, N - 1) * W + (kc >> 5) + j);
    }
    if (!TMAB)
#pragma unroll
      for (int u = 0; u < BU; ++u) {
        const int i = tid + u * kUmmaThreads, b = i / CPR, c = i - b * CPR;
        rv[u] = __ldg(reinterpret_cast<const uint4*>(q + (size_t)(b0 + min(b, nb - 1)) * K + kc) + c);
      }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int u = 0; u < AW; ++u) {
      const int i = tid + u * kUmmaThreads, r = i / WPR, j = i - r * WPR;
      const uint32_t x = rw[u];
      const uint4 lo = make_uint4(x & 0x01010101u, (x >> 1) & 0x01010101u, (x >> 2) & 0x01010101u,
                                  (x >> 3) & 0x01010101u);
      const uint4 hi = make_uint4((x >> 4) & 0x01010101u, (x >> 5) & 0x01010101u, (x >> 6) & 0x01010101u,
                                  (x >> 7) & 0x01010101u);
      if (TMAB) {  // units 2j, 2j + 1 of row r, swizzled
        unsigned char* rowp = sA(buf) + (r >> 3) * 1024 + (r & 7) * 128;
        *reinterpret_cast<uint4*>(rowp + (((2 * j) ^ (r & 7)) << 4)) = lo;
        *reinterpret_cast<uint4*>(rowp + (((2 * j + 1) ^ (r & 7)) << 4)) = hi;
      } else {
        unsigned char* dst = sA(buf) + (r >> 3) * SBO + (2 * j) * 128 + (r & 7) * 16;
        *reinterpret_cast<uint4*>(dst) = lo;
        *reinterpret_cast<uint4*>(dst + 128) = hi;
      }
    }
    if (!TMAB)
#pragma unroll
      for (int u = 0; u < BU; ++u) {
        const int i = tid + u * kUmmaThreads, b = i / CPR, c = i - b * CPR;
        *reinterpret_cast<uint4*>(sB(buf) + (b >> 3) * SBO + c * 128 + (b & 7) * 16) = rv[u];
      }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
  };

  const int klen = K / ksplit, kbeg = blockIdx.z * klen;
  const int nch = klen / kUmmaKC;
  bool ok = true;
  unsigned ph0 = 0u, ph1 = 0u;  // next phase to wait for on bars[0] / bars[1]
  auto wait_buf = [&](int k) {
    const bool r = umma_wait(&bars[k], k ? ph1 : ph0);
    if (k) ph1 ^= 1u;
    else ph0 ^= 1u;
    return r;
  };
  unsigned fph0 = 0u, fph1 = 0u;  // TMAB: next phase of fulls[0] / fulls[1]
  auto issue_b = [&](int kc, int buf) {  // thread 0: the B tile of chunk kc into buffer buf
    if (TMAB && tid == 0) {
      mbar_expect_tx(&fulls[buf], (unsigned)BBYTES);
      asm volatile(
          "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
              smem_u32(sB(buf))),
          "l"(reinterpret_cast<uint64_t>(&tmq)), "r"(kc), "r"(b0), "r"(smem_u32(&fulls[buf]))
          : "memory");
    }
  };
  issue_b(kbeg, 0);
  load(kbeg);
  store(0);
  if (nch > 1) {
    issue_b(kbeg + kUmmaKC, 1);
    load(kbeg + kUmmaKC);
  }
  for (int c = 0; c < nch; ++c) {
    const int buf = c & 1;
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    if (tid == 0) {
      if (TMAB) {  // the chunk's B tile
        ok = umma_wait(&fulls[buf], buf ? fph1 : fph0) && ok;
        if (buf) fph1 ^= 1u;
        else fph0 ^= 1u;
      }
#pragma unroll
      for (int s = 0; s < kUmmaKC / 32; ++s) {
        // no swizzle: the K step is 2 core matrices (256 B); swizzled: 32 bytes along the 128-byte row
        const uint64_t da = TMAB ? umma_sdesc(smem_u32(sA(buf)) + s * 32, 16, 1024, 2)
                                 : umma_sdesc(smem_u32(sA(buf)) + s * 256, 128, SBO);
        const uint64_t db = TMAB ? umma_sdesc(smem_u32(sB(buf)) + s * 32, 16, 1024, 2)
                                 : umma_sdesc(smem_u32(sB(buf)) + s * 256, 128, SBO);
        const uint32_t accum = (c > 0 || s > 0) ? 1u : 0u;
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
                     "l"(da), "l"(db), "r"(idesc), "r"(accum));
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(&bars[buf]))
                   : "memory");
    }
    if (c + 1 < nch) {
      // the other buffer was last read by the MMAs of chunk c - 1
      if (c >= 1) {
        ok = wait_buf(buf ^ 1) && ok;
        issue_b(kbeg + (c + 1) * kUmmaKC, buf ^ 1);
      }
      store(buf ^ 1);
      if (c + 2 < nch) load(kbeg + (c + 2) * kUmmaKC);
    }
  }
  // the last chunk's MMAs (and with them all earlier ones) complete
  {
    const int lb = (nch - 1) & 1;
    if (nch >= 2) ok = wait_buf(lb ^ 1) && ok;  // chunk nch - 2, not yet waited for
    ok = wait_buf(lb) && ok;
  }
  asm volatile("tcgen05.fence::after_thread_sync;");
  if (!ok && tid == 0) atomicOr(err, 1u);
  // warp w and w + 4 share TMEM lanes 32 (w % 4)..: thread = output row lr, w < 4 takes the
  // batch columns [0, NT/2), w >= 4 the rest
  const int quarter = wid & 3, half = wid >> 2;
  const int lr = quarter * 32 + lane, row = row0 + lr;
  const bool rvalid = row < N;
  const int rr = min(row, N - 1);
  const int tile = blockIdx.y * gridDim.x + blockIdx.x;
  bool emit_here = ksplit == 1 || MODE == 2;
  if (!emit_here) {
    // partial sums -> ws; the last CTA of the tile emits
    for (int c0 = half * (NT / 2); c0 < (half + 1) * (NT / 2); c0 += 8) {
      uint32_t v[8];
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                   : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                   : "r"(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int jj = 0; jj < 8; ++jj)
        if (rvalid && c0 + jj < nb) atomicAdd(ws + (size_t)(b0 + c0 + jj) * N + row, (int)v[jj]);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(cnt + tile, 1u) == (unsigned)(ksplit - 1);
    __syncthreads();
    if (!s_last) goto done;
    __threadfence();
  }
  {
    float scale = 0.f, a[DFSSM_RANK], cw[4] = {0.f, 0.f, 0.f, 0.f}, cb = 0.f;
    int ch = -1;
    if (MODE != 2) {
      scale = h2f(p.scale[rr]);
      const uint4 a0 = reinterpret_cast<const uint4*>(p.A16 + (size_t)rr * DFSSM_RANK)[0];
      const uint4 a1 = reinterpret_cast<const uint4*>(p.A16 + (size_t)rr * DFSSM_RANK)[1];
      const unsigned aw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&aw[i]));
        a[2 * i] = f.x;
        a[2 * i + 1] = f.y;
      }
      if (MODE == 0 && rr - d_inner >= 0 && rr - d_inner < d_xbc) {
        ch = rr - d_inner;
#pragma unroll
        for (int k = 0; k < 4; ++k) cw[k] = h2f(conv_w[ch * DFSSM_DCONV + k]);
        cb = h2f(conv_b[ch]);
      }
    }
    for (int c0 = half * (NT / 2); c0 < (half + 1) * (NT / 2); c0 += 8) {
      uint32_t v[8];
      if (ksplit == 1 || MODE == 2) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                     : "r"(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      } else {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          int* wp = ws + (size_t)(b0 + min(c0 + jj, nb - 1)) * N + rr;
          v[jj] = (rvalid && c0 + jj < nb) ? (uint32_t)__ldcg(wp) : 0u;
          if (rvalid && c0 + jj < nb) *wp = 0;  // clean for the next use
        }
      }
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int j = c0 + jj, b = b0 + j;
        if (!rvalid || j >= nb) continue;
        if (MODE == 2) {
          const int part = 2 * (int)v[jj] - (blockIdx.z == 0 ? e_qsum[j] : 0);
          int* o = reinterpret_cast<int*>(out) + (size_t)b * ld_out + row;
          if (ksplit == 1) *o = part;
          else atomicAdd(o, part);
          continue;
        }
        const int dot = 2 * (int)v[jj] - e_qsum[j];
        const float base = round_h(round_h(round_h((float)dot) * e_xs[j]) * scale);
        float la = 0.f;
#pragma unroll
        for (int r = 0; r < DFSSM_RANK; ++r) la = fmaf(e_t[j * DFSSM_RANK + r], a[r], la);
        const float vv = round_h(base + la);
        if (MODE == 0) {
          float res = vv;
          if (ch >= 0) {
            float* cs = conv_state + (size_t)b * 3 * d_xbc;
            const float s0 = cs[ch], s1 = cs[d_xbc + ch], s2 = cs[2 * d_xbc + ch];
            cs[ch] = s1;
            cs[d_xbc + ch] = s2;
            cs[2 * d_xbc + ch] = vv;
            const float o2 = s0 * cw[0] + s1 * cw[1] + s2 * cw[2] + vv * cw[3] + cb;
            const float sig = 1.0f / (1.0f + expf(-o2));
            res = o2 * sig;
          }
          out[(size_t)b * ld_out + row] = f2h(res);
        } else if (MODE == 3) {
          out[(size_t)b * ld_out + row] = f2h(vv);
        } else {
          __half* xo = out + (size_t)b * ld_out + row;
          *xo = f2h(h2f(*xo) + vv);
        }
      }
    }
    if (ksplit > 1 && MODE != 2 && tid == 0) cnt[tile] = 0u;
  }
done:
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (wid == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(NT));
}

}  // namespace dfssm
