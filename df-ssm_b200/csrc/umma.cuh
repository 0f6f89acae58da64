// Batched scaffold projection on the 5th-generation tensor cores (tcgen05, kind::i8), for batches
// of 96 and more (decode at large batch, prompt prefill rows, the stand-alone scaffold GEMM).
//
// One CTA computes a 128-row x NT-column tile of D = mask . q^T with the accumulator in tensor
// memory (TMEM): MMA M = 128 weight rows, N = NT batch rows, K in 128-byte chunks.
//   A (weights): the 0/1 sign masks as u8, built in shared memory from the packed bits: word w of
//     a row gives the 32 bytes (w >> j) & 0x01010101, j = 0..7 -- the permuted column order that
//     the quantised activations are stored in (qperm_index), so A and B columns line up.
//   B (activations): the permuted int8 q rows, as s8.
//   D (s32): sum over k of mask * q; the signed product is 2 D - sum_k q, as in the GEMV paths,
//     so the int32 result equals torch._int_mm on the +-1 weights bit for bit.
// Both operands use the K-major 128-byte-swizzled layout (8-row atoms of 1 KB; 16-byte unit u of
// row r sits at unit u ^ (r % 8)), one 128-byte row per K chunk.  Data movement per CTA:
//   - per K chunk, one ring slot receives by TMA the activation tile (NT rows x 128 bytes, tensor
//     map over q, 128-byte swizzle) and the weight rows' packed bits (128 rows x 16 bytes, tensor
//     map over the bits, no swizzle) on one mbarrier; the ring is kUmmaSB slots deep, and a slot is
//     refilled (kUmmaSB chunks on) as soon as the MMAs that read it have committed;
//   - the threads expand a chunk's bits into the u8 masks (shared to shared) in one of two A buffers.
// tcgen05.commit of chunk c's MMAs on an mbarrier frees its A buffer and ring slot.  The epilogue
// reads D with tcgen05.ld (warp w and w + 4 own TMEM lanes 32(w % 4).., i.e. output rows; each
// thread holds its row's dequant/LoRA/conv operands in registers) and runs the same per-element
// arithmetic as proj_mma_kernel.
#pragma once
#include <cuda.h>  // CUtensorMap (the map is encoded on the host through the driver entry point)

#include "common.cuh"

namespace dfssm {

constexpr int kUmmaThreads = 256;
constexpr int kUmmaKC = 128;        // K bytes per chunk (4 MMAs of K = 32; one 128-byte swizzle row)
constexpr int kUmmaMinBatch = 96;   // batches below this use proj_mma_kernel (mma.sync)
constexpr int kUmmaSpin = 1 << 22;  // bound of every mbarrier wait
constexpr int kUmmaSB = 3;          // ring depth (chunks in flight)
constexpr int kUmmaRawBytes = 128 * kUmmaKC / 8;  // one chunk of the 128 weight rows' bits

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
  return 1024 + (size_t)2 * 128 * kUmmaKC + (size_t)kUmmaSB * (NT * kUmmaKC + kUmmaRawBytes) + 2 * NT * 4 +
         NT * DFSSM_RANK * 4;  // + base alignment
}

// MODE as proj_mma_kernel: 0 in_proj + conv1d, 1 out_proj + residual, 2 raw int32, 3 plain.
// Grid (ceil(N / 128), ceil(B / NT), ksplit); (K / ksplit) % 128 == 0.  With ksplit > 1 the CTAs
// of a tile each take a K range (narrow projections would otherwise leave most SMs idle): the
// integer partials meet exactly, in any order, through atomicAdd -- into `out` for MODE 2 (zeroed
// by the caller), else into ws [B][N] int32 with a per-tile counter cnt, and the last CTA of the
// tile runs the epilogue and clears its part of ws and its counter.  err: set to 1 if a wait ran
// out.
// tmq: tensor map over q [B][K] int8, box 128 bytes x NT rows, 128-byte swizzle (rows past B read
// as zeros).  tmw: tensor map over the packed bits [N][K / 8] bytes, box 16 bytes x 128 rows, no
// swizzle (rows past N read as zeros).  K / ksplit is a multiple of 128.
template <int MODE, int NT>
__global__ void __launch_bounds__(kUmmaThreads, 1)
proj_umma_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmw, ProjW p,
                 const int* __restrict__ qsum, const __half* __restrict__ xs,
                 const __half* __restrict__ t, int B, __half* __restrict__ out, int ld_out,
                 float* __restrict__ conv_state, const __half* __restrict__ conv_w, const __half* __restrict__ conv_b,
                 int d_inner, int d_xbc, int ksplit, int* __restrict__ ws, unsigned* __restrict__ cnt,
                 unsigned* __restrict__ err) {
  static_assert(kUmmaKC == 128, "the swizzled layout holds one 128-byte row per chunk");
  constexpr int ABYTES = 128 * kUmmaKC, BBYTES = NT * kUmmaKC;
  constexpr int WPR = kUmmaKC / 32;  // bit words per row and chunk
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // 1 KB-aligned base (the 128-byte swizzle atoms and TMA destinations need it)
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int N = p.N, K = p.K;
  const int klen = K / ksplit, kbeg = blockIdx.z * klen, nch = klen / kUmmaKC;
  auto sA = [&](int k) { return smem + k * ABYTES; };                          // 2 mask buffers
  auto sB = [&](int k) { return smem + 2 * ABYTES + k * BBYTES; };              // ring: activation tiles
  auto sW = [&](int k) { return smem + 2 * ABYTES + kUmmaSB * BBYTES + k * kUmmaRawBytes; };  // ring: bits
  float* e_xs = reinterpret_cast<float*>(sW(kUmmaSB));                           // [NT]
  int* e_qsum = reinterpret_cast<int*>(e_xs + NT);                               // [NT]
  float* e_t = reinterpret_cast<float*>(e_qsum + NT);                            // [NT][16]
  __shared__ uint64_t mbars[kUmmaSB];  // MMAs of the chunk in slot s complete
  __shared__ uint64_t fulls[kUmmaSB];  // activation tile and weight bits of slot s landed
  __shared__ uint32_t s_tmem;
  __shared__ int s_last;
  const int tid = threadIdx.x, wid = tid >> 5, lane = tid & 31;
  const int row0 = blockIdx.x * 128, b0 = blockIdx.y * NT, nb = min(NT, B - b0);
  if (wid == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)), "r"(NT));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int i = 0; i < kUmmaSB; ++i) {
      mbar_init(&mbars[i], 1);
      mbar_init(&fulls[i], 1);
    }
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

  auto issue = [&](int c) {  // thread 0: chunk c's activation tile and weight bits into slot c % kUmmaSB
    const int sl = c % kUmmaSB, kc = kbeg + c * kUmmaKC;
    mbar_expect_tx(&fulls[sl], (unsigned)(BBYTES + kUmmaRawBytes));
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(sB(sl))),
        "l"(reinterpret_cast<uint64_t>(&tmq)), "r"(kc), "r"(b0), "r"(smem_u32(&fulls[sl]))
        : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(sW(sl))),
        "l"(reinterpret_cast<uint64_t>(&tmw)), "r"(kc >> 3), "r"(row0), "r"(smem_u32(&fulls[sl]))
        : "memory");
  };
  if (tid == 0)
    for (int c = 0; c < kUmmaSB && c < nch; ++c) issue(c);
  // chunk c's masks into A buffer c & 1: thread i expands word j = i % WPR of row i / WPR (+64)
  auto expand = [&](int c) {
    const unsigned char* raw = sW(c % kUmmaSB);
#pragma unroll
    for (int u = 0; u < 128 * WPR / kUmmaThreads; ++u) {
      const int i = tid + u * kUmmaThreads, r = i / WPR, j = i - r * WPR;
      const uint32_t x = *reinterpret_cast<const uint32_t*>(raw + r * (kUmmaKC / 8) + 4 * j);
      const uint4 lo = make_uint4(x & 0x01010101u, (x >> 1) & 0x01010101u, (x >> 2) & 0x01010101u,
                                  (x >> 3) & 0x01010101u);
      const uint4 hi = make_uint4((x >> 4) & 0x01010101u, (x >> 5) & 0x01010101u, (x >> 6) & 0x01010101u,
                                  (x >> 7) & 0x01010101u);
      unsigned char* rowp = sA(c & 1) + (r >> 3) * 1024 + (r & 7) * 128;  // units 2j, 2j + 1, swizzled
      *reinterpret_cast<uint4*>(rowp + (((2 * j) ^ (r & 7)) << 4)) = lo;
      *reinterpret_cast<uint4*>(rowp + (((2 * j + 1) ^ (r & 7)) << 4)) = hi;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
  };
  auto slot_par = [](int c) { return (unsigned)((c / kUmmaSB) & 1); };
  // warp w and w + 4 share TMEM lanes 32 (w % 4)..: thread = output row lr, w < 4 takes the
  // batch columns [0, NT/2), w >= 4 the rest
  const int quarter = wid & 3, half = wid >> 2;
  const int lr = quarter * 32 + lane, row = row0 + lr;
  const bool rvalid = row < N;
  const int rr = min(row, N - 1);
  // this row's epilogue operands, loaded before the main loop so their latency overlaps it
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
  bool ok = umma_wait(&fulls[0], 0u);
  expand(0);
  for (int c = 0; c < nch; ++c) {
    const int sl = c % kUmmaSB;
    __syncthreads();  // chunk c's masks are stored
    asm volatile("tcgen05.fence::after_thread_sync;");
    if (tid == 0) {
      // chunk c's activation tile (its slot's barrier completed before expand(c) read the bits)
#pragma unroll
      for (int k = 0; k < kUmmaKC / 32; ++k) {  // K = 32 per MMA: 32 bytes along the 128-byte row
        const uint64_t da = umma_sdesc(smem_u32(sA(c & 1)) + k * 32, 16, 1024, 2);
        const uint64_t db = umma_sdesc(smem_u32(sB(sl)) + k * 32, 16, 1024, 2);
        const uint32_t accum = (c > 0 || k > 0) ? 1u : 0u;
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
                     "l"(da), "l"(db), "r"(idesc), "r"(accum));
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(&mbars[sl]))
                   : "memory");
    }
    if (c >= 1) {
      // chunk c - 1's MMAs are done: its A buffer (that of chunk c + 1) and its ring slot (that of
      // chunk c - 1 + kUmmaSB) are free
      const int pc = c - 1;
      ok = umma_wait(&mbars[pc % kUmmaSB], slot_par(pc)) && ok;
      if (tid == 0 && pc + kUmmaSB < nch) issue(pc + kUmmaSB);
    }
    if (c + 1 < nch) {
      ok = umma_wait(&fulls[(c + 1) % kUmmaSB], slot_par(c + 1)) && ok;
      expand(c + 1);
    }
  }
  // the last chunk's MMAs (and with them all earlier ones) complete
  ok = umma_wait(&mbars[(nch - 1) % kUmmaSB], (unsigned)(((nch - 1) / kUmmaSB) & 1)) && ok;
  asm volatile("tcgen05.fence::after_thread_sync;");
  if (!ok && tid == 0) atomicOr(err, 1u);
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
    for (int c0 = half * (NT / 2); c0 < (half + 1) * (NT / 2); c0 += 8) {
      uint32_t v[8];
      if (ksplit == 1 || MODE == 2) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                     : "r"(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      } else {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj)
          v[jj] = (rvalid && c0 + jj < nb) ? (uint32_t)__ldcg(ws + (size_t)(b0 + c0 + jj) * N + rr) : 0u;
#pragma unroll
        for (int jj = 0; jj < 8; ++jj)  // clean for the next use (after all 8 loads are out)
          if (rvalid && c0 + jj < nb) ws[(size_t)(b0 + c0 + jj) * N + rr] = 0;
      }
      // the group's other global operands (conv taps, residual), all requested before any is used
      float g0[8], g1[8], g2[8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        g0[jj] = g1[jj] = g2[jj] = 0.f;
        const int b = b0 + c0 + jj;
        if (!rvalid || c0 + jj >= nb) continue;
        if (MODE == 0 && ch >= 0) {
          const float* cs = conv_state + (size_t)b * 3 * d_xbc;
          g0[jj] = cs[ch];
          g1[jj] = cs[d_xbc + ch];
          g2[jj] = cs[2 * d_xbc + ch];
        } else if (MODE == 1) {
          g0[jj] = h2f(out[(size_t)b * ld_out + row]);
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
        const float vv = round_h(base + round_h(la));
        if (MODE == 0) {
          float res = vv;
          if (ch >= 0) {
            float* cs = conv_state + (size_t)b * 3 * d_xbc;
            const float s0 = g0[jj], s1 = g1[jj], s2 = g2[jj];
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
          out[(size_t)b * ld_out + row] = f2h(g0[jj] + vv);
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
